"""GPU, one process per GPU: expert parallelism across processes (BASELINE config 4's layout,
PP x EP). Every stage's home process runs the stage and expert range 0 of each sparse-MoE
layer; a partner process per further range receives the layer's token rows and routing by
peer copies, runs its experts and stores its contribution rows into the home's buffer over
NVLink, with bounded device flags on both sides (multistage.ExpertPartner, RemoteExperts).
The tiny Qwen3-MoE model (16 experts top-4 in every layer) must give the oracle's greedy
tokens: 1 stage x 2 expert ranges on 2 GPUs, and 2 stages x 2 on 4 GPUs."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle.model import OraclePipeline, quantize_state_dict
from superl8_serve_b200.config import tiny_moe
from superl8_serve_b200.weights import random_state_dict

pytestmark = pytest.mark.gpu

STEPS = 6
M = 16


def _first_ids(n, vocab):
    return ((5 * np.arange(n) + 1) % vocab).astype(np.int32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, ep, port, out_path):
    import torch.distributed as dist

    from superl8_serve_b200.multistage import ExpertPartner, RankPipeline, plan_roles

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    cfg = tiny_moe()
    sd = random_state_dict(cfg, 13, w_std=0.1)
    S, role, _, _ = plan_roles(rank, world, ep)
    if role == "home":
        pipe = RankPipeline(cfg, rank, S, m=M, max_len=STEPS + 16, ctx=0, scheme="int8-had",
                            state_dict=sd, fill_kv=False, ep=ep)
    else:
        pipe = ExpertPartner(cfg, rank, S, ep, m=M, state_dict=sd)
    first = role == "home" and pipe.plan.first
    ids_h = torch.from_numpy(_first_ids(M * S, cfg.vocab_size)).pin_memory()
    out_h = torch.zeros(M * S, dtype=torch.int32).pin_memory()
    if first:
        pipe.put_ids(ids_h)
    torch.cuda.synchronize()
    dist.barrier()
    toks = []
    for _ in range(STEPS):
        pipe.enqueue_step()
        if first:
            pipe.get_tokens(out_h)
        torch.cuda.synchronize()
        if first:
            toks.append(out_h.numpy().copy())
    pipe.check_status()
    if rank == 0:
        np.save(out_path, np.stack(toks))
    pipe.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("stages,ep", [(1, 2), (2, 2)])
def test_expert_parallel_processes_match_oracle(tmp_path, stages, ep):
    world = stages * ep
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out_path = str(tmp_path / "toks.npy")
    mp.spawn(_rank_main, args=(world, ep, _free_port(), out_path), nprocs=world, join=True)
    got = np.load(out_path)  # [STEPS, stages * M]
    cfg = tiny_moe()
    qw = quantize_state_dict(random_state_dict(cfg, 13, w_std=0.1), cfg)
    first = _first_ids(M * stages, cfg.vocab_size)
    ref, _ = OraclePipeline(cfg, qw, n_stages=stages, wire_scheme="int8-had",
                            num_slots=M * stages, max_len=STEPS + 16).generate(
        [[int(t)] for t in first], STEPS)
    assert got.T.tolist() == ref
