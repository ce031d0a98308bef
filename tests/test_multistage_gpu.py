"""GPU, one process per GPU: the multi-process pipeline (multistage.RankPipeline: receive and
token slots exported with CUDA IPC, the boundary encoder and the last stage's argmax storing
into the peer over NVLink, device flags with bounded waits) produces the oracle's greedy
tokens for the tiny Qwen3 model, 2 stages (layers 0-1 / 2-3), 2 micro-batches of 16
sequences each, int8-had and int4-had boundaries."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle.model import OraclePipeline, quantize_state_dict
from superl8_serve_b200.config import tiny
from superl8_serve_b200.weights import random_state_dict

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

STEPS = 8
M = 16  # sequences per micro-batch (tensor-core GEMM and persistent attention)


def _first_ids(n, vocab):
    return ((7 * np.arange(n) + 3) % vocab).astype(np.int32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, scheme, out_path):
    import torch.distributed as dist

    from superl8_serve_b200.multistage import RankPipeline

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    cfg = tiny()
    sd = random_state_dict(cfg, 11, w_std=0.1)
    pipe = RankPipeline(cfg, rank, world, m=M, max_len=STEPS + 16, ctx=0, scheme=scheme,
                        state_dict=sd, fill_kv=False)
    ids_h = torch.from_numpy(_first_ids(M * world, cfg.vocab_size)).pin_memory()
    out_h = torch.zeros(M * world, dtype=torch.int32).pin_memory()
    if pipe.plan.first:
        pipe.put_ids(ids_h)
    torch.cuda.synchronize()
    dist.barrier()
    toks = []
    for _ in range(STEPS):
        pipe.enqueue_step()  # the last stage's argmax lands in stage 0's token slots
        if pipe.plan.first:
            pipe.get_tokens(out_h)
        torch.cuda.synchronize()
        if pipe.plan.first:
            toks.append(out_h.numpy().copy())
    pipe.check_status()
    if rank == 0:
        np.save(out_path, np.stack(toks))
    pipe.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("scheme", ["int8-had", "int4-had"])
def test_two_process_pipeline_matches_oracle(tmp_path, scheme):
    world = 2
    out_path = str(tmp_path / "toks.npy")
    mp.spawn(_rank_main, args=(world, _free_port(), scheme, out_path), nprocs=world, join=True)
    got = np.load(out_path)  # [STEPS, world * M]
    cfg = tiny()
    qw = quantize_state_dict(random_state_dict(cfg, 11, w_std=0.1), cfg)
    first = _first_ids(M * world, cfg.vocab_size)
    ref, _ = OraclePipeline(cfg, qw, n_stages=world, wire_scheme=scheme, num_slots=M * world,
                            max_len=STEPS + 16).generate([[int(t)] for t in first], STEPS)
    assert got.T.tolist() == ref
