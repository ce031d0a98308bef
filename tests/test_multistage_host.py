"""CPU: host-side logic of the one-process-per-GPU pipeline: per-rank layout and the handle
exchange between ranks, run as world-size-2 (and 4) gloo process groups on 127.0.0.1."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from superl8_serve_b200.dist.pipeline import stage_bounds
from superl8_serve_b200.multistage import RankPlan, peer_handles, plan_rank


def _sizes(T, D, scheme):
    return (T * D, T) if scheme.startswith("int8") else (T * D // 2, T * D // 128)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_rank_layout(world):
    bounds = stage_bounds(36, world)
    for r in range(world):
        p = plan_rank(36, 4096, r, world, 64, "int8-had", payload_bytes_fn=_sizes)
        assert p.layers == (bounds[r], bounds[r + 1])
        assert p.n_micro == world
        assert p.slot_payload == 64 * 8192 and p.slot_scales == 64
        assert p.slot_bytes % 256 == 0 and p.slot_bytes >= 64 * 8192 + 256
        assert (p.recv_bytes > 0) == (r > 0)
        assert (p.tok_bytes > 0) == (r == 0)
    with pytest.raises(ValueError):
        plan_rank(4, 4096, 0, 8, 64, "int8-had", payload_bytes_fn=_sizes)


def test_plan_rank_int4_scales():
    p = plan_rank(64, 5120, 3, 8, 32, "int4-had", payload_bytes_fn=_sizes)
    assert p.slot_payload == 32 * 10240 // 2 and p.slot_scales == 32 * 80


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from superl8_serve_b200.multistage import exchange_infos

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    plan = plan_rank(36, 4096, rank, world, 64, "int8-had", payload_bytes_fn=_sizes)
    info = {"rank": rank, "recv": bytes([rank, 1]) if rank else b"",
            "tok": bytes([rank, 2]) if rank == 0 else b"", "flag": bytes([rank, 3])}
    infos = exchange_infos(info, world)
    q.put((rank, [i["rank"] for i in infos], peer_handles(plan, infos)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_handle_exchange_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict((r, (ranks, h)) for r, ranks, h in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        ranks, h = got[r]
        assert ranks == list(range(world))
        if r < world - 1:
            assert h["next_recv"] == bytes([r + 1, 1]) and h["next_flag"] == bytes([r + 1, 3])
        if r == world - 1:
            assert h["first_tok"] == bytes([0, 2]) and h["first_flag"] == bytes([0, 3])
            assert "next_recv" not in h


def test_balanced_stage_bounds():
    from superl8_serve_b200.dist.pipeline import balanced_stage_bounds

    assert balanced_stage_bounds(36, 1, last_extra=0.9) == [0, 36]
    assert balanced_stage_bounds(36, 2) == stage_bounds(36, 2)
    for S in (2, 4, 8):
        b = balanced_stage_bounds(36, S, last_extra=0.9)
        assert b[0] == 0 and b[-1] == 36 and all(b[i] < b[i + 1] for i in range(S))
        cost = [b[i + 1] - b[i] + (0.9 if i == S - 1 else 0.0) for i in range(S)]
        even = stage_bounds(36, S)
        even_cost = [even[i + 1] - even[i] + (0.9 if i == S - 1 else 0.0) for i in range(S)]
        assert max(cost) <= max(even_cost)
    assert balanced_stage_bounds(36, 8, last_extra=0.9)[-2] >= 32  # head stage gets <= 4
    with pytest.raises(ValueError):
        balanced_stage_bounds(4, 8)
    p = plan_rank(36, 4096, 7, 8, 64, "int8-had", payload_bytes_fn=_sizes,
                  bounds=balanced_stage_bounds(36, 8, last_extra=0.9))
    assert p.layers[1] == 36
    with pytest.raises(ValueError):
        plan_rank(36, 4096, 0, 2, 64, "int8-had", payload_bytes_fn=_sizes, bounds=[0, 40, 36])
