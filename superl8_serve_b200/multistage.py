"""One-process-per-GPU pipeline decode (torchrun): rank r runs stage r of S = world size.

Stage-to-stage data never touches the host:

* rank r > 0 owns S receive slots (one per micro-batch: boundary codes + scales) and rank 0
  owns S token slots (next input ids). They are allocated with ``s8b_ipc_alloc``; the handles
  are exchanged once over the process group and mapped by the producer (``s8b_ipc_open``).
* the producer's codec encoder (or, on the last stage, the greedy argmax) stores straight into
  the consumer's slot over NVLink, then raises the slot's ready flag to the step's epoch with a
  system-scope release store (``s8b_flag_set``);
* the consumer's first kernel for that micro-batch is a bounded device-side wait on its own
  flag (``s8b_flag_wait``); a missing producer ends in S8B_ERR_TIMEOUT in a status word, never
  a hang.

Epochs live in device memory and advance by one per step inside the captured graph, so each
rank replays one CUDA graph per step. Slots need no "free" handshake: micro-batch k of step
t+1 starts from the tokens that micro-batch k produced at the end of step t, so every stage has
consumed its step-t slot before the slot is written again.

Micro-batches: S of ``m`` rows each (global batch m*S): per-GPU work is fixed as S grows.
"""

from __future__ import annotations

import ctypes as C
import json
import math
import os
import time
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import CODEC, call, load, ptr, stream
from .dist.pipeline import balanced_stage_bounds, stage_bounds
from .ops import codec_sizes
from .runtime import (KVPool, MicroBatch, RemoteExperts, StageModel, StageRunner, moe_experts,
                      moe_expert_buffers)

FLAG_TIMEOUT_NS = 20_000_000_000  # 20 s: generous for cold first steps, still bounded


class DevPtr:
    """A raw device pointer with the few tensor-like attributes the launch helpers use."""

    def __init__(self, addr: int, numel: int = 0):
        self.addr = int(addr)
        self.numel_ = numel
        self.is_cuda = True

    def data_ptr(self) -> int:
        return self.addr

    def is_contiguous(self) -> bool:
        return True

    def numel(self) -> int:
        return self.numel_

    def offset(self, nbytes: int, numel: int = 0) -> "DevPtr":
        return DevPtr(self.addr + nbytes, numel)


@dataclass
class RankPlan:
    """Pure host-side layout of one rank (testable without a GPU)."""

    rank: int
    world: int
    layers: tuple[int, int]
    m: int
    n_micro: int
    slot_payload: int
    slot_scales: int
    slot_bytes: int
    recv_bytes: int
    tok_bytes: int
    flag_bytes: int

    @property
    def first(self) -> bool:
        return self.rank == 0

    @property
    def last(self) -> bool:
        return self.rank == self.world - 1


# last-stage extra work (final norm, LM head, sampler) in Qwen3-8B layer units at the bench
# shape: LM head ~140 us against ~158 us per layer on B200
HEAD_LAYERS = 0.9


def plan_rank(n_layers: int, hidden: int, rank: int, world: int, m: int, scheme: str,
              payload_bytes_fn=None, bounds: list[int] | None = None) -> RankPlan:
    """``bounds``: layer split (default: the reference's even split, stage_bounds)."""
    if world > n_layers:
        raise ValueError("pipeline stage count cannot exceed the model layer count")
    b = stage_bounds(n_layers, world) if bounds is None else list(bounds)
    if len(b) != world + 1 or b[0] != 0 or b[-1] != n_layers or any(
            b[i] >= b[i + 1] for i in range(world)):
        raise ValueError(f"bad stage bounds {b} for {n_layers} layers / {world} stages")
    fn = payload_bytes_fn or (lambda T, D, s: codec_sizes(T, D, s))
    pay, nsc = fn(m, 2 * hidden, scheme)
    pay_al = (pay + 255) // 256 * 256
    sc_al = (max(nsc, 1) * 4 + 255) // 256 * 256
    slot = pay_al + sc_al
    n_micro = world
    return RankPlan(rank, world, (b[rank], b[rank + 1]), m, n_micro, pay, max(nsc, 1), slot,
                    slot * n_micro if rank > 0 else 0,
                    ((m * 4 + 255) // 256 * 256) * n_micro if rank == 0 else 0,
                    ((2 * n_micro * 4 + 255) // 256) * 256)


def exchange_infos(info: dict, world: int, pg=None) -> list[dict]:
    """All-gather every rank's exported handles (bytes) over the process group."""
    import torch.distributed as dist

    infos = [None] * world
    dist.all_gather_object(infos, info, group=pg)
    return infos


def peer_handles(plan: RankPlan, infos: list[dict]) -> dict[str, bytes]:
    """Handles this rank maps: the next stage's receive slots and flags (all but the last
    stage), stage 0's token slots and flags (the last stage of a multi-stage pipeline)."""
    out: dict[str, bytes] = {}
    if not plan.last:
        out["next_recv"] = infos[plan.rank + 1]["recv"]
        out["next_flag"] = infos[plan.rank + 1]["flag"]
    if plan.last and plan.world > 1:
        out["first_tok"] = infos[0]["tok"]
        out["first_flag"] = infos[0]["flag"]
    return out


def _alloc_ipc(nbytes: int):
    lib = load()
    hsz = lib.s8b_ipc_handle_size()
    handle = (C.c_uint8 * hsz)()
    p = C.c_void_p()
    call("s8b_ipc_alloc", max(nbytes, 256), C.byref(p), handle)
    return p.value, bytes(handle)


def _open_ipc(handle: bytes) -> int:
    buf = (C.c_uint8 * len(handle)).from_buffer_copy(handle)
    p = C.c_void_p()
    call("s8b_ipc_open", buf, C.byref(p))
    return p.value


class RankPipeline:
    """Stage ``rank`` of an S-stage pipeline on the current CUDA device."""

    def __init__(self, cfg, rank: int, world: int, *, m: int, max_len: int, ctx: int,
                 scheme: str = "int8-had", seed: int = 0, pg=None, state_dict=None,
                 fill_kv: bool = True, bounds: list[int] | None = None, ep: int = 1):
        """``state_dict`` (HF-style float weights) selects real weights for this rank's layer
        range; without it the weights are synthetic (benchmarks). ``fill_kv`` pre-fills the
        KV pool with random codes for a synthetic context of ``ctx`` tokens; with
        ``fill_kv=False`` and ``ctx=0`` every sequence starts empty. ``world`` is the stage
        count; with ``ep`` > 1 the process group has ep * world ranks and ranks world ..
        ep * world - 1 are ExpertPartner processes holding the further expert ranges of the
        sparse-MoE layers (``plan_roles``)."""
        self.cfg, self.rank, self.world = cfg, rank, world
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self.plan = plan_rank(cfg.num_hidden_layers, cfg.hidden_size, rank, world, m, scheme,
                              bounds=bounds)
        self.scheme = scheme
        S, H = world, cfg.hidden_size
        lo, hi = self.plan.layers
        if state_dict is not None:
            self.model = StageModel.from_state_dict(cfg, state_dict, lo, hi, self.dev,
                                                    first=self.plan.first, last=self.plan.last)
        else:
            self.model = StageModel.synthetic(cfg, lo, hi, self.dev, first=self.plan.first,
                                              last=self.plan.last, seed=seed)
        self.m = m
        self.max_blocks = (max_len + 15) // 16
        nb = m * S * self.max_blocks
        self.pool = KVPool(hi - lo, nb, cfg.num_key_value_heads, cfg.resolved_head_dim(), 16,
                           self.dev)
        if fill_kv:
            self.pool.fill_random(seed=seed * 7 + rank)
        self.ep = ep
        self.ep_cuts = ep_cuts(cfg.num_experts, ep) if ep > 1 else None
        if ep > 1:  # keep this GPU's expert range [cuts[0], cuts[1]) of every MoE layer
            h = self.ep_cuts[1]
            for L in self.model.layers:
                mw = L.moe
                if mw is not None:
                    mw.gu_w, mw.gu_s = mw.gu_w[:h].clone(), mw.gu_s[:h].clone()
                    mw.d_w, mw.d_s = mw.d_w[:h].clone(), mw.d_s[:h].clone()
            torch.cuda.empty_cache()
        self.runner = StageRunner(self.model, self.pool, m, max_len)
        # device-side per micro-batch state: sequence j = k*m + i owns blocks
        # [j*max_blocks, (j+1)*max_blocks) (identical layout on every stage)
        self.mbs = []
        for k in range(S):
            base = torch.arange(m, dtype=torch.int32).unsqueeze(1) + k * m
            bt = (base * self.max_blocks + torch.arange(self.max_blocks, dtype=torch.int32)).to(self.dev)
            pos = torch.full((m,), ctx, dtype=torch.int32, device=self.dev)
            self.mbs.append(MicroBatch(ids=torch.zeros(m, dtype=torch.int32, device=self.dev),
                                       positions=pos, context_lens=pos + 1, block_table=bt))
        # IPC buffers: receive slots (r > 0), token slots (r == 0), flags (everyone)
        self.own = []
        self.recv_ptr = self.tok_ptr = None
        recv_h = tok_h = b""
        if self.plan.recv_bytes:
            self.recv_ptr, recv_h = _alloc_ipc(self.plan.recv_bytes)
            self.own.append(self.recv_ptr)
        if self.plan.tok_bytes:
            self.tok_ptr, tok_h = _alloc_ipc(self.plan.tok_bytes)
            self.own.append(self.tok_ptr)
        self.flag_ptr, flag_h = _alloc_ipc(self.plan.flag_bytes)
        self.own.append(self.flag_ptr)
        info = {"rank": rank, "recv": recv_h, "tok": tok_h, "flag": flag_h}
        moe = [L.moe for L in self.model.layers if L.moe is not None]
        if ep > 1 and moe:
            # the contribution rows partners store into, and this GPU's completion flags
            k, H = moe[0].top_k, cfg.hidden_size
            self.contrib_ptr, info["ep_contrib"] = _alloc_ipc(m * k * H * 2)
            self.epflag_ptr, info["ep_flag"] = _alloc_ipc(256)
            self.own += [self.contrib_ptr, self.epflag_ptr]
            self.runner.moe_buf["contrib"] = DevPtr(self.contrib_ptr, m * k * H)
        infos = exchange_infos(info, world * ep, pg)
        mapped = {k: _open_ipc(h) for k, h in peer_handles(self.plan, infos).items()}
        self.opened = list(mapped.values())
        self.next_recv, self.next_flag = mapped.get("next_recv"), mapped.get("next_flag")
        self.first_tok, self.first_flag = mapped.get("first_tok"), mapped.get("first_flag")
        if self.plan.last and world == 1:
            self.first_tok, self.first_flag = self.tok_ptr, self.flag_ptr
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.status = torch.zeros(4, dtype=torch.int32, device=self.dev)
        self.moe_epoch = torch.zeros(1, dtype=torch.int32, device=self.dev)
        if ep > 1 and moe:  # map every partner's input block and flag; hand the ranges out
            for j in range(1, ep):
                inf = infos[j * world + rank]
                base, fl = _open_ipc(inf["ep_in"]), _open_ipc(inf["ep_flag"])
                self.opened += [base, fl]
                lay = ep_input_layout(m, moe[0].top_k, cfg.hidden_size, cfg.num_experts)
                for mw in moe:
                    mw.remote.append(RemoteExperts(
                        self.ep_cuts[j], self.ep_cuts[j + 1], base + lay["xq"], base + lay["xs"],
                        base + lay["offsets"], base + lay["sorted_token"], fl,
                        self.epflag_ptr + 4 * (j - 1), ptr(self.moe_epoch), ptr(self.status),
                        FLAG_TIMEOUT_NS))
        # token slots: stage 0 reads its ids there; the last stage writes the next ids there
        tok_stride = (m * 4 + 255) // 256 * 256
        for k in range(S):
            if self.plan.first:
                self.mbs[k].ids = DevPtr(self.tok_ptr + k * tok_stride, m)
            elif self.plan.last:
                self.mbs[k].ids = DevPtr(self.first_tok + k * tok_stride, m)
        self.graph = self.graph_io = None

    # flags: [ready[S] | tok_ready[S]] uint32 in each rank's flag block
    def _ready_flag(self, base: int, k: int) -> DevPtr:
        return DevPtr(base + 4 * k)

    def _tok_flag(self, base: int, k: int) -> DevPtr:
        return DevPtr(base + 4 * (self.world + k))

    def _slot(self, base: int, k: int):
        p = self.plan
        s = base + k * p.slot_bytes
        pay_al = (p.slot_payload + 255) // 256 * 256
        return (DevPtr(s, p.slot_payload), DevPtr(s + pay_al, p.slot_scales), self.scheme)

    @property
    def tok_stride(self) -> int:
        return (self.m * 4 + 255) // 256 * 256

    def put_ids(self, ids_host: torch.Tensor):
        """Stage 0: copy the step's input ids (pinned host, m*S int32) into the token slots."""
        st = stream()
        for k in range(self.world):
            call("s8b_memcpy_async", self.tok_ptr + k * self.tok_stride,
                 ids_host.data_ptr() + 4 * k * self.m, 4 * self.m, st)

    def get_tokens(self, out_host: torch.Tensor, epoch_add: int = 0):
        """Stage 0: wait (on the device, bounded) until the last stage delivered this step's
        tokens, then copy them to pinned host memory."""
        st = stream()
        for k in range(self.world):
            if self.world > 1:
                call("s8b_flag_wait", self._tok_flag(self.flag_ptr, k).addr, ptr(self.epoch),
                     epoch_add, FLAG_TIMEOUT_NS, ptr(self.status), st)
            call("s8b_memcpy_async", out_host.data_ptr() + 4 * k * self.m,
                 self.tok_ptr + k * self.tok_stride, 4 * self.m, st)

    def enqueue_step(self, *, token_return: bool = True, host_io: torch.Tensor | None = None,
                     solo: bool = False):
        """Enqueue this rank's share of one step. On stage 0, ``host_io`` (pinned int32, m*S)
        routes every micro-batch's input ids through host memory once they have arrived: the
        token slot is copied device -> host into ``host_io`` and back, stream-ordered, so the
        host holds each step's tokens without draining the pipeline. ``solo`` runs this
        stage's work for every micro-batch with no flag waits or sets (its own device time per
        step, for the stage-time report; the boundary slots are read and written as usual)."""
        S, st = self.world, stream()
        for k in range(S):
            mb = self.mbs[k]
            if self.plan.first and S > 1 and token_return and not solo:
                call("s8b_flag_wait", self._tok_flag(self.flag_ptr, k).addr, ptr(self.epoch), 0,
                     FLAG_TIMEOUT_NS, ptr(self.status), st)
            if self.plan.first and host_io is not None:
                slot = self.tok_ptr + k * self.tok_stride
                dst = host_io.data_ptr() + 4 * k * self.m
                call("s8b_memcpy_async", dst, slot, 4 * self.m, st)
                call("s8b_memcpy_async", slot, dst, 4 * self.m, st)
            bin_ = bout = None
            if not self.plan.first:
                if not solo:
                    call("s8b_flag_wait", self._ready_flag(self.flag_ptr, k).addr,
                         ptr(self.epoch), 1, FLAG_TIMEOUT_NS, ptr(self.status), st)
                bin_ = self._slot(self.recv_ptr, k)
            if not self.plan.last:
                bout = self._slot(self.next_recv, k)
            self.runner.run(mb, self.m, boundary_in=bin_, boundary_out=bout)
            if solo:
                pass
            elif not self.plan.last:
                call("s8b_flag_set", self._ready_flag(self.next_flag, k).addr, ptr(self.epoch), 1, st)
            elif S > 1:
                call("s8b_flag_set", self._tok_flag(self.first_flag, k).addr, ptr(self.epoch), 1, st)
            call("s8b_advance", ptr(mb.positions), ptr(mb.context_lens), self.m, 1, st)
        if not solo:
            call("s8b_counter_add", ptr(self.epoch), 1, st)

    def solo_ms(self, reps: int) -> float:
        """Device time of this stage's work for one step with no waits (see enqueue_step);
        MoE layers run this GPU's expert range only."""
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        g = torch.cuda.CUDAGraph()
        self.runner.skip_remote = True
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.enqueue_step(solo=True)
        self.runner.skip_remote = False
        torch.cuda.current_stream(self.dev).wait_stream(s)
        g.replay()
        torch.cuda.synchronize(self.dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        b.synchronize()
        del g
        return a.elapsed_time(b) / reps

    def capture(self, host_io: torch.Tensor | None = None):
        """Capture one step into a CUDA graph; with ``host_io`` (stage 0's pinned token
        buffer; other ranks pass None) the graph is replayed by step_host_io()."""
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.enqueue_step(host_io=host_io)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        if host_io is None and not getattr(self, "_capturing_io", False):
            self.graph = g
        else:
            self.graph_io = g

    def capture_host_io(self, host_io: torch.Tensor | None):
        """The host-I/O variant of the step graph on every rank (stage 0 gets the copies)."""
        self._capturing_io = True
        try:
            self.capture(host_io if self.plan.first else None)
        finally:
            self._capturing_io = False

    def step(self):
        self.graph.replay()

    def step_host_io(self):
        self.graph_io.replay()

    def check_status(self):
        st = self.status.cpu().tolist()
        if st[0] != 0:
            raise RuntimeError(f"rank {self.rank}: device wait timed out (awaited epoch {st[1]}, "
                               f"saw {st[2]})")

    def close(self, pg=None):
        import torch.distributed as dist

        torch.cuda.synchronize(self.dev)
        self.graph = self.graph_io = None
        for p in self.opened:
            call("s8b_ipc_close", p)
        dist.barrier(group=pg)
        for p in self.own:
            call("s8b_ipc_free", p)
        self.own, self.opened = [], []


def plan_roles(rank: int, world: int, ep: int) -> tuple[int, str, int, int]:
    """(stages S, role, stage, range j) of a rank in a pipeline of S = world / ep stages with
    the experts of each stage split over ep GPUs: ranks [0, S) are the stages' home GPUs
    (the whole stage and expert range 0), rank j * S + s holds expert range j of stage s."""
    if ep < 1 or world % ep:
        raise ValueError(f"world size {world} is not a multiple of the expert split {ep}")
    S = world // ep
    j, s = divmod(rank, S)
    return S, "home" if j == 0 else "partner", s, j


def ep_cuts(E: int, ep: int) -> list[int]:
    """Expert range boundaries: range j is experts [cuts[j], cuts[j + 1])."""
    return [j * E // ep for j in range(ep + 1)]


def ep_input_layout(m: int, k: int, H: int, E: int) -> dict[str, int]:
    """Byte offsets of a partner's input block (filled by the home's peer copies): token rows,
    their scales, the expert offsets and the sorted-token list; and its total size."""
    out, off = {}, 0
    for name, n in (("xq", m * H), ("xs", 4 * m), ("offsets", 4 * (E + 1)),
                    ("sorted_token", 4 * m * k)):
        out[name] = off
        off += (n + 255) // 256 * 256
    out["bytes"] = off
    return out


class ExpertPartner:
    """Expert range j of every sparse-MoE layer of stage s, in a process of its own (one GPU).

    Per MoE call of the home GPU (each MoE layer of each micro-batch, in the home's order) it
    waits (bounded) until the home has copied the call's token rows and routing into this
    GPU's input block and raised this GPU's flag, runs its experts (gather, gate_up, SwiGLU,
    down) with the down projection storing straight into the home's contribution buffer over
    NVLink, and raises the home's flag. Both sides count calls in device memory, so one CUDA
    graph per step replays on each."""

    def __init__(self, cfg, rank: int, world: int, ep: int, *, m: int, seed: int = 0, pg=None,
                 state_dict=None, bounds: list[int] | None = None):
        self.cfg, self.rank = cfg, rank
        self.S, _, self.stage, self.j = plan_roles(rank, world * ep, ep)
        self.world, self.ep, self.m = world, ep, m
        self.dev = torch.device("cuda", torch.cuda.current_device())
        b = stage_bounds(cfg.num_hidden_layers, world) if bounds is None else list(bounds)
        lo, hi = b[self.stage], b[self.stage + 1]
        cuts = ep_cuts(cfg.num_experts, ep)
        self.e_lo, self.e_hi = cuts[self.j], cuts[self.j + 1]
        if state_dict is not None:
            full = StageModel.from_state_dict(cfg, state_dict, lo, hi, self.dev, first=False,
                                              last=False)
        else:
            full = StageModel.synthetic(cfg, lo, hi, self.dev, first=False, last=False,
                                        seed=seed * 31 + self.j)
        self.layers = []
        for L in full.layers:
            mw = L.moe
            if mw is None:
                continue
            e0, e1 = self.e_lo, self.e_hi
            self.layers.append((mw.gu_w[e0:e1].clone(), mw.gu_s[e0:e1].clone(),
                                mw.d_w[e0:e1].clone(), mw.d_s[e0:e1].clone(), mw.top_k, mw.ffn))
        del full
        torch.cuda.empty_cache()
        E, H = cfg.num_experts, cfg.hidden_size
        k = self.layers[0][4] if self.layers else cfg.num_experts_per_tok
        Fe = self.layers[0][5] if self.layers else cfg.moe_intermediate_size
        self.k, self.Fe, self.H = k, Fe, H
        self.buf = moe_expert_buffers(m, k, H, Fe, E, self.dev)
        lay = ep_input_layout(m, k, H, E)
        self.in_ptr, in_h = _alloc_ipc(lay["bytes"])
        self.flag_ptr, flag_h = _alloc_ipc(256)
        self.own = [self.in_ptr, self.flag_ptr]
        for name in ("xq", "xs", "offsets", "sorted_token"):  # the home fills these
            self.buf[name] = DevPtr(self.in_ptr + lay[name])
        infos = exchange_infos({"rank": rank, "ep_in": in_h, "ep_flag": flag_h}, world * ep, pg)
        home = infos[self.stage]
        self.opened = []
        self.contrib = self.home_flag = None
        if "ep_contrib" in home:  # (a stage without MoE layers has nothing to exchange)
            self.contrib = _open_ipc(home["ep_contrib"])
            fl = _open_ipc(home["ep_flag"])
            self.home_flag = fl + 4 * (self.j - 1)
            self.opened = [self.contrib, fl]
        self.plan = None  # (no pipeline slots: the home GPU carries the stage's boundaries)
        self.moe_epoch = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.status = torch.zeros(4, dtype=torch.int32, device=self.dev)
        self.graph = self.graph_io = None

    def enqueue_step(self, *, solo: bool = False, **_):
        st = stream()
        off = ptr(self.buf["offsets"]) + 4 * self.e_lo
        for _k in range(self.world):  # micro-batches
            for gu_w, gu_s, d_w, d_s, k, Fe in self.layers:
                if not solo:
                    call("s8b_flag_wait", self.flag_ptr, ptr(self.moe_epoch), 1, FLAG_TIMEOUT_NS,
                         ptr(self.status), st)
                moe_experts(self.buf, off, self.e_hi - self.e_lo, gu_w, gu_s, d_w, d_s,
                            self.contrib, self.m, k, Fe, self.H, st)
                if not solo:
                    call("s8b_flag_set", self.home_flag, ptr(self.moe_epoch), 1, st)
                    call("s8b_counter_add", ptr(self.moe_epoch), 1, st)

    def _graph(self, solo=False):
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.enqueue_step(solo=solo)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        return g

    def capture(self, host_io=None):
        self.graph = self._graph()

    def capture_host_io(self, host_io=None):
        self.graph_io = self._graph()

    def step(self):
        self.graph.replay()

    def step_host_io(self):
        self.graph_io.replay()

    def solo_ms(self, reps: int) -> float:
        g = self._graph(solo=True)
        g.replay()
        torch.cuda.synchronize(self.dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        b.synchronize()
        del g
        return a.elapsed_time(b) / reps

    def check_status(self):
        st = self.status.cpu().tolist()
        if st[0] != 0:
            raise RuntimeError(f"rank {self.rank}: device wait timed out (awaited {st[1]}, "
                               f"saw {st[2]})")

    def close(self, pg=None):
        import torch.distributed as dist

        torch.cuda.synchronize(self.dev)
        self.graph = self.graph_io = None
        for p in self.opened:
            call("s8b_ipc_close", p)
        dist.barrier(group=pg)
        for p in self.own:
            call("s8b_ipc_free", p)
        self.own, self.opened = [], []


def attention_rate(pipe) -> dict:
    """Paged attention of micro-batch 0 on this rank's layers, launched back to back and
    timed with CUDA events on the launching stream (each layer's pool streams from HBM):
    ms per launch, algorithmic bytes per launch (K/V codes and scales over the rows'
    contexts, queries, outputs) and GB/s."""
    r, mb = pipe.runner, pipe.mbs[0]
    M, L = pipe.m, len(r.model.layers)
    st = stream()

    def launch(li):
        kc, ks, vc, vs = r.pool.layer(li % L)
        call("s8b_paged_decode_q8", ptr(r.q_i8), ptr(r.q_s), ptr(kc), ptr(ks), ptr(vc), ptr(vs),
             ptr(mb.block_table), ptr(mb.context_lens), ptr(r.attn), ptr(r.xq), ptr(r.xs), M,
             r.Hq, r.Hkv, r.D, r.pool.block_size, mb.block_table.shape[1], r.max_ctx, r.scale,
             ptr(r.ws), r.ws.numel(), 0, st)

    launch(0)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 4 * L
    a.record()
    for i in range(reps):
        launch(i)
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b) / reps
    ctx = int(mb.context_lens[0].item())
    byts = M * ctx * r.Hkv * (2 * 128 + 2 * 4) + M * r.Hq * (128 + 4) + M * r.Hq * 128 * 3
    return {"ms": ms, "bytes": byts, "gbs": byts / ms / 1e6}


def run_bench_multi(args, metric, step_bytes, peaks, ClockSampler, cpu_sample):
    """bench.py at N > 1: each rank one stage; rank 0 prints the JSON line."""
    import datetime

    import torch.distributed as dist

    from . import config as model_configs

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch with torchrun")
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    model = getattr(args, "model", "qwen3-8b")
    cfg = getattr(model_configs, {"qwen3-8b": "qwen3_8b", "qwen3-30b-a3b": "qwen3_30b_a3b",
                                  "qwen3-27b": "qwen3_27b_dense"}[model])()
    if args.layers:
        cfg = cfg.with_(num_hidden_layers=args.layers)
    m, ctx = args.batch, args.ctx
    ep = max(1, getattr(args, "ep", 1))
    S, role, stage, _ = plan_roles(rank, world, ep)
    total_steps = 1 + 2 * args.warmup + 3 * args.steps + 8  # graph, host-I/O and host-wait loops
    # the last stage also runs the final norm, the LM head and the sampler for every
    # micro-batch (~0.9 of a Qwen3-8B layer at this shape, measured): balance on that
    bounds = balanced_stage_bounds(cfg.num_hidden_layers, S, last_extra=HEAD_LAYERS)
    if role == "home":
        pipe = RankPipeline(cfg, rank, S, m=m, max_len=ctx + total_steps + 16, ctx=ctx,
                            scheme=args.scheme, seed=1, bounds=bounds, ep=ep)
    else:
        pipe = ExpertPartner(cfg, rank, S, ep, m=m, seed=1, bounds=bounds)
    first = role == "home" and pipe.plan.first
    rng = np.random.default_rng(3)
    ids_h = torch.from_numpy(rng.integers(0, cfg.vocab_size, m * S).astype(np.int32)).pin_memory()
    out_h = torch.zeros(m * S, dtype=torch.int32).pin_memory()
    if first:
        pipe.put_ids(ids_h)
    lib = load()
    dist.barrier()
    pipe.enqueue_step()  # eager warm-up step (kernel attributes, lazy module loads)
    torch.cuda.synchronize()
    n0 = lib.s8b_launch_count()
    pipe.capture()
    launches_per_step = int(lib.s8b_launch_count() - n0)
    for _ in range(args.warmup):
        pipe.step()
    torch.cuda.synchronize()
    pipe.check_status()
    dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        time.sleep(0.3)
        # every rank's clock sampler is up (their start-up times differ by tens of ms): line
        # the ranks up again so that no rank's timed region includes another's late start
        dist.barrier()
        torch.cuda.synchronize()
        a.record()
        for _ in range(args.steps):
            pipe.step()
        b.record()
        b.synchronize()
    ms = a.elapsed_time(b) / args.steps
    torch.cuda.synchronize()
    pipe.check_status()
    dist.barrier()
    # e2e through the host API. Stage 0 routes every micro-batch's input ids through pinned
    # host memory inside its step graph (stream-ordered D2H of the delivered tokens, H2D of
    # the ids), so the host holds every step's tokens while the pipeline stays full.
    if first:
        pipe.put_ids(ids_h)
    torch.cuda.synchronize()
    dist.barrier()
    pipe.capture_host_io(ids_h)
    for _ in range(args.warmup):
        pipe.step_host_io()
    torch.cuda.synchronize()
    pipe.check_status()
    dist.barrier()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record()
    for _ in range(args.steps):
        pipe.step_host_io()
    eb.record()
    eb.synchronize()
    e2e_ms = ea.elapsed_time(eb) / args.steps
    pipe.check_status()
    dist.barrier()
    # the same with every rank waiting on the host for each step: stage 0 copies the step's
    # ids in and, once the last stage's tokens landed (device-side flag wait), copies them out
    torch.cuda.synchronize()
    dist.barrier()
    ea.record()
    for _ in range(args.steps):
        if first:
            pipe.put_ids(ids_h)
        pipe.step()
        if first:
            pipe.get_tokens(out_h)
        torch.cuda.current_stream().synchronize()
        if first:
            ids_h.copy_(out_h)
    eb.record()
    eb.synchronize()
    e2e_sync_ms = ea.elapsed_time(eb) / args.steps
    pipe.check_status()
    t = torch.tensor([ms, e2e_ms, e2e_sync_ms], dtype=torch.float64, device=pipe.dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, e2e_sync_ms = t.tolist()
    # each stage's own device time per step (its S micro-batches, no waits): the slowest
    # stage bounds the pipelined step; the rest of the step time is fill, drain and the
    # boundary and token-return hops on the critical path
    dist.barrier()
    solo = torch.tensor([pipe.solo_ms(max(3, args.steps // 2))], dtype=torch.float64,
                        device=pipe.dev)
    solos = [torch.zeros_like(solo) for _ in range(world)]
    dist.all_gather(solos, solo)
    stage_ms = [float(x.item()) for x in solos]
    clocks = clk.summary()
    hbm, _, peak_kind = peaks()
    sb = 0
    if role == "home":
        lo, hi = pipe.plan.layers
        sb = step_bytes(cfg, m * S, ctx, hi - lo, pipe.plan.last)
    # the dominant kernel (paged attention) timed live on rank 0's own layers and buffers
    attn = attention_rate(pipe) if rank == 0 else None
    pipe.close()
    B = m * S
    if rank == 0:
        line = {
            "metric": metric, "value": B / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8 x int8 -> int32 GEMM, bf16 activations",
            "data": "synthetic (random int8 weights, KV pre-filled with random codes)",
            "config": {"workload": f"{model}-shaped W8A8 decode",
                       "micro_batch": m, "n_micro": S, "global_batch": B, "ctx": ctx,
                       "stage_bounds": bounds,
                       "layers": cfg.num_hidden_layers, "block_size": 16,
                       "parallelism": f"pp{S}" + (f" x ep{ep}" if ep > 1 else ""),
                       "wire_scheme": args.scheme,
                       "cuda_graph": True, "transport": "NVLink P2P stores + device flags",
                       "l2": "inputs > L2, no flush"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "e2e": {"value": B / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B,
                    "mode": "ids round-trip through pinned host memory per micro-batch inside "
                            "each step on stage 0 (stream-ordered, no per-step host wait)",
                    "host_wait_per_step_value": B / (e2e_sync_ms / 1e3)},
            "stages": {"stage_ms": stage_ms, "slowest": int(np.argmax(stage_ms)),
                       "pipelined_ms": ms,
                       "wait_frac": 1.0 - max(stage_ms) / ms,
                       "note": "stage_ms: each rank's own device time for its S micro-batches "
                               "per step with no flag waits; wait_frac: the share of the "
                               "pipelined step not covered by the slowest stage's work"},
            "step_roofline": {"bytes_rank0": sb, "achieved_gbs_rank0": sb / ms / 1e6,
                              "frac_rank0": sb / ms / 1e6 / hbm, "peak": hbm,
                              "peak_kind": peak_kind},
            "roofline": {"bound": "hbm", "kernel": "paged_decode_attention (rank 0)",
                         "achieved": attn["gbs"], "peak": hbm, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": attn["gbs"] / hbm, "traffic": None,
                         "bytes_per_launch": attn["bytes"], "ms_per_launch": attn["ms"]},
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()
