#!/usr/bin/env python
"""Benchmark: Qwen3-8B-shaped W8A8 pipeline decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl s8b|reference]
    torchrun --nproc-per-node N ... bench.py --gpus N ...     (N > 1: one stage per rank)

A step is one decode step of every sequence: ``micro_batch`` (64) rows per micro-batch,
``N`` micro-batches in flight through ``N`` stages of 36/N layers (``i*L//S`` split), KV cache
pre-filled synthetically to 2048 tokens, random int8 weights. Per-GPU work is fixed as N grows
(weak scaling): global batch = 64*N. Inputs (7.6 GB of weights, 10 GB of KV) are far larger
than L2, so no flush is needed between steps.

Prints ONE JSON line (rank 0). `value` is whole-job tokens/s with inputs resident in HBM
(CUDA-graph replay, device timed with CUDA events, max over ranks); `e2e` is the same step
through the engine's host API (token ids H2D from pinned memory, next tokens D2H, each step).
`roofline` is the dominant kernel timed live with CUDA events; `cpu_baseline` is the CPU
oracle on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "decode tokens/s (whole box) at 1/2/4/8 pipeline stages; % HBM roofline per stage"


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms during the timed region. The
    sampler is running (its first sample written) before __enter__ returns, so a short timed
    region still falls between samples of its own."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = tempfile.mktemp(suffix=".csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return self
        t0 = time.time()
        while time.time() - t0 < 10.0 and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.05)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ----------------------------------------------------------------------- CPU baseline ----

class CpuOracleSample:
    """CPU oracle on a bounded sample of the config-3 step: one Qwen3-8B layer at batch
    `batch`, context `ctx`, plus 1/`head_frac` of the LM head, extrapolated to the full
    36-layer step. Weights and the KV pool are built once; each run() is one sample."""

    def __init__(self, batch=64, ctx=2048, head_frac=16, seed=0, cfg=None):
        from oracle.kernels import rope_tables
        from oracle.model import PagedPool, Shape
        from superl8_serve_b200.config import qwen3_8b

        self.cfg = cfg = cfg or qwen3_8b()
        self.batch, self.ctx, self.head_frac = batch, ctx, head_frac
        self.s = Shape(cfg.vocab_size, cfg.hidden_size, 1, cfg.num_attention_heads,
                       cfg.num_key_value_heads, 128, cfg.intermediate_size, 1e-6, 1e6, ctx + 8,
                       False, cfg.num_experts, cfg.num_experts_per_tok, cfg.norm_topk_prob)
        rng = np.random.default_rng(seed)
        H, F, D = self.s.hidden_size, self.s.intermediate_size, 128
        nh, nkv = self.s.num_attention_heads, self.s.num_key_value_heads

        def w(n, k):
            return (rng.integers(-127, 128, (n, k), dtype=np.int8),
                    np.full(n, 0.02 / 73.3, dtype=np.float32))

        g = lambda n: (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)  # noqa: E731
        self.L = {"qkv": w((nh + 2 * nkv) * D, H), "o": w(H, nh * D), "in_norm": g(H),
                  "post_norm": g(H), "q_norm": g(D), "k_norm": g(D)}
        if cfg.num_experts:
            Fe = cfg.moe_intermediate_size
            self.L["router"] = (0.02 * rng.standard_normal((cfg.num_experts, H))).astype(np.float32)
            self.L["experts"] = [(w(2 * Fe, H), w(H, Fe)) for _ in range(cfg.num_experts)]
        else:
            self.L["gu"], self.L["down"] = w(2 * F, H), w(H, F)
        pool = PagedPool(1, batch, nkv, ctx + 8, D)
        pool.kc[:] = rng.integers(-127, 128, pool.kc.shape, dtype=np.int8)
        pool.vc[:] = rng.integers(-127, 128, pool.vc.shape, dtype=np.int8)
        pool.ks[:] = rng.uniform(0.01, 0.05, pool.ks.shape)
        pool.vs[:] = rng.uniform(0.01, 0.05, pool.vs.shape)
        slots = [pool.alloc() for _ in range(batch)]
        pool.ensure_capacity(slots, [ctx + 1] * batch)
        self.pool = pool
        self.sm = pool.slot_mapping(slots, [ctx] * batch)
        self.bt = pool.block_table(slots)
        self.cl = np.full(batch, ctx + 1, dtype=np.int32)
        self.tabs = rope_tables(D, ctx + 8, 1e6)
        self.h = (0.5 * rng.standard_normal((batch, H))).astype(np.float32)
        self.res = (rng.standard_normal((batch, H))).astype(np.float32)
        self.hw, _ = w(cfg.vocab_size // head_frac, H)
        self.xq = rng.integers(-127, 128, (batch, H), dtype=np.int8)
        self.desc = (f"oracle (numpy, BLAS GEMMs on {os.cpu_count()} host threads, Python "
                     f"attention loop): 1 of {cfg.num_hidden_layers} layers"
                     f"{' (sparse MoE)' if cfg.num_experts else ''} + "
                     f"1/{head_frac} of the LM head at batch {batch}, ctx {ctx}, extrapolated "
                     f"to one {cfg.num_hidden_layers}-layer decode step")

    def run(self):
        """One sample: returns (tokens/s, seconds spent)."""
        from oracle.kernels import gemm_acc
        from oracle.model import layer_decode

        t0 = time.perf_counter()
        layer_decode(self.L, 0, self.h.copy(), self.res.copy(), [self.ctx] * self.batch, self.sm,
                     self.bt, self.cl, self.pool, self.s, self.tabs)
        t_layer = time.perf_counter() - t0
        t1 = time.perf_counter()
        gemm_acc(self.xq, self.hw)
        t_head = (time.perf_counter() - t1) * self.head_frac
        step = t_layer * self.cfg.num_hidden_layers + t_head
        return self.batch / step, time.perf_counter() - t0


def cpu_sample_tokens_per_s(batch=64, ctx=2048, n_layers=1, head_frac=16, seed=0, cfg=None):
    """One CPU-oracle sample (see CpuOracleSample). Returns (tokens/s, seconds, description)."""
    smp = CpuOracleSample(batch, ctx, head_frac, seed, cfg=cfg)
    v, spent = smp.run()
    return v, spent, smp.desc


REF_MAX_SAMPLES = 6


def host_threads() -> dict:
    """Host threads the CPU oracle may use: cores, torch's intra-op pool, and numpy's BLAS
    pool (the oracle's GEMMs) where threadpoolctl can read it."""
    out = {"cores": os.cpu_count(), "torch_threads": torch.get_num_threads()}
    try:
        from threadpoolctl import threadpool_info

        blas = [p for p in threadpool_info() if p.get("user_api") == "blas"]
        if blas:
            out["blas_threads"] = max(int(p.get("num_threads", 0)) for p in blas)
            out["blas"] = blas[0].get("internal_api")
    except Exception:
        pass
    return out


def run_reference(args):
    """The reference arm: the CPU oracle (the superl8 kernels are not vendored, so the
    oracle's restatement stands in for them) on the host cores. A full 36-layer config-3 step
    takes minutes on the CPU, so each timed step is a bounded sample: one layer at the same
    batch and context plus 1/16 of the LM head. `ms_per_step` and `value` are the full step
    those samples extrapolate to; `sample_ms` is what one sample took; `steps` is the number
    of samples actually timed (at most REF_MAX_SAMPLES of the requested --steps)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    t_start = time.perf_counter()
    smp = CpuOracleSample(batch=args.batch, ctx=args.ctx, cfg=model_config(args.model))
    smp.run()
    vals, spent = [], []
    for _ in range(min(args.steps, REF_MAX_SAMPLES)):
        v, t = smp.run()
        vals.append(v)
        spent.append(t)
    v = statistics.median(vals)
    threads = host_threads()
    L = smp.cfg.num_hidden_layers
    extrap = (f"each timed sample runs 1 of {L} layers at batch {args.batch}, ctx {args.ctx} "
              f"(all of its kernels) and 1/{smp.head_frac} of the LM head GEMM; the full step "
              f"is estimated as {L} x layer time + {smp.head_frac} x head-slice time")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": len(vals), "steps_requested": args.steps, "warmup": 1,
        "warmup_requested": args.warmup,
        "ms_per_step": args.batch / v * 1000.0, "ms_per_step_kind": "extrapolated full step",
        "sample_ms": statistics.median(spent) * 1000.0, "extrapolated_from": extrap,
        "wall_s": time.perf_counter() - t_start, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": CONFIG_NAMES[args.model], "micro_batch": args.batch,
                   "ctx": args.ctx, "stages": 1, "note": "superl8 kernels are not vendored; "
                   "the reference arm is the CPU oracle restating them"},
        "cpu_baseline": {"value": v, "unit": "tokens/s", "kind": "port",
                         "sample": smp.desc + f"; median of {len(vals)} samples after 1 "
                                              "warm-up sample", **threads},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_config1(args):
    """BASELINE config 1 in full, on the GPU pipeline and on the CPU oracle in the same run:
    Qwen3-0.6B shape (28 layers), random N(0, 0.02) weights quantized per row, 2 pipeline
    stages (layers 0-13 / 14-27, both on cuda:0 unless a second GPU is visible), batch 4,
    prompts of 128 uniform-random ids, int8 paged KV (block 16), 32 greedy steps. Each side
    prefills the prompts and decodes; the line reports both throughputs (generated tokens
    per second of the whole generate call, prefill included) and whether the greedy tokens
    are identical."""
    from oracle.model import OraclePipeline, quantize_state_dict
    from superl8_serve_b200.config import qwen3_0_6b
    from superl8_serve_b200.dist.pipeline import stage_bounds
    from superl8_serve_b200.engine import DecodePipeline
    from superl8_serve_b200.runtime import StageModel
    from superl8_serve_b200.weights import random_state_dict

    cfg = qwen3_0_6b()
    B, plen, new = 4, 128, 32
    sd = random_state_dict(cfg, 0, w_std=0.02)
    prompts = np.random.default_rng(1).integers(0, cfg.vocab_size, (B, plen)).tolist()
    b = stage_bounds(cfg.num_hidden_layers, 2)
    devs = ["cuda:0", "cuda:1" if torch.cuda.device_count() > 1 else "cuda:0"]
    models = [StageModel.from_state_dict(cfg, sd, b[i], b[i + 1], devs[i], first=i == 0,
                                         last=i == 1) for i in range(2)]
    pipe = DecodePipeline(models, batch=B, n_micro=1, max_len=plen + new + 16,
                          wire_scheme=args.scheme)
    pipe.generate(prompts, 2, prefill=True)  # warm-up (kernel attributes, lazy init)
    pipe = DecodePipeline(models, batch=B, n_micro=1, max_len=plen + new + 16,
                          wire_scheme=args.scheme)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    gpu_out = pipe.generate(prompts, new, prefill=True)
    torch.cuda.synchronize()
    gpu_s = time.perf_counter() - t0
    qw = quantize_state_dict(sd, cfg)
    t0 = time.perf_counter()
    cpu_out, _ = OraclePipeline(cfg, qw, n_stages=2, wire_scheme=args.scheme, num_slots=B,
                                max_len=plen + new + 16).generate_prefilled(prompts, new)
    cpu_s = time.perf_counter() - t0
    same = [list(map(int, g)) for g in gpu_out] == [list(map(int, c)) for c in cpu_out]
    line = {
        "metric": "generated tokens/s, BASELINE config 1 (prefill + 32 greedy decode steps)",
        "value": B * new / gpu_s, "unit": "tokens/s", "n_gpus": len(set(devs)),
        "steps": new, "warmup": 1, "ms_per_step": gpu_s * 1000.0 / new,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 GEMM, bf16 activations", "data": "synthetic",
        "config": {"workload": "qwen3-0.6b-shaped W8A8, 2 stages, batch 4, 128-token prompts",
                   "wire_scheme": args.scheme, "timing": "host wall clock around generate() "
                   "(host-driven loop: a synchronising read of the tokens every step)"},
        "greedy_tokens_identical": same,
        "cpu_baseline": {"value": B * new / cpu_s, "unit": "tokens/s", "kind": "port",
                         "sample": "config 1 in full on the CPU oracle (prefill + 32 steps)",
                         "seconds": cpu_s, **host_threads()},
    }
    print(json.dumps(line), flush=True)
    if not same:
        raise SystemExit("config 1: GPU and CPU greedy tokens differ")


# ------------------------------------------------------------------------ GPU (N=1) ----

def time_kernel(fn, reps: int) -> float:
    """Average ms of fn() (one launch per call) with CUDA events on the current stream."""
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / reps


# dram__bytes_read.sum + dram__bytes_write.sum per launch from one ncu capture of the same
# launch shape (the attention and gate_up captures summarised under profiles/); re-captured
# whenever the kernel changes.
NCU_TRAFFIC = {
    "paged_decode_attention": {"bytes": 279405056 + 10110464,
                               "source": "ncu dram bytes of attn_persistent_kernel (the row "
                                         "merge reads its 8.4 MB of partials from L2)"},
    "gemm_w8a8_tc_gate_up": {"bytes": 100976128 + 4385024,
                             "source": "ncu dram bytes of gemm_tc_kernel (gate_up launch)"},
}


def kernel_rooflines(pipe, hbm_peak):
    """Live CUDA-event timing of the two HBM-heavy kernels on the bench's own buffers,
    rotating through all layers so every launch streams its operands from HBM."""
    from superl8_serve_b200._lib import call, ptr, stream

    r = pipe.runners[0]
    mb = pipe.mbs[0][0]
    M = pipe.rows[0]
    L = len(r.model.layers)
    out = {}
    lw = r.model.layers[0]
    if lw.moe is None:
        # W8A8 gate_up GEMM (largest weight matrix: 2F x H int8)
        it = iter(range(10 ** 9))

        def gemm():
            li = next(it) % L
            lw = r.model.layers[li]
            r._gemm(r.xq, r.xs, lw.gu_w, lw.gu_s, r.gu, M)

        ms = time_kernel(gemm, 4 * L)
        N, K = lw.gu_w.shape
        byts = N * K + N * 4 + M * K + M * 4 + M * N * 2
        name = ("gemm_w8a8_tc_gate_up" if r.tc_ws is not None and M >= r.tc_min
                else "gemm_w8a8_gate_up")
    else:
        # grouped expert gate_up GEMM on the routing the last step left behind
        b, mw = r.moe_buf, lw.moe
        A, Fe, E = M * mw.top_k, mw.ffn, mw.local_experts  # this GPU's experts only
        it = iter(range(10 ** 9))

        tc = r.MOE_TC and r.H % 128 == 0 and Fe % 128 == 0 and E <= 512

        def gemm():
            w = r.model.layers[next(it) % L].moe
            if tc:  # the step's kernel: tensor cores on the rows it gathered
                call("s8b_moe_gemm_grouped_tc", ptr(b["xg"]), ptr(b["xgs"]), ptr(w.gu_w),
                     ptr(w.gu_s), ptr(b["offsets"]), ptr(b["gu"]), A, 2 * Fe, r.H, E, M,
                     ptr(b["status"]), 0, stream())
            else:
                call("s8b_moe_gemm_grouped", ptr(r.xq), ptr(r.xs), ptr(b["sorted_token"]),
                     ptr(w.gu_w), ptr(w.gu_s), ptr(b["offsets"]), ptr(b["gu"]), A, 2 * Fe, r.H,
                     E, 0, stream())

        ms = time_kernel(gemm, 4 * L)
        off = b["offsets"].cpu()[: E + 1]
        hit = int(((off[1:] - off[:-1]) > 0).sum())
        byts = hit * (2 * Fe * r.H + 2 * Fe * 4) + M * r.H + 4 * M + A * 2 * Fe * 2 + 4 * A
        name = "moe_gemm_grouped_tc_gate_up" if tc else "moe_gemm_grouped_gate_up"
    out[name] = {"ms": ms, "bytes": byts, "gbs": byts / ms / 1e6, "launches_per_step": L}
    # paged decode attention (partition + combine) for one layer
    it2 = iter(range(10 ** 9))

    def attn():
        li = next(it2) % L
        kc, ks, vc, vs = r.pool.layer(li)
        call("s8b_paged_decode_q8", ptr(r.q_i8), ptr(r.q_s), ptr(kc), ptr(ks), ptr(vc), ptr(vs),
             ptr(mb.block_table), ptr(mb.context_lens), ptr(r.attn), ptr(r.xq), ptr(r.xs), M,
             r.Hq, r.Hkv, r.D, r.pool.block_size, mb.block_table.shape[1], r.max_ctx, r.scale,
             ptr(r.ws), r.ws.numel(), 0, stream())

    ms = time_kernel(attn, 4 * L)
    ctx = int(mb.context_lens[0].item())
    byts = M * ctx * r.Hkv * (2 * 128 + 2 * 4) + M * r.Hq * (128 + 4) + M * r.Hq * 128 * 3
    out["paged_decode_attention"] = {"ms": ms, "bytes": byts, "gbs": byts / ms / 1e6,
                                     "launches_per_step": L}
    for v in out.values():
        v["frac"] = v["gbs"] / hbm_peak
    return out


MODELS = {"qwen3-8b": "qwen3_8b", "qwen3-30b-a3b": "qwen3_30b_a3b",
          "qwen3-27b": "qwen3_27b_dense"}
CONFIG_NAMES = {"qwen3-8b": "qwen3-8b-shaped W8A8 decode (BASELINE config 3)",
                "qwen3-30b-a3b": "qwen3-30b-a3b-shaped MoE W8A8 decode (BASELINE config 4)",
                "qwen3-27b": "27b-dense-shaped W8A8 long-context decode (BASELINE config 5)"}


def model_config(name: str):
    from superl8_serve_b200 import config

    return getattr(config, MODELS[name])()


def experts_hit(cfg, tokens: int) -> float:
    """Expected number of distinct experts routed to by `tokens` tokens choosing top-k of E
    uniformly (the synthetic router's regime)."""
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    return E * (1.0 - (1.0 - k / E) ** tokens)


def step_bytes(cfg, batch, ctx, layers, last):
    """Algorithmic HBM bytes of one decode step of one stage (weights + scales + KV read +
    KV write + LM head on the last stage). A sparse-MoE layer streams the router and the
    experts that the step's tokens route to (expected count for uniform routing)."""
    H, F, D = cfg.hidden_size, cfg.intermediate_size, 128
    nh, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    attn_w = ((nh + 2 * nkv) * D) * H + H * nh * D + 4 * ((nh + 2 * nkv) * D + H)
    if getattr(cfg, "num_experts", 0):
        Fe = cfg.moe_intermediate_size
        expert = 2 * Fe * H + H * Fe + 4 * (2 * Fe + H)
        ffn_w = 4 * cfg.num_experts * H + experts_hit(cfg, batch) * expert
    else:
        ffn_w = 2 * F * H + H * F + 4 * (2 * F + H)
    w = layers * (attn_w + ffn_w)
    kv = layers * batch * (ctx * nkv * (2 * D + 8) + nkv * (2 * D + 8))
    head = (cfg.vocab_size * H + 4 * cfg.vocab_size) if last else 0
    return int(w + kv + head)


def run_single(args):
    from superl8_serve_b200 import _lib
    from superl8_serve_b200.config import qwen3_8b
    from superl8_serve_b200.engine import DecodePipeline
    from superl8_serve_b200.runtime import StageModel

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cfg = model_config(args.model)
    if args.layers:
        cfg = cfg.with_(num_hidden_layers=args.layers)
    B, ctx = args.batch, args.ctx
    max_len = ctx + args.warmup + args.steps + 16
    model = StageModel.synthetic(cfg, 0, cfg.num_hidden_layers, dev, first=True, last=True, seed=1)
    ep = max(1, args.ep)
    if ep > 1:
        # expert parallelism inside the stage: experts split over cuda:0..cuda:ep-1; the step
        # spans several GPUs, so it runs eagerly (no CUDA graph)
        model.shard_experts([f"cuda:{i}" for i in range(1, ep)])
    pipe = DecodePipeline([model], batch=B, n_micro=1, max_len=max_len, wire_scheme=args.scheme)
    pipe.pools[0].fill_random(seed=2)
    pipe.add_sequences()
    ids0 = np.random.default_rng(3).integers(0, cfg.vocab_size, B).tolist()
    pipe.set_state([ctx] * B, ids0, reserve=args.warmup + args.steps + 8)
    pipe._enqueue()  # eager warm-up: kernel attributes, lazy init
    torch.cuda.synchronize()
    pipe.set_state([ctx] * B, ids0, reserve=args.warmup + args.steps + 8)
    if ep == 1:
        pipe.capture()
    for _ in range(args.warmup):
        pipe.step()
    torch.cuda.synchronize()
    n0 = _lib.load().s8b_launch_count()
    pipe._enqueue()  # count launches of one step (eager), then restore state
    per_step_launches = _lib.load().s8b_launch_count() - n0
    torch.cuda.synchronize()
    pipe.set_state([ctx] * B, ids0, reserve=args.warmup + args.steps + 8)
    for _ in range(args.warmup):
        pipe.step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        time.sleep(0.3)
        a.record()
        for _ in range(args.steps):
            pipe.step()
        b.record()
        b.synchronize()
    ms = a.elapsed_time(b) / args.steps
    value = B / (ms / 1e3)
    clocks = clk.summary()

    # e2e through the engine's host API. Every step, every micro-batch's input ids make a
    # device -> host -> device round trip through pinned memory inside the step graph
    # (stream-ordered D2H of the previous tokens, H2D of the ids), so the host holds every
    # step's tokens while the pipeline stays full; the host reads the buffer after the loop.
    ids_h = torch.tensor(ids0, dtype=torch.int32).pin_memory()
    pipe.set_state([ctx] * B, ids0, reserve=args.warmup + args.steps + 8)
    if ep == 1:
        pipe.capture(host_io=ids_h)
    else:
        pipe.step_host_io = lambda: pipe._enqueue(ids_h)
    for _ in range(args.warmup):
        pipe.step_host_io()
    torch.cuda.synchronize()
    pipe.set_state([ctx] * B, ids0, reserve=args.warmup + args.steps + 8)
    torch.cuda.synchronize()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record()
    for _ in range(args.steps):
        pipe.step_host_io()
    eb.record()
    eb.synchronize()
    e2e_ms = ea.elapsed_time(eb) / args.steps
    # the same with the host waiting for each step's tokens before issuing the next step
    pipe.set_state([ctx] * B, ids0, reserve=args.warmup + args.steps + 8)
    ids_h.copy_(torch.tensor(ids0, dtype=torch.int32))
    out_h = torch.empty(B, dtype=torch.int32).pin_memory()
    mbids = pipe.mbs[0][0].ids
    torch.cuda.synchronize()
    ea.record()
    for _ in range(args.steps):
        mbids[:B].copy_(ids_h, non_blocking=True)
        pipe.step()
        out_h.copy_(pipe.mbs[-1][0].ids[:B], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        ids_h.copy_(out_h)
    eb.record()
    eb.synchronize()
    e2e_sync_ms = ea.elapsed_time(eb) / args.steps
    hbm, _, peak_kind = peaks()
    kr = kernel_rooflines(pipe, hbm)
    top_name, top = max(kr.items(), key=lambda kv: kv[1]["ms"] * kv[1]["launches_per_step"])
    sb = step_bytes(cfg, B, ctx, cfg.num_hidden_layers, True)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ep, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 x int8 -> int32 GEMM, bf16 activations",
        "data": "synthetic (random int8 weights, KV pre-filled with random codes)",
        "config": {"workload": CONFIG_NAMES[args.model],
                   "micro_batch": B, "n_micro": 1, "global_batch": B, "ctx": ctx,
                   "layers": cfg.num_hidden_layers,
                   "block_size": 16, "parallelism": "pp1" + (f" x ep{ep}" if ep > 1 else ""),
                   "wire_scheme": args.scheme, "cuda_graph": ep == 1,
                   "l2": f"inputs ({step_bytes(cfg, B, ctx, cfg.num_hidden_layers, True) / 1e9:.1f}"
                         " GB) > L2, no flush"},
        "gpu_launches": int(per_step_launches) * args.steps,
        "clocks": clocks,
        "e2e": {"value": B / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 4 * B,
                "d2h_bytes_per_step": 4 * B,
                "mode": "ids round-trip through pinned host memory per micro-batch inside each "
                        "step (stream-ordered, no per-step host wait)",
                "host_wait_per_step_value": B / (e2e_sync_ms / 1e3)},
        "roofline": {"bound": "hbm", "kernel": top_name, "achieved": top["gbs"], "peak": hbm,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": top["frac"],
                     "traffic": NCU_TRAFFIC.get(top_name, {}).get("bytes"),
                     "traffic_source": NCU_TRAFFIC.get(top_name, {}).get("source"),
                     "bytes_per_launch": top["bytes"], "ms_per_launch": top["ms"]},
        "kernels": kr,
        "step_roofline": {"bytes": sb, "achieved_gbs": sb / ms / 1e6, "frac": sb / ms / 1e6 / hbm},
    }
    if not args.no_cpu_baseline:
        v, spent, desc = cpu_sample_tokens_per_s(batch=B, ctx=ctx, n_layers=1,
                                                 cfg=model_config(args.model))
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "kind": "port",
                                "sample": desc, "seconds": spent, **host_threads()}
    print(json.dumps(line), flush=True)


def run_prefill(args):
    """Varlen prefill of ``--batch`` prompts of ``--ctx`` random tokens each (Qwen3-8B shape,
    one GPU, 256-row chunks): prompt tokens/s, device-timed with CUDA events around whole
    ``prefill()`` calls (host ids H2D at the start, first tokens D2H at the end)."""
    from superl8_serve_b200 import _lib
    from superl8_serve_b200.engine import DecodePipeline
    from superl8_serve_b200.runtime import StageModel

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    cfg = model_config(args.model)
    if args.layers:
        cfg = cfg.with_(num_hidden_layers=args.layers)
    B, P = args.batch, args.ctx
    model = StageModel.synthetic(cfg, 0, cfg.num_hidden_layers, dev, first=True, last=True, seed=1)
    pipe = DecodePipeline([model], batch=B, n_micro=1, max_len=P + 16, wire_scheme=args.scheme)
    rng = np.random.default_rng(3)
    prompts = rng.integers(0, cfg.vocab_size, (B, P)).tolist()
    for _ in range(args.warmup):
        pipe.prefill(prompts)
    torch.cuda.synchronize()
    n0 = _lib.load().s8b_launch_count()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        time.sleep(0.3)
        a.record()
        for _ in range(args.steps):
            pipe.prefill(prompts)
        b.record()
        b.synchronize()
    launches = _lib.load().s8b_launch_count() - n0
    ms = a.elapsed_time(b) / args.steps
    tokens = B * P
    H, F, D = cfg.hidden_size, cfg.intermediate_size, 128
    nh, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    params = cfg.num_hidden_layers * (((nh + 2 * nkv) * D + 2 * F) * H + H * nh * D + H * F)
    gemm_ops = 2.0 * params * tokens + 2.0 * cfg.vocab_size * H * B
    # attention: q.k and p.v over the causal prefix of every row, every head
    attn_ops = cfg.num_hidden_layers * B * nh * 4.0 * D * (P * (P + 1) / 2)
    _, bf16_peak, peak_kind = peaks()
    line = {
        "metric": "prefill tokens/s (varlen prefill, one GPU)", "value": tokens / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 x int8 -> int32 GEMM, bf16 activations",
        "data": "synthetic (random int8 weights, uniform-random prompt ids)",
        "config": {"workload": "qwen3-8b-shaped W8A8 varlen prefill", "prompts": B,
                   "prompt_len": P, "layers": cfg.num_hidden_layers,
                   "chunk_rows": pipe.prefill_chunk, "parallelism": "pp1"},
        "gpu_launches": int(launches), "clocks": clk.summary(),
        "tensor": {"gemm_tops": gemm_ops / ms / 1e9, "attn_tops": attn_ops / ms / 1e9,
                   "int8_peak_tops": 2 * bf16_peak, "peak_kind": peak_kind + " (2 x bf16)",
                   "gemm_frac": gemm_ops / ms / 1e9 / (2 * bf16_peak)},
    }
    print(json.dumps(line), flush=True)


def time_graph(fn, reps: int, device) -> float:
    """Average ms of fn() (one launch per call) from a CUDA graph holding `reps` calls, so the
    host launch rate does not enter the figure."""
    fn()
    torch.cuda.synchronize(device)
    s = torch.cuda.Stream(device=device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.device(device), torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(reps):
                fn()
    g.replay()
    torch.cuda.synchronize(device)
    with torch.cuda.device(device):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
    return a.elapsed_time(b) / reps


def run_codec(args):
    """the inter-stage codec. x bf16 [T, 4096], N(0,1) with 0.1% of the
    channels (4) scaled x20; block-128 Hadamard, per-token absmax, int8 and int4 (and the
    reference's nf4 scheme beside them). The
    encoder on GPU 0 stores its codes straight into GPU 1's buffer over NVLink (local when
    only one GPU is visible); GPU 1 decodes. Device time (CUDA events around a CUDA graph of
    repeated launches) of encode (codes crossing NVLink inside it) and of decode, per T; bytes
    moved per token; round-trip SQNR against the reference's bars."""
    from superl8_serve_b200 import ops
    from superl8_serve_b200._lib import call
    from superl8_serve_b200.dist import accuracy_report

    src = torch.device("cuda", 0)
    dst = torch.device("cuda", 1 if torch.cuda.device_count() > 1 else 0)
    if dst != src:
        call("s8b_enable_peer_access", 0, 1)
    D, reps = 4096, 50
    rng = np.random.default_rng(0)
    cols = rng.choice(D, 4, replace=False)
    rows = []
    for scheme in ("int8-had", "int4-had", "nf4"):  # config 2's two codecs, and nf4
        for T in (1, 16, 64, 256, 1024):
            xh = rng.standard_normal((T, D)).astype(np.float32)
            xh[:, cols] *= 20
            x = torch.from_numpy(xh).to(torch.bfloat16).to(src)
            nbytes, nsc = ops.codec_sizes(T, D, scheme)
            pay = torch.empty(nbytes, dtype=torch.uint8, device=dst)
            sc = torch.empty(max(nsc, 1), dtype=torch.float32, device=dst)
            ms_enc = time_graph(lambda: ops.codec_encode(x, None, scheme, payload=pay, scales=sc),
                                reps, src)
            out = torch.empty(T, D, dtype=torch.bfloat16, device=dst)
            ms_dec = time_graph(lambda: ops.codec_decode(pay, sc, T, D, 0, scheme, torch.bfloat16,
                                                         out_a=out), reps, dst)
            torch.cuda.synchronize(dst)
            rep = accuracy_report(x.float().cpu(), out.float().cpu(), scheme)
            wire = nbytes + 4 * nsc
            rows.append({"scheme": scheme, "T": T, "encode_us": ms_enc * 1e3,
                         "decode_us": ms_dec * 1e3, "wire_bytes_per_token": wire / T,
                         "encode_gbs": (2 * T * D + wire) / ms_enc / 1e6,
                         "sqnr_db": rep["sqnr_db"], "sqnr_pass": rep["sqnr_pass"],
                         "cos": rep["cos"]})
    big = [r for r in rows if r["T"] == 1024 and r["scheme"] == "int8-had"][0]
    line = {
        "metric": "inter-stage codec: encode + NVLink store + decode (BASELINE config 2)",
        "value": 1024 / ((big["encode_us"] + big["decode_us"]) / 1e6), "unit": "tokens/s",
        "n_gpus": 2 if dst != src else 1, "steps": reps, "warmup": 1,
        "ms_per_step": (big["encode_us"] + big["decode_us"]) / 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 -> int8 / int4 codes",
        "data": "synthetic N(0,1), 4 outlier channels x20",
        "config": {"workload": "codec microbench, D = 4096", "transfer":
                   "peer stores GPU0 -> GPU1" if dst != src else "local (one GPU visible)"},
        "rows": rows,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="s8b", choices=["s8b", "reference"])
    ap.add_argument("--batch", type=int, default=64, help="rows per micro-batch")
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--scheme", default="int8-had")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--model", default="qwen3-8b", choices=sorted(MODELS),
                    help="qwen3-8b (config 3, default), qwen3-30b-a3b (config 4, MoE), "
                         "qwen3-27b (config 5, dense long-context)")
    ap.add_argument("--ep", type=int, default=1,
                    help="MoE models: experts of each layer split over this many GPUs of the "
                         "stage (in-process, cuda:0..ep-1)")
    ap.add_argument("--mode", default="decode", choices=["decode", "prefill", "codec", "config1"],
                    help="prefill: varlen prefill throughput of --batch prompts of --ctx tokens; "
                         "codec: the inter-stage codec microbench (config 2); config1: BASELINE "
                         "config 1 in full on the GPU and on the CPU oracle")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: fewer layers than the model's 36 (small ncu case)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.mode == "prefill":
        return run_prefill(args)
    if args.mode == "codec":
        return run_codec(args)
    if args.mode == "config1":
        return run_config1(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 or args.gpus > 1:
        from superl8_serve_b200.multistage import run_bench_multi

        return run_bench_multi(args, METRIC, step_bytes, peaks, ClockSampler,
                               cpu_sample_tokens_per_s)
    return run_single(args)


if __name__ == "__main__":
    main()
