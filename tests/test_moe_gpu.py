"""GPU: the sparse-MoE kernels (router + grouping, grouped W8A8 GEMM, combine) and the MoE
decoder layer against the CPU oracle and the reference graph's golden tokens, through the C
ABI. Everything is compared bit for bit."""

import numpy as np
import pytest
import torch

from oracle import moe as om
from oracle import numerics as on
from oracle.kernels import gemm_w8a8
from oracle.model import OraclePipeline, quantize_state_dict
from superl8_serve_b200 import ops
from superl8_serve_b200.config import tiny_moe
from superl8_serve_b200.dist.pipeline import stage_bounds
from superl8_serve_b200.engine import DecodePipeline
from superl8_serve_b200.runtime import StageModel
from superl8_serve_b200.weights import random_state_dict

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
PROMPTS = [[3, 1, 4, 1, 5], [9, 2, 6], [5, 3, 5, 8, 9, 7, 9]]


def bf16(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).to(DEV)


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def f32(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("T,H,E,k", [(1, 256, 16, 4), (7, 512, 60, 4), (128, 2048, 128, 8),
                                     (33, 1024, 256, 16)])
def test_route_and_grouping_bit_exact(T, H, E, k):
    rng = np.random.default_rng(T * 7 + E)
    y = on.round_bf16(rng.standard_normal((T, H)).astype(np.float32))
    gate = on.round_bf16((0.05 * rng.standard_normal((E, H))).astype(np.float32))
    r = ops.moe_route(bf16(y), dev(gate), k)
    topi, topw, _ = om.moe_route(y, gate, k)
    assert np.array_equal(r["topi"].cpu().numpy(), topi)
    assert np.array_equal(f32(r["topw"]), topw)
    off, order, rowpos = om.group_assignments(topi, E)
    assert np.array_equal(r["offsets"].cpu().numpy(), off)
    assert np.array_equal(r["sorted_assign"].cpu().numpy(), order)
    assert np.array_equal(r["sorted_token"].cpu().numpy(), order // k)
    assert np.array_equal(r["assign_pos"].cpu().numpy(), rowpos)


def test_route_without_renormalisation_and_scaling():
    rng = np.random.default_rng(3)
    y = on.round_bf16(rng.standard_normal((5, 256)).astype(np.float32))
    gate = on.round_bf16((0.1 * rng.standard_normal((32, 256))).astype(np.float32))
    r = ops.moe_route(bf16(y), dev(gate), 6, norm_topk_prob=False, scaling=2.5)
    topi, topw, _ = om.moe_route(y, gate, 6, norm_topk_prob=False, scaling=2.5)
    assert np.array_equal(r["topi"].cpu().numpy(), topi)
    assert np.array_equal(f32(r["topw"]), topw)


@pytest.mark.parametrize("gather", [True, False])
@pytest.mark.parametrize("T,N,K,E,k", [(1, 96, 256, 8, 2), (32, 1536, 2048, 128, 8),
                                       (64, 256, 768, 16, 4)])
def test_grouped_gemm_bit_exact(gather, T, N, K, E, k):
    rng = np.random.default_rng(N + K + E)
    topi = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    off, order, _ = om.group_assignments(topi, E)
    A = T * k
    rows = T if gather else A
    xq = rng.integers(-127, 128, (rows, K), dtype=np.int8)
    xs = rng.uniform(0.001, 0.1, rows).astype(np.float32)
    w = rng.integers(-127, 128, (E, N, K), dtype=np.int8)
    ws = rng.uniform(1e-4, 1e-3, (E, N)).astype(np.float32)
    src = order // k if gather else np.arange(A)
    y = ops.moe_gemm_grouped(dev(xq), dev(xs), dev(w), dev(ws), dev(off),
                             row_index=dev(src.astype(np.int32)) if gather else None, A=A)
    want = np.zeros((A, N), np.float32)
    for e in range(E):
        lo, hi = off[e], off[e + 1]
        if lo < hi:
            want[lo:hi] = gemm_w8a8(xq[src[lo:hi]], xs[src[lo:hi]], w[e], ws[e])
    assert np.array_equal(f32(y), want)


def _skewed_topi(rng, T, E, k, hot):
    """Top-k choices where expert `hot` is picked by every token (T rows: several 64-row
    passes when T > 64) and the rest spread at random; some experts get no rows."""
    topi = np.zeros((T, k), np.int32)
    for t in range(T):
        others = rng.permutation([e for e in range(E) if e != hot])[: k - 1]
        topi[t] = np.concatenate([[hot], others])
    return topi


@pytest.mark.parametrize("T,N,K,E,k,skew", [
    (1, 96, 256, 8, 2, False),        # one token: 2 experts of 1 row, 6 empty
    (32, 1536, 2048, 128, 8, False),  # config-4 gate_up shape, batch 32
    (128, 1536, 2048, 128, 8, False), # config-4 gate_up shape, batch 128 (about 8 rows each)
    (128, 2048, 768, 128, 8, False),  # config-4 down shape
    (130, 256, 384, 16, 4, True),     # one expert with 130 rows: three passes (64, 64, 2)
    (65, 200, 128, 8, 3, True),       # 65 rows (a pass of 64 and one of 1); N not a tile multiple
])
def test_grouped_gemm_tensor_cores_bit_exact(T, N, K, E, k, skew):
    """s8b_moe_gemm_grouped_tc on rows gathered by s8b_moe_gather_rows: bit-exact against the
    oracle (the same integer sums and dequantization as the CUDA-core grouped kernel)."""
    rng = np.random.default_rng(T * 3 + N + K + E)
    topi = (_skewed_topi(rng, T, E, k, hot=E // 2) if skew else
            np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32))
    off, order, _ = om.group_assignments(topi, E)
    A = T * k
    xq = rng.integers(-127, 128, (T, K), dtype=np.int8)
    xs = rng.uniform(0.001, 0.1, T).astype(np.float32)
    w = rng.integers(-127, 128, (E, N, K), dtype=np.int8)
    ws = rng.uniform(1e-4, 1e-3, (E, N)).astype(np.float32)
    src = (order // k).astype(np.int32)
    xg, xgs = ops.moe_gather_rows(dev(xq), dev(xs), dev(src), A)
    assert np.array_equal(xg.cpu().numpy(), xq[src])
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    y = ops.moe_gemm_grouped_tc(xg, xgs, dev(w), dev(ws), dev(off), A=A, max_rows=T,
                                status=status)
    want = np.zeros((A, N), np.float32)
    for e in range(E):
        lo, hi = off[e], off[e + 1]
        if lo < hi:
            want[lo:hi] = gemm_w8a8(xq[src[lo:hi]], xs[src[lo:hi]], w[e], ws[e])
    got = f32(y)
    bad = np.argwhere(got != want)
    assert bad.size == 0, (len(bad), bad[:4])
    assert int(status.item()) == 0
    # an expert range of a shard: experts [e_lo, E) with the offsets from e_lo on (absolute
    # row numbers), as the expert-parallel partner runs them
    e_lo = E // 2
    y2 = torch.full((A, N), float("nan"), dtype=torch.bfloat16, device=DEV)
    offd = dev(off)
    from superl8_serve_b200._lib import call, ptr, stream
    call("s8b_moe_gemm_grouped_tc", ptr(xg), ptr(xgs), ptr(dev(w[e_lo:].copy())),
         ptr(dev(ws[e_lo:].copy())), offd.data_ptr() + 4 * e_lo, ptr(y2), A, N, K, E - e_lo, T,
         ptr(status), 0, stream(xg.device))
    lo = off[e_lo]
    assert np.array_equal(f32(y2)[lo:], want[lo:])


def test_combine_bit_exact():
    rng = np.random.default_rng(9)
    T, k, E, H = 19, 8, 128, 2048
    topi = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    topw = on.round_bf16(rng.uniform(0, 0.5, (T, k)).astype(np.float32))
    _, _, rowpos = om.group_assignments(topi, E)
    contrib = on.round_bf16(rng.standard_normal((T * k, H)).astype(np.float32))
    out = ops.moe_combine(bf16(contrib), bf16(topw), dev(topi), dev(rowpos))
    assert np.array_equal(f32(out), om.combine(contrib, topi, topw, rowpos))


def test_qwen3_30b_a3b_shaped_moe_ffn_bit_exact():
    """One MoE FFN at the BASELINE config-4 shape (128 experts top-8, hidden 2048, expert FFN
    768) for a 32-token micro-batch: route, grouped gate_up, SwiGLU + quant, grouped down,
    combine — the oracle's ``moe_ffn`` bit for bit."""
    rng = np.random.default_rng(30)
    T, H, E, Fe, k = 32, 2048, 128, 768, 8
    y = on.round_bf16(rng.standard_normal((T, H)).astype(np.float32))
    gate = on.round_bf16((0.02 * rng.standard_normal((E, H))).astype(np.float32))
    gu_w = rng.integers(-127, 128, (E, 2 * Fe, H), dtype=np.int8)
    gu_s = rng.uniform(1e-4, 3e-4, (E, 2 * Fe)).astype(np.float32)
    d_w = rng.integers(-127, 128, (E, H, Fe), dtype=np.int8)
    d_s = rng.uniform(1e-4, 3e-4, (E, H)).astype(np.float32)
    xq, xs = on.quant_rows_i8(y)
    r = ops.moe_route(bf16(y), dev(gate), k)
    A = T * k
    gu = ops.moe_gemm_grouped(dev(xq), dev(xs), dev(gu_w), dev(gu_s), r["offsets"],
                              row_index=r["sorted_token"], A=A)
    aq, a_s, _ = ops.silu_mul_quant(gu)
    part = ops.moe_gemm_grouped(aq, a_s, dev(d_w), dev(d_s), r["offsets"], A=A)
    out = ops.moe_combine(part, r["topw"], r["topi"], r["assign_pos"])
    experts = [((gu_w[e], gu_s[e]), (d_w[e], d_s[e])) for e in range(E)]
    want = om.moe_ffn(y, xq, xs, gate, experts, k)
    assert np.array_equal(f32(out), want)


def stage_models(cfg, sd, n_stages):
    b = stage_bounds(cfg.num_hidden_layers, n_stages)
    return [StageModel.from_state_dict(cfg, sd, b[i], b[i + 1], DEV, first=i == 0,
                                       last=i == n_stages - 1) for i in range(n_stages)]


@pytest.fixture(scope="module")
def moe_sd():
    return tiny_moe(), random_state_dict(tiny_moe(), 13, w_std=0.1)


@pytest.mark.parametrize("tag,stages,scheme,prefill", [
    ("moe_s1", 1, "int8", False), ("moe_s2_int8had", 2, "int8-had", False),
    ("moe_s2_int8had", 2, "int8-had", True)])
def test_tiny_moe_model_matches_reference_graph(golden_dir, moe_sd, tag, stages, scheme, prefill):
    """Tiny Qwen3-MoE (16 experts top-4 in every layer) through the stage runtime: the
    reference graph's greedy tokens and logits, bit for bit (decode-fed and prefilled)."""
    g = np.load(golden_dir / "tiny_qwen3_moe.npz")
    cfg, sd = moe_sd
    pipe = DecodePipeline(stage_models(cfg, sd, stages), batch=3, n_micro=1, max_len=64,
                          wire_scheme=scheme)
    if prefill:
        pipe.prefill_chunk = 5
    outs, logits = pipe.generate(PROMPTS, 8, keep_logits=True, prefill=prefill)
    assert np.array_equal(np.array(outs), g[f"{tag}_tokens"])
    got = np.stack([np.stack([t.numpy() for t in row]) for row in logits])
    assert np.array_equal(got, g[f"{tag}_logits"])


def test_tiny_moe_tensor_core_micro_batch_matches_oracle(moe_sd):
    """24 rows per micro-batch: the attention projections run on the tcgen05 GEMM with
    split-K partials feeding the post-attention norm that also emits the router input."""
    cfg, sd = moe_sd
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, cfg.vocab_size, 6).tolist() for _ in range(24)]
    pipe = DecodePipeline(stage_models(cfg, sd, 2), batch=24, n_micro=1, max_len=64,
                          wire_scheme="int8-had")
    assert pipe.runners[0].tc_ws is not None
    outs = pipe.generate(prompts, 4)
    ref, _ = OraclePipeline(cfg, quantize_state_dict(sd, cfg), n_stages=2,
                            wire_scheme="int8-had", num_slots=24, max_len=64).generate(prompts, 4)
    assert outs == ref


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("stages", [1, 2])
def test_expert_parallel_two_gpus_matches_reference_graph(golden_dir, moe_sd, stages):
    """Experts of every MoE layer split over cuda:0 (0-7) and cuda:1 (8-15): the partner's
    down projection stores its rows into cuda:0's buffer over NVLink and cuda:0 combines in
    ascending expert order — the single-GPU result, bit for bit."""
    g = np.load(golden_dir / "tiny_qwen3_moe.npz")
    tag = {1: "moe_s1", 2: "moe_s2_int8had"}[stages]
    cfg, sd = moe_sd
    models = [m.shard_experts(["cuda:1"]) for m in stage_models(cfg, sd, stages)]
    assert models[0].layers[0].moe.local_experts == 8
    pipe = DecodePipeline(models, batch=3, n_micro=1, max_len=64,
                          wire_scheme="int8" if stages == 1 else "int8-had")
    outs, logits = pipe.generate(PROMPTS, 8, keep_logits=True)
    assert np.array_equal(np.array(outs), g[f"{tag}_tokens"])
    got = np.stack([np.stack([t.numpy() for t in row]) for row in logits])
    assert np.array_equal(got, g[f"{tag}_logits"])
