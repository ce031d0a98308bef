"""GPU: the tcgen05 kind::i8 GEMM against the oracle: int32 accumulators and dequantized
outputs bit-identical, across whole-tile and split-tile work ranges, token counts 16..300."""

import numpy as np
import pytest
import torch

from oracle import kernels as ok

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("M,N,K", [
    (16, 128, 128),       # one unit
    (64, 4096, 4096),     # o_proj: tiles split across several CTAs
    (64, 24576, 4096),    # gate_up: ~1.3 tiles per CTA
    (64, 4096, 12288),    # down
    (64, 6144, 4096),     # qkv
    (13, 1024, 256),      # ragged token count (padded to 16)
    (40, 1536, 1024),     # 40 -> 64-token tile
    (100, 2048, 512),     # 128-token tile
    (256, 1024, 384),     # full 256-token tile
    (300, 640, 256),      # two passes (256 + 44)
])
def test_tc_gemm_bit_exact(M, N, K):
    from superl8_serve_b200 import ops

    rng = np.random.default_rng(M * 7 + N)
    xq = rng.integers(-127, 128, (M, K), dtype=np.int8)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    xq[0] = 127
    w[0] = -127
    xs = rng.uniform(0.001, 0.05, M).astype(np.float32)
    ws = rng.uniform(0.0001, 0.001, N).astype(np.float32)
    wsp = ops.gemm_tc_workspace(M, N, DEV)
    acc = ops.gemm_w8a8_tc(_t(xq), _t(xs), _t(w), _t(ws), raw=True, workspace=wsp)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), ok.gemm_acc(xq, w))
    y = ops.gemm_w8a8_tc(_t(xq), _t(xs), _t(w), _t(ws), workspace=wsp)
    torch.cuda.synchronize()
    assert np.array_equal(y.float().cpu().numpy(), ok.gemm_w8a8(xq, xs, w, ws))
    # every completed launch leaves the workspace zero (status, counters, accumulators)
    assert int(wsp.count_nonzero()) == 0


def test_tc_gemm_matches_dp4a_path():
    from superl8_serve_b200 import ops

    rng = np.random.default_rng(5)
    M, N, K = 64, 3072, 1024
    xq, w = rng.integers(-127, 128, (M, K), dtype=np.int8), rng.integers(-127, 128, (N, K), dtype=np.int8)
    xs = rng.uniform(0.001, 0.05, M).astype(np.float32)
    ws = rng.uniform(0.0001, 0.001, N).astype(np.float32)
    a = ops.gemm_w8a8_tc(_t(xq), _t(xs), _t(w), _t(ws))
    b = ops.gemm_w8a8(_t(xq), _t(xs), _t(w), _t(ws))
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_tiny_model_on_tensor_core_path_matches_oracle():
    """20 rows per micro-batch: every GEMM of the step runs on tcgen05; tokens and logits
    must equal the oracle's."""
    from oracle.model import OraclePipeline, quantize_state_dict
    from superl8_serve_b200.config import tiny
    from superl8_serve_b200.engine import DecodePipeline
    from superl8_serve_b200.runtime import StageModel
    from superl8_serve_b200.weights import random_state_dict

    cfg = tiny()
    sd = random_state_dict(cfg, 3, w_std=0.1)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, cfg.vocab_size, int(n)).tolist() for n in rng.integers(2, 6, 20)]
    models = [StageModel.from_state_dict(cfg, sd, 0, 2, DEV, first=True, last=False),
              StageModel.from_state_dict(cfg, sd, 2, 4, DEV, first=False, last=True)]
    pipe = DecodePipeline(models, batch=20, n_micro=1, max_len=64, wire_scheme="int8-had")
    assert pipe.runners[0].tc_ws is not None
    outs, logits = pipe.generate(prompts, 4, keep_logits=True)
    ref, ref_logits = OraclePipeline(cfg, quantize_state_dict(sd, cfg), n_stages=2,
                                     wire_scheme="int8-had", num_slots=20,
                                     max_len=64).generate(prompts, 4)
    assert outs == ref
    got = np.stack([np.stack([t.numpy() for t in row]) for row in logits])
    assert np.array_equal(got, np.array(ref_logits, dtype=np.float32))


@pytest.mark.parametrize("M,N,K", [(64, 24576, 4096), (64, 4096, 12288), (16, 1000, 256),
                                   (200, 640, 384)])
def test_tc_gemm_packed_weights_bit_exact(M, N, K):
    """Pre-packed unit images (contiguous bulk loads) give the same int32 sums and outputs."""
    from superl8_serve_b200 import ops

    rng = np.random.default_rng(N + K)
    xq = rng.integers(-127, 128, (M, K), dtype=np.int8)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    xs = rng.uniform(0.001, 0.05, M).astype(np.float32)
    ws = rng.uniform(0.0001, 0.001, N).astype(np.float32)
    wd = _t(w)
    packed = ops.pack_weights_tc(wd)
    wsp = ops.gemm_tc_workspace(M, N, DEV)
    acc = ops.gemm_w8a8_tc(_t(xq), _t(xs), wd, _t(ws), raw=True, workspace=wsp, packed=packed)
    y = ops.gemm_w8a8_tc(_t(xq), _t(xs), wd, _t(ws), workspace=wsp, packed=packed)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), ok.gemm_acc(xq, w))
    assert np.array_equal(y.float().cpu().numpy(), ok.gemm_w8a8(xq, xs, w, ws))
    assert int(wsp.count_nonzero()) == 0


@pytest.mark.parametrize("M,N,K,packed", [
    (64, 4096, 4096, True), (64, 6144, 4096, True), (64, 24576, 4096, True),
    (64, 4096, 12288, True), (20, 1000, 256, False), (300, 640, 384, False)])
def test_tc_gemm_split_partials_sum_to_accumulators(M, N, K, packed):
    """out_kind 2: C int32 partial tiles whose sum is the oracle's accumulator."""
    from superl8_serve_b200 import ops

    rng = np.random.default_rng(N * 3 + K)
    xq = rng.integers(-127, 128, (M, K), dtype=np.int8)
    w = rng.integers(-127, 128, (N, K), dtype=np.int8)
    xs = rng.uniform(0.001, 0.05, M).astype(np.float32)
    wd = _t(w)
    part = ops.gemm_w8a8_tc_split(_t(xq), _t(xs), wd,
                                  packed=ops.pack_weights_tc(wd) if packed else None)
    torch.cuda.synchronize()
    assert 1 <= part.shape[0] <= 8
    assert np.array_equal(part.sum(0, dtype=torch.int64).cpu().numpy(), ok.gemm_acc(xq, w))


def _gemm_inputs(rng, M, N, K):
    xq = _t(rng.integers(-127, 128, (M, K), dtype=np.int8))
    xs = _t(rng.uniform(0.001, 0.02, M).astype(np.float32))
    w = _t(rng.integers(-127, 128, (N, K), dtype=np.int8))
    ws = _t(rng.uniform(0.0002, 0.002, N).astype(np.float32))
    return xq, xs, w, ws


def test_rmsnorm_and_silu_split_consumers_match_dtype_path():
    """Reading the GEMM's partials (sum, dequant) inside the row kernel gives exactly what the
    GEMM's own dtype output followed by the plain row kernel gives."""
    from superl8_serve_b200 import ops

    rng = np.random.default_rng(21)
    M, H, F = 64, 4096, 12288
    xq, xs, w, ws = _gemm_inputs(rng, M, H, 4096)
    res = _t((rng.standard_normal((M, H)) * 2).astype(np.float32)).to(torch.bfloat16)
    gain = _t((1 + 0.1 * rng.standard_normal(H)).astype(np.float32)).to(torch.bfloat16)
    h = ops.gemm_w8a8_tc(xq, xs, w, ws)
    r1, q1, s1, _ = ops.rmsnorm_quant(h, res, gain, 1e-6, residual_out=torch.empty_like(res))
    part = ops.gemm_w8a8_tc_split(xq, xs, w)
    r2, q2, s2 = ops.rmsnorm_quant_split(part, xs, ws, res, gain, 1e-6,
                                         residual_out=torch.empty_like(res))
    torch.cuda.synchronize()
    assert torch.equal(r1, r2) and torch.equal(q1, q2) and torch.equal(s1, s2)
    xq, xs, w, ws = _gemm_inputs(rng, M, 2 * F, 4096)
    gu = ops.gemm_w8a8_tc(xq, xs, w, ws)
    qa, sa, ya = ops.silu_mul_quant(gu, y_out=True)
    qb, sb, yb = ops.silu_mul_quant_split(ops.gemm_w8a8_tc_split(xq, xs, w), xs, ws)
    torch.cuda.synchronize()
    assert torch.equal(qa, qb) and torch.equal(sa, sb) and torch.equal(ya, yb)


def test_qkv_post_split_consumer_matches_dtype_path():
    from superl8_serve_b200 import ops
    from superl8_serve_b200.layers import rope_tables

    rng = np.random.default_rng(22)
    M, Hq, Hkv, D, bs = 64, 32, 8, 128, 16
    xq, xs, w, ws = _gemm_inputs(rng, M, (Hq + 2 * Hkv) * D, 4096)
    cos, sin = (t.to(DEV) for t in rope_tables(D, 4096, 1e6))
    qn = _t((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)).to(torch.bfloat16)
    kn = _t((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)).to(torch.bfloat16)
    pos = _t(rng.integers(0, 4000, M).astype(np.int32))
    bt = _t(np.arange(M * 256, dtype=np.int32).reshape(M, 256))
    pools = [[torch.zeros((M * 256, Hkv, bs, D), dtype=torch.int8, device=DEV),
              torch.zeros((M * 256, Hkv, bs), dtype=torch.float32, device=DEV),
              torch.zeros((M * 256, Hkv, bs, D), dtype=torch.int8, device=DEV),
              torch.zeros((M * 256, Hkv, bs), dtype=torch.float32, device=DEV)] for _ in range(2)]
    qkv = ops.gemm_w8a8_tc(xq, xs, w, ws)
    qa, sa, _ = ops.qkv_post(qkv, pos, cos, sin, qn, kn, 1e-6, Hq, Hkv, *pools[0], block_table=bt)
    qb, sb = ops.qkv_post_split(ops.gemm_w8a8_tc_split(xq, xs, w), xs, ws, pos, cos, sin, qn, kn,
                                1e-6, Hq, Hkv, *pools[1], block_table=bt)
    torch.cuda.synchronize()
    assert torch.equal(qa, qb) and torch.equal(sa, sb)
    for a, b in zip(pools[0], pools[1]):
        assert torch.equal(a, b)
