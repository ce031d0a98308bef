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
