"""GPU: the no-allocation paged-decode entry point (s8b_paged_decode_q8_noalloc).

Some callers cannot allocate device memory on the decode path: a host-language binding that is
handed device buffers but owns no allocator, or a serving runtime that reserved all of HBM up
front. For them the library offers one attention entry point that takes no workspace and keeps
its scratch in a fixed array inside the library's own device memory. These tests call it
through the C ABI and check every call against both the workspace-taking entry point and the
CPU oracle, bit for bit:

* on each attention implementation (the persistent tensor-core kernel, the per-partition
  tensor-core kernel and the CUDA-core kernel; the last two keep completion counters in the
  array);
* on call sequences whose shape grows (more rows, more heads), so that a call's counters land
  where the previous call left partials, and that shrink again;
* on a block size of 4, which the persistent kernel does not take (automatic fallback);
* on 288 work units (about two per SM of the persistent kernel).

They also check the array's status word through s8b_paged_decode_noalloc_status, and that a
request beyond the fixed limit is refused without launching anything.

The file name sorts last so that a run stopping at the first failure has run everything else
first; the tests also pass on their own in a fresh process, where the first call is the one
that looks up the array's device address.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import kernels as ok
from oracle import numerics as on

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TIMEOUT_CODE = -6  # S8B_ERR_TIMEOUT


def _case(rng, B, Hq, Hkv, lens, bs=16):
    maxb = (max(lens) + bs - 1) // bs
    nb = B * maxb + 2
    kc = rng.integers(-127, 128, (nb, Hkv, bs, 128), dtype=np.int8)
    vc = rng.integers(-127, 128, (nb, Hkv, bs, 128), dtype=np.int8)
    ks = rng.uniform(0.01, 0.05, (nb, Hkv, bs)).astype(np.float32)
    vs = rng.uniform(0.01, 0.05, (nb, Hkv, bs)).astype(np.float32)
    perm = rng.permutation(nb)
    bt = np.zeros((B, maxb + 1), dtype=np.int32)
    for b in range(B):
        bt[b, :maxb] = perm[b * maxb:(b + 1) * maxb]
    qq = rng.integers(-127, 128, (B, Hq, 128), dtype=np.int8)
    qs = rng.uniform(0.002, 0.02, (B, Hq)).astype(np.float32)
    cl = np.array(lens, dtype=np.int32)
    return qq, qs, kc, ks, vc, vs, bt, cl


def _noalloc(lib, dev_args, B, Hq, Hkv, bs, maxb, max_ctx, scale):
    qq, qs, kc, ks, vc, vs, bt, cl = dev_args
    out = torch.full((B, Hq * 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    out_q = torch.zeros((B, Hq * 128), dtype=torch.int8, device=DEV)
    out_s = torch.zeros(B, dtype=torch.float32, device=DEV)
    rc = lib.s8b_paged_decode_q8_noalloc(
        qq.data_ptr(), qs.data_ptr(), kc.data_ptr(), ks.data_ptr(), vc.data_ptr(),
        vs.data_ptr(), bt.data_ptr(), cl.data_ptr(), out.data_ptr(), out_q.data_ptr(),
        out_s.data_ptr(), B, Hq, Hkv, 128, bs, maxb, max_ctx, scale, 0,
        torch.cuda.current_stream().cuda_stream)
    return rc, out, out_q, out_s


def _status(lib, replace_with=0):
    prev = ctypes.c_int32(12345)
    rc = lib.s8b_paged_decode_noalloc_status(ctypes.byref(prev), replace_with)
    assert rc == 0
    return prev.value


def _check_sequence(cases, bs=16, seed=99):
    """Runs each case through the no-allocation entry point, the workspace entry point and the
    oracle; every output must be identical."""
    from superl8_serve_b200 import _lib, ops

    lib = _lib.load()
    rng = np.random.default_rng(seed)
    scale = 128 ** -0.5
    for B, Hq, Hkv, lens in cases:
        host = _case(rng, B, Hq, Hkv, lens, bs)
        dev = [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in host]
        qq, qs, kc, ks, vc, vs, bt, cl = dev
        max_ctx = max(lens) + 3
        ref_q = torch.empty((B, Hq * 128), dtype=torch.int8, device=DEV)
        ref_s = torch.empty(B, dtype=torch.float32, device=DEV)
        ref = ops.paged_decode_q8(qq, qs, kc, ks, vc, vs, bt, cl, max_ctx, scale,
                                  out_q=ref_q, out_s=ref_s)
        rc, out, out_q, out_s = _noalloc(lib, dev, B, Hq, Hkv, bs, bt.shape[1], max_ctx, scale)
        assert rc == 0, _lib.strerror(rc)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert torch.equal(out_q, ref_q) and torch.equal(out_s, ref_s)
        want = ok.paged_decode(*host, bs, scale).reshape(B, -1)
        assert np.array_equal(out.float().cpu().numpy(), want)
        wq, wsc = on.quant_rows_i8(want)
        assert np.array_equal(out_q.cpu().numpy(), wq)
        assert np.array_equal(out_s.cpu().numpy(), wsc)
    assert _status(lib) == 0


@pytest.fixture(params=["auto", "tc_partition", "cuda_core"])
def attn_impl(request):
    from superl8_serve_b200 import ops

    ops.set_attention_impl(request.param)
    yield request.param
    ops.set_attention_impl("auto")


def test_noalloc_calls_in_a_row_with_growing_and_shrinking_shapes(attn_impl):
    # rows grow (3 -> 4), heads grow (16 -> 32), then the shape shrinks again: each call's
    # counters start where an earlier call kept partials or counters
    _check_sequence([(3, 32, 8, [17, 700, 256]),
                     (4, 32, 8, [2049, 1, 300, 1000]),
                     (4, 16, 8, [600, 33, 1000, 5]),
                     (4, 32, 8, [257, 512, 1, 90]),
                     (2, 32, 8, [1500, 3])])


def test_noalloc_block_size_4_takes_the_partition_kernels():
    # the persistent kernel needs blocks of >= 8 tokens; "auto" falls back here
    _check_sequence([(3, 32, 8, [40, 300, 129]), (4, 32, 8, [513, 2, 77, 256])], bs=4, seed=5)


def test_noalloc_288_units():
    # 4 rows x 8 kv heads x 9 partitions: about two units per SM of the persistent kernel
    _check_sequence([(4, 32, 8, [2049, 2000, 1900, 2048])], seed=7)


def test_noalloc_status_word_reads_and_clears():
    """The status word is sticky: a decode call leaves a set word as it is, the status call
    returns it and replaces it. A value is planted by the status call itself (no device wait
    is made to time out)."""
    from superl8_serve_b200 import _lib

    lib = _lib.load()
    _check_sequence([(2, 32, 8, [100, 300])], seed=3)  # ends by reading a clear word
    assert _status(lib, TIMEOUT_CODE) == 0  # plant the timeout code
    assert _status(lib, TIMEOUT_CODE) == TIMEOUT_CODE
    rng = np.random.default_rng(4)
    host = _case(rng, 2, 32, 8, [64, 700])
    dev = [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in host]
    rc, *_ = _noalloc(lib, dev, 2, 32, 8, 16, dev[6].shape[1], 703, 128 ** -0.5)
    assert rc == 0
    torch.cuda.synchronize()
    assert _status(lib, 0) == TIMEOUT_CODE  # a call does not clear it
    assert _status(lib, 0) == 0


def test_noalloc_refuses_requests_beyond_the_static_limit():
    from superl8_serve_b200 import _lib

    lib = _lib.load()
    # 64 rows x 32 heads x 16 partitions x 130 floats = 17 MiB > 16 MiB: refused before launch
    dummy = torch.zeros(16, dtype=torch.int8, device=DEV)
    p = dummy.data_ptr()
    rc = lib.s8b_paged_decode_q8_noalloc(p, p, p, p, p, p, p, p, p, None, None, 64, 32, 8, 128,
                                         16, 256, 4096, 0.088, 0,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == -9
    assert "static limit" in _lib.strerror(rc)
