"""GPU: the no-allocation paged-decode entry point (s8b_paged_decode_q8_noalloc).

Some callers cannot allocate device memory on the decode path: a host-language binding that is
handed device buffers but owns no allocator, or a serving runtime that reserved all of HBM up
front. For them the library offers one attention entry point that takes no workspace and keeps
its scratch in a fixed array inside the library's own device memory. This test calls it
through the C ABI and checks it against the workspace-taking entry point, on two calls in a
row with different inputs (the second call reuses the array the first one filled), and checks
that a request beyond the fixed limit is refused without launching anything.

The file name sorts last so that a run stopping at the first failure has run everything else
first; the test also passes on its own in a fresh process, where its first call is the one
that looks up the array's device address.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


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
    return [torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
            for a in (qq, qs, kc, ks, vc, vs, bt, cl)]


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    from superl8_serve_b200 import _lib, ops

    lib = _lib.load()
    rng = np.random.default_rng(99)
    cases = [(4, 32, 8, [2049, 1, 300, 1000]), (3, 32, 8, [17, 700, 256])]
    for B, Hq, Hkv, lens in cases:
        qq, qs, kc, ks, vc, vs, bt, cl = _case(rng, B, Hq, Hkv, lens)
        max_ctx = max(lens) + 3
        scale = 128 ** -0.5
        ref_q = torch.empty((B, Hq * 128), dtype=torch.int8, device=DEV)
        ref_s = torch.empty(B, dtype=torch.float32, device=DEV)
        ref = ops.paged_decode_q8(qq, qs, kc, ks, vc, vs, bt, cl, max_ctx, scale,
                                  out_q=ref_q, out_s=ref_s)
        out = torch.full((B, Hq * 128), float("nan"), dtype=torch.bfloat16, device=DEV)
        out_q = torch.zeros((B, Hq * 128), dtype=torch.int8, device=DEV)
        out_s = torch.zeros(B, dtype=torch.float32, device=DEV)
        rc = lib.s8b_paged_decode_q8_noalloc(
            qq.data_ptr(), qs.data_ptr(), kc.data_ptr(), ks.data_ptr(), vc.data_ptr(),
            vs.data_ptr(), bt.data_ptr(), cl.data_ptr(), out.data_ptr(), out_q.data_ptr(),
            out_s.data_ptr(), B, Hq, Hkv, 128, 16, bt.shape[1], max_ctx, scale, 0,
            torch.cuda.current_stream().cuda_stream)
        assert rc == 0, _lib.strerror(rc)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert torch.equal(out_q, ref_q) and torch.equal(out_s, ref_s)


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
