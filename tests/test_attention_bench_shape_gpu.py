"""GPU: paged decode attention at the benchmarked shape, against the CPU oracle, bit for bit.

Qwen3-8B attention (32 query heads, 8 kv heads, head dim 128, block 16) over contexts of about
2048 tokens, at batch 64 (4,096 work units of (row, kv head, 256-token partition)) and batch
256 (16,384 units). The persistent kernel runs one CTA per SM, so every CTA walks about 28
(or 111) units: its three-stage K/V ring wraps many times and its double-buffered TMEM score
and output tiles are handed back and forth between the MMA, softmax and epilogue roles on
every unit, which small cases never reach. Block tables come in the orders an allocator
produces (consecutive ascending ids, the reference allocator's descending runs, a random
permutation), so full partitions take both the 4-D run copies and the per-block copies.
Contexts are ragged, so partial partitions and tail masks occur in the same launch.

The oracle result is computed once per case and every attention implementation is compared
with it.
"""

import numpy as np
import pytest
import torch

from oracle import kernels as ok
from oracle import numerics as on

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
IMPLS = ("auto", "tc_partition", "cuda_core")


def _table(layout, B, maxb, nb, rng):
    bt = np.zeros((B, maxb + 2), dtype=np.int32)
    if layout == "ascending":
        for b in range(B):
            bt[b, :maxb] = np.arange(b * maxb, (b + 1) * maxb)
    elif layout == "descending":  # free list range(nb), popped from the end
        free = list(range(nb))
        for b in range(B):
            bt[b, :maxb] = [free.pop() for _ in range(maxb)]
    else:
        perm = rng.permutation(nb)
        for b in range(B):
            bt[b, :maxb] = perm[b * maxb:(b + 1) * maxb]
    return bt


@pytest.mark.parametrize("B,layout", [(64, "ascending"), (64, "descending"), (64, "random"),
                                      (256, "descending"), (256, "random")])
def test_paged_decode_at_bench_shape(B, layout):
    from superl8_serve_b200 import ops

    Hq, Hkv, bs = 32, 8, 16
    rng = np.random.default_rng(2048 + B)
    lens = (2049 - rng.integers(0, 260, B)).astype(np.int32)
    lens[: B // 4] = 2049  # a quarter of the rows have every partition full but the last
    lens[B // 4: B // 2] = 2048  # and a quarter end exactly on a partition edge
    maxb = (int(lens.max()) + bs - 1) // bs
    nb = B * maxb + 3
    kc = rng.integers(-127, 128, (nb, Hkv, bs, 128), dtype=np.int8)
    vc = rng.integers(-127, 128, (nb, Hkv, bs, 128), dtype=np.int8)
    ks = rng.uniform(0.01, 0.05, (nb, Hkv, bs)).astype(np.float32)
    vs = rng.uniform(0.01, 0.05, (nb, Hkv, bs)).astype(np.float32)
    bt = _table(layout, B, maxb, nb, rng)
    qq = rng.integers(-127, 128, (B, Hq, 128), dtype=np.int8)
    qs = rng.uniform(0.002, 0.02, (B, Hq)).astype(np.float32)
    scale = 128 ** -0.5
    dev = [torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
           for a in (qq, qs, kc, ks, vc, vs, bt, lens)]
    want = ok.paged_decode(qq, qs, kc, ks, vc, vs, bt, lens, bs, scale).reshape(B, -1)
    wq, wsc = on.quant_rows_i8(want)
    max_ctx = 2049 + 16
    ws = torch.zeros(ops.decode_workspace_bytes(B, Hq, 128, max_ctx), dtype=torch.uint8,
                     device=DEV)
    try:
        # the decode-step form (older partitions streamed before the previous kernel ends)
        # with the persistent kernel, then every implementation through the plain form
        for impl, step in [("auto", True)] + [(i, False) for i in IMPLS]:
            ops.set_attention_impl(impl)
            oq = torch.zeros((B, Hq * 128), dtype=torch.int8, device=DEV)
            osc = torch.zeros(B, dtype=torch.float32, device=DEV)
            for _ in range(2):  # a second launch on the same workspace
                out = ops.paged_decode_q8(*dev, max_ctx, scale, out_q=oq, out_s=osc,
                                          workspace=ws, step=step)
            assert ops.decode_status(ws, B, Hq) == 0, impl
            got = out.float().cpu().numpy()
            bad = np.argwhere(got != want)
            assert bad.size == 0, (impl, len(bad), bad[:4])
            assert np.array_equal(oq.cpu().numpy(), wq), impl
            assert np.array_equal(osc.cpu().numpy(), wsc), impl
    finally:
        ops.set_attention_impl("auto")
