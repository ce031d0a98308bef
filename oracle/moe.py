"""Oracle sparse-MoE FFN (TEST INFRASTRUCTURE ONLY): the reference's ``SparseMoE.forward``
(``superl8serve/models/moe.py:88-138``) with the softmax scoring path of Qwen3-MoE, restated
step by step with every rounding fixed.

* Router logits ``F.linear(xf.float(), gate.float())`` (``moe.py:97-101``). Fixed order:
  lane j of 32 accumulates, in float64, the exact products y[k]*g[e, k] for
  k = 256*i + 8*j + u (i ascending, then u = 0..7), the 32 lane sums meet in an xor
  butterfly (16, 8, 4, 2, 1) in float64, and the result is rounded once to float32.
* ``F.softmax(logits, -1)`` over all experts in float32 (``moe.py:106``):
  m = max; e = exp_s8b(l - m); S = lane-order sum (lane j adds e[j + 32c] for c ascending,
  then the same xor butterfly, float32); p = e / S.
* ``torch.topk(p, k)`` (``moe.py:130``): the k largest in descending order, equal values in
  ascending expert index.
* ``norm_topk_prob`` (``moe.py:131-132``): w = p_j / max(sum_j p_j, 1e-9) with the sum taken
  left to right in rank order; ``* routed_scaling_factor``; cast to bf16 (``moe.py:133``).
* Each expert is a ``GatedMLP`` (``superl8serve/layers/mlp.py:39-40``): W8A8 gate_up on the
  token rows, SwiGLU, W8A8 down; the W8A8 recipe is per-token (``oracle.kernels``).
* ``out.index_add_(0, tok_idx, contrib * w)`` over experts in ascending index
  (``moe.py:135-141``): per token, v = bf16(contrib * w) and out = bf16(out + v) with the
  add done in float32, starting from zero.
"""

from __future__ import annotations

import numpy as np

from .kernels import gemm_w8a8, silu_mul
from .numerics import exp_s8b, quant_rows_i8, round_bf16

_LANE = np.arange(32)


def router_logits(y: np.ndarray, gate: np.ndarray) -> np.ndarray:
    """y [T, H] (bf16-valued), gate [E, H] float32 -> float32 logits [T, E] in the lane order
    above."""
    y = np.asarray(y, np.float64)
    g = np.asarray(gate, np.float64)
    T, H = y.shape
    E = g.shape[0]
    Hp = -(-H // 256) * 256
    if Hp != H:
        y = np.pad(y, ((0, 0), (0, Hp - H)))
        g = np.pad(g, ((0, 0), (0, Hp - H)))
    out = np.empty((T, E), np.float32)
    for t0 in range(0, T, 16):
        yt = y[t0:t0 + 16].reshape(-1, 1, Hp // 256, 32, 8)
        gt = g.reshape(1, E, Hp // 256, 32, 8)
        prod = yt * gt  # exact: bf16 x f32 products fit in float64
        acc = np.zeros(prod.shape[:2] + (32,), np.float64)
        for i in range(Hp // 256):
            for u in range(8):
                acc = acc + prod[:, :, i, :, u]
        for off in (16, 8, 4, 2, 1):
            acc = acc + acc[..., _LANE ^ off]
        out[t0:t0 + 16] = acc[..., 0].astype(np.float32)
    return out


def lane_sum32(e: np.ndarray) -> np.ndarray:
    """float32 sum over the last axis: lane j adds e[j + 32c] (c ascending), then an xor
    butterfly."""
    T, E = e.shape
    Ep = -(-E // 32) * 32
    ep = np.zeros((T, Ep), np.float32)
    ep[:, :E] = e
    acc = np.zeros((T, 32), np.float32)
    for c in range(Ep // 32):
        acc = (acc + ep[:, 32 * c:32 * c + 32]).astype(np.float32)
    for off in (16, 8, 4, 2, 1):
        acc = (acc + acc[:, _LANE ^ off]).astype(np.float32)
    return acc[:, 0]


def moe_route(y: np.ndarray, gate: np.ndarray, top_k: int, norm_topk_prob: bool = True,
              scaling: float = 1.0):
    """Returns (topi int32 [T, k], topw float32 bf16-valued [T, k], probs float32 [T, E])."""
    logits = router_logits(y, gate)
    m = logits.max(axis=1, keepdims=True)
    e = exp_s8b((logits - m).astype(np.float32))
    S = lane_sum32(e)
    p = (e / S[:, None]).astype(np.float32)
    order = np.argsort(-p, axis=1, kind="stable")
    topi = order[:, :top_k].astype(np.int32)
    topw = np.take_along_axis(p, topi, axis=1).astype(np.float32)
    if norm_topk_prob:
        s = np.zeros(len(p), np.float32)
        for j in range(top_k):
            s = (s + topw[:, j]).astype(np.float32)
        s = np.maximum(s, np.float32(1e-9))
        topw = (topw / s[:, None]).astype(np.float32)
    topw = (topw * np.float32(scaling)).astype(np.float32)
    return topi, round_bf16(topw), p


def group_assignments(topi: np.ndarray, n_experts: int):
    """Assignments a = t*k + j sorted by (expert, token): (offsets [E+1], order [A] = the a at
    each sorted position, rowpos [A] = sorted position of each a)."""
    T, k = topi.shape
    a = np.arange(T * k)
    e = topi.reshape(-1)
    order = np.lexsort((a // k, e)).astype(np.int32)
    counts = np.bincount(e, minlength=n_experts)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    rowpos = np.empty(T * k, np.int32)
    rowpos[order] = np.arange(T * k, dtype=np.int32)
    return offsets, order, rowpos


def experts_ffn(xq, xs, order, offsets, k, experts):
    """Grouped expert FFN over the sorted assignments: rows of expert e are
    [offsets[e], offsets[e+1]); the input of sorted row p is token order[p] // k.
    experts[e] = ((gu_q, gu_s), (down_q, down_s)). Returns contributions [A, H] (bf16-valued)."""
    tok = order // k
    A = len(order)
    H = experts[0][1][0].shape[0]
    out = np.zeros((A, H), np.float32)
    for e, ((gq, gs), (dq, ds)) in enumerate(experts):
        lo, hi = offsets[e], offsets[e + 1]
        if lo == hi:
            continue
        gu = gemm_w8a8(xq[tok[lo:hi]], xs[tok[lo:hi]], gq, gs)
        a = silu_mul(gu)
        out[lo:hi] = gemm_w8a8(*quant_rows_i8(a), dq, ds)
    return out


def combine(contrib, topi, topw, rowpos):
    """out[t] = bf16 running sum, in ascending expert index, of bf16(contrib * w)."""
    T, k = topi.shape
    H = contrib.shape[1]
    out = np.zeros((T, H), np.float32)
    ranks = np.argsort(topi, axis=1, kind="stable")
    for r in range(k):
        j = ranks[:, r]
        a = np.arange(T) * k + j
        w = topw[np.arange(T), j]
        v = round_bf16((contrib[rowpos[a]] * w[:, None]).astype(np.float32))
        out = round_bf16((out + v).astype(np.float32))
    return out


def moe_ffn(y, xq, xs, router, experts, top_k, norm_topk_prob=True, scaling=1.0):
    """The whole MoE FFN of one layer: y is the bf16 post-attention RMSNorm output (router
    input), (xq, xs) its per-token int8 quantization (expert input)."""
    topi, topw, _ = moe_route(y, router, top_k, norm_topk_prob, scaling)
    offsets, order, rowpos = group_assignments(topi, len(experts))
    contrib = experts_ffn(xq, xs, order, offsets, top_k, experts)
    return combine(contrib, topi, topw, rowpos)
