"""The reference's float contract for the paged decode attention (TEST INFRASTRUCTURE ONLY).

The ``superl8`` attention kernel is absent, so ``oracle.kernels.paged_decode`` DEFINES the
bit-level recipe the CUDA kernels reproduce (per-head int8 query, 256-token partitions,
15-bit p.v weights). This module states the float computation that recipe approximates, as
the reference's own float code path spells it out: ``PagedKVCache.read_dense``
(``superl8serve/engine/kv_cache.py:1233-1299``) dequantizes the int8 cache (K = code x
scale, then the orthonormal Hadamard un-rotates it; V = code x scale) and the attention is
softmax(q . K^T * scale) . V with an fp32 softmax, rounded to the activation dtype
(``superl8serve/engine/kv_cache.py:1148-1201`` names the contract of
``attn_paged_decode_cached``). ``acc`` selects fp32 (the contract) or fp64 (to measure how
far two float evaluations of the same contract already are apart).

``TeacherForced`` drives a model with the float contract and, at every layer of every step,
also evaluates the recipe on exactly the same query and cache: the recipe's own error, layer
by layer, without the compounding of a free-running comparison.

Why the comparison is made per layer: every W8A8 linear quantizes its input row per token
(amax / 127). A change anywhere in a row, however small, that moves the row's amax or
crosses a rounding boundary re-draws that row's rounding pattern, so the model's output
moves by the size of the quantization noise (about 1-4% of the logits here), not by the size
of the change. Two evaluations of a W8A8 model agree to 1e-2 in the logits only if every
quantizer sees bit-identical inputs; that is the bar the CUDA path meets against the oracle.
"""

from __future__ import annotations

import numpy as np

from .model import recipe_attention
from .numerics import hadamard128, round_bf16


def float_attention(q, kc, ks, vc, vs, block_table, ctx_lens, block_size, scale, li=None,
                    acc=np.float32):
    """q [B, Hq, D] (float32, bf16-valued, not rotated) over the paged int8 cache ->
    [B, Hq, D] bf16-valued: read_dense dequantization, then softmax(q K^T scale) V in `acc`."""
    B, Hq, D = q.shape
    _, Hkv, bs, _ = kc.shape
    G = Hq // Hkv
    kf, vf = kc.reshape(-1, D), vc.reshape(-1, D)
    ksf, vsf = ks.reshape(-1), vs.reshape(-1)
    out = np.zeros((B, Hq, D), np.float32)
    heads = np.arange(Hq) // G
    for b in range(B):
        n = int(ctx_lens[b])
        j = np.arange(n)
        blk = np.asarray(block_table[b], np.int64)[j // block_size]
        rows = (blk[:, None] * Hkv + np.arange(Hkv)[None]) * block_size + (j % block_size)[:, None]
        k = hadamard128((kf[rows].astype(np.float32) * ksf[rows][..., None]).astype(np.float32))
        k = k.astype(acc)
        v = vf[rows].astype(acc) * vsf[rows][..., None].astype(acc)
        s = np.einsum("hd,nhd->nh", q[b].astype(acc), k[:, heads]) * acc(scale)
        p = np.exp(s - s.max(axis=0))
        p = p / p.sum(axis=0)
        out[b] = round_bf16(np.einsum("nh,nhd->hd", p, v[:, heads]).astype(np.float32))
    return out


def float64_attention(*args, **kw):
    return float_attention(*args, acc=np.float64, **kw)


class TeacherForced:
    """Attention callable for ``OraclePipeline(attention=...)``: returns the float contract
    (so the model runs on it) and records, per call, the relative error of the recipe on the
    same query and cache: ||recipe - float|| / ||float|| over the batch's rows."""

    def __init__(self):
        self.errors: list[float] = []

    def __call__(self, q, kc, ks, vc, vs, block_table, ctx_lens, block_size, scale, li=None):
        ref = float_attention(q, kc, ks, vc, vs, block_table, ctx_lens, block_size, scale)
        got = recipe_attention(q, kc, ks, vc, vs, block_table, ctx_lens, block_size, scale)
        self.errors.append(float(np.linalg.norm(got - ref) / np.linalg.norm(ref)))
        return ref


def logits_rel(a, b) -> float:
    """max over rows of ||a - b|| / ||b|| (rows of logits)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.linalg.norm(a - b, axis=-1) / np.linalg.norm(b, axis=-1)))
