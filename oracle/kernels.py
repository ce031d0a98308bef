"""Oracle restatements of the decode-step kernels (TEST INFRASTRUCTURE ONLY).

Each function states the arithmetic the CUDA kernel of the same name must reproduce bit for
bit. Shapes follow the reference call sites cited per function.
"""

from __future__ import annotations

import numpy as np

from .numerics import (
    F32,
    exp_s8b,
    fwht128,
    hadamard128,
    quant_rows_i8,
    quant_sym,
    dequant_acc,
    round_bf16,
)

ATTN_PART = 256  # tokens per attention partition (fixes the accumulation order)


# ------------------------------------------------------------------------ W8A8 GEMM ----

_F32_CACHE: dict[int, tuple[np.ndarray, np.ndarray]] = {}
_KCHUNK = 1024  # 1024 * 127^2 < 2^24: every fp32 partial sum of a chunk is an exact integer


def _f32_weight(wq: np.ndarray) -> np.ndarray:
    hit = _F32_CACHE.get(id(wq))
    if hit is not None and hit[0] is wq:
        return hit[1]
    wf = wq.astype(np.float32)
    if wq.size >= (1 << 20):
        _F32_CACHE[id(wq)] = (wq, wf)
    return wf


def gemm_acc(xq: np.ndarray, wq: np.ndarray) -> np.ndarray:
    """int32 accumulators acc[m, n] = sum_k xq[m, k] * wq[n, k] (exact: |acc| < 2^31).

    Computed as float32 GEMMs over K-chunks of 1024 (each chunk's partial sums are integers
    below 2^24, hence exact in any summation order) and summed in int64."""
    wf = _f32_weight(wq)
    xf = xq.astype(np.float32)
    K = xq.shape[-1]
    acc = np.zeros((xq.shape[0], wq.shape[0]), dtype=np.int64)
    for k0 in range(0, K, _KCHUNK):
        acc += (xf[:, k0:k0 + _KCHUNK] @ wf[:, k0:k0 + _KCHUNK].T).astype(np.int64)
    return acc.astype(np.int32)


def linear_w8a8(x: np.ndarray, wq: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """``LinearW8A8.forward`` (``superl8serve/layers/linear.py:112-124``): per-token int8
    quant of x, int32 GEMM, dequant by x-scale and row scale, output rounded to bf16."""
    xq, xs = quant_rows_i8(x)
    return round_bf16(dequant_acc(gemm_acc(xq, wq), xs, ws))


def gemm_w8a8(xq, xs, wq, ws):
    """GEMM on already-quantized activations, output bf16-valued float32 [M, N]."""
    return round_bf16(dequant_acc(gemm_acc(xq, wq), xs, ws))


# -------------------------------------------------------------------------- RMSNorm ----

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """RMSNorm over the last axis (``superl8serve/layers/norm.py:38-43``), binary32 math:
    ss = sum x^2 (float64 accumulation), ms = f32(ss / n), r = 1 / sqrt(ms + eps),
    y = bf16((x * r) * w)."""
    x = np.asarray(x, dtype=np.float32)
    n = x.shape[-1]
    ss = np.sum(np.square(x.astype(np.float64)), axis=-1)
    ms = (ss / float(n)).astype(np.float32)
    r = (F32(1.0) / np.sqrt((ms + F32(eps)).astype(np.float32))).astype(np.float32)
    y = (x * r[..., None]).astype(np.float32)
    return round_bf16((y * np.asarray(w, dtype=np.float32)).astype(np.float32))


def add_residual(h: np.ndarray, residual):
    """Fused residual add of ``RMSNorm.forward(x, residual)`` (``layers/norm.py:53-58``):
    x = bf16(h + residual); the sum is also the new residual."""
    if residual is None:
        return h
    return round_bf16((h + residual).astype(np.float32))


def rmsnorm_quant(h, residual, w, eps):
    """Kernel ``s8b_rmsnorm_quant``: (new residual, int8 codes, scale) of RMSNorm(h + res)."""
    x = add_residual(h, residual)
    y = rmsnorm(x, w, eps)
    q, s = quant_rows_i8(y)
    return x, q, s, y


# ----------------------------------------------------------------------------- RoPE ----

def rope_tables(head_dim: int, max_position: int, base: float):
    """cos/sin tables exactly as ``RotaryEmbedding.__init__`` builds them
    (``superl8serve/layers/rotary.py:31-37``): binary32 inv_freq, outer product and
    cat(freqs, freqs). Computed with torch on the CPU, as the reference does."""
    import torch

    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().numpy().astype(np.float32), emb.sin().numpy().astype(np.float32)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """rotate-half RoPE ``x*cos + rotate_half(x)*sin`` (``layers/rotary.py:16-19,39-42``)
    with binary32 tables: out = bf16(x*cos + (-x_other)*sin). x [..., D]; cos/sin [..., D]
    broadcastable."""
    d = x.shape[-1]
    h = d // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1).astype(np.float32)
    a = (x * cos).astype(np.float32)
    b = (rot * sin).astype(np.float32)
    return round_bf16((a + b).astype(np.float32))


# ------------------------------------------------------------------------ paged KV ----

def flat_rows(slot_mapping: np.ndarray, nkv: int, block_size: int) -> np.ndarray:
    """Row index of each (token, head) in a layer's [num_blocks*Hkv*block_size, D] store:
    row = (block*Hkv + h)*block_size + off (``superl8serve/engine/kv_cache.py:570-585``).
    Returns [T, Hkv] int64."""
    sm = np.asarray(slot_mapping, dtype=np.int64)
    blk = sm // block_size
    off = sm % block_size
    heads = np.arange(nkv, dtype=np.int64)
    return (blk[:, None] * nkv + heads[None, :]) * block_size + off[:, None]


def kv_write_paged(k, v, kc, ks, vc, vs, slot_mapping, block_size, rotate_k=True):
    """``quantize_kv_write_paged`` (``engine/kv_cache.py:587-604,1095-1116``): K is Hadamard
    rotated (``hadamard128``, rounded to bf16), then K and V are quantized per (token, head)
    to int8 with an fp32 scale and scattered to their rows. k, v: [T, Hkv, D] bf16-valued.
    kc/vc: [num_blocks, Hkv, block_size, D] int8; ks/vs: [num_blocks, Hkv, block_size] fp32.
    Updated in place."""
    T, nkv, D = k.shape
    rows = flat_rows(slot_mapping, nkv, block_size).reshape(-1)
    kk = round_bf16(hadamard128(k)) if rotate_k else k
    kq, ksc = quant_sym(kk.reshape(-1, D), 127)
    vq, vsc = quant_sym(v.reshape(-1, D), 127)
    kc.reshape(-1, D)[rows] = kq.astype(np.int8)
    ks.reshape(-1)[rows] = ksc
    vc.reshape(-1, D)[rows] = vq.astype(np.int8)
    vs.reshape(-1)[rows] = vsc


def qkv_post(qkv, positions, nh, nkv, hd, q_norm_w, k_norm_w, eps, cos_tab, sin_tab):
    """Decode-branch head processing of ``GQAAttention.forward``
    (``superl8serve/layers/gqa_attention.py:65-74``): split [q | k | v], per-head RMSNorm
    on q and k before RoPE, RoPE at each row's position. Returns bf16-valued q, k, v
    [M, H, D]."""
    M = qkv.shape[0]
    q = qkv[:, : nh * hd].reshape(M, nh, hd)
    k = qkv[:, nh * hd : (nh + nkv) * hd].reshape(M, nkv, hd)
    v = qkv[:, (nh + nkv) * hd :].reshape(M, nkv, hd)
    q = rmsnorm(q, q_norm_w, eps)
    k = rmsnorm(k, k_norm_w, eps)
    pos = np.asarray(positions, dtype=np.int64)
    c = cos_tab[pos][:, None, :]
    s = sin_tab[pos][:, None, :]
    return rope(q, c, s), rope(k, c, s), v.astype(np.float32)


def quant_q_for_attn(q: np.ndarray):
    """Attention query prologue: rotate each head by the same orthonormal Hadamard as the
    stored K (so q_rot . k_rot = q . k), keep binary32, and quantize per (token, head) to
    int8. q [M, H, D] -> (codes int8 [M, H, D], scale fp32 [M, H])."""
    qr = hadamard128(q)
    qq, qs = quant_sym(qr, 127)
    return qq.astype(np.int8), qs


def lane_sum(e: np.ndarray) -> np.ndarray:
    """Denominator order of one partition: pad the (<= 256) values of each head to 256, lane
    l (0..31) sums e[l], e[32+l], ..., e[224+l] in that order, then the 32 lane sums are
    combined by the xor butterfly (offsets 16, 8, 4, 2, 1), all in binary32. e: [n, H] ->
    [H]."""
    n, H = e.shape
    pad = np.zeros((ATTN_PART, H), dtype=np.float32)
    pad[:n] = e
    lanes = pad.reshape(ATTN_PART // 32, 32, H)
    acc = lanes[0].copy()
    for i in range(1, ATTN_PART // 32):
        acc = (acc + lanes[i]).astype(np.float32)
    idx = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        acc = (acc + acc[idx ^ off]).astype(np.float32)
    return acc[0]


def paged_decode(qq, qs, kc, ks, vc, vs, block_table, context_lens, block_size, scale,
                 return_parts=False):
    """Paged int8 GQA decode attention (``attn_paged_decode_cached`` call site,
    ``superl8serve/engine/kv_cache.py:1190-1201``). Accumulation order is fixed:

    * score s_j = (f32(qq . kq_j) * (qs * scale)) * ks_j, the dot an exact int32;
    * the context is cut into partitions of ATTN_PART tokens; in partition p, per query head:
      m_p = max s_j, e_j = exp(s_j - m_p), l_p = sum e_j in the order of ``lane_sum``
      (binary32); the value weights w_j = e_j * vs_j are quantized relative to their
      maximum, W_j = clamp(rint(w_j * (32767 / wmax)), 0, 32767), the numerator is the exact
      integer o_int = sum_j W_j * vq_j and o_p = f32(o_int) * (wmax / 32767);
    * combine: M = max m_p, w_p = exp(m_p - M), L = sum w_p*l_p, O = sum w_p*o_p over p in
      order; out = bf16(O / L).
    The 15-bit weights keep every product exact (|o_int| < 2^31) so the numerator may be summed
    in any order; the weight rounding is at most 1.5e-5 of the partition's largest weight.

    qq [B, Hq, D] int8, qs [B, Hq]; caches as in ``kv_write_paged``; block_table
    [B, max_blocks] int32; context_lens [B] int32 (>= 1). Returns [B, Hq, D] bf16-valued.
    """
    B, Hq, D = qq.shape
    NB, Hkv, bs, _ = kc.shape
    G = Hq // Hkv
    out = np.zeros((B, Hq, D), dtype=np.float32)
    parts = []
    kc_f = kc.reshape(-1, D)
    vc_f = vc.reshape(-1, D)
    ks_f = ks.reshape(-1)
    vs_f = vs.reshape(-1)
    qsc = (qs.astype(np.float32) * F32(scale)).astype(np.float32)  # [B, Hq]
    for b in range(B):
        n = int(context_lens[b])
        j = np.arange(n)
        blk = np.asarray(block_table[b], dtype=np.int64)[j // block_size]
        off = j % block_size
        # rows[j, g]
        rows = (blk[:, None] * Hkv + np.arange(Hkv)[None, :]) * block_size + off[:, None]
        kq = kc_f[rows].astype(np.int64)  # [n, Hkv, D]
        vq = vc_f[rows].astype(np.float32)  # [n, Hkv, D]
        ksj = ks_f[rows]  # [n, Hkv]
        vsj = vs_f[rows]
        g_of_h = np.arange(Hq) // G
        dots = np.einsum("hd,nhd->nh", qq[b].astype(np.int64), kq[:, g_of_h, :])  # [n, Hq]
        s = (dots.astype(np.float32) * qsc[b][None, :]).astype(np.float32)
        s = (s * ksj[:, g_of_h]).astype(np.float32)
        vcodes = vq[:, g_of_h, :].astype(np.int64)  # [n, Hq, D]
        vsh = vsj[:, g_of_h]  # [n, Hq]
        nparts = (n + ATTN_PART - 1) // ATTN_PART
        ms, ls, os_ = [], [], []
        for p in range(nparts):
            lo, hi = p * ATTN_PART, min(n, (p + 1) * ATTN_PART)
            sp = s[lo:hi]
            m = sp.max(axis=0)
            e = exp_s8b((sp - m[None, :]).astype(np.float32))  # [np, Hq]
            l = lane_sum(e)
            w = (e * vsh[lo:hi]).astype(np.float32)
            wmax = w.max(axis=0)
            winv = (F32(32767.0) / wmax).astype(np.float32)
            qsc_p = (wmax / F32(32767.0)).astype(np.float32)
            W = np.clip(np.rint((w * winv[None, :]).astype(np.float32)), 0, 32767).astype(np.int64)
            o_int = np.einsum("nh,nhd->hd", W, vcodes[lo:hi])
            o = (o_int.astype(np.float32) * qsc_p[:, None]).astype(np.float32)
            ms.append(m)
            ls.append(l)
            os_.append(o)
        M = np.max(np.stack(ms), axis=0)
        L = np.zeros(Hq, dtype=np.float32)
        O = np.zeros((Hq, D), dtype=np.float32)
        for p in range(nparts):
            w = exp_s8b((ms[p] - M).astype(np.float32))
            L = (L + (w * ls[p]).astype(np.float32)).astype(np.float32)
            O = (O + (w[:, None] * os_[p]).astype(np.float32)).astype(np.float32)
        out[b] = round_bf16((O / L[:, None]).astype(np.float32))
        parts.append((ms, ls, os_))
    if return_parts:
        return out, parts
    return out


# ------------------------------------------------------------------------------ MLP ----

def silu_mul(gu: np.ndarray) -> np.ndarray:
    """``SiluAndMul`` (``superl8serve/layers/activation.py:20-26``) on the merged
    [gate | up] output: a = bf16(g / (1 + exp(-g))), y = bf16(a * u)."""
    F = gu.shape[-1] // 2
    g = gu[..., :F].astype(np.float32)
    u = gu[..., F:].astype(np.float32)
    den = (F32(1.0) + exp_s8b(-g)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        a = round_bf16((g / den).astype(np.float32))
    return round_bf16((a * u).astype(np.float32))


# ------------------------------------------------------------------------- sampling ----

def argmax_rows(logits: np.ndarray) -> np.ndarray:
    """Greedy sampler fast path (``superl8serve/layers/sampler.py:51-63``): argmax over
    the vocab, lowest index on ties."""
    return np.argmax(logits, axis=-1).astype(np.int32)


def embed(table: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """``VocabEmbedding.forward`` (``superl8serve/layers/embedding.py:60-69``): row gather."""
    return table[np.asarray(ids, dtype=np.int64)]
