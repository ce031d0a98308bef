"""Tensor-level wrappers over the s8b C ABI (CUDA tensors only; outputs allocated here when
not passed in). The stage runner passes preallocated buffers; tests and the reference-shaped
layer API use the allocating forms."""

from __future__ import annotations

import torch

from ._lib import CODEC, call, dtype_code, ptr, stream

__all__ = [
    "quant_rows", "rmsnorm_quant", "gemm_w8a8", "gemm_w8a8_tc", "gemm_tc_workspace",
    "silu_mul_quant", "qkv_post", "kv_write_paged",
    "paged_decode_q8", "paged_decode", "embed", "argmax", "codec_encode", "codec_decode",
    "codec_sizes", "decode_workspace_bytes", "moe_route", "moe_gemm_grouped", "moe_combine",
    "sample",
]


def quant_rows(x: torch.Tensor):
    x = x.contiguous()
    K = x.shape[-1]
    M = x.numel() // K
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    call("s8b_quant_rows", ptr(x), dtype_code(x.dtype), ptr(q), ptr(s), M, K, stream(x.device))
    return q, s


def rmsnorm_quant(h, residual, w, eps, *, residual_out=None, y_out=False, q=None, s=None):
    """Returns (new residual, q, s, y or None). residual None = first layer (no add)."""
    h = h.contiguous()
    H = h.shape[-1]
    M = h.numel() // H
    if residual_out is None:
        residual_out = torch.empty_like(h)
    q = torch.empty(h.shape, dtype=torch.int8, device=h.device) if q is None else q
    s = torch.empty(h.shape[:-1], dtype=torch.float32, device=h.device) if s is None else s
    y = torch.empty_like(h) if y_out else None
    call("s8b_rmsnorm_quant", ptr(h), ptr(residual), ptr(residual_out), ptr(w), float(eps),
         ptr(q), ptr(s), ptr(y), M, H, dtype_code(h.dtype), stream(h.device))
    return residual_out, q, s, y


def gemm_w8a8(xq, xs, w, ws, *, out=None, out_dtype=torch.bfloat16, raw=False):
    """y = dequant(xq @ w^T). raw=True returns the int32 accumulators."""
    K = xq.shape[-1]
    M = xq.numel() // K
    N = w.shape[0]
    if out is None:
        out = torch.empty((*xq.shape[:-1], N), dtype=torch.int32 if raw else out_dtype,
                          device=xq.device)
    dt = dtype_code(out_dtype if raw else out.dtype)
    call("s8b_gemm_w8a8", ptr(xq), ptr(xs), ptr(w), ptr(ws), ptr(out), 1 if raw else 0, M, N, K,
         dt, stream(xq.device))
    return out


def gemm_tc_workspace(M: int, N: int, device) -> torch.Tensor:
    """Zero-filled workspace for s8b_gemm_w8a8_tc (kept zero by every completed launch)."""
    from ._lib import load

    n = int(load().s8b_gemm_tc_workspace_size(M, N))
    return torch.zeros(n, dtype=torch.uint8, device=device)


def pack_weights_tc(w: torch.Tensor) -> torch.Tensor:
    """Pre-pack an int8 [N, K] weight into the tensor-core GEMM's unit images."""
    from ._lib import load

    N, K = w.shape
    packed = torch.empty(int(load().s8b_tc_packed_bytes(N, K)), dtype=torch.int8, device=w.device)
    call("s8b_pack_weights_tc", ptr(w.contiguous()), N, K, ptr(packed), stream(w.device))
    return packed


def gemm_w8a8_tc(xq, xs, w, ws, *, out=None, out_dtype=torch.bfloat16, raw=False, workspace=None,
                 packed: torch.Tensor | None = None):
    """Tensor-core (tcgen05 kind::i8) form of gemm_w8a8; identical results. With `packed`
    (from pack_weights_tc(w)) the weight stream is read as contiguous unit images."""
    K = xq.shape[-1]
    M = xq.numel() // K
    N = w.shape[0]
    if out is None:
        out = torch.empty((*xq.shape[:-1], N), dtype=torch.int32 if raw else out_dtype,
                          device=xq.device)
    if workspace is None:
        workspace = gemm_tc_workspace(M, N, xq.device)
    dt = dtype_code(out_dtype if raw else out.dtype)
    if packed is not None:
        call("s8b_gemm_w8a8_tc_packed", ptr(xq), ptr(xs), ptr(packed), ptr(ws), ptr(out),
             1 if raw else 0, M, N, K, dt, ptr(workspace), workspace.numel(), stream(xq.device))
    else:
        call("s8b_gemm_w8a8_tc", ptr(xq), ptr(xs), ptr(w), ptr(ws), ptr(out), 1 if raw else 0, M,
             N, K, dt, ptr(workspace), workspace.numel(), stream(xq.device))
    return out


def gemm_w8a8_tc_split(xq, xs, w, *, packed=None, workspace=None):
    """Tensor-core GEMM, split-K partials left unreduced (out_kind 2): returns int32
    [C, M, N] with sum over C = the int32 accumulators."""
    from ._lib import load

    K = xq.shape[-1]
    M = xq.numel() // K
    N = w.shape[0]
    C = int(load().s8b_gemm_tc_split_count(M, N, K))
    part = torch.empty((C, M, N), dtype=torch.int32, device=xq.device)
    if workspace is None:
        workspace = gemm_tc_workspace(M, N, xq.device)
    if packed is not None:
        call("s8b_gemm_w8a8_tc_packed", ptr(xq), ptr(xs), ptr(packed), None, ptr(part), 2, M, N, K,
             0, ptr(workspace), workspace.numel(), stream(xq.device))
    else:
        call("s8b_gemm_w8a8_tc", ptr(xq), ptr(xs), ptr(w), None, ptr(part), 2, M, N, K, 0,
             ptr(workspace), workspace.numel(), stream(xq.device))
    return part


def rmsnorm_quant_split(part, xs, ws, residual, w, eps, *, residual_out, dtype=torch.bfloat16):
    """rmsnorm_quant with h = dequant(sum of the GEMM partials part [C, M, H])."""
    C, M, H = part.shape
    q = torch.empty((M, H), dtype=torch.int8, device=part.device)
    s = torch.empty(M, dtype=torch.float32, device=part.device)
    call("s8b_rmsnorm_quant_split", ptr(part), C, ptr(xs), ptr(ws), ptr(residual),
         ptr(residual_out), ptr(w), float(eps), ptr(q), ptr(s), None, M, H, dtype_code(dtype),
         stream(part.device))
    return residual_out, q, s


def silu_mul_quant_split(part, xs, ws, *, dtype=torch.bfloat16):
    C, M, F2 = part.shape
    F = F2 // 2
    q = torch.empty((M, F), dtype=torch.int8, device=part.device)
    s = torch.empty(M, dtype=torch.float32, device=part.device)
    y = torch.empty((M, F), dtype=dtype, device=part.device)
    call("s8b_silu_mul_quant_split", ptr(part), C, ptr(xs), ptr(ws), M, F, ptr(y), ptr(q), ptr(s),
         dtype_code(dtype), stream(part.device))
    return q, s, y


def silu_mul_quant(gu, *, y_out=False, q=None, s=None):
    F = gu.shape[-1] // 2
    M = gu.numel() // (2 * F)
    shp = (*gu.shape[:-1], F)
    q = torch.empty(shp, dtype=torch.int8, device=gu.device) if q is None else q
    s = torch.empty(shp[:-1], dtype=torch.float32, device=gu.device) if s is None else s
    y = torch.empty(shp, dtype=gu.dtype, device=gu.device) if y_out else None
    call("s8b_silu_mul_quant", ptr(gu), M, F, ptr(y), ptr(q), ptr(s), dtype_code(gu.dtype),
         stream(gu.device))
    return q, s, y


def qkv_post(qkv, positions, cos, sin, q_norm_w, k_norm_w, eps, Hq, Hkv, kc, ks, vc, vs, *,
             slot_mapping=None, block_table=None, q_out=False, q_i8=None, q_s=None):
    """Returns (q_i8 [M,Hq,D], q_s [M,Hq], q_out or None); writes K/V into the paged stores."""
    M = qkv.shape[0]
    D = cos.shape[-1]
    dev = qkv.device
    q_i8 = torch.empty((M, Hq, D), dtype=torch.int8, device=dev) if q_i8 is None else q_i8
    q_s = torch.empty((M, Hq), dtype=torch.float32, device=dev) if q_s is None else q_s
    qo = torch.empty((M, Hq, D), dtype=qkv.dtype, device=dev) if q_out else None
    bs = kc.shape[-2]
    maxb = block_table.shape[-1] if block_table is not None else 0
    call("s8b_qkv_post", ptr(qkv), ptr(positions), ptr(cos), ptr(sin), cos.shape[0], ptr(q_norm_w),
         ptr(k_norm_w), float(eps), M, Hq, Hkv, D, ptr(q_i8), ptr(q_s), ptr(qo), ptr(kc), ptr(ks),
         ptr(vc), ptr(vs), ptr(slot_mapping), ptr(block_table), maxb, bs, dtype_code(qkv.dtype),
         stream(dev))
    return q_i8, q_s, qo


def qkv_post_split(part, xs, ws, positions, cos, sin, q_norm_w, k_norm_w, eps, Hq, Hkv, kc, ks,
                   vc, vs, *, block_table, dtype=torch.bfloat16):
    """qkv_post with the merged qkv rows given as GEMM split-K partials [C, M, (Hq+2Hkv)*D]."""
    C, M, _ = part.shape
    D = cos.shape[-1]
    dev = part.device
    q_i8 = torch.empty((M, Hq, D), dtype=torch.int8, device=dev)
    q_s = torch.empty((M, Hq), dtype=torch.float32, device=dev)
    call("s8b_qkv_post_split", ptr(part), C, ptr(xs), ptr(ws), ptr(positions), ptr(cos), ptr(sin),
         cos.shape[0], ptr(q_norm_w), ptr(k_norm_w), float(eps), M, Hq, Hkv, D, ptr(q_i8),
         ptr(q_s), None, ptr(kc), ptr(ks), ptr(vc), ptr(vs), None, ptr(block_table),
         block_table.shape[-1], kc.shape[-2], dtype_code(dtype), stream(dev))
    return q_i8, q_s


def kv_write_paged(k, v, kc, ks, vc, vs, slot_mapping, *, rotate_k=True):
    T, Hkv, D = k.shape
    call("s8b_kv_write_paged", ptr(k.contiguous()), ptr(v.contiguous()), ptr(kc), ptr(ks), ptr(vc),
         ptr(vs), ptr(slot_mapping), T, Hkv, D, kc.shape[-2], 1 if rotate_k else 0,
         dtype_code(k.dtype), stream(k.device))


def decode_workspace_bytes(B, Hq, D, max_ctx, *, ref=False) -> int:
    from ._lib import load

    fn = load().s8b_paged_decode_ref_workspace_size if ref else load().s8b_paged_decode_workspace_size
    return int(fn(B, Hq, D, max_ctx))


ATTENTION_IMPLS = {"auto": 0, "cuda_core": 1, "tc_partition": 2}


def set_attention_impl(impl: str) -> None:
    """"auto" (persistent tensor-core kernel where the shape allows, the default),
    "cuda_core" or "tc_partition"; results are bit-identical."""
    call("s8b_set_attention_impl", ATTENTION_IMPLS[impl])


def decode_status(workspace, B, Hq) -> int:
    """The workspace's status word (0, or the timeout code of a bounded tensor-core wait)."""
    from ._lib import load

    off = int(load().s8b_paged_decode_status_offset(B, Hq))
    return int(workspace[off:off + 4].view(torch.int32).item())


def paged_decode_q8(q_i8, q_s, kc, ks, vc, vs, block_table, context_lens, max_ctx, scale, *,
                    out=None, out_q=None, out_s=None, workspace=None, dtype=torch.bfloat16,
                    step=False):
    """``step``: the decode-step form (``s8b_paged_decode_q8_step``), for a call whose
    preceding kernel wrote only each row's newest K/V; same results."""
    B, Hq, D = q_i8.shape
    Hkv, bs = kc.shape[-3], kc.shape[-2]
    dev = q_i8.device
    out = torch.empty((B, Hq * D), dtype=dtype, device=dev) if out is None else out
    need = decode_workspace_bytes(B, Hq, D, max_ctx)
    if workspace is None:  # zero-filled once; the kernel leaves its counters at zero
        workspace = torch.zeros(need, dtype=torch.uint8, device=dev)
    call("s8b_paged_decode_q8_step" if step else "s8b_paged_decode_q8", ptr(q_i8), ptr(q_s),
         ptr(kc), ptr(ks), ptr(vc), ptr(vs),
         ptr(block_table), ptr(context_lens), ptr(out), ptr(out_q), ptr(out_s), B, Hq, Hkv, D, bs,
         block_table.shape[-1], int(max_ctx), float(scale), ptr(workspace), workspace.numel(),
         dtype_code(out.dtype), stream(dev))
    return out


def prefill_block_rows(Hq: int, Hkv: int) -> int:
    """Most rows one row block of ``paged_prefill_q8`` may hold at this head shape."""
    from ._lib import load

    return int(load().s8b_paged_prefill_block_rows(Hq, Hkv))


def prefill_row_blocks(seq_lens, block_rows: int) -> list[tuple[int, int]]:
    """Row blocks for rows packed sequence after sequence (``seq_lens`` rows each): runs of
    at most ``block_rows`` consecutive rows that never cross a sequence."""
    blocks, r0 = [], 0
    for n in seq_lens:
        for i in range(0, n, block_rows):
            blocks.append((r0 + i, min(block_rows, n - i)))
        r0 += n
    return blocks


def paged_prefill_q8(q_i8, q_s, kc, ks, vc, vs, block_table, context_lens, row_blocks,
                     max_ctx, scale, *, out=None, out_q=None, out_s=None, workspace=None,
                     dtype=torch.bfloat16):
    """``paged_decode_q8`` over prefill rows grouped into ``row_blocks`` (int32 [n, 2] device
    tensor of (first row, row count), rows of one sequence each); identical results, each
    block's K/V partitions read once for all its rows."""
    B, Hq, D = q_i8.shape
    Hkv, bs = kc.shape[-3], kc.shape[-2]
    dev = q_i8.device
    out = torch.empty((B, Hq * D), dtype=dtype, device=dev) if out is None else out
    need = decode_workspace_bytes(B, Hq, D, max_ctx)
    if workspace is None:
        workspace = torch.zeros(need, dtype=torch.uint8, device=dev)
    call("s8b_paged_prefill_q8", ptr(q_i8), ptr(q_s), ptr(kc), ptr(ks), ptr(vc), ptr(vs),
         ptr(block_table), ptr(context_lens), ptr(row_blocks), row_blocks.shape[0], ptr(out),
         ptr(out_q), ptr(out_s), B, Hq, Hkv, D, bs, block_table.shape[-1], int(max_ctx),
         float(scale), ptr(workspace), workspace.numel(), dtype_code(out.dtype), stream(dev))
    return out


def paged_decode(q, kc, ks, vc, vs, block_table, context_lens, max_ctx, scale, *, out=None,
                 workspace=None):
    """Reference layout: q [B, Hq, D] (or [B, Hq, 1, D]) -> [B, Hq, D]."""
    qq = q.reshape(q.shape[0], q.shape[1], q.shape[-1]).contiguous()
    B, Hq, D = qq.shape
    Hkv, bs = kc.shape[-3], kc.shape[-2]
    out = torch.empty_like(qq) if out is None else out
    need = decode_workspace_bytes(B, Hq, D, max_ctx, ref=True)
    if workspace is None:  # zero-filled once; the kernel leaves its counters at zero
        workspace = torch.zeros(need, dtype=torch.uint8, device=q.device)
    call("s8b_paged_decode", ptr(qq), ptr(kc), ptr(ks), ptr(vc), ptr(vs), ptr(block_table),
         ptr(context_lens), ptr(out), B, Hq, Hkv, D, bs, block_table.shape[-1], int(max_ctx),
         float(scale), ptr(workspace), workspace.numel(), dtype_code(qq.dtype), stream(q.device))
    return out


def embed(ids, table, *, out=None):
    M = ids.numel()
    H = table.shape[-1]
    out = torch.empty((M, H), dtype=table.dtype, device=table.device) if out is None else out
    call("s8b_embed", ptr(ids), ptr(table), M, H, ptr(out), dtype_code(table.dtype),
         stream(table.device))
    return out


def argmax(logits, *, out=None):
    V = logits.shape[-1]
    M = logits.numel() // V
    out = torch.empty(M, dtype=torch.int32, device=logits.device) if out is None else out
    call("s8b_argmax", ptr(logits), M, V, ptr(out), dtype_code(logits.dtype), stream(logits.device))
    return out


def exp_s8b(x):
    """The library's binary32 exponential, elementwise (fp32 CUDA tensor in, same shape out)."""
    if x.dtype != torch.float32 or not x.is_cuda:
        raise RuntimeError("exp_s8b: fp32 CUDA tensor required")
    x = x.contiguous()
    y = torch.empty_like(x)
    call("s8b_exp_f32", ptr(x), ptr(y), x.numel(), stream(x.device))
    return y


def codec_sizes(T: int, D: int, scheme: str) -> tuple[int, int]:
    """(payload bytes, fp32 scale count) of one encoded [T, D] block."""
    from ._lib import load

    sc = CODEC[scheme]
    return int(load().s8b_codec_payload_bytes(T, D, sc, 0)), int(load().s8b_codec_scale_count(T, D, sc))


def codec_encode(a, b, scheme, *, payload=None, scales=None, dtype=None):
    """Encode rows [a | b] (b may be None). payload/scales may live on another GPU."""
    T, Da = a.shape[0], a.shape[-1]
    Db = 0 if b is None else b.shape[-1]
    nbytes, nsc = codec_sizes(T, Da + Db, scheme)
    if payload is None:
        payload = torch.empty(nbytes, dtype=torch.uint8, device=a.device)
    if scales is None:
        scales = torch.empty(max(nsc, 1), dtype=torch.float32, device=a.device)
    call("s8b_codec_encode", ptr(a.contiguous()), ptr(None if b is None else b.contiguous()), T, Da,
         Db, CODEC[scheme], payload.data_ptr(), scales.data_ptr(), dtype_code(a.dtype),
         stream(a.device))
    return payload, scales


def codec_decode(payload, scales, T, Da, Db, scheme, dtype, *, out_a=None, out_b=None):
    dev = payload.device
    out_a = torch.empty((T, Da), dtype=dtype, device=dev) if out_a is None else out_a
    if Db:
        out_b = torch.empty((T, Db), dtype=dtype, device=dev) if out_b is None else out_b
    call("s8b_codec_decode", ptr(payload), ptr(scales), T, Da, Db, CODEC[scheme], ptr(out_a),
         ptr(out_b) if Db else None, dtype_code(dtype), stream(dev))
    return out_a, out_b


# ------------------------------------------------------------------------- sparse MoE ----
def moe_route(y, gate, top_k: int, *, norm_topk_prob: bool = True, scaling: float = 1.0):
    """Router + grouping (``s8b_moe_route``). Returns a dict of device tensors: topi, topw,
    offsets [E+1], sorted_assign, sorted_token, assign_pos."""
    T, H = y.shape
    E = gate.shape[0]
    dev = y.device
    i32 = lambda n: torch.empty(n, dtype=torch.int32, device=dev)  # noqa: E731
    r = {"topi": i32(T * top_k).view(T, top_k),
         "topw": torch.empty(T, top_k, dtype=y.dtype, device=dev),
         "offsets": i32(E + 1), "sorted_assign": i32(T * top_k),
         "sorted_token": i32(T * top_k), "assign_pos": i32(T * top_k)}
    call("s8b_moe_route", ptr(y), dtype_code(y.dtype), ptr(gate), T, H, E, top_k, int(norm_topk_prob),
         scaling, ptr(r["topi"]), ptr(r["topw"]), ptr(r["offsets"]), ptr(r["sorted_assign"]),
         ptr(r["sorted_token"]), ptr(r["assign_pos"]), stream(dev))
    return r


def moe_gemm_grouped(xq, xs, w, ws, offsets, *, row_index=None, A: int, out_dtype=torch.bfloat16):
    """y [A, N] = grouped W8A8 over expert row groups (``s8b_moe_gemm_grouped``)."""
    E, N, K = w.shape
    y = torch.empty(A, N, dtype=out_dtype, device=xq.device)
    call("s8b_moe_gemm_grouped", ptr(xq), ptr(xs), None if row_index is None else ptr(row_index),
         ptr(w), ptr(ws), ptr(offsets), ptr(y), A, N, K, E, dtype_code(y.dtype),
         stream(xq.device))
    return y


def moe_gather_rows(xq, xs, index, A: int):
    """Rows in assignment order: (xq[index], xs[index]) (``s8b_moe_gather_rows``)."""
    K = xq.shape[-1]
    xg = torch.empty(A, K, dtype=torch.int8, device=xq.device)
    xgs = torch.empty(A, dtype=torch.float32, device=xq.device)
    call("s8b_moe_gather_rows", ptr(xq), ptr(xs), ptr(index), A, K, ptr(xg), ptr(xgs),
         stream(xq.device))
    return xg, xgs


def moe_gemm_grouped_tc(xg, xgs, w, ws, offsets, *, A: int, max_rows: int, status=None,
                        out_dtype=torch.bfloat16):
    """The tensor-core grouped GEMM on gathered rows (``s8b_moe_gemm_grouped_tc``)."""
    E, N, K = w.shape
    y = torch.empty(A, N, dtype=out_dtype, device=xg.device)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=xg.device)
    call("s8b_moe_gemm_grouped_tc", ptr(xg), ptr(xgs), ptr(w), ptr(ws), ptr(offsets), ptr(y), A,
         N, K, E, int(max_rows), ptr(status), dtype_code(y.dtype), stream(xg.device))
    return y


def moe_combine(contrib, topw, topi, assign_pos):
    T, k = topi.shape
    H = contrib.shape[1]
    out = torch.empty(T, H, dtype=contrib.dtype, device=contrib.device)
    call("s8b_moe_combine", ptr(contrib), ptr(topw), ptr(topi), ptr(assign_pos), ptr(out), T, k,
         H, dtype_code(out.dtype), stream(out.device))
    return out


# ---------------------------------------------------------------------------- sampler ----
def sample(logits, temperature, *, top_k=None, top_p=None, penalty=None, input_ids, positions,
           history, seeds, out=None, workspace=None):
    """Next tokens [M] int32 (``s8b_sample``). history: int32 [M, cap], updated in place at
    each row's position with its input id."""
    M, V = logits.shape
    dev = logits.device
    if workspace is None:
        from ._lib import load

        workspace = torch.empty(int(load().s8b_sample_workspace_size(M, V)), dtype=torch.uint8,
                                device=dev)
    out = torch.empty(M, dtype=torch.int32, device=dev) if out is None else out
    call("s8b_sample", ptr(logits), dtype_code(logits.dtype), M, V, ptr(temperature), ptr(top_k),
         ptr(top_p), ptr(penalty), ptr(input_ids), ptr(positions), ptr(history),
         history.shape[1], ptr(seeds), ptr(workspace), workspace.numel(), ptr(out), stream(dev))
    return out
