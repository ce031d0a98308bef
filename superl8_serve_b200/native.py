"""ctypes mirrors of ``S8bLayerDesc`` / ``S8bStageDesc`` (``include/s8b.h``) and the builder
that fills them from a ``runtime.StageRunner``: with ``StageRunner.native`` set, a stage step is
one ``s8b_stage_step`` call (the C++ replay of the Python launch sequence) instead of one
ctypes call per kernel."""

from __future__ import annotations

import ctypes as C

_p, _i, _f, _sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t


class LayerDesc(C.Structure):
    _fields_ = [(n, _p) for n in ("qkv_w", "qkv_packed", "qkv_s", "o_w", "o_packed", "o_s",
                                  "gu_w", "gu_packed", "gu_s", "d_w", "d_packed", "d_s",
                                  "in_norm", "post_norm", "q_norm", "k_norm",
                                  "kc", "ks", "vc", "vs")] + [
        ("moe_experts", _i), ("moe_top_k", _i), ("moe_ffn", _i), ("moe_norm_topk", _i),
        ("moe_scaling", _f), ("router", _p), ("moe_gu_w", _p), ("moe_gu_s", _p),
        ("moe_d_w", _p), ("moe_d_s", _p)]


class StageDesc(C.Structure):
    _fields_ = [(n, _i) for n in ("n_layers", "M", "H", "Hq", "Hkv", "D", "F", "V",
                                  "block_size", "max_blocks", "max_ctx", "rope_len", "dtype",
                                  "tc_min", "first_model_layer", "head")] + [
        ("eps", _f), ("scale", _f), ("layers", _p), ("cos_tab", _p), ("sin_tab", _p),
        ("embed", _p), ("final_norm", _p), ("head_w", _p), ("head_packed", _p), ("head_s", _p),
        ("ids", _p), ("positions", _p), ("context_lens", _p), ("block_table", _p),
        ("in_payload", _p), ("in_scales", _p), ("out_payload", _p), ("out_scales", _p),
        ("scheme", _i),
        ("h", _p), ("res", _p), ("qkv", _p), ("attn", _p), ("gu", _p), ("logits", _p),
        ("xq", _p), ("xs", _p), ("q_i8", _p), ("q_s", _p), ("part", _p),
        ("attn_ws", _p), ("attn_ws_bytes", _sz), ("tc_ws", _p), ("tc_ws_bytes", _sz),
        ("moe_y", _p), ("moe_topw", _p), ("moe_gu", _p), ("moe_contrib", _p), ("moe_aq", _p),
        ("moe_as", _p), ("moe_topi", _p), ("moe_offsets", _p), ("moe_sorted_assign", _p),
        ("moe_sorted_token", _p), ("moe_assign_pos", _p),
        ("temperature", _p), ("top_p", _p), ("penalty", _p), ("top_k", _p),
        ("input_ids", _p), ("history", _p), ("history_cap", _i), ("seeds", _p),
        ("sample_ws", _p), ("sample_ws_bytes", _sz)]


def _a(t):
    return None if t is None else t.data_ptr()


def layer_descs(runner) -> C.Array:
    """The runner's layers as an ``S8bLayerDesc`` array (weights and KV pools do not move)."""
    arr = (LayerDesc * max(1, len(runner.model.layers)))()
    for li, L in enumerate(runner.model.layers):
        d = arr[li]
        pk = lambda w: (None if w is None or id(w) not in runner.packed  # noqa: E731
                        else _a(runner.packed[id(w)][1]))
        d.qkv_w, d.qkv_packed, d.qkv_s = _a(L.qkv_w), pk(L.qkv_w), _a(L.qkv_s)
        d.o_w, d.o_packed, d.o_s = _a(L.o_w), pk(L.o_w), _a(L.o_s)
        d.gu_w, d.gu_packed, d.gu_s = _a(L.gu_w), pk(L.gu_w), _a(L.gu_s)
        d.d_w, d.d_packed, d.d_s = _a(L.d_w), pk(L.d_w), _a(L.d_s)
        d.in_norm, d.post_norm = _a(L.in_norm), _a(L.post_norm)
        d.q_norm, d.k_norm = _a(L.q_norm), _a(L.k_norm)
        d.kc, d.ks, d.vc, d.vs = (_a(t) for t in runner.pool.layer(li))
        mw = L.moe
        if mw is not None:
            if mw.shards:
                raise NotImplementedError("s8b_stage_step keeps every expert on the stage's GPU")
            d.moe_experts, d.moe_top_k, d.moe_ffn = mw.num_experts, mw.top_k, mw.ffn
            d.moe_norm_topk, d.moe_scaling = int(mw.norm_topk_prob), mw.scaling
            d.router, d.moe_gu_w, d.moe_gu_s = _a(mw.router), _a(mw.gu_w), _a(mw.gu_s)
            d.moe_d_w, d.moe_d_s = _a(mw.d_w), _a(mw.d_s)
    return arr


def stage_desc(runner, mb, M, boundary_in, boundary_out, head) -> StageDesc:
    from ._lib import CODEC, dtype_code

    r, m = runner, runner.model
    d = StageDesc()
    if getattr(r, "_layer_descs", None) is None:
        r._layer_descs = layer_descs(r)
    d.n_layers, d.M, d.H, d.Hq, d.Hkv, d.D = len(m.layers), M, r.H, r.Hq, r.Hkv, r.D
    d.F, d.V = r.F, r.V
    d.block_size, d.max_blocks = r.pool.block_size, mb.block_table.shape[1]
    d.max_ctx, d.rope_len, d.dtype = r.max_ctx, r.cos.shape[0], dtype_code(r.dtype)
    d.tc_min = r.tc_min if r.tc_ws is not None else 0
    d.first_model_layer, d.head = int(m.start == 0), int(head)
    d.eps, d.scale = r.eps, r.scale
    d.layers = C.cast(r._layer_descs, _p)
    d.cos_tab, d.sin_tab = _a(r.cos), _a(r.sin)
    d.embed = _a(m.embed)
    d.final_norm, d.head_w, d.head_s = _a(m.norm), _a(m.head_w), _a(m.head_s)
    d.head_packed = (_a(r.packed[id(m.head_w)][1])
                     if m.head_w is not None and id(m.head_w) in r.packed else None)
    d.ids, d.positions, d.context_lens = _a(mb.ids), _a(mb.positions), _a(mb.context_lens)
    d.block_table = _a(mb.block_table)
    scheme = None
    if boundary_in is not None:
        pay, sc, scheme = boundary_in
        d.in_payload, d.in_scales = pay.data_ptr(), sc.data_ptr()
    if boundary_out is not None:
        pay, sc, scheme = boundary_out
        d.out_payload, d.out_scales = pay.data_ptr(), sc.data_ptr()
    d.scheme = CODEC[scheme] if scheme is not None else 0
    d.h, d.res, d.qkv, d.attn, d.gu = _a(r.h), _a(r.res), _a(r.qkv), _a(r.attn), _a(r.gu)
    d.logits = _a(getattr(r, "logits", None))
    d.xq, d.xs, d.q_i8, d.q_s, d.part = _a(r.xq), _a(r.xs), _a(r.q_i8), _a(r.q_s), _a(r.part)
    d.attn_ws, d.attn_ws_bytes = _a(r.ws), r.ws.numel()
    if r.tc_ws is not None:
        d.tc_ws, d.tc_ws_bytes = _a(r.tc_ws), r.tc_ws.numel()
    b = r.moe_buf
    if b is not None:
        d.moe_y, d.moe_topw, d.moe_gu, d.moe_contrib = _a(b["y"]), _a(b["topw"]), _a(b["gu"]), _a(b["contrib"])
        d.moe_aq, d.moe_as, d.moe_topi = _a(b["aq"]), _a(b["as"]), _a(b["topi"])
        d.moe_offsets, d.moe_sorted_assign = _a(b["offsets"]), _a(b["sorted_assign"])
        d.moe_sorted_token, d.moe_assign_pos = _a(b["sorted_token"]), _a(b["assign_pos"])
    smp = mb.extra.get("sampling") if m.is_last else None
    if smp is not None:
        d.temperature, d.top_p, d.penalty = _a(smp["temperature"]), _a(smp["top_p"]), _a(smp["penalty"])
        d.top_k, d.input_ids, d.history = _a(smp["top_k"]), _a(smp["input_ids"]), _a(smp["history"])
        d.history_cap, d.seeds = smp["history"].shape[1], _a(smp["seeds"])
        d.sample_ws, d.sample_ws_bytes = _a(smp["workspace"]), smp["workspace"].numel()
    return d
