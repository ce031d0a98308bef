"""Generate golden fixtures by running the superl8-serve reference's own Python code.

Run in a container where the reference checkout is available:

    S8B_REFERENCE=/path/to/superl8-serve python tests/golden/make_golden.py

The reference cannot be imported as shipped: its package ``__init__`` insists on a
torch+cu129 build and every module imports the un-vendored ``superl8`` kernel package.
This script therefore

* registers bare package objects for ``superl8serve`` and its sub-packages (so their
  ``__init__`` files, which pull in unrelated model families, are not executed), and
* installs a stand-in ``superl8`` module whose kernels are the oracle restatements in
  ``oracle/`` (the only definition of those kernels this build has).

Everything else runs as the reference wrote it: ``Qwen3ForCausalLM`` / ``Qwen3DecoderLayer``
/ ``GQAAttention`` / ``LinearW8A8`` / ``PagedKVCache`` / ``make_pipeline`` stage slicing /
``_pack_boundary`` / ``peer_routes`` / ``TransferHandle`` / ``accuracy_report`` and the
reference's eager RMSNorm / RoPE / SwiGLU / Sampler. The fixtures therefore pin how the
reference composes the kernels (layer order, residual threading, head split, cache row
layout, stage bounds, boundary packing, route policy), which the oracle's own model driver
and the CUDA path are then tested against. Outputs go next to this script.
"""

from __future__ import annotations

import dataclasses
import importlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import codec as ocodec  # noqa: E402
from oracle import kernels as ok  # noqa: E402
from oracle import numerics as on  # noqa: E402


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _bf16(a: np.ndarray, like: torch.Tensor | None = None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return t.to(like.dtype if like is not None else torch.bfloat16)


# ------------------------------------------------------------- stand-in `superl8` ----

def make_superl8_stub() -> types.ModuleType:
    sl8 = types.ModuleType("superl8")

    @dataclasses.dataclass
    class QTensor:
        data: torch.Tensor
        scale: torch.Tensor | None
        scheme: str = "per_row_i8"
        group_size: int | None = None
        codebook: str | None = None

    @dataclasses.dataclass
    class Compressed:
        scheme: str
        shape: tuple
        dtype: torch.dtype
        group_size: int | None
        payload: torch.Tensor
        scales: torch.Tensor
        d: int

    def linear(x, qt, bias=None, out_dtype=None):
        shp = x.shape
        y = ok.linear_w8a8(_np(x).reshape(-1, shp[-1]), qt.data.numpy(), qt.scale.numpy())
        return _bf16(y).to(out_dtype or x.dtype).reshape(*shp[:-1], -1)

    def rmsnorm(x, weight, eps, residual=None, unit_offset=False):
        assert not unit_offset
        shp = x.shape
        xf = _np(x).reshape(-1, shp[-1])
        rf = None if residual is None else _np(residual).reshape(-1, shp[-1])
        s, _, _, y = ok.rmsnorm_quant(xf, rf, _np(weight), eps)
        y = _bf16(y).to(x.dtype).reshape(shp)
        if residual is None:
            return y
        return y, _bf16(s).to(x.dtype).reshape(shp)

    def rope(positions, q, k, cos, sin, rotary_dim):
        assert rotary_dim == q.shape[-1]
        pos = positions.reshape(-1).long()
        c = _np(cos)[pos.numpy()]
        s = _np(sin)[pos.numpy()]
        B = pos.numel()

        def app(x):
            xf = _np(x).reshape(B, -1, x.shape[-2], x.shape[-1])
            return _bf16(ok.rope(xf, c[:, None, None, :], s[:, None, None, :])).to(x.dtype).reshape(x.shape)

        return app(q), app(k)

    def act_and_mul(x, kind):
        assert kind == "silu"
        return _bf16(ok.silu_mul(_np(x))).to(x.dtype)

    def quantize_kv_write_paged(k, v, kc, ks, vc, vs, slot_mapping):
        kcn, ksn, vcn, vsn = kc.numpy(), ks.numpy(), vc.numpy(), vs.numpy()
        ok.kv_write_paged(_np(k), _np(v), kcn, ksn, vcn, vsn, slot_mapping.numpy(),
                          kc.shape[2], rotate_k=True)

    def attn_paged_decode_cached(q, kc, ks, vc, vs, block_table, context_lens, block_size,
                                 max_context_len=None, scale=None):
        B, H, S, D = q.shape
        assert S == 1
        qq, qs = ok.quant_q_for_attn(_np(q)[:, :, 0, :])
        out = ok.paged_decode(qq, qs, kc.numpy(), ks.numpy(), vc.numpy(), vs.numpy(),
                              block_table.numpy(), context_lens.numpy(), block_size, scale)
        return _bf16(out).to(q.dtype).reshape(B, H, 1, D)

    def quantize_int8_rowwise(w):
        q, s = on.quantize_weight_rowwise(_np(w))
        return torch.from_numpy(q), torch.from_numpy(s).unsqueeze(-1)

    def compress_activation(x, scheme="int8", group_size=None):
        d = x.shape[-1]
        pay, sc = ocodec.encode(_np(x), scheme)
        return Compressed(scheme, tuple(x.shape), x.dtype, group_size,
                          torch.from_numpy(np.ascontiguousarray(pay)), torch.from_numpy(sc), d)

    def decompress_activation(c):
        rec = ocodec.decode(c.payload.numpy(), c.scales.numpy(), c.scheme, c.d)
        return _bf16(rec).to(c.dtype).reshape(c.shape)

    def hadamard_matrix(d, device="cpu", dtype=torch.float32):
        i = torch.arange(d)
        pc = torch.zeros(d, d, dtype=torch.int64)
        a = i[:, None] & i[None, :]
        while bool(a.any()):
            pc += a & 1
            a = a >> 1
        return ((1 - 2 * (pc % 2)).to(dtype) / d ** 0.5).to(device)

    def rotate_last(x):
        return _bf16(on.hadamard128(_np(x))).to(x.dtype)

    for f in (linear, rmsnorm, rope, act_and_mul, quantize_kv_write_paged,
              attn_paged_decode_cached, compress_activation, decompress_activation):
        setattr(sl8, f.__name__, f)
    sl8.QTensor = QTensor
    sl8.Compressed = Compressed
    quant = types.ModuleType("superl8.quant")
    rot = types.ModuleType("superl8.quant.rotation")
    rot.rotate_last = rotate_last
    rot.hadamard_matrix = hadamard_matrix
    core = types.ModuleType("superl8.quant.core")
    core.quantize_int8_rowwise = quantize_int8_rowwise
    lowbit = types.ModuleType("superl8.quant.lowbit")
    quant.rotation, quant.core, quant.lowbit = rot, core, lowbit
    sl8.quant = quant
    sys.modules.update({"superl8": sl8, "superl8.quant": quant, "superl8.quant.rotation": rot,
                        "superl8.quant.core": core, "superl8.quant.lowbit": lowbit})
    return sl8


def import_reference(ref_root: Path):
    make_superl8_stub()
    base = ref_root / "superl8serve"
    for name, sub in (("superl8serve", ""), ("superl8serve.layers", "layers"),
                      ("superl8serve.models", "models"), ("superl8serve.engine", "engine"),
                      ("superl8serve.dist", None)):
        if sub is None:
            continue
        m = types.ModuleType(name)
        m.__path__ = [str(base / sub) if sub else str(base)]
        sys.modules[name] = m
    import importlib

    mods = {}
    for n in ("layers.linear", "layers.norm", "layers.rotary", "layers.activation",
              "layers.embedding", "layers.sampler", "layers.gqa_attention", "models.config",
              "models.base", "models.qwen3", "models.weights", "engine.kv_cache"):
        mods[n] = importlib.import_module(f"superl8serve.{n}")
    # dist/__init__ holds send/recv/TransferHandle/accuracy_report; import it as a module.
    spec = importlib.util.spec_from_file_location(
        "superl8serve.dist", base / "dist" / "__init__.py",
        submodule_search_locations=[str(base / "dist")])
    dist = importlib.util.module_from_spec(spec)
    sys.modules["superl8serve.dist"] = dist
    spec.loader.exec_module(dist)
    mods["dist"] = dist
    mods["dist.peer_routes"] = importlib.import_module("superl8serve.dist.peer_routes")
    mods["dist.pipeline"] = importlib.import_module("superl8serve.dist.pipeline")
    return mods


def force_kernel_paths(mods):
    """Route the reference layers to the `superl8` kernels on CPU tensors (their CUDA
    branch), which is where the stand-in kernels live."""
    sl8 = sys.modules["superl8"]
    mods["layers.linear"].LinearW8A8._dp4a_ok = lambda self, x: True
    norm = mods["layers.norm"].RMSNorm
    norm.forward = lambda self, x, residual=None: sl8.rmsnorm(
        x, self.weight, self.eps, residual=residual, unit_offset=self.add_unit_offset)
    rot = mods["layers.rotary"].RotaryEmbedding
    rot.forward = lambda self, positions, q, k: sl8.rope(positions, q, k, self.cos, self.sin,
                                                          self.rotary_dim)
    act = mods["layers.activation"].SiluAndMul
    act.forward = lambda self, x: sl8.act_and_mul(x, "silu")


# ------------------------------------------------------------------------ fixtures ----

def tiny_cfg_ref(mods, moe: bool = False, **kw):
    from superl8_serve_b200.config import tiny, tiny_moe

    c = (tiny_moe if moe else tiny)(**kw)
    MC = mods["models.config"].ModelConfig
    extra = {}
    if moe:
        extra = dict(num_experts=c.num_experts, num_experts_per_tok=c.num_experts_per_tok,
                     moe_intermediate_size=c.moe_intermediate_size,
                     norm_topk_prob=c.norm_topk_prob)
    return c, MC(arch="qwen3", **extra, vocab_size=c.vocab_size, hidden_size=c.hidden_size,
                 num_hidden_layers=c.num_hidden_layers,
                 num_attention_heads=c.num_attention_heads,
                 num_key_value_heads=c.num_key_value_heads,
                 intermediate_size=c.intermediate_size,
                 max_position_embeddings=c.max_position_embeddings, head_dim=c.head_dim,
                 qk_norm=True, tie_word_embeddings=c.tie_word_embeddings,
                 rms_norm_eps=c.rms_norm_eps, rope_theta=c.rope_theta,
                 torch_dtype="bfloat16")


def gen_model_golden(mods, out: dict, n_stages: int, scheme: str, seed: int, tag: str,
                     moe: bool = False):
    """Greedy decode through the reference module graph, stage-sliced like make_pipeline.
    ``moe``: the tiny Qwen3-MoE shape (every layer's MLP is the reference ``SparseMoE``)."""
    from superl8_serve_b200.weights import random_state_dict

    pipe = mods["dist.pipeline"]
    kvm = mods["engine.kv_cache"]
    base = mods["models.base"]
    cfg, rcfg = tiny_cfg_ref(mods, moe=moe)
    sd = {k: torch.from_numpy(v).to(torch.bfloat16) for k, v in random_state_dict(cfg, seed, w_std=0.1).items()}

    pipe._move_stage_groups = lambda groups, devices: None
    pipe._build_stage_cache = lambda n, slots, nkv, max_len, hd, *, device, block_size=16, \
        num_blocks=None: kvm.PagedKVCache(n, slots, nkv, max_len, hd, device="cpu",
                                           block_size=block_size, num_blocks=num_blocks)
    if n_stages == 1:
        model = mods["models.qwen3"].Qwen3ForCausalLM(rcfg, dict(sd))
        stages = [types.SimpleNamespace(embed=model.model.embed_tokens, layers=model.model.layers,
                                        norm=model.model.norm, lm_head=model.lm_head,
                                        layer_offset=0, is_first=True, is_last=True,
                                        kv_cache=kvm.PagedKVCache(cfg.num_hidden_layers, 4,
                                                                  cfg.num_key_value_heads, 64,
                                                                  128, device="cpu"))]
    else:
        stages = list(pipe.make_pipeline(rcfg, dict(sd), devices=tuple(range(n_stages)),
                                         max_num_seqs=4, max_len=64))
    prompts = [[3, 1, 4, 1, 5], [9, 2, 6], [5, 3, 5, 8, 9, 7, 9]]
    max_new = 8
    slots = [stages[0].kv_cache.alloc() for _ in prompts]
    for st in stages[1:]:
        for _ in prompts:
            st.kv_cache.alloc()
    seqs = [list(p) for p in prompts]
    outs = [[] for _ in prompts]
    logits_log = [[] for _ in prompts]
    step = 0
    H = cfg.hidden_size
    while any(len(o) < max_new for o in outs):
        positions = torch.tensor([[step]] * len(prompts))
        lengths = [step] * len(prompts)
        hidden = residual = None
        for st in stages:
            st.kv_cache.ensure_capacity(slots, [n + 1 for n in lengths])
            ctx = base.ForwardContext(is_prefill=False, kv_cache=st.kv_cache, slots=slots,
                                      slot_lengths=lengths)
            if st.embed is not None and st.layer_offset == 0:
                ids = torch.tensor([[sq[step]] for sq in seqs])
                hidden = st.embed(ids)
            rc = pipe.LayerRemappedCache(st.kv_cache, st.layer_offset)
            sctx = pipe._remap_ctx(ctx, rc)
            for layer in st.layers:
                hidden, residual = layer(hidden, positions, sctx, residual)
            if st.lm_head is None:
                packed = pipe._pack_boundary(hidden.contiguous(), residual)
                sl8 = sys.modules["superl8"]
                c = sl8.compress_activation(packed, scheme=scheme)
                hidden, residual = pipe._unpack_boundary(sl8.decompress_activation(c), H)
        last = stages[-1]
        h, _ = last.norm(hidden, residual)
        logits = last.lm_head(h[:, -1])
        toks = mods["layers.sampler"].Sampler()(logits, torch.zeros(len(prompts)),
                                                  all_greedy=True)
        for i, sq in enumerate(seqs):
            if step >= len(prompts[i]) - 1 and len(outs[i]) < max_new:
                outs[i].append(int(toks[i]))
                logits_log[i].append(_np(logits[i]))
            if step + 1 >= len(sq):
                sq.append(int(toks[i]))
        step += 1
    out[f"{tag}_tokens"] = np.array(outs, dtype=np.int32)
    out[f"{tag}_logits"] = np.array(logits_log, dtype=np.float32)
    out[f"{tag}_bounds"] = np.array([st.layer_offset for st in stages] + [cfg.num_hidden_layers])


def gen_moe_module_golden(mods, out: dict):
    """The reference ``SparseMoE.forward`` (``superl8serve/models/moe.py:88-141``) on random
    bf16 rows: its output and the router's top-k choice and weights, recorded by wrapping
    ``torch.topk`` for the duration of the call (the wrapper returns torch's own result)."""
    from superl8_serve_b200.weights import random_tensor

    moe_mod = importlib.import_module("superl8serve.models.moe")
    weights = mods["models.weights"]
    T, H, E, Fe, k = 24, 256, 16, 128, 4
    g = torch.Generator().manual_seed(21)
    x = (torch.randn(T, H, generator=g) * 1.5).to(torch.bfloat16)
    gate = torch.from_numpy(random_tensor(21, "gate", (E, H), "w", 0.1)).to(torch.bfloat16)
    raw = {}
    experts = []
    for e in range(E):
        gp = random_tensor(21, f"e{e}.gate", (Fe, H), "w", 0.1)
        up = random_tensor(21, f"e{e}.up", (Fe, H), "w", 0.1)
        dn = random_tensor(21, f"e{e}.down", (H, Fe), "w", 0.1)
        raw[f"moe_e{e}_gate"], raw[f"moe_e{e}_up"], raw[f"moe_e{e}_down"] = gp, up, dn
        t = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
        experts.append((weights.merge_qtensor([t(gp), t(up)]), weights.to_qtensor(t(dn))))
    m = moe_mod.SparseMoE(gate=gate, experts=experts, top_k=k, norm_topk_prob=True)
    seen = []
    real_topk = torch.topk

    def rec_topk(*a, **kw):
        r = real_topk(*a, **kw)
        seen.append((r[0].detach().clone(), r[1].detach().clone()))
        return r

    torch.topk = rec_topk
    try:
        with torch.no_grad():
            y = m(x.reshape(1, T, H))
    finally:
        torch.topk = real_topk
    assert len(seen) == 1
    topv, topi = seen[0]
    topw = topv / topv.sum(dim=-1, keepdim=True).clamp_min(1e-9)
    out.update(raw)
    out["moe_x"] = _np(x)
    out["moe_gate"] = _np(gate)
    out["moe_out"] = _np(y.reshape(T, H))
    out["moe_topi"] = topi.numpy().astype(np.int32)
    out["moe_topw"] = _np(topw.to(torch.bfloat16))
    out["moe_shape"] = np.array([T, H, E, Fe, k])


def gen_entropy_golden(ref_root: Path) -> dict:
    """The reference's rANS stage (``superl8serve/dist/entropy.py``) on payloads of the
    kinds it codes: int8 wire codes of activations with outliers, int4-packed codes, a
    constant buffer (its documented low-entropy case), uniform and skewed bytes, one byte,
    an empty buffer. Records each payload, the reference's normalised frequency table and
    its encoded byte stream."""
    spec = importlib.util.spec_from_file_location("ref_entropy", ref_root / "superl8serve" /
                                                  "dist" / "entropy.py")
    ent = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ent)
    rng = np.random.default_rng(17)
    x = rng.standard_normal((4, 1024)).astype(np.float32)
    x[:, rng.choice(1024, 3, replace=False)] *= 20
    pay8, _ = ocodec.encode(on.round_bf16(x), "int8-had")
    pay4, _ = ocodec.encode(on.round_bf16(x), "int4-had")
    cases = {
        "int8_codes": np.asarray(pay8).view(np.uint8).ravel(),
        "int4_codes": np.asarray(pay4).view(np.uint8).ravel(),
        "constant42": np.full(1000, 42, np.uint8),
        "uniform": rng.integers(0, 256, 4096).astype(np.uint8),
        "skewed": np.minimum(rng.geometric(0.3, 10000), 255).astype(np.uint8),
        "one_byte": np.array([7], np.uint8),
        "empty": np.zeros(0, np.uint8),
    }
    out = {}
    for name, data in cases.items():
        enc, freqs = ent.encode(data)
        dec = ent.decode(enc, freqs, data.size)
        assert np.array_equal(dec, data)
        out[f"{name}_data"] = data
        out[f"{name}_freqs"] = np.asarray(freqs, np.int32)
        out[f"{name}_enc"] = np.frombuffer(enc, np.uint8).copy()
    return out


def gen_eager_golden(mods, out: dict):
    """The reference's own eager (CPU) numerics for norm / RoPE / SwiGLU / sampler."""
    g = torch.Generator().manual_seed(7)
    x = torch.randn(6, 256, generator=g).to(torch.bfloat16)
    r = torch.randn(6, 256, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(256, generator=g)).to(torch.bfloat16)
    norm = mods["layers.norm"].RMSNorm.__new__(mods["layers.norm"].RMSNorm)
    torch.nn.Module.__init__(norm)
    norm.eps, norm.add_unit_offset, norm.weight = 1e-6, False, torch.nn.Parameter(w)
    y, res = (norm._norm(x + r), x + r)
    out.update(norm_x=_np(x), norm_r=_np(r), norm_w=_np(w), norm_y=_np(y), norm_res=_np(res))
    Rot = mods["layers.rotary"].RotaryEmbedding
    rope = Rot(128, 4096, base=1e6)
    q = torch.randn(5, 1, 4, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(5, 1, 2, 128, generator=g).to(torch.bfloat16)
    pos = torch.tensor([[0], [1], [17], [1000], [4095]])
    cos = rope.cos[pos].unsqueeze(-2)
    sin = rope.sin[pos].unsqueeze(-2)
    qr, kr = rope._rotate(q, cos.to(q.dtype), sin.to(q.dtype)), rope._rotate(k, cos.to(k.dtype), sin.to(k.dtype))
    out.update(rope_q=_np(q), rope_k=_np(k), rope_pos=pos.numpy(), rope_qr=_np(qr),
               rope_kr=_np(kr), rope_cos=rope.cos.numpy(), rope_sin=rope.sin.numpy())
    gu = (2 * torch.randn(4, 2 * 192, generator=g)).to(torch.bfloat16)
    gate, up = gu.chunk(2, dim=-1)
    out.update(silu_in=_np(gu), silu_out=_np(torch.nn.functional.silu(gate) * up))
    logits = torch.randn(3, 1000, generator=g).to(torch.bfloat16)
    logits[1, 10] = logits[1, 20] = 50.0  # tie -> lowest index
    out.update(samp_logits=_np(logits), samp_tok=mods["layers.sampler"].Sampler()(
        logits, torch.zeros(3), all_greedy=True).numpy())


def gen_codec_gate_golden() -> dict:
    """The reference's wire-scheme gate (``superl8serve/dist/codec_quality.py``:
    ``verify_boundary_fidelity`` and ``select_wire_scheme``) on seeded activations, with the
    oracle codec standing in for ``superl8``. The module refers to the codec as ``fni8``, a
    name it never binds (an unfinished rename); the stand-in is bound to that name here."""
    cq = importlib.import_module("superl8serve.dist.codec_quality")
    cq.fni8 = sys.modules["superl8"]
    res = {}
    for kind in ocodec.GATE_INPUTS:
        x = torch.from_numpy(ocodec.gate_activation(kind, seed=3)).to(torch.bfloat16)
        out = {"seed": 3, "scheme": cq.select_wire_scheme(x)}
        for scheme in ("int4", "int8"):
            sq, cos = cq.verify_boundary_fidelity(x, scheme)
            out[scheme] = [sq if np.isfinite(sq) else "inf", cos]
        res[kind] = out
    return res


def gen_host_golden(mods) -> dict:
    """Pure host logic: stage bounds, peer-route policy, cache addressing, wire bytes, the
    wire-scheme gate."""
    res: dict = {"codec_gate": gen_codec_gate_golden()}
    pipe = mods["dist.pipeline"]
    res["stage_bounds"] = {f"{L}_{S}": [i * L // S for i in range(S + 1)]
                           for L in (2, 6, 28, 36, 48, 64) for S in (1, 2, 3, 4, 8) if S <= L}
    # make_pipeline itself on the tiny config (CPU, moves disabled)
    pr = mods["dist.peer_routes"]
    specs = ["", " ", "0,1", "1,0", "0,1;2,3", " 0 , 1 ; 1,2 ", "0,1;", ";", "0", "a,b",
             "0,0", "-1,2", "0,1,2"]
    parsed = {}
    for s in specs:
        try:
            parsed[s] = sorted(map(list, pr.parse_validated_pairs(s)))
        except ValueError as e:
            parsed[s] = f"ValueError: {e}"
    res["parse_validated_pairs"] = parsed
    routes = []
    for spec in ("0,1", "0,1;1,2", ""):
        val = pr.parse_validated_pairs(spec)
        for src in range(3):
            for dst in range(3):
                for cap in (True, False, None):
                    routes.append([spec, src, dst, cap,
                                   list(pr.select_route(src, dst, validated=val, capability=cap))])
    res["select_route"] = routes
    kvm = mods["engine.kv_cache"]
    cache = kvm.PagedKVCache(2, 4, 2, 64, 128, device="cpu", block_size=16)
    a, b = cache.alloc(), cache.alloc()
    cache.ensure_capacity([a, b], [20, 33])
    c = cache.alloc()
    cache.free(a)
    cache.ensure_capacity([c, b], [5, 50])
    res["kv_alloc"] = {"slots": [a, b, c], "slot_blocks": cache._slot_blocks,
                       "block_table_bc": cache.block_table([b, c]).tolist(),
                       "slot_mapping": cache._slot_mapping([b, c, b], [0, 3, 49]).tolist(),
                       "flat_rows": cache._flat_rows(torch.tensor([0, 17, 49], dtype=torch.int32)).tolist(),
                       "used_blocks": cache.used_blocks}
    dist = mods["dist"]
    TH = dist.TransferHandle
    wb = []
    for scheme, pay, sc in (("int8", (4, 8192), (4,)), ("int4", (4, 4096), (4, 64)),
                            ("fp16", (4, 8192), (0,))):
        h = TH(src_device=0, dst_device=1, scheme=scheme, shape=torch.Size((4, 1, 8192)),
               dtype=torch.bfloat16, group_size=None,
               d_payload=torch.empty(pay, dtype=torch.int8 if scheme != "fp16" else torch.bfloat16),
               d_scales=torch.empty(sc, dtype=torch.float32), compress_elapsed_ms=0.0,
               p2p_elapsed_ms=0.0)
        wb.append([scheme, h.on_wire_bytes, h.theoretical_wire_ms])
    res["on_wire_bytes"] = wb
    g = torch.Generator().manual_seed(3)
    x = torch.randn(4, 256, generator=g)
    xr = x + 0.01 * torch.randn(4, 256, generator=g)
    rep = dist.accuracy_report(x, xr, "int8")
    res["accuracy_report"] = {k: (v if not isinstance(v, float) or np.isfinite(v) else str(v))
                              for k, v in rep.items()}
    res["accuracy_report_exact"] = dist.accuracy_report(x, x.clone(), "fp16")["sqnr_db"] == float("inf")
    np.savez_compressed(HERE / "acc_inputs.npz", x=x.numpy(), xr=xr.numpy())
    return res


def main():
    if "S8B_REFERENCE" not in os.environ:
        raise SystemExit("set S8B_REFERENCE to a superl8-serve checkout (the directory that "
                         "holds the superl8serve package)")
    ref = Path(os.environ["S8B_REFERENCE"])
    if not (ref / "superl8serve").is_dir():
        raise SystemExit(f"reference checkout not found under {ref}")
    os.environ.setdefault("SUPERL8_SERVE_SKIP_TORCH_CHECK", "1")
    mods = import_reference(ref)
    force_kernel_paths(mods)
    arrays: dict = {}
    gen_eager_golden(mods, arrays)
    np.savez_compressed(HERE / "eager_numerics.npz", **arrays)
    model_arrays: dict = {}
    gen_model_golden(mods, model_arrays, 1, "int8", seed=11, tag="s1")
    gen_model_golden(mods, model_arrays, 2, "int8", seed=11, tag="s2_int8")
    gen_model_golden(mods, model_arrays, 2, "int8-had", seed=11, tag="s2_int8had")
    gen_model_golden(mods, model_arrays, 3, "int4-had", seed=11, tag="s3_int4had")
    np.savez_compressed(HERE / "tiny_qwen3_decode.npz", **model_arrays)
    moe_arrays: dict = {}
    gen_moe_module_golden(mods, moe_arrays)
    gen_model_golden(mods, moe_arrays, 1, "int8", seed=13, tag="moe_s1", moe=True)
    gen_model_golden(mods, moe_arrays, 2, "int8-had", seed=13, tag="moe_s2_int8had", moe=True)
    np.savez_compressed(HERE / "tiny_qwen3_moe.npz", **moe_arrays)
    np.savez_compressed(HERE / "rans.npz", **gen_entropy_golden(ref))
    host = gen_host_golden(mods)
    (HERE / "host_logic.json").write_text(json.dumps(host, indent=1, sort_keys=True))
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    main()
