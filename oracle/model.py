"""Oracle Qwen3 W8A8 pipeline decode (TEST INFRASTRUCTURE ONLY).

Restates, on the CPU, one decode step of superl8-serve's layer-split pipeline:

* stage split ``bounds[i] = i*L//S`` (``superl8serve/dist/pipeline.py:452``), a paged KV pool
  per stage sized to its own layers (``:486-494``);
* per stage, the Qwen3 decoder layers (``superl8serve/models/qwen3.py:70-80``): input
  RMSNorm with fused residual, merged-QKV W8A8, per-head q/k RMSNorm, RoPE, int8 paged KV
  write and paged decode attention, o_proj, post-attention RMSNorm, merged gate_up W8A8,
  SwiGLU, down W8A8;
* between stages the packed ``[hidden | residual]`` boundary (``:246-250,301-305``) goes
  through the wire codec (``oracle.codec``);
* last stage: final RMSNorm with the residual, int8 LM head (quantized even when tied,
  ``superl8serve/models/qwen3.py:161-166``), greedy argmax.

``generate`` consumes prompts by decode steps (token t of every prompt at step t);
``prefill`` restates the varlen prefill, which gives the same tokens and logits;
``generate_sampled`` restates the sampler (``oracle.sampler``).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import codec as ocodec
from .kernels import (
    add_residual,
    argmax_rows,
    embed,
    gemm_w8a8,
    kv_write_paged,
    paged_decode,
    qkv_post,
    quant_q_for_attn,
    rmsnorm,
    rope_tables,
    silu_mul,
)
from .moe import moe_ffn
from .numerics import quant_rows_i8, quantize_weight_rowwise, round_bf16


@dataclass
class Shape:
    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position_embeddings: int = 4096
    tie_word_embeddings: bool = False
    num_experts: int = 0
    num_experts_per_tok: int = 8
    norm_topk_prob: bool = True


def shape_of(cfg) -> Shape:
    return Shape(**{f: getattr(cfg, f) for f in Shape.__dataclass_fields__
                    if hasattr(cfg, f)})


def quantize_state_dict(sd: dict, cfg) -> dict:
    """HF-style float state dict -> quantized oracle weights (merged qkv / gate_up rows,
    per-row int8; ``superl8serve/models/weights.py:49-138``)."""
    s = shape_of(cfg)
    out = {"embed": np.asarray(sd["model.embed_tokens.weight"], dtype=np.float32),
           "norm": np.asarray(sd["model.norm.weight"], dtype=np.float32), "layers": []}
    for i in range(s.num_hidden_layers):
        p = f"model.layers.{i}"
        qkv = np.concatenate([sd[f"{p}.self_attn.{n}_proj.weight"] for n in "qkv"], axis=0)
        L = {}
        L["qkv"] = quantize_weight_rowwise(qkv)
        L["o"] = quantize_weight_rowwise(sd[f"{p}.self_attn.o_proj.weight"])
        if f"{p}.mlp.gate.weight" in sd:
            # sparse MoE layer (``superl8serve/models/qwen3.py:53-64``): router + per-expert
            # merged gate_up / down, each quantized per row
            L["router"] = np.asarray(sd[f"{p}.mlp.gate.weight"], dtype=np.float32)
            L["experts"] = []
            for e in range(L["router"].shape[0]):
                q = f"{p}.mlp.experts.{e}"
                gu = np.concatenate([sd[f"{q}.gate_proj.weight"], sd[f"{q}.up_proj.weight"]], 0)
                L["experts"].append((quantize_weight_rowwise(gu),
                                     quantize_weight_rowwise(sd[f"{q}.down_proj.weight"])))
        else:
            gu = np.concatenate([sd[f"{p}.mlp.gate_proj.weight"], sd[f"{p}.mlp.up_proj.weight"]], 0)
            L["gu"] = quantize_weight_rowwise(gu)
            L["down"] = quantize_weight_rowwise(sd[f"{p}.mlp.down_proj.weight"])
        L["in_norm"] = np.asarray(sd[f"{p}.input_layernorm.weight"], dtype=np.float32)
        L["post_norm"] = np.asarray(sd[f"{p}.post_attention_layernorm.weight"], dtype=np.float32)
        L["q_norm"] = np.asarray(sd[f"{p}.self_attn.q_norm.weight"], dtype=np.float32)
        L["k_norm"] = np.asarray(sd[f"{p}.self_attn.k_norm.weight"], dtype=np.float32)
        out["layers"].append(L)
    head = sd["model.embed_tokens.weight"] if s.tie_word_embeddings else sd["lm_head.weight"]
    out["head"] = quantize_weight_rowwise(head)
    return out


class PagedPool:
    """Host block allocator + int8 pools of one stage, following ``PagedKVCache``
    (``superl8serve/engine/kv_cache.py:439-559,703-749,1118-1127``)."""

    def __init__(self, n_layers, num_slots, nkv, max_len, hd, block_size=16, num_blocks=None):
        self.block_size = block_size
        self.max_blocks_per_seq = (max_len + block_size - 1) // block_size
        self.num_blocks = num_blocks or num_slots * self.max_blocks_per_seq
        shp = (n_layers, self.num_blocks, nkv, block_size, hd)
        self.kc = np.zeros(shp, np.int8)
        self.vc = np.zeros(shp, np.int8)
        self.ks = np.ones(shp[:-1], np.float32)
        self.vs = np.ones(shp[:-1], np.float32)
        self._free_blocks = list(range(self.num_blocks))
        self._free_slots = list(range(num_slots))
        self._slot_blocks = [[] for _ in range(num_slots)]

    def alloc(self):
        return self._free_slots.pop()

    def ensure_capacity(self, slots, lengths):
        for slot, n in zip(slots, lengths):
            blocks = self._slot_blocks[slot]
            need = (n + self.block_size - 1) // self.block_size
            while len(blocks) < need:
                blocks.append(self._free_blocks.pop())

    def slot_mapping(self, slots, positions):
        bs = self.block_size
        return np.array([self._slot_blocks[s][p // bs] * bs + p % bs
                         for s, p in zip(slots, positions)], dtype=np.int32)

    def block_table(self, slots):
        bt = np.zeros((len(slots), self.max_blocks_per_seq), dtype=np.int32)
        for i, s in enumerate(slots):
            b = self._slot_blocks[s]
            bt[i, : len(b)] = b
        return bt


def recipe_attention(q, kc, ks, vc, vs, block_table, ctx_lens, block_size, scale, li=None):
    """The attention recipe the kernels reproduce: the query rotated and quantized per head
    (``quant_q_for_attn``), then ``paged_decode``. q [M, Hq, D] float32 (bf16-valued)."""
    qq, qs = quant_q_for_attn(q)
    return paged_decode(qq, qs, kc, ks, vc, vs, block_table, ctx_lens, block_size, scale)


def layer_decode(L, li, h, residual, positions, slot_mapping, block_table, ctx_lens, pool,
                 s: Shape, tabs, attention=None):
    """One ``Qwen3DecoderLayer.forward`` in decode (``superl8serve/models/qwen3.py:70-80``).
    ``attention`` replaces ``recipe_attention`` (same arguments), e.g. with the float
    contract of ``oracle.float_contract``."""
    nh, nkv, hd, eps = s.num_attention_heads, s.num_key_value_heads, s.head_dim, s.rms_norm_eps
    x = h if residual is None else add_residual(h, residual)
    residual = x
    y = rmsnorm(x, L["in_norm"], eps)
    qkv = gemm_w8a8(*quant_rows_i8(y), *L["qkv"])
    q, k, v = qkv_post(qkv, positions, nh, nkv, hd, L["q_norm"], L["k_norm"], eps, *tabs)
    kv_write_paged(k, v, pool.kc[li], pool.ks[li], pool.vc[li], pool.vs[li], slot_mapping,
                   pool.block_size)
    att = (attention or recipe_attention)(q, pool.kc[li], pool.ks[li], pool.vc[li],
                                          pool.vs[li], block_table, ctx_lens, pool.block_size,
                                          hd ** -0.5, li=li)
    o = gemm_w8a8(*quant_rows_i8(att.reshape(att.shape[0], -1)), *L["o"])
    x = add_residual(o, residual)
    residual = x
    y = rmsnorm(x, L["post_norm"], eps)
    if "experts" in L:
        h = moe_ffn(y, *quant_rows_i8(y), L["router"], L["experts"], s.num_experts_per_tok,
                    s.norm_topk_prob)
        return h, residual
    gu = gemm_w8a8(*quant_rows_i8(y), *L["gu"])
    a = silu_mul(gu)
    h = gemm_w8a8(*quant_rows_i8(a), *L["down"])
    return h, residual


class OraclePipeline:
    """Greedy W8A8 decode through S contiguous stages with a codec at each boundary."""

    def __init__(self, cfg, qw: dict, *, n_stages=1, wire_scheme="int8-had", num_slots=8,
                 max_len=256, block_size=16, attention=None):
        self.attention = attention  # None: the recipe (``recipe_attention``)
        self.s = shape_of(cfg)
        self.qw = qw
        L = self.s.num_hidden_layers
        if n_stages > L:
            raise ValueError("pipeline stage count cannot exceed the model layer count")
        self.bounds = [i * L // n_stages for i in range(n_stages + 1)]
        self.wire_scheme = wire_scheme
        self.pools = [PagedPool(self.bounds[i + 1] - self.bounds[i], num_slots,
                                self.s.num_key_value_heads, max_len, self.s.head_dim,
                                block_size) for i in range(n_stages)]
        self.tabs = rope_tables(self.s.head_dim, self.s.max_position_embeddings,
                                self.s.rope_theta)

    def decode(self, ids, slots, positions):
        """One decode step for a batch: returns (next token ids, logits bf16-valued)."""
        s = self.s
        lengths = [p + 1 for p in positions]
        h = round_bf16(embed(self.qw["embed"], ids))
        residual = None
        for si, pool in enumerate(self.pools):
            pool.ensure_capacity(slots, lengths)
            sm = pool.slot_mapping(slots, positions)
            bt = pool.block_table(slots)
            cl = np.array(lengths, dtype=np.int32)
            for li in range(self.bounds[si], self.bounds[si + 1]):
                h, residual = layer_decode(self.qw["layers"][li], li - self.bounds[si], h,
                                           residual, positions, sm, bt, cl, pool, s, self.tabs,
                                           attention=self.attention)
            if si != len(self.pools) - 1:
                packed = np.concatenate([h, residual], axis=-1)
                pay, sc = ocodec.encode(packed, self.wire_scheme)
                rec = ocodec.decode(pay, sc, self.wire_scheme, packed.shape[-1])
                h, residual = rec[:, : s.hidden_size], rec[:, s.hidden_size:]
        x = add_residual(h, residual)
        y = rmsnorm(x, self.qw["norm"], s.rms_norm_eps)
        logits = gemm_w8a8(*quant_rows_i8(y), *self.qw["head"])
        return argmax_rows(logits), logits

    def generate(self, prompts, max_new_tokens):
        """Greedy generation; every sequence advances one token per step (prompt tokens are
        teacher-forced). Returns (outputs per prompt, logits of every generated token)."""
        slots = [self.pools[0].alloc() for _ in prompts]
        for p in self.pools[1:]:
            for _ in prompts:
                p.alloc()
        seqs = [list(p) for p in prompts]
        outs = [[] for _ in prompts]
        logit_log = [[] for _ in prompts]
        step = 0
        while any(len(o) < max_new_tokens for o in outs):
            ids = np.array([sq[step] for sq in seqs], dtype=np.int64)
            toks, logits = self.decode(ids, slots, [step] * len(prompts))
            for i, sq in enumerate(seqs):
                if step >= len(prompts[i]) - 1 and len(outs[i]) < max_new_tokens:
                    outs[i].append(int(toks[i]))
                    logit_log[i].append(logits[i])
                if step + 1 >= len(sq):
                    sq.append(int(toks[i]))
            step += 1
        return outs, logit_log

    def prefill(self, prompts):
        """``PipelineEngine._prefill`` (``superl8serve/dist/pipeline.py:908-984``): all prompt
        tokens of all sequences as one varlen batch of rows (``cu_seqlens`` order), each row
        writing its K/V at its position and attending over positions [0, t] of its sequence;
        the argmax of each sequence's last row is its first generated token. Returns
        (first tokens, their logits, slots)."""
        slots = [self.pools[0].alloc() for _ in prompts]
        for p in self.pools[1:]:
            for _ in prompts:
                p.alloc()
        ids = np.array([t for p in prompts for t in p], dtype=np.int64)
        row_slots = [slots[i] for i, p in enumerate(prompts) for _ in p]
        positions = [t for p in prompts for t in range(len(p))]
        toks, logits = self.decode(ids, row_slots, positions)
        last = np.cumsum([len(p) for p in prompts]) - 1
        return [int(toks[j]) for j in last], [logits[j] for j in last], slots

    def generate_prefilled(self, prompts, max_new_tokens):
        """Prefill, then greedy decode with every sequence at its own position."""
        first, first_logits, slots = self.prefill(prompts)
        outs = [[t] for t in first]
        logit_log = [[lg] for lg in first_logits]
        positions = [len(p) for p in prompts]
        ids = np.array(first, dtype=np.int64)
        for _ in range(max_new_tokens - 1):
            toks, logits = self.decode(ids, slots, positions)
            for i in range(len(prompts)):
                outs[i].append(int(toks[i]))
                logit_log[i].append(logits[i])
            ids = np.asarray(toks, dtype=np.int64)
            positions = [p + 1 for p in positions]
        return outs, logit_log

    def generate_sampled(self, prompts, max_new_tokens, params):
        """Teacher-forced generation with the sampling recipe of ``oracle.sampler`` per row
        (params[i]: temperature, top_k, top_p, repetition_penalty, seed); the history of a
        row at a step is every token up to and including that step's input."""
        from .sampler import sample_row

        slots = [self.pools[0].alloc() for _ in prompts]
        for p in self.pools[1:]:
            for _ in prompts:
                p.alloc()
        seqs = [list(p) for p in prompts]
        outs = [[] for _ in prompts]
        step = 0
        while any(len(o) < max_new_tokens for o in outs):
            ids = np.array([sq[step] for sq in seqs], dtype=np.int64)
            _, logits = self.decode(ids, slots, [step] * len(prompts))
            for i, sq in enumerate(seqs):
                if step >= len(prompts[i]) - 1:
                    # every row past its prompt keeps stepping (as the pipeline does); only
                    # the first max_new_tokens are its output
                    pr = params[i]
                    tok = sample_row(logits[i], pr.get("temperature", 0.0), pr.get("top_k", 0),
                                     pr.get("top_p", 1.0), pr.get("repetition_penalty", 1.0),
                                     sq[:step + 1], step, int(pr.get("seed", i)))
                    if len(outs[i]) < max_new_tokens:
                        outs[i].append(tok)
                    if step + 1 >= len(sq):
                        sq.append(tok)
            step += 1
        return outs
