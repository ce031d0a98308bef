"""Weights: the ``QTensor`` container, the per-row int8 quantizer and seeded random init.

``QTensor`` keeps the fields the reference reads (``data``, ``scale``, ``scheme``,
``group_size``, ``codebook``; ``superl8serve/layers/linear.py:37-72``,
``superl8serve/dist/pipeline.py:333-342``), since the ``superl8`` package that defines it
upstream is not part of this build.

Random init follows the Hugging Face convention for Qwen3 (linear and embedding weights
N(0, 0.02)); RMSNorm gains are 1 + N(0, 0.1) so that a wrong gain index cannot hide behind
an all-ones vector. Every tensor is rounded to bf16 (the model's storage dtype) and drawn
from its own stream seeded by (seed, crc32(name)), so generation order does not matter.
"""

from __future__ import annotations

import zlib
from dataclasses import dataclass, field
from typing import Iterator

import numpy as np
import torch


@dataclass
class QTensor:
    data: torch.Tensor
    scale: torch.Tensor | None
    scheme: str = "per_row_i8"
    group_size: int | None = None
    codebook: str | None = None
    meta: dict = field(default_factory=dict)

    def to(self, device) -> "QTensor":
        return QTensor(self.data.to(device), None if self.scale is None else self.scale.to(device),
                       self.scheme, self.group_size, self.codebook, dict(self.meta))


def _bf16_round(x: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(torch.bfloat16).float().numpy()


def quantize_rowwise_np(w: np.ndarray):
    """Per-output-row symmetric int8: s = max(absmax, 1e-6)/127, q = clamp(rint(w/s)),
    binary32 arithmetic (the reference's recipe, ``tests/test_layers.py:29-33``)."""
    w = np.asarray(w, dtype=np.float32)
    amax = np.max(np.abs(w), axis=-1).astype(np.float32)
    s = (np.maximum(amax, np.float32(1e-6)) / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint((w / s[:, None]).astype(np.float32)), -127, 127).astype(np.int8)
    return q, s


def to_qtensor(w) -> QTensor:
    """float weight [out, in] -> per_row_i8 QTensor (``superl8serve/models/weights.py:49-56``).
    An existing QTensor passes through."""
    if isinstance(w, QTensor):
        return w
    arr = w.float().cpu().numpy() if isinstance(w, torch.Tensor) else np.asarray(w)
    q, s = quantize_rowwise_np(arr)
    return QTensor(torch.from_numpy(q), torch.from_numpy(s), scheme="per_row_i8")


def merge_qtensor(rows: list) -> QTensor:
    """Concatenate q/k/v (or gate/up) on the output axis; each row keeps its own scale, so the
    merge is exact (``superl8serve/models/weights.py:75-115``)."""
    qs = [to_qtensor(r) for r in rows]
    return QTensor(torch.cat([q.data for q in qs], 0).contiguous(),
                   torch.cat([q.scale for q in qs], 0).contiguous(), scheme="per_row_i8")


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def state_dict_names(cfg) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, kind) of every HF-style tensor of a Qwen3 dense or Qwen3-MoE model
    (``mlp.gate`` router and ``mlp.experts.{e}.*`` in sparse layers)."""
    H, hd = cfg.hidden_size, cfg.resolved_head_dim()
    nh, nkv, F, V = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size, cfg.vocab_size
    out = [("model.embed_tokens.weight", (V, H), "w"), ("model.norm.weight", (H,), "g")]
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}"
        out += [
            (f"{p}.input_layernorm.weight", (H,), "g"),
            (f"{p}.post_attention_layernorm.weight", (H,), "g"),
            (f"{p}.self_attn.q_proj.weight", (nh * hd, H), "w"),
            (f"{p}.self_attn.k_proj.weight", (nkv * hd, H), "w"),
            (f"{p}.self_attn.v_proj.weight", (nkv * hd, H), "w"),
            (f"{p}.self_attn.o_proj.weight", (H, nh * hd), "w"),
            (f"{p}.self_attn.q_norm.weight", (hd,), "g"),
            (f"{p}.self_attn.k_norm.weight", (hd,), "g"),
        ]
        if cfg.layer_is_moe(i):
            Fe = cfg.moe_intermediate_size
            out.append((f"{p}.mlp.gate.weight", (cfg.num_experts, H), "w"))
            for e in range(cfg.num_experts):
                q = f"{p}.mlp.experts.{e}"
                out += [(f"{q}.gate_proj.weight", (Fe, H), "w"), (f"{q}.up_proj.weight", (Fe, H), "w"),
                        (f"{q}.down_proj.weight", (H, Fe), "w")]
        else:
            out += [
                (f"{p}.mlp.gate_proj.weight", (F, H), "w"),
                (f"{p}.mlp.up_proj.weight", (F, H), "w"),
                (f"{p}.mlp.down_proj.weight", (H, F), "w"),
            ]
    if not cfg.tie_word_embeddings:
        out.append(("lm_head.weight", (V, H), "w"))
    return out


def random_tensor(seed: int, name: str, shape, kind: str, w_std: float = 0.02) -> np.ndarray:
    g = _rng(seed, name)
    x = g.standard_normal(shape, dtype=np.float32)
    if kind == "w":
        x *= np.float32(w_std)
    else:
        x = np.float32(1.0) + np.float32(0.1) * x
    return _bf16_round(x)


def iter_random_state_dict(cfg, seed: int = 0, w_std: float = 0.02
                           ) -> Iterator[tuple[str, np.ndarray]]:
    for name, shape, kind in state_dict_names(cfg):
        yield name, random_tensor(seed, name, shape, kind, w_std)


def random_state_dict(cfg, seed: int = 0, w_std: float = 0.02) -> dict[str, np.ndarray]:
    """Whole HF-style float32 (bf16-valued) state dict; use only for small models."""
    return dict(iter_random_state_dict(cfg, seed, w_std))
