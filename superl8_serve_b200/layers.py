"""Reference-shaped layer API over the s8b kernels.

Each class keeps the constructor and ``forward`` signature of its superl8-serve counterpart
so model code written against the reference runs unchanged; the arithmetic is the s8b CUDA
kernels (CUDA tensors only: there is no CPU path).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import ops
from .weights import QTensor, to_qtensor


def rope_tables(head_dim: int, max_position: int, base: float = 1e6):
    """binary32 cos/sin tables exactly as ``RotaryEmbedding.__init__`` builds them
    (``superl8serve/layers/rotary.py:31-37``); computed on the host, uploaded once."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().contiguous(), emb.sin().contiguous()


def _cuda(x: torch.Tensor, what: str):
    if not x.is_cuda:
        raise RuntimeError(f"{what}: s8b layers run on CUDA tensors only (no CPU fallback)")


class LinearW8A8(nn.Module):
    """``LinearW8A8`` (``superl8serve/layers/linear.py:75-124``): per-token int8 activation
    quant + int8 GEMM with int32 accumulation + dequant, output in the activation dtype."""

    def __init__(self, weight: QTensor, bias: torch.Tensor | None = None):
        super().__init__()
        if weight.scheme != "per_row_i8":
            raise ValueError(f"LinearW8A8 supports per_row_i8 weights, got {weight.scheme!r}")
        self.weight = weight
        self.bias = bias
        self.out_features, self.in_features = weight.data.shape

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _cuda(x, "LinearW8A8")
        q, s = ops.quant_rows(x)
        y = ops.gemm_w8a8(q, s, self.weight.data, self.weight.scale, out_dtype=x.dtype)
        return y if self.bias is None else y + self.bias


class RMSNorm(nn.Module):
    """``RMSNorm`` (``superl8serve/layers/norm.py:21-58``) with fused residual add:
    ``forward(x)`` -> normed; ``forward(x, residual)`` -> (normed, x + residual)."""

    def __init__(self, dim: int, eps: float = 1e-6, weight: torch.Tensor | None = None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(weight if weight is not None else torch.ones(dim, dtype=torch.bfloat16),
                                   requires_grad=False)

    def forward(self, x, residual=None):
        _cuda(x, "RMSNorm")
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        r2 = None if residual is None else residual.reshape(-1, shp[-1]).contiguous()
        res, _, _, y = ops.rmsnorm_quant(x2, r2, self.weight.data, self.eps, y_out=True)
        y = y.reshape(shp)
        return y if residual is None else (y, res.reshape(shp))


class SiluAndMul(nn.Module):
    """``SiluAndMul`` (``superl8serve/layers/activation.py:20-26``) on [gate | up]."""

    def forward(self, x):
        _cuda(x, "SiluAndMul")
        shp = x.shape
        _, _, y = ops.silu_mul_quant(x.reshape(-1, shp[-1]).contiguous(), y_out=True)
        return y.reshape(*shp[:-1], shp[-1] // 2)


class VocabEmbedding(nn.Module):
    """``VocabEmbedding`` (``superl8serve/layers/embedding.py:22-69``), bf16/fp16 table."""

    def __init__(self, weight: torch.Tensor, embed_scale: float = 1.0, out_dtype=torch.bfloat16):
        super().__init__()
        if embed_scale != 1.0:
            raise ValueError("embed_scale != 1 is outside the Qwen3 decode path")
        self.weight = nn.Parameter(weight.to(out_dtype), requires_grad=False)

    def forward(self, input_ids):
        _cuda(input_ids, "VocabEmbedding")
        ids = input_ids.reshape(-1).to(torch.int32).contiguous()
        return ops.embed(ids, self.weight.data).reshape(*input_ids.shape, -1)


class LMHead(nn.Module):
    """``LMHead`` (``superl8serve/layers/embedding.py:72-91``): int8 head GEMM."""

    def __init__(self, weight: QTensor | torch.Tensor):
        super().__init__()
        self.proj = LinearW8A8(to_qtensor(weight))

    def forward(self, hidden):
        return self.proj(hidden)


class Sampler(nn.Module):
    """``Sampler`` (``superl8serve/layers/sampler.py:20-156``) with its signature. An
    all-greedy batch is the argmax kernel (lowest index on ties, ``:51-63``); otherwise
    ``s8b_sample`` applies the repetition penalty over each row's ``input_ids`` history,
    temperature, top-k and top-p, and draws one token per row. The draw is an inverse-CDF
    draw keyed by a per-row seed taken from torch's RNG (``torch.manual_seed`` makes it
    repeatable) instead of the reference's Gumbel noise; the distribution is the same.
    Host-side ``logit_processors`` are not supported."""

    def forward(self, logits, temperatures=None, top_p=None, top_k=None,
                repetition_penalty=None, logit_processors=None, input_ids=None, *,
                all_greedy=None, **kw):
        _cuda(logits, "Sampler")
        if logit_processors is not None and any(logit_processors):
            raise NotImplementedError("host logit processors are not on the s8b decode path")
        logits = logits.contiguous()
        M, V = logits.shape
        dev = logits.device
        greedy = temperatures is None or bool((temperatures == 0).all())
        no_pen = repetition_penalty is None or bool((repetition_penalty == 1.0).all())
        if greedy and no_pen:
            return ops.argmax(logits).long()
        if not no_pen and input_ids is None:
            raise ValueError("input_ids are required for repetition_penalty")
        hist_rows = input_ids if input_ids is not None else [[] for _ in range(M)]
        cap = max(1, max(len(h) for h in hist_rows))
        hist = torch.zeros(M, cap, dtype=torch.int32)
        for i, h in enumerate(hist_rows):
            if h:
                hist[i, : len(h)] = torch.tensor(h, dtype=torch.int32)
        pos = torch.tensor([max(len(h) - 1, 0) for h in hist_rows], dtype=torch.int32)
        last = torch.tensor([h[-1] if h else 0 for h in hist_rows], dtype=torch.int32)
        f32 = lambda t, d: (torch.full((M,), d, dtype=torch.float32) if t is None  # noqa: E731
                            else t.detach().float().reshape(M).cpu())
        seeds = torch.randint(0, 2 ** 62, (M,), dtype=torch.int64)
        out = ops.sample(logits, f32(temperatures, 0.0).to(dev),
                         top_k=None if top_k is None else top_k.to(torch.int32).reshape(M).to(dev),
                         top_p=None if top_p is None else f32(top_p, 1.0).to(dev),
                         penalty=None if repetition_penalty is None else f32(repetition_penalty, 1.0).to(dev),
                         input_ids=last.to(dev), positions=pos.to(dev), history=hist.to(dev),
                         seeds=seeds.to(dev))
        return out.long()
