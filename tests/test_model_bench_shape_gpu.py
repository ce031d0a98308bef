"""GPU: decode steps at the benchmarked shape against the CPU oracle, bit for bit.

The bench's own setup (Qwen3-8B layer shapes, vocabulary 151,936, batch 64, KV pre-filled
with random codes to 2048 tokens, the whole step captured in one CUDA graph) cut to two
layers so the oracle finishes in about a minute. Three steps in a row: every step's greedy
tokens and bf16 logits must equal the oracle's, which runs the same layers on copies of the
device's weights and KV pool. This is the kernel sequence the throughput figure is measured
on: the tensor-core GEMMs with their split-K partial mode and the row kernels that reduce
them, the persistent attention at 4,096+ work units, the LM head over the full vocabulary.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle.kernels import add_residual, argmax_rows, gemm_w8a8, rmsnorm, rope_tables
from oracle.model import Shape, layer_decode
from oracle.numerics import quant_rows_i8, round_bf16

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy() if t.is_floating_point() else t.cpu().numpy()


def _oracle_layers(model):
    out = []
    for L in model.layers:
        out.append({"qkv": (_np(L.qkv_w), _np(L.qkv_s)), "o": (_np(L.o_w), _np(L.o_s)),
                    "gu": (_np(L.gu_w), _np(L.gu_s)), "down": (_np(L.d_w), _np(L.d_s)),
                    "in_norm": _np(L.in_norm), "post_norm": _np(L.post_norm),
                    "q_norm": _np(L.q_norm), "k_norm": _np(L.k_norm)})
    return out


def test_config3_shaped_decode_two_layers_matches_oracle():
    from superl8_serve_b200.config import qwen3_8b
    from superl8_serve_b200.engine import DecodePipeline
    from superl8_serve_b200.runtime import StageModel

    cfg = qwen3_8b(num_hidden_layers=2)
    B, ctx, steps, bs = 64, 2048, 3, 16
    dev = torch.device("cuda", 0)
    model = StageModel.synthetic(cfg, 0, 2, dev, first=True, last=True, seed=1)
    pipe = DecodePipeline([model], batch=B, n_micro=1, max_len=ctx + steps + 16)
    pipe.pools[0].fill_random(seed=2)
    pipe.add_sequences()
    ids = np.random.default_rng(3).integers(0, cfg.vocab_size, B)
    pipe.set_state([ctx] * B, ids.tolist(), reserve=steps + 8)
    torch.cuda.synchronize()

    # oracle copies of the device state (before any step writes the pool)
    pool = pipe.pools[0]
    opool = SimpleNamespace(kc=_np(pool.kc), ks=_np(pool.ks), vc=_np(pool.vc), vs=_np(pool.vs),
                            block_size=bs)
    bt = _np(pipe.mbs[0][0].block_table)
    layers = _oracle_layers(model)
    norm = _np(model.norm)
    head = (_np(model.head_w), _np(model.head_s))
    s = Shape(cfg.vocab_size, cfg.hidden_size, 2, cfg.num_attention_heads,
              cfg.num_key_value_heads, 128, cfg.intermediate_size, cfg.rms_norm_eps,
              cfg.rope_theta, cfg.max_position_embeddings)
    tabs = rope_tables(128, cfg.max_position_embeddings, cfg.rope_theta)

    pipe.capture()  # the bench's path: one CUDA graph per step
    for t in range(steps):
        pipe.step()
        torch.cuda.synchronize()
        got_tok = _np(pipe.tokens())
        got_logits = _np(pipe.logits())

        pos = ctx + t
        positions = [pos] * B
        sm = (bt[:, pos // bs] * bs + pos % bs).astype(np.int32)
        cl = np.full(B, pos + 1, dtype=np.int32)
        h = round_bf16(_np(model.embed[torch.from_numpy(ids).to(dev)]))
        res = None
        for li, L in enumerate(layers):
            h, res = layer_decode(L, li, h, res, positions, sm, bt, cl, opool, s, tabs)
        y = rmsnorm(add_residual(h, res), norm, s.rms_norm_eps)
        want_logits = gemm_w8a8(*quant_rows_i8(y), *head)
        want_tok = argmax_rows(want_logits)
        assert np.array_equal(got_tok, want_tok), t
        bad = np.argwhere(got_logits != want_logits)
        assert bad.size == 0, (t, len(bad), bad[:4])
        ids = want_tok.astype(np.int64)
