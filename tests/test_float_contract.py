"""CPU: the attention recipe against the reference's float contract, inside a model.

``oracle.kernels.paged_decode`` (what the CUDA kernels reproduce bit for bit) quantizes the
rotated query per head to int8 and the softmax weights to 15 bits. The reference's float
path (``PagedKVCache.read_dense`` dequantization, fp32 softmax; ``oracle.float_contract``)
is the contract it approximates. Here a Qwen3-0.6B-shaped model (config 1's widths and
vocabulary, two layers in two stages, random N(0, 0.02) weights) runs on the float contract
while every layer, at every prefill and decode call, also evaluates the recipe on the same
query and cache (teacher forcing, so errors do not compound).

Bound: the recipe's attention output is within 1e-2 relative (L2 over the batch) of the
float contract at every layer. Measured: at most 0.7%, mean 0.5%, dominated by the int8
query.

Not asserted at model level: per-token int8 activation quantization makes a W8A8 model's
logits jump by its quantization noise whenever a row's quantizer input changes at all. On
this model two float evaluations of the same contract (fp32 against fp64 attention) already
differ by 1.8% in the step-0 logits; the recipe differs by 4.8%. The one-layer model below
shows the float contract itself is resolved (fp32 and fp64 agree exactly there).
"""

import numpy as np
import pytest

from oracle import float_contract as fc
from oracle.model import OraclePipeline, quantize_state_dict

PROMPT_LEN, STEPS = 32, 8


@pytest.fixture(scope="module")
def model2():
    from superl8_serve_b200.config import qwen3_0_6b
    from superl8_serve_b200.weights import random_state_dict

    cfg = qwen3_0_6b(num_hidden_layers=2)
    qw = quantize_state_dict(random_state_dict(cfg, 0, w_std=0.02), cfg)
    prompts = np.random.default_rng(1).integers(0, cfg.vocab_size, (4, PROMPT_LEN)).tolist()
    return cfg, qw, prompts


def _pipe(cfg, qw, attention=None, stages=2):
    return OraclePipeline(cfg, qw, n_stages=stages, num_slots=4,
                          max_len=PROMPT_LEN + STEPS + 16, attention=attention)


def test_recipe_attention_within_1e2_of_float_contract_at_every_layer(model2):
    cfg, qw, prompts = model2
    tf = fc.TeacherForced()
    toks, _ = _pipe(cfg, qw, tf).generate_prefilled(prompts, STEPS)
    L = cfg.num_hidden_layers
    assert len(tf.errors) == L * STEPS  # prefill (all prompt rows) + STEPS - 1 decode calls
    assert max(tf.errors) < 1e-2, tf.errors
    assert all(len(t) == STEPS for t in toks)


def test_float_contract_is_resolved_on_one_layer():
    """fp32 and fp64 evaluations of the float contract give the same logits and tokens on a
    one-layer model, so the comparison above is not limited by the contract's own rounding."""
    from superl8_serve_b200.config import qwen3_0_6b
    from superl8_serve_b200.weights import random_state_dict

    cfg = qwen3_0_6b(num_hidden_layers=1)
    qw = quantize_state_dict(random_state_dict(cfg, 0, w_std=0.02), cfg)
    prompts = np.random.default_rng(1).integers(0, cfg.vocab_size, (4, PROMPT_LEN)).tolist()
    t32, l32 = _pipe(cfg, qw, fc.float_attention, 1).generate_prefilled(prompts, 4)
    t64, l64 = _pipe(cfg, qw, fc.float64_attention, 1).generate_prefilled(prompts, 4)
    assert t32 == t64
    assert fc.logits_rel(np.array(l64)[:, 0], np.array(l32)[:, 0]) < 1e-6
