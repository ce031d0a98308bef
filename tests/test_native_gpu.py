"""GPU: ``s8b_stage_step`` (one C call per stage step, from a plain-pointer descriptor) gives
the reference graph's tokens and logits, like the Python launch sequence it replays: dp4a and
tensor-core (split-K) paths, several micro-batches and stages, prefill, a sparse-MoE model."""

import numpy as np
import pytest

from superl8_serve_b200.config import tiny, tiny_moe
from superl8_serve_b200.dist.pipeline import stage_bounds
from superl8_serve_b200.engine import DecodePipeline
from superl8_serve_b200.runtime import StageModel
from superl8_serve_b200.weights import random_state_dict

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
PROMPTS = [[3, 1, 4, 1, 5], [9, 2, 6], [5, 3, 5, 8, 9, 7, 9]]


def _models(cfg, sd, n):
    b = stage_bounds(cfg.num_hidden_layers, n)
    return [StageModel.from_state_dict(cfg, sd, b[i], b[i + 1], DEV, first=i == 0,
                                       last=i == n - 1) for i in range(n)]


@pytest.mark.parametrize("moe,tag,stages,scheme,n_micro,prefill", [
    (False, "s1", 1, "int8", 1, False), (False, "s2_int8had", 2, "int8-had", 3, False),
    (False, "s3_int4had", 3, "int4-had", 1, True), (True, "moe_s2_int8had", 2, "int8-had", 1, True)])
def test_native_stage_step_matches_reference_graph(golden_dir, moe, tag, stages, scheme, n_micro,
                                                   prefill):
    cfg = tiny_moe() if moe else tiny()
    sd = random_state_dict(cfg, 13 if moe else 11, w_std=0.1)
    g = np.load(golden_dir / ("tiny_qwen3_moe.npz" if moe else "tiny_qwen3_decode.npz"))
    pipe = DecodePipeline(_models(cfg, sd, stages), batch=3, n_micro=n_micro, max_len=64,
                          wire_scheme=scheme)
    pipe.set_native()
    pipe.prefill_chunk = 4
    outs, logits = pipe.generate(PROMPTS, 8, keep_logits=True, prefill=prefill)
    assert np.array_equal(np.array(outs), g[f"{tag}_tokens"])
    if n_micro == 1:
        got = np.stack([np.stack([t.numpy() for t in row]) for row in logits])
        assert np.array_equal(got, g[f"{tag}_logits"])


def test_native_tensor_core_path_equals_python_launches():
    cfg = tiny()
    sd = random_state_dict(cfg, 11, w_std=0.1)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, cfg.vocab_size, 6).tolist() for _ in range(24)]
    res = []
    for native in (False, True):
        pipe = DecodePipeline(_models(cfg, sd, 2), batch=24, n_micro=1, max_len=64,
                              wire_scheme="int8-had")
        assert pipe.runners[0].tc_ws is not None
        pipe.set_native(native)
        outs, logits = pipe.generate(prompts, 4, keep_logits=True)
        res.append((outs, np.stack([np.stack([t.numpy() for t in row]) for row in logits])))
    assert res[0][0] == res[1][0] and np.array_equal(res[0][1], res[1][1])
