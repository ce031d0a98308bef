"""GPU: continuous batching — requests join and leave the running decode batch through the
scheduler; every request's tokens equal a run of that request alone (oracle)."""

import numpy as np
import pytest

from oracle.model import OraclePipeline, quantize_state_dict
from superl8_serve_b200.config import tiny
from superl8_serve_b200.dist.pipeline import SamplingParams, stage_bounds
from superl8_serve_b200.runtime import StageModel
from superl8_serve_b200.scheduler import ContinuousEngine
from superl8_serve_b200.weights import random_state_dict

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def test_requests_joining_and_leaving_match_solo_runs():
    cfg = tiny()
    sd = random_state_dict(cfg, 11, w_std=0.1)
    b = stage_bounds(cfg.num_hidden_layers, 2)
    models = [StageModel.from_state_dict(cfg, sd, b[i], b[i + 1], DEV, first=i == 0,
                                         last=i == 1) for i in range(2)]
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (5, 1, 9, 3, 7, 2, 6)]
    params = [SamplingParams(max_tokens=m) for m in (6, 4, 8, 3, 5, 7, 4)]
    params[2] = SamplingParams(temperature=0.8, top_k=20, top_p=0.9, max_tokens=8, seed=4)
    params[4] = SamplingParams(temperature=0.0, repetition_penalty=1.3, max_tokens=5)
    eng = ContinuousEngine(models, max_num_seqs=3, max_len=64, max_batch_tokens=12)
    outs = eng.generate(prompts, params)
    qw = quantize_state_dict(sd, cfg)
    for p, sp, got in zip(prompts, params, outs):
        ref = OraclePipeline(cfg, qw, n_stages=2, wire_scheme="int8-had", num_slots=2,
                             max_len=64).generate_sampled(
            [p], sp.max_tokens, [{"temperature": sp.temperature, "top_k": sp.top_k,
                                  "top_p": sp.top_p,
                                  "repetition_penalty": sp.repetition_penalty,
                                  "seed": 0 if sp.seed is None else sp.seed}])
        assert got == ref[0]
    assert not eng.sched.has_work() and len(eng.pipe.alloc._free_slots) == 3
