"""GPU: the sampler kernel (temperature, top-k, top-p, repetition penalty, counter-seeded
draw) against the oracle's recipe, row by row, and sampled generation through the pipeline
against the oracle pipeline."""

import numpy as np
import pytest
import torch

from oracle import numerics as on
from oracle.model import OraclePipeline, quantize_state_dict
from oracle.sampler import sample_row
from superl8_serve_b200 import ops
from superl8_serve_b200.config import tiny
from superl8_serve_b200.dist.pipeline import stage_bounds
from superl8_serve_b200.engine import DecodePipeline
from superl8_serve_b200.runtime import StageModel
from superl8_serve_b200.weights import random_state_dict

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

ROWS = [  # temperature, top_k, top_p, penalty
    (0.0, 0, 1.0, 1.0), (0.7, 0, 1.0, 1.0), (1.0, 50, 1.0, 1.0), (0.9, 0, 0.8, 1.0),
    (1.2, 1000, 0.95, 1.3), (1.0, 1, 1.0, 1.0), (0.5, 0, 0.5, 0.8), (2.0, 40, 0.9, 1.1)]


@pytest.mark.parametrize("V", [512, 151936])
def test_sample_rows_match_oracle(V):
    rng = np.random.default_rng(V)
    M, cap = len(ROWS), 64
    logits = on.round_bf16((3.0 * rng.standard_normal((M, V))).astype(np.float32))
    pos = rng.integers(3, 40, M).astype(np.int32)
    hist = rng.integers(0, V, (M, cap)).astype(np.int32)
    inp = rng.integers(0, V, M).astype(np.int32)
    seeds = rng.integers(0, 2 ** 62, M).astype(np.int64)
    col = lambda j, dt: torch.tensor([r[j] for r in ROWS], dtype=dt, device=DEV)  # noqa: E731
    hist_d = torch.from_numpy(hist.copy()).to(DEV)
    for rep in range(2):  # the draw depends on the position: two positions per row
        p = pos + rep
        out = ops.sample(torch.from_numpy(logits).to(torch.bfloat16).to(DEV),
                         col(0, torch.float32), top_k=col(1, torch.int32),
                         top_p=col(2, torch.float32), penalty=col(3, torch.float32),
                         input_ids=torch.from_numpy(inp).to(DEV),
                         positions=torch.from_numpy(p).to(DEV), history=hist_d,
                         seeds=torch.from_numpy(seeds).to(DEV))
        got = out.cpu().numpy()
        for i, (t, k, tp, pen) in enumerate(ROWS):
            h = hist[i].copy()
            h[p[i]] = inp[i]
            want = sample_row(logits[i], t, k, tp, pen, h[:p[i] + 1], int(p[i]), int(seeds[i]))
            assert got[i] == want, (i, rep)
        assert np.array_equal(hist_d.cpu().numpy()[np.arange(M), p], inp)
        hist[np.arange(M), p] = inp


def test_sampled_draws_follow_the_distribution():
    """Many seeds on one small row: the empirical frequencies of the kept tokens follow the
    renormalised softmax (chi-square well inside its 99.9% bound)."""
    V, n = 16, 4000
    logits = on.round_bf16(np.linspace(-2, 2, V).astype(np.float32))
    x = torch.from_numpy(np.tile(logits, (n, 1))).to(torch.bfloat16).to(DEV)
    t = torch.full((n,), 1.0, device=DEV)
    out = ops.sample(x, t, input_ids=torch.zeros(n, dtype=torch.int32, device=DEV),
                     positions=torch.zeros(n, dtype=torch.int32, device=DEV),
                     history=torch.zeros(n, 4, dtype=torch.int32, device=DEV),
                     seeds=torch.arange(n, dtype=torch.int64, device=DEV) * 7919).cpu().numpy()
    p = np.exp(logits - logits.max())
    p /= p.sum()
    counts = np.bincount(out, minlength=V)
    chi2 = ((counts - n * p) ** 2 / (n * p)).sum()
    assert chi2 < 37.7  # 15 degrees of freedom, p = 0.001


@pytest.mark.parametrize("prefill", [False, True])
def test_sampled_generation_matches_oracle_pipeline(prefill):
    cfg = tiny()
    sd = random_state_dict(cfg, 11, w_std=0.1)
    b = stage_bounds(cfg.num_hidden_layers, 2)
    models = [StageModel.from_state_dict(cfg, sd, b[i], b[i + 1], DEV, first=i == 0,
                                         last=i == 1) for i in range(2)]
    prompts = [[3, 1, 4, 1, 5], [9, 2, 6], [5, 3, 5, 8, 9, 7, 9]]
    params = [{"temperature": 0.8, "top_k": 40, "top_p": 0.9, "repetition_penalty": 1.2,
               "seed": 5},
              {"temperature": 0.0},
              {"temperature": 1.3, "top_p": 0.7, "seed": 99}]
    pipe = DecodePipeline(models, batch=3, n_micro=1, max_len=64, wire_scheme="int8-had")
    pipe.set_sampling(params, prompts)
    outs = pipe.generate(prompts, 8, prefill=prefill)
    ref = OraclePipeline(cfg, quantize_state_dict(sd, cfg), n_stages=2, wire_scheme="int8-had",
                         num_slots=4, max_len=64).generate_sampled(prompts, 8, params)
    assert outs == ref


def test_pipeline_engine_sampling_params():
    """PipelineEngine with the reference's SamplingParams fields: sampled requests equal the
    oracle's recipe with the request's seed; a greedy request in the same batch stays greedy."""
    from superl8_serve_b200.dist.pipeline import PipelineEngine, SamplingParams, make_pipeline

    cfg = tiny()
    sd = random_state_dict(cfg, 11, w_std=0.1)
    stages = make_pipeline(cfg, sd, devices=(0, 0), max_num_seqs=4, max_len=64)
    eng = PipelineEngine.from_stages(stages, cfg, max_num_seqs=4, max_len=64,
                                     wire_scheme="int8-had")
    prompts = [[3, 1, 4, 1, 5], [9, 2, 6]]
    ps = [SamplingParams(temperature=0.9, top_k=30, top_p=0.9, repetition_penalty=1.1,
                         max_tokens=6, seed=3), SamplingParams(max_tokens=6)]
    sids = [eng.add_request(p, sp) for p, sp in zip(prompts, ps)]
    eng.run_pending()
    outs = [eng._out[s] for s in sids]
    ref = OraclePipeline(cfg, quantize_state_dict(sd, cfg), n_stages=2, wire_scheme="int8-had",
                         num_slots=4, max_len=64).generate_sampled(
        prompts, 6, [{"temperature": 0.9, "top_k": 30, "top_p": 0.9, "repetition_penalty": 1.1,
                      "seed": 3}, {"temperature": 0.0}])
    assert outs == ref


def test_sampler_layer_reference_signature():
    """``layers.Sampler`` with the reference's arguments: greedy rows are the argmax; a
    top_k = 1 row is its argmax too; a penalised greedy row follows the oracle recipe."""
    from superl8_serve_b200.layers import Sampler

    rng = np.random.default_rng(2)
    V = 1000
    logits = on.round_bf16((2.0 * rng.standard_normal((3, V))).astype(np.float32))
    x = torch.from_numpy(logits).to(torch.bfloat16).to(DEV)
    hist = [[5, 9, int(np.argmax(logits[2]))], [1], [int(np.argmax(logits[2])), 4]]
    torch.manual_seed(0)
    out = Sampler()(x, torch.tensor([0.0, 1.0, 0.0], device=DEV),
                    top_k=torch.tensor([0, 1, 0], device=DEV),
                    repetition_penalty=torch.tensor([1.0, 1.0, 3.0], device=DEV),
                    input_ids=hist).cpu().tolist()
    assert out[0] == int(np.argmax(logits[0])) and out[1] == int(np.argmax(logits[1]))
    assert out[2] == sample_row(logits[2], 0.0, 0, 1.0, 3.0, hist[2], len(hist[2]) - 1, 0)
