"""GPU: whole decode steps through the stage runtime against the oracle and the golden
fixtures of the reference's module graph: greedy tokens identical, logits bit-identical."""

import numpy as np
import pytest
import torch

from oracle.model import OraclePipeline, quantize_state_dict
from superl8_serve_b200.config import qwen3_0_6b, tiny
from superl8_serve_b200.dist.pipeline import PipelineEngine, SamplingParams, make_pipeline, stage_bounds
from superl8_serve_b200.engine import DecodePipeline
from superl8_serve_b200.runtime import StageModel
from superl8_serve_b200.weights import random_state_dict

pytestmark = pytest.mark.gpu
PROMPTS = [[3, 1, 4, 1, 5], [9, 2, 6], [5, 3, 5, 8, 9, 7, 9]]


def stage_models(cfg, sd, n_stages, devices=None):
    b = stage_bounds(cfg.num_hidden_layers, n_stages)
    devices = devices or ["cuda:0"] * n_stages
    return [StageModel.from_state_dict(cfg, sd, b[i], b[i + 1], devices[i], first=i == 0,
                                       last=i == n_stages - 1) for i in range(n_stages)]


@pytest.fixture(scope="module")
def tiny_sd():
    return tiny(), random_state_dict(tiny(), 11, w_std=0.1)


@pytest.mark.parametrize("tag,stages,scheme,n_micro", [
    ("s1", 1, "int8", 1), ("s2_int8", 2, "int8", 1), ("s2_int8had", 2, "int8-had", 3),
    ("s3_int4had", 3, "int4-had", 1)])
def test_tiny_pipeline_matches_golden(golden_dir, tiny_sd, tag, stages, scheme, n_micro):
    d = np.load(golden_dir / "tiny_qwen3_decode.npz")
    cfg, sd = tiny_sd
    pipe = DecodePipeline(stage_models(cfg, sd, stages), batch=3, n_micro=n_micro, max_len=64,
                          wire_scheme=scheme)
    outs, logits = pipe.generate(PROMPTS, 8, keep_logits=True)
    assert np.array_equal(np.array(outs), d[f"{tag}_tokens"])
    if n_micro == 1:
        got = np.stack([np.stack([t.numpy() for t in row]) for row in logits])
        assert np.array_equal(got, d[f"{tag}_logits"])


@pytest.mark.parametrize("tag,stages,scheme,chunk", [
    ("s1", 1, "int8", 256), ("s2_int8had", 2, "int8-had", 4), ("s3_int4had", 3, "int4-had", 7)])
def test_prefill_then_decode_matches_golden(golden_dir, tiny_sd, tag, stages, scheme, chunk):
    """Varlen chunked prefill (chunks of 4 and 7 rows cut sequences mid-prompt) then decode
    from each sequence's own length: the reference graph's tokens and logits, bit for bit."""
    d = np.load(golden_dir / "tiny_qwen3_decode.npz")
    cfg, sd = tiny_sd
    pipe = DecodePipeline(stage_models(cfg, sd, stages), batch=3, n_micro=1, max_len=64,
                          wire_scheme=scheme)
    pipe.prefill_chunk = chunk
    outs, logits = pipe.generate(PROMPTS, 8, keep_logits=True, prefill=True)
    assert np.array_equal(np.array(outs), d[f"{tag}_tokens"])
    got = np.stack([np.stack([t.numpy() for t in row]) for row in logits])
    assert np.array_equal(got, d[f"{tag}_logits"])


def test_prefill_tensor_core_chunks_match_oracle(tiny_sd):
    """Prompts of 40, 17 and 70 tokens in 64-row chunks: every chunk runs the tcgen05 GEMMs
    with split-K partials; tokens and logits equal the oracle's prefill + decode."""
    cfg, sd = tiny_sd
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (40, 17, 70)]
    pipe = DecodePipeline(stage_models(cfg, sd, 2), batch=3, n_micro=1, max_len=128,
                          wire_scheme="int8-had")
    pipe.prefill_chunk = 64
    outs, logits = pipe.generate(prompts, 6, keep_logits=True, prefill=True)
    assert pipe._pf[0][0].tc_ws is not None
    ref, ref_logits = OraclePipeline(cfg, quantize_state_dict(sd, cfg), n_stages=2,
                                     wire_scheme="int8-had", num_slots=4,
                                     max_len=128).generate_prefilled(prompts, 6)
    assert outs == ref
    got = np.stack([np.stack([t.numpy() for t in row]) for row in logits])
    assert np.array_equal(got, np.array(ref_logits, dtype=np.float32))


def test_prefill_rejects_empty_prompt(tiny_sd):
    cfg, sd = tiny_sd
    pipe = DecodePipeline(stage_models(cfg, sd, 1), batch=2, max_len=64)
    with pytest.raises(ValueError):
        pipe.prefill([[1, 2], []])


def test_graph_replay_equals_eager(tiny_sd):
    cfg, sd = tiny_sd
    outs = []
    for use_graph in (False, True):
        pipe = DecodePipeline(stage_models(cfg, sd, 2), batch=4, n_micro=2, max_len=128,
                              wire_scheme="int8-had")
        pipe.add_sequences()
        pipe.set_state([0, 0, 0, 0], [1, 2, 3, 4], reserve=40)
        if use_graph:
            pipe._enqueue()  # warm-up (sets kernel attributes) outside capture
            torch.cuda.synchronize()
            pipe.set_state([0, 0, 0, 0], [1, 2, 3, 4], reserve=40)
            pipe.capture()
        seq = []
        for _ in range(20):
            pipe.step()
            seq.append(pipe.tokens().cpu().tolist())
        torch.cuda.synchronize()
        outs.append(seq)
    assert outs[0] == outs[1]


def test_pipeline_engine_api(tiny_sd):
    """make_pipeline / PipelineEngine.from_stages / generate with the reference's signatures
    (superl8serve/dist/pipeline.py:430,535,1042), two stages on one GPU."""
    cfg, sd = tiny_sd
    stages = make_pipeline(cfg, sd, devices=(0, 0), max_num_seqs=4, max_len=64)
    assert [s.layer_offset for s in stages] == [0, 2]
    eng = PipelineEngine.from_stages(stages, cfg, max_num_seqs=4, max_len=64, wire_scheme="int8")
    out = eng.generate(PROMPTS, SamplingParams(temperature=0.0, max_tokens=5))
    qw = quantize_state_dict(sd, cfg)
    ref, _ = OraclePipeline(cfg, qw, n_stages=2, wire_scheme="int8", num_slots=4,
                            max_len=64).generate(PROMPTS, 5)
    assert out == ref


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_in_process_pipeline(tiny_sd):
    cfg, sd = tiny_sd
    d = stage_models(cfg, sd, 2, ["cuda:0", "cuda:1"])
    pipe = DecodePipeline(d, batch=3, n_micro=3, max_len=64, wire_scheme="int8")
    outs = pipe.generate(PROMPTS, 8)
    qw = quantize_state_dict(sd, cfg)
    ref, _ = OraclePipeline(cfg, qw, n_stages=2, wire_scheme="int8", num_slots=4,
                            max_len=64).generate(PROMPTS, 8)
    assert outs == ref
    pipe = DecodePipeline(stage_models(cfg, sd, 2, ["cuda:0", "cuda:1"]), batch=3, n_micro=1,
                          max_len=64, wire_scheme="int8")
    pipe.prefill_chunk = 4
    assert pipe.generate(PROMPTS, 8, prefill=True) == ref


@pytest.mark.slow
def test_config1_qwen3_0_6b_two_stage_greedy_parity():
    """Qwen3-0.6B shape, 2 stages (layers 0-13 / 14-27), batch 4, prompts
    of 128 uniform-random ids, int8 paged KV (block 16), greedy decoding for 64 steps (the
    north star's greedy-identity length): GPU tokens == oracle tokens and logits within 1e-2
    relative (they are in fact identical), token by token and through the varlen prefill."""
    cfg = qwen3_0_6b(max_position_embeddings=4096)
    sd = random_state_dict(cfg, 0)
    rng = np.random.default_rng(0)
    prompts = rng.integers(0, cfg.vocab_size, (4, 128)).tolist()
    steps = 64
    pipe = DecodePipeline(stage_models(cfg, sd, 2), batch=4, n_micro=1, max_len=208,
                          wire_scheme="int8-had")
    assert stage_bounds(28, 2) == [0, 14, 28]
    outs, logits = pipe.generate(prompts, steps, keep_logits=True)
    # the same prompts through the varlen prefill: 512 rows in two 256-row chunks
    del pipe
    pipe = DecodePipeline(stage_models(cfg, sd, 2), batch=4, n_micro=1, max_len=208,
                          wire_scheme="int8-had")
    outs_p, logits_p = pipe.generate(prompts, steps, keep_logits=True, prefill=True)
    del pipe
    qw = quantize_state_dict(sd, cfg)
    del sd
    ref, ref_logits = OraclePipeline(cfg, qw, n_stages=2, wire_scheme="int8-had", num_slots=4,
                                     max_len=208).generate_prefilled(prompts, steps)
    assert all(len(r) == steps for r in ref)
    assert outs == ref
    got = np.stack([np.stack([t.numpy() for t in row]) for row in logits])
    want = np.array(ref_logits, dtype=np.float32)
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= 1e-2
    assert np.array_equal(got, want)
    assert outs_p == ref
    got = np.stack([np.stack([t.numpy() for t in row]) for row in logits_p])
    assert np.array_equal(got, want)
