"""CPU: the MoE oracle (router, grouped experts, combine) against the reference's own
``SparseMoE`` and Qwen3-MoE model graph (tests/golden/make_golden.py,
``tiny_qwen3_moe.npz``)."""

import numpy as np
import pytest

from oracle import moe as om
from oracle.model import OraclePipeline, quantize_state_dict
from oracle.numerics import quant_rows_i8, quantize_weight_rowwise
from superl8_serve_b200.config import tiny_moe
from superl8_serve_b200.weights import random_state_dict

PROMPTS = [[3, 1, 4, 1, 5], [9, 2, 6], [5, 3, 5, 8, 9, 7, 9]]


@pytest.fixture(scope="module")
def g(golden_dir):
    return np.load(golden_dir / "tiny_qwen3_moe.npz")


def _experts(g, E):
    out = []
    for e in range(E):
        gu = np.concatenate([g[f"moe_e{e}_gate"], g[f"moe_e{e}_up"]], 0)
        out.append((quantize_weight_rowwise(gu), quantize_weight_rowwise(g[f"moe_e{e}_down"])))
    return out


def test_router_matches_reference_sparse_moe(g):
    """Same experts chosen, in the same rank order, with the same bf16 weights as the
    reference's fp32 F.linear / softmax / topk / renormalise."""
    T, H, E, Fe, k = g["moe_shape"]
    topi, topw, p = om.moe_route(g["moe_x"], g["moe_gate"], int(k))
    assert np.array_equal(topi, g["moe_topi"])
    assert np.array_equal(topw, g["moe_topw"])
    assert np.allclose(p.sum(1), 1.0, atol=1e-5)


def test_moe_ffn_bit_exact_against_reference(g):
    T, H, E, Fe, k = g["moe_shape"]
    x = g["moe_x"]
    out = om.moe_ffn(x, *quant_rows_i8(x), g["moe_gate"], _experts(g, int(E)), int(k))
    assert np.array_equal(out, g["moe_out"])


def test_grouping_sorted_by_expert_then_token():
    rng = np.random.default_rng(0)
    T, k, E = 37, 4, 9
    topi = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    off, order, rowpos = om.group_assignments(topi, E)
    e_sorted = topi.reshape(-1)[order]
    assert np.all(np.diff(e_sorted) >= 0)
    for e in range(E):
        seg = order[off[e]:off[e + 1]]
        assert np.all(topi.reshape(-1)[seg] == e) and np.all(np.diff(seg // k) > 0)
    assert np.array_equal(order[rowpos], np.arange(T * k))


def test_topk_ties_prefer_lower_expert_index():
    y = np.zeros((1, 256), np.float32)
    gate = np.zeros((8, 256), np.float32)
    topi, topw, _ = om.moe_route(y, gate, 3)
    assert topi.tolist() == [[0, 1, 2]]
    assert np.allclose(topw, 1 / 3, rtol=1e-2)


@pytest.mark.parametrize("tag,stages,scheme", [("moe_s1", 1, "int8"),
                                               ("moe_s2_int8had", 2, "int8-had")])
def test_tiny_moe_model_matches_reference_graph(g, tag, stages, scheme):
    """Whole tiny Qwen3-MoE through the reference's Qwen3ForCausalLM / make_pipeline graph:
    greedy tokens identical and logits within 1e-2 relative (the bar for a router whose
    float32 GEMM and softmax torch rounds its own way); on these inputs they are identical."""
    cfg = tiny_moe()
    qw = quantize_state_dict(random_state_dict(cfg, 13, w_std=0.1), cfg)
    p = OraclePipeline(cfg, qw, n_stages=stages, wire_scheme=scheme, num_slots=4, max_len=64)
    outs, logits = p.generate(PROMPTS, 8)
    assert np.array_equal(np.array(outs), g[f"{tag}_tokens"])
    got = np.array(logits, dtype=np.float32)
    want = g[f"{tag}_logits"]
    assert np.abs(got - want).max() <= 1e-2 * np.abs(want).max()
    assert np.array_equal(got, want)
