"""CPU: the algorithmic byte counts behind bench.py's roofline figures."""

import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_config3_step_bytes(bench):
    """Qwen3-8B, batch 64, ctx 2048, 36 layers + head: 6.95 GB of layer weights, 0.62 GB of
    head, 2112 B per token per layer of KV."""
    cfg = bench.model_config("qwen3-8b")
    b = bench.step_bytes(cfg, 64, 2048, 36, True)
    assert b == 17544840704
    w = bench.step_bytes(cfg, 0, 2048, 36, False)
    kv_per_token_layer = (bench.step_bytes(cfg, 1, 2048, 1, False)
                          - bench.step_bytes(cfg, 0, 2048, 1, False)) / 2049
    assert abs(w / 1e9 - 6.95) < 0.01 and kv_per_token_layer == 2112


def test_moe_step_bytes_count_only_routed_experts(bench):
    cfg = bench.model_config("qwen3-30b-a3b")
    assert 127.9 < bench.experts_hit(cfg, 128) <= 128
    assert bench.experts_hit(cfg, 1) == pytest.approx(8.0)
    full = bench.step_bytes(cfg, 128, 4096, 48, True)
    one = bench.step_bytes(cfg, 1, 4096, 48, True)
    assert abs(full / 1e9 - 56.92) < 0.01 and one < full / 4
