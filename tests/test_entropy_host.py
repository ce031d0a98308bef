"""CPU: the rANS oracle and the host-side frequency normalisation against the reference's
own entropy coder (golden streams from ``superl8serve/dist/entropy.py``,
tests/golden/make_golden.py)."""

import numpy as np
import pytest

from oracle import entropy as oe
from superl8_serve_b200.dist.entropy import normalize_freqs

CASES = ["int8_codes", "int4_codes", "constant42", "uniform", "skewed", "one_byte", "empty"]


@pytest.fixture(scope="module")
def g(golden_dir):
    return np.load(golden_dir / "rans.npz")


@pytest.mark.parametrize("case", CASES)
def test_oracle_reproduces_reference_streams(g, case):
    data = g[f"{case}_data"]
    streams, freqs = oe.encode(data)
    assert np.array_equal(freqs, g[f"{case}_freqs"])
    assert streams[0] == g[f"{case}_enc"].tobytes()
    if data.size:
        assert np.array_equal(oe.decode([g[f"{case}_enc"].tobytes()], freqs, data.size), data)


@pytest.mark.parametrize("case", CASES)
def test_host_normalisation_matches_reference_table(g, case):
    counts = np.bincount(g[f"{case}_data"], minlength=256)
    assert np.array_equal(normalize_freqs(counts), g[f"{case}_freqs"])


def test_normalised_tables_sum_to_4096_and_keep_every_symbol():
    rng = np.random.default_rng(0)
    for _ in range(50):
        counts = rng.integers(0, 1000, 256) * (rng.random(256) < rng.random())
        if counts.sum() == 0:
            continue
        f = normalize_freqs(counts)
        assert f.sum() == 4096 and np.all(f[counts > 0] >= 1) and np.all(f[counts == 0] == 0)


@pytest.mark.parametrize("S", [1, 3, 16])
def test_oracle_multi_stream_round_trip(g, S):
    data = g["int8_codes_data"]
    streams, freqs = oe.encode(data, n_streams=S)
    assert len(streams) == S
    assert np.array_equal(oe.decode(streams, freqs, data.size), data)


def test_decode_rejects_a_table_that_does_not_sum_to_4096():
    """Tables are checked on the host before any kernel sees them."""
    import torch

    from superl8_serve_b200.dist import entropy as ent

    bad = np.zeros(256, np.int32)
    bad[7] = 4095
    with pytest.raises(ValueError):
        ent.decode(torch.zeros(8, dtype=torch.uint8), bad, 10)
    with pytest.raises(ValueError):
        ent.decode(torch.zeros(8, dtype=torch.uint8), np.full(255, 16, np.int32), 10)
