"""CPU: the sampling recipe (``oracle.sampler``, which ``s8b_sample`` reproduces bit for bit)
against the behaviour the reference's own sampler tests require (superl8-serve
``tests/test_sampler.py``): greedy = argmax, per-row top-k, sign-aware once-per-token
repetition penalty, default controls as no-ops, top-p = 1 as a no-op."""

import numpy as np

from oracle.sampler import sample_row


def test_greedy_matches_argmax():
    rows = np.array([[0.1, 0.9, 0.2], [0.5, 0.1, 0.3]], np.float32)
    assert [sample_row(r, 0.0) for r in rows] == [1, 0]


def test_greedy_full_vocab_rows_are_argmax():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 151936)).astype(np.float32)
    assert [sample_row(r, 0.0, top_p=0.5, top_k=7) for r in x] == list(x.argmax(1))


def test_top_k_keeps_each_rows_top_k():
    rng = np.random.default_rng(1)
    x = rng.standard_normal(64).astype(np.float32)
    top2 = set(np.argsort(-x)[:2].tolist())
    assert all(sample_row(x, 1.0, top_k=1, seed=s) == int(x.argmax()) for s in range(20))
    draws = {sample_row(x, 5.0, top_k=2, seed=s) for s in range(200)}
    assert draws <= top2 and len(draws) == 2


def test_repetition_penalty_is_sign_aware_and_once_per_token():
    # [4, 3, -0.5] with token 0 twice and token 2 once in the history, penalty 2:
    # 4 / 2 = 2 (once, not twice) and -0.5 * 2 = -1 -> the greedy pick moves to token 1
    assert sample_row(np.array([4.0, 3.0, -0.5], np.float32), 0.0, penalty=2.0,
                      history=[0, 0, 2]) == 1
    # once per token: 4 / 1.5 = 2.67 beats 2.5; penalised twice (1.78) it would not
    assert sample_row(np.array([4.0, 2.5], np.float32), 0.0, penalty=1.5,
                      history=[0, 0]) == 0
    # a negative repeated logit gets more negative, not less
    x = np.array([-1.0, -1.5], np.float32)
    assert sample_row(x, 0.0, penalty=2.0, history=[0]) == 1


def test_repetition_penalty_changes_greedy_pick():
    assert sample_row(np.array([4.0, 3.0, 1.0], np.float32), 0.0, penalty=2.0,
                      history=[0]) == 1


def test_default_controls_are_no_ops():
    rng = np.random.default_rng(3)
    x = rng.standard_normal(32).astype(np.float32)
    for s in range(10):
        base = sample_row(x, 0.8, seed=s, position=4)
        assert sample_row(x, 0.8, top_k=0, top_p=1.0, penalty=1.0, history=[1, 2], seed=s,
                          position=4) == base


def test_top_p_keeps_only_the_nucleus():
    x = np.array([3.0, 2.9, 0.0, -1.0, -2.0], np.float32)
    # probabilities 0.505, 0.457, 0.025, ...: token 1 has 0.505 of mass ahead of it, so
    # top_p = 0.6 keeps tokens 0 and 1 only, and top_p = 0.5 (< 0.505) keeps token 0 only
    # (the reference removes a token when cumsum - p > top_p)
    assert {sample_row(x, 1.0, top_p=0.6, seed=s) for s in range(200)} == {0, 1}
    assert {sample_row(x, 1.0, top_p=0.5, seed=s) for s in range(100)} == {0}
    assert {sample_row(x, 1.0, top_p=1e-6, seed=s) for s in range(50)} == {0}
