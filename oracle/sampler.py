"""Oracle token sampler (TEST INFRASTRUCTURE ONLY): the repo's sampling recipe, which follows
the reference's ``Sampler.forward`` (``superl8serve/layers/sampler.py:22-86``) step by step
but replaces its torch-RNG Gumbel draw with a counter-seeded inverse-CDF draw and its float
sums with integer masses, so that every result is reproducible:

* repetition penalty on each distinct id of the history (``sampler.py:96-125``, the Hugging
  Face rule: ``x * p`` if x < 0 else ``x / p``); greedy = argmax (first index on ties);
  temperature 0 -> greedy (``:59-68``);
* ``s = x / max(t, 1e-5)`` (``:70-71``); top-k keeps ``s >= k-th largest`` (``:127-145``);
* e = exp_s8b(s - max s), q = floor(e * 2^32); top-p keeps every e whose strictly larger
  masses sum to at most floor(p * Q) (``:147-156``: the sorted-cumsum rule, tie-symmetric);
* draw: u24 = splitmix64(seed + position) >> 40 (Steele, Lea and Flood's SplitMix64),
  target = min(floor(u24 * Q * 2^-24), Q - 1), token = first index whose running mass
  exceeds target (categorical by inverse CDF; the reference draws Gumbel-max noise).
"""

from __future__ import annotations

import numpy as np

from .numerics import exp_s8b

_M64 = (1 << 64) - 1


def splitmix64(x: int) -> int:
    z = (x + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def sample_row(logits, temperature, top_k=0, top_p=1.0, penalty=1.0, history=(), position=0,
               seed=0) -> int:
    """logits: bf16-valued float32 [V]; history: the ids at positions 0..position."""
    x = np.asarray(logits, np.float32).copy()
    V = x.size
    pen = np.float32(penalty)
    if pen != np.float32(1.0):
        for tok in dict.fromkeys(int(t) for t in history):
            if 0 <= tok < V:
                v = x[tok]
                x[tok] = np.float32(v * pen) if v < 0 else np.float32(v / pen)
    greedy = int(np.argmax(x))
    if np.float32(temperature) == 0:
        return greedy
    s = (x / np.float32(max(np.float32(temperature), np.float32(1e-5)))).astype(np.float32)
    if 0 < top_k < V:
        cutoff = np.sort(s)[::-1][top_k - 1]
        s = np.where(s < cutoff, np.float32(-np.inf), s).astype(np.float32)
    m = s.max()
    e = np.where(s == -np.inf, np.float32(0), exp_s8b((s - m).astype(np.float32))).astype(np.float32)
    q = (e.astype(np.float64) * 4294967296.0).astype(np.uint64)
    Q = int(q.sum(dtype=np.uint64))
    if np.float32(top_p) < np.float32(1.0):
        Tp = int(np.floor(np.float64(np.float32(top_p)) * np.float64(Q)))
        vals, inv = np.unique(e, return_inverse=True)  # distinct values, ascending
        mass = np.zeros(vals.size, np.uint64)
        np.add.at(mass, inv, q)  # exact integer sums per distinct value
        above, vstar = 0, vals[-1]
        for j in range(vals.size - 1, -1, -1):  # descending
            if above > Tp:
                break
            vstar = vals[j]
            above += int(mass[j])
        q = np.where(e >= vstar, q, np.uint64(0))
        Q = int(q.sum(dtype=np.uint64))
    if Q == 0:
        return greedy
    u24 = splitmix64((seed + position) & _M64) >> 40
    target = int(np.floor(np.float64(u24) * np.float64(Q) * 2.0 ** -24))
    target = min(target, Q - 1)
    run = np.cumsum(q.astype(np.uint64), dtype=np.uint64)
    return int(np.searchsorted(run, np.uint64(target), side="right"))
