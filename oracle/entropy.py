"""Oracle static rANS (TEST INFRASTRUCTURE ONLY): the reference's entropy stage
(``superl8serve/dist/entropy.py``) restated, plus the chunked multi-stream layout of the
GPU coder (chunk i = symbols [i*n/S, (i+1)*n/S) coded as an independent stream).

Format (``entropy.py:1-26,103-152``): frequencies normalised to M = 2^12; 32-bit state in
[2^23, 2^31); symbols coded last to first; before coding symbol s, bytes of the state are
emitted low byte first while state >= 2^19 * freq(s); state = (state // f << 12) +
state % f + cum(s); the final state is flushed as 4 bytes, low byte first. Decode starts
from the last 4 bytes and reads backwards.
"""

from __future__ import annotations

import numpy as np

SCALE_BITS = 12
M = 1 << SCALE_BITS
L = 1 << 23
X_MAX_FACTOR = (L >> SCALE_BITS) << 8


def normalize_freqs(counts: np.ndarray) -> np.ndarray:
    """``_normalize_freqs`` (``entropy.py:54-91``): floor(count * M / total), present symbols
    at least 1, then the drift to M spread one unit at a time over the present symbols in
    ``np.argsort(-counts)`` order (never below 1)."""
    counts = np.asarray(counts, np.int64)
    total = int(counts.sum())
    f = np.zeros(256, np.int64)
    if total == 0:
        return f.astype(np.int32)
    present = counts > 0
    f[present] = np.maximum(counts[present] * M // total, 1)
    drift = M - int(f.sum())
    order = np.argsort(-counts)
    n_present = int(present.sum())
    i = 0
    while drift:
        s = order[i % n_present]
        if drift > 0:
            f[s] += 1
            drift -= 1
        elif f[s] > 1:
            f[s] -= 1
            drift += 1
        i += 1
    return f.astype(np.int32)


def encode_stream(sym: np.ndarray, freqs: np.ndarray) -> bytes:
    f = [int(v) for v in freqs]
    cum = [0] * 257
    for s in range(256):
        cum[s + 1] = cum[s] + f[s]
    state, out = L, bytearray()
    for s in np.asarray(sym, np.uint8)[::-1].tolist():
        while state >= X_MAX_FACTOR * f[s]:
            out.append(state & 0xFF)
            state >>= 8
        state = ((state // f[s]) << SCALE_BITS) + state % f[s] + cum[s]
    for _ in range(4):
        out.append(state & 0xFF)
        state >>= 8
    return bytes(out)


def decode_stream(buf: bytes, freqs: np.ndarray, n: int) -> np.ndarray:
    f = [int(v) for v in freqs]
    cum = [0] * 257
    for s in range(256):
        cum[s + 1] = cum[s] + f[s]
    slot_sym = np.repeat(np.arange(256), f).tolist()
    pos = len(buf) - 4
    state = buf[pos] | buf[pos + 1] << 8 | buf[pos + 2] << 16 | buf[pos + 3] << 24
    out = np.empty(n, np.uint8)
    for i in range(n):
        slot = state & (M - 1)
        s = slot_sym[slot]
        state = f[s] * (state >> SCALE_BITS) + slot - cum[s]
        while state < L:
            pos -= 1
            state = (state << 8) | buf[pos]
        out[i] = s
    return out


def encode(sym: np.ndarray, n_streams: int = 1):
    """Returns (list of per-stream byte strings, freqs). One stream: the reference's
    ``encode`` output (``b""`` for an empty input)."""
    sym = np.asarray(sym, np.uint8).ravel()
    freqs = normalize_freqs(np.bincount(sym, minlength=256))
    if sym.size == 0:
        return [b""], freqs
    n = sym.size
    lo = [n * i // n_streams for i in range(n_streams + 1)]
    return [encode_stream(sym[lo[i]:lo[i + 1]], freqs) for i in range(n_streams)], freqs


def decode(streams: list, freqs: np.ndarray, n: int) -> np.ndarray:
    S = len(streams)
    lo = [n * i // S for i in range(S + 1)]
    return np.concatenate([decode_stream(streams[i], freqs, lo[i + 1] - lo[i])
                           for i in range(S)]) if n else np.zeros(0, np.uint8)
