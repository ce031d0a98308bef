"""Bit-level numeric primitives shared by every oracle kernel (TEST INFRASTRUCTURE ONLY).

Every floating-point value is a numpy ``float32`` array and every operation below is one
correctly rounded IEEE-754 binary32 operation (round to nearest, ties to even), applied
in the order written. The CUDA kernels perform the same operations in the same order with
``__fmul_rn`` / ``__fadd_rn`` / ``__fdiv_rn`` / ``__fsqrt_rn`` (no FMA contraction), so
the two sides agree bit for bit. Activations of the act dtype (bf16) are carried as float32
arrays whose values are bf16-representable.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------- bf16 ----

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit pattern (uint16), round to nearest even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    """bf16 bit pattern (uint16) -> float32 (exact)."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 value, returned as float32."""
    return bf16_to_f32(bf16_bits(x))


# ----------------------------------------------------------------------------- exp ----
#
# exp(x) by Cody-Waite style range reduction to a power of two and a Taylor polynomial:
#   exp(x) = 2^t,  t = x*log2(e) = k + f,  k = rint(t),  |f| <= 1/2,
#   2^f = sum_i (f ln2)^i / i!   (degree 7; truncation error < 6e-9 for |f| <= 1/2).
# Coefficients are the binary32 roundings of ln(2)^i / i!, evaluated by Horner's rule with
# separate multiply and add. 2^k is exact (k is kept in the normal exponent range).

LOG2E = F32(1.4426950408889634)
EXP_COEF = [F32(math.log(2.0) ** i / math.factorial(i)) for i in range(8)]
EXP_T_MIN = F32(-125.0)  # t below this -> 0
EXP_T_MAX = F32(127.0)  # t above this -> +inf


def exp_s8b(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    t = (x * LOG2E).astype(np.float32)
    tc = np.clip(t, EXP_T_MIN, EXP_T_MAX)
    k = np.rint(tc).astype(np.float32)
    f = (tc - k).astype(np.float32)
    p = np.full_like(f, EXP_COEF[7])
    for c in EXP_COEF[6::-1]:
        p = (p * f).astype(np.float32)
        p = (p + c).astype(np.float32)
    r = np.ldexp(p, k.astype(np.int32)).astype(np.float32)
    r = np.where(t < EXP_T_MIN, F32(0.0), r)
    r = np.where(t > EXP_T_MAX, F32(np.inf), r)
    return r.astype(np.float32)


# -------------------------------------------------------------------- Hadamard-128 ----

HAD_SCALE = F32(1.0 / math.sqrt(128.0))  # binary32 rounding of 128^-1/2


def fwht128(x: np.ndarray) -> np.ndarray:
    """Unnormalised fast Walsh-Hadamard transform over the last axis (length 128).

    Stage h = 1, 2, 4, ..., 64 replaces each pair (j, j+h) with j's bit h clear by
    (a + b, a - b), in binary32. The result equals x @ H128 for the natural-order
    Sylvester matrix H128[i, j] = (-1)^popcount(i & j) up to per-stage rounding.
    """
    x = np.asarray(x, dtype=np.float32)
    lead = x.shape[:-1]
    assert x.shape[-1] == 128
    y = x.reshape(-1, 128)
    h = 1
    while h < 128:
        y = y.reshape(-1, 128 // (2 * h), 2, h)
        a = y[:, :, 0, :]
        b = y[:, :, 1, :]
        y = np.stack([(a + b).astype(np.float32), (a - b).astype(np.float32)], axis=2)
        h *= 2
    return y.reshape(*lead, 128)


def hadamard128(x: np.ndarray) -> np.ndarray:
    """Orthonormal block Hadamard: fwht128(x) * 128^-1/2 (binary32). An involution up to
    rounding, as the reference's ``rotate_last`` (``superl8serve/engine/kv_cache.py:274-278``)."""
    return (fwht128(x) * HAD_SCALE).astype(np.float32)


def hadamard_blocks(x: np.ndarray) -> np.ndarray:
    """Apply ``hadamard128`` to every 128-wide block of the last axis."""
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    assert d % 128 == 0
    return hadamard128(x.reshape(*x.shape[:-1], d // 128, 128)).reshape(x.shape)


# ----------------------------------------------------------------------- quantizers ----

def quant_sym(x: np.ndarray, qmax: int):
    """Symmetric round-to-nearest quantizer over the last axis.

    amax = max|x| (exact); inv = qmax / amax; code = clamp(rint(x * inv), -qmax, qmax);
    scale = amax / qmax. An all-zero row gets scale 1 and zero codes.
    Returns (codes int32, scale float32).
    """
    x = np.asarray(x, dtype=np.float32)
    amax = np.max(np.abs(x), axis=-1).astype(np.float32)
    nz = amax > 0
    safe = np.where(nz, amax, F32(1.0)).astype(np.float32)
    inv = np.where(nz, (F32(qmax) / safe).astype(np.float32), F32(0.0)).astype(np.float32)
    scale = np.where(nz, (safe / F32(qmax)).astype(np.float32), F32(1.0)).astype(np.float32)
    q = np.rint((x * inv[..., None]).astype(np.float32))
    q = np.clip(q, -qmax, qmax).astype(np.int32)
    return q, scale


def quant_rows_i8(x: np.ndarray):
    """Per-token int8 activation quantizer (W8A8 contract, ``layers/linear.py:1-13``)."""
    q, s = quant_sym(x, 127)
    return q.astype(np.int8), s


def quantize_weight_rowwise(w: np.ndarray):
    """Per-output-row int8 weight quantizer, restating the reference's test recipe
    (``tests/test_layers.py:29-33``: s = absmax.clamp_min(1e-6)/127,
    q = round(w/s).clamp(-127,127)) in binary32."""
    w = np.asarray(w, dtype=np.float32)
    amax = np.max(np.abs(w), axis=-1).astype(np.float32)
    s = (np.maximum(amax, F32(1e-6)) / F32(127.0)).astype(np.float32)
    q = np.clip(np.rint((w / s[:, None]).astype(np.float32)), -127, 127).astype(np.int8)
    return q, s


def dequant_acc(acc: np.ndarray, sx: np.ndarray, sw: np.ndarray) -> np.ndarray:
    """y = (float(acc) * sx[m]) * sw[n] in binary32 (float(acc) rounds to nearest even)."""
    a = acc.astype(np.float32)
    y = (a * sx[:, None].astype(np.float32)).astype(np.float32)
    return (y * sw[None, :].astype(np.float32)).astype(np.float32)
