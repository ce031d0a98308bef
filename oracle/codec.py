"""Oracle restatement of the inter-stage activation codec (TEST INFRASTRUCTURE ONLY).

The reference delegates ``compress_activation`` / ``decompress_activation`` to the absent
``superl8`` package (call sites ``superl8serve/dist/__init__.py:189,300``). What is visible
fixes the wire format: ``int8`` carries one fp32 scale per row
(``tests/test_transport.py:137-153``), ``int4`` / ``int4-had`` carry nibble-packed codes and
one fp32 scale per 128-element group (``superl8serve/dist/transfer_model.py:25-41``,
nibble order low-first as in ``superl8serve/layers/linear.py:43-50``), ``fp16`` is the raw
activation (bit-exact). ``int8-had`` is the block-Hadamard per-token-absmax int8 codec the
pipeline boundary uses. ``nf4`` (listed with its 16 dB / 0.985 bars at
``superl8serve/dist/__init__.py:51`` and its 4-bit, 128-group wire at
``superl8serve/dist/transfer_model.py:31,40``) follows the NF4 recipe the reference applies
to adapter weights (``superl8serve/training/qlora.py:14-36``): absmax scale per group,
nearest entry of the NF4 codebook to x / absmax (``argmin``, so the lowest index on ties).
The codebook itself lives in the absent ``superl8.quant.lowbit``; it is rebuilt here from
its published construction (QLoRA, Dettmers et al. 2023), see ``nf4_codebook``.

Encode of a row x (bf16-valued, length d, d % 128 == 0):
  z = hadamard128 per 128-block (``-had`` schemes) or z = x;
  int8*:  (codes, scale) = quant_sym(z, 127) over the whole row -> scales [rows];
  int4*:  (codes, scale) = quant_sym(z, 7) per 128-group -> scales [rows, d/128];
          byte i of the payload = (code[2i] & 0xF) | (code[2i+1] & 0xF) << 4.
  nf4:    scale = max|z| per 128-group; code = argmin_i |f32(z / scale) - NF4[i]| (0.0 for an
          all-zero group: code 7); packed as int4.
Decode: z' = f32(code) * scale (nf4: NF4[code] * scale); x' = bf16(hadamard128(z')) for
``-had``, else bf16(z').
"""

from __future__ import annotations

import numpy as np

from .numerics import hadamard_blocks, quant_sym, round_bf16

SCHEMES = ("fp16", "int8", "int8-had", "int4", "int4-had", "nf4")
GROUP = 128

# NF4 codebook, binary32, ascending (the values of ``nf4_codebook()``, pinned so the GPU
# kernels' constants and this oracle cannot drift apart).
NF4 = np.array([
    -1.0, -0.6961929202079773, -0.5250730514526367, -0.39491748809814453,
    -0.28444135189056396, -0.18477343022823334, -0.09104999154806137, 0.0,
    0.07958032935857773, 0.16093017160892487, 0.24611228704452515, 0.33791518211364746,
    0.44070979952812195, 0.5626169443130493, 0.7229567170143127, 1.0], dtype=np.float32)


def nf4_codebook() -> np.ndarray:
    """The published NF4 construction: 8 positive standard-normal quantiles at probabilities
    linspace(0.9677083, 0.5, 9)[:-1], the 7 negated quantiles at linspace(0.9677083, 0.5,
    8)[:-1], and 0; normalised by the largest magnitude; binary32, ascending."""
    from scipy.stats import norm

    off = 0.9677083
    pos = norm.ppf(np.linspace(off, 0.5, 9)[:-1])
    neg = -norm.ppf(np.linspace(off, 0.5, 8)[:-1])
    v = np.sort(np.concatenate([pos, [0.0], neg]))
    return (v / np.max(np.abs(v))).astype(np.float32)


def _pack4(codes: np.ndarray) -> np.ndarray:
    lo = (codes[:, 0::2] & 0xF).astype(np.uint8)
    hi = (codes[:, 1::2] & 0xF).astype(np.uint8)
    return (lo | (hi << 4)).astype(np.uint8)


def _nf4_encode(z: np.ndarray):
    rows, d = z.shape
    g = z.reshape(rows, d // GROUP, GROUP).astype(np.float32)
    amax = np.max(np.abs(g), axis=-1, keepdims=True).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        y = np.where(amax > 0, g / np.where(amax > 0, amax, np.float32(1)), np.float32(0))
    y = y.astype(np.float32)
    dist = np.abs((y[..., None] - NF4).astype(np.float32))
    codes = np.argmin(dist, axis=-1).reshape(rows, d).astype(np.int32)
    return _pack4(codes), amax.reshape(rows, d // GROUP).astype(np.float32)


def _rows(x):
    x = np.asarray(x, dtype=np.float32)
    return x.reshape(-1, x.shape[-1])


def encode(x: np.ndarray, scheme: str):
    """Returns (payload, scales). payload: int8 [rows, d] / uint8 [rows, d/2] / bf16 bits."""
    from .numerics import bf16_bits

    if scheme not in SCHEMES:
        raise ValueError(f"unknown codec scheme {scheme!r}")
    r = _rows(x)
    if scheme == "fp16":
        return bf16_bits(r), np.zeros((0,), dtype=np.float32)
    z = hadamard_blocks(r) if scheme.endswith("-had") else r
    if scheme.startswith("int8"):
        q, s = quant_sym(z, 127)
        return q.astype(np.int8), s
    if scheme == "nf4":
        return _nf4_encode(z)
    rows, d = z.shape
    q, s = quant_sym(z.reshape(rows, d // GROUP, GROUP), 7)
    return _pack4(q.reshape(rows, d).astype(np.int32)), s.astype(np.float32)


def decode(payload: np.ndarray, scales: np.ndarray, scheme: str, d: int) -> np.ndarray:
    from .numerics import bf16_to_f32

    if scheme == "fp16":
        return bf16_to_f32(payload).reshape(-1, d)
    if scheme.startswith("int8"):
        z = (payload.astype(np.float32) * scales.reshape(-1, 1)).astype(np.float32)
    else:
        p = payload.astype(np.int32)
        lo = p & 0xF
        hi = (p >> 4) & 0xF
        codes = np.stack([lo, hi], axis=-1).reshape(p.shape[0], -1)
        if scheme == "nf4":
            codes = NF4[codes]
        else:
            codes = np.where(codes >= 8, codes - 16, codes).astype(np.float32)
        rows = codes.shape[0]
        z = (codes.reshape(rows, d // GROUP, GROUP) * scales.reshape(rows, d // GROUP, 1))
        z = z.astype(np.float32).reshape(rows, d)
    if scheme.endswith("-had"):
        z = hadamard_blocks(z)
    return round_bf16(z)


def wire_bytes(rows: int, d: int, scheme: str) -> int:
    """Bytes on the wire: payload plus fp32 scales (``TransferHandle.on_wire_bytes``,
    ``superl8serve/dist/__init__.py:115-129``)."""
    if scheme == "fp16":
        return rows * d * 2
    if scheme.startswith("int8"):
        return rows * d + rows * 4
    return rows * d // 2 + rows * (d // GROUP) * 4


def accuracy(original: np.ndarray, reconstructed: np.ndarray):
    """(SQNR dB, cosine) as ``accuracy_report`` computes them
    (``superl8serve/dist/__init__.py:55-85``)."""
    x = np.asarray(original, dtype=np.float64).ravel()
    xr = np.asarray(reconstructed, dtype=np.float64).ravel()
    noise = float(np.sum((x - xr) ** 2))
    sqnr = float("inf") if noise == 0.0 else float(10.0 * np.log10(np.sum(x * x) / noise))
    den = max(np.linalg.norm(x) * np.linalg.norm(xr), 1e-12)
    return sqnr, float(np.dot(x, xr) / den)


GATE_INPUTS = ("gauss", "outliers", "laplace", "const")


def gate_activation(kind: str, seed: int = 0, T: int = 8, D: int = 2048) -> np.ndarray:
    """Seeded bf16-valued activations [T, D] for the wire-scheme gate
    (``superl8serve/dist/codec_quality.py:68-93``): ``gauss`` N(0, 1); ``outliers`` N(0, 1)
    with 0.1% of the channels scaled x20 (BASELINE config 2's distribution); ``laplace``
    Laplace(0, 1); ``const`` every element 0.5 (exact round trip)."""
    rng = np.random.default_rng(seed)
    if kind == "gauss":
        x = rng.standard_normal((T, D))
    elif kind == "outliers":
        x = rng.standard_normal((T, D))
        x[:, rng.choice(D, max(1, D // 1000), replace=False)] *= 20.0
    elif kind == "laplace":
        x = rng.laplace(0.0, 1.0, (T, D))
    elif kind == "const":
        x = np.full((T, D), 0.5)
    else:
        raise ValueError(kind)
    return round_bf16(x.astype(np.float32))
