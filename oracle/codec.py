"""Oracle restatement of the inter-stage activation codec (TEST INFRASTRUCTURE ONLY).

The reference delegates ``compress_activation`` / ``decompress_activation`` to the absent
``superl8`` package (call sites ``superl8serve/dist/__init__.py:189,300``). What is visible
fixes the wire format: ``int8`` carries one fp32 scale per row
(``tests/test_transport.py:137-153``), ``int4`` / ``int4-had`` carry nibble-packed codes and
one fp32 scale per 128-element group (``superl8serve/dist/transfer_model.py:25-41``,
nibble order low-first as in ``superl8serve/layers/linear.py:43-50``), ``fp16`` is the raw
activation (bit-exact). ``int8-had`` is the block-Hadamard per-token-absmax int8 codec the
pipeline boundary uses.

Encode of a row x (bf16-valued, length d, d % 128 == 0):
  z = hadamard128 per 128-block (``-had`` schemes) or z = x;
  int8*:  (codes, scale) = quant_sym(z, 127) over the whole row -> scales [rows];
  int4*:  (codes, scale) = quant_sym(z, 7) per 128-group -> scales [rows, d/128];
          byte i of the payload = (code[2i] & 0xF) | (code[2i+1] & 0xF) << 4.
Decode: z' = f32(code) * scale; x' = bf16(hadamard128(z')) for ``-had``, else bf16(z').
"""

from __future__ import annotations

import numpy as np

from .numerics import hadamard_blocks, quant_sym, round_bf16

SCHEMES = ("fp16", "int8", "int8-had", "int4", "int4-had")
GROUP = 128


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
    rows, d = z.shape
    q, s = quant_sym(z.reshape(rows, d // GROUP, GROUP), 7)
    q = q.reshape(rows, d).astype(np.int32)
    lo = (q[:, 0::2] & 0xF).astype(np.uint8)
    hi = (q[:, 1::2] & 0xF).astype(np.uint8)
    return (lo | (hi << 4)).astype(np.uint8), s.astype(np.float32)


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
