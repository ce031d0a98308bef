"""Wire-codec accuracy gate (``superl8serve/dist/codec_quality.py``): round-trip an
activation through a scheme and report (SQNR dB, cosine); pick int4 when it clears the bars
(14 dB, 0.98), else int8. On the s8b codec kernels. This gate synchronises the host (it reads
the metrics back), so the captured pipeline step uses a fixed ``wire_scheme`` instead."""

from __future__ import annotations

import torch

from . import compress_activation, decompress_activation


def verify_boundary_fidelity(activation: torch.Tensor, compressor: str,
                             group_size: int | None = None) -> tuple[float, float]:
    if group_size is None and compressor in ("int4", "int4-had", "nf4"):
        group_size = 128
    c = compress_activation(activation, scheme=compressor, group_size=group_size)
    xr = decompress_activation(c)
    x = activation.detach().float().flatten()
    r = xr.detach().float().flatten()
    noise = (x - r).pow(2).sum()
    if noise.item() == 0.0:
        sqnr = float("inf")
    else:
        sqnr = float(10.0 * torch.log10(x.pow(2).sum() / noise))
    cos = float(torch.nn.functional.cosine_similarity(x, r, dim=0, eps=1e-12))
    return sqnr, cos


def select_wire_scheme(activation: torch.Tensor, group_size: int | None = None) -> str:
    sqnr, cos = verify_boundary_fidelity(activation, "int4", group_size=group_size)
    return "int4" if sqnr >= 14.0 and cos >= 0.98 else "int8"
