"""Engine-boundary transport: compress -> copy -> decompress, with the reference's API
(``superl8serve/dist/__init__.py``: ``send``, ``recv``, ``TransferHandle``,
``accuracy_report``), on the s8b codec kernels.

``send`` compresses on the source GPU with ``s8b_codec_encode``; when the route is allowed
(``peer_routes``) the encoder stores the codes straight into a buffer on the destination GPU
over NVLink, otherwise the codes are staged through pinned host memory. ``recv`` decodes on the
destination. Both record CUDA-event timings in the handle like the reference. This is the
reference-shaped, host-synchronising seam; the pipeline hot path (``engine.DecodePipeline``,
``multistage``) fuses the same kernels into the stage step without host involvement.

The reference's opt-in rANS entropy stage (``entropy=True``) codes the payload's bytes
after compression; here it runs on the GPU (``dist.entropy``) in the reference's format, and
``recv`` inverts it on the destination GPU before decoding.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from .peer_routes import peer_route_allowed

_WIRE_BYTES_PER_S = 250e6  # the reference's modeled PCIe-1.0-x1 link, for theoretical_wire_ms

def _grouped(scheme: str) -> bool:
    """Schemes with one scale per 128-element group (the 4-bit ones)."""
    return scheme.startswith("int4") or scheme == "nf4"


_BARS: dict[str, tuple[float, float]] = {
    "fp16": (float("inf"), 1.0),
    "int8": (35.0, 0.999),
    "int8-had": (35.0, 0.999),
    "int4": (14.0, 0.98),
    "int4-had": (14.0, 0.98),
    "nf4": (16.0, 0.985),
}


def accuracy_report(original: torch.Tensor, reconstructed: torch.Tensor, scheme: str) -> dict:
    """SQNR (dB) / cosine of a round-trip against the scheme's bars
    (``superl8serve/dist/__init__.py:55-85``)."""
    x = original.detach().float().flatten()
    xr = reconstructed.detach().float().flatten()
    noise_power = (x - xr).pow(2).sum()
    if noise_power.item() == 0.0:
        sqnr_db = float("inf")
    else:
        sqnr_db = float(10.0 * torch.log10(x.pow(2).sum() / noise_power))
    cos = float(torch.nn.functional.cosine_similarity(x, xr, dim=0, eps=1e-12))
    sqnr_bar, cos_bar = _BARS.get(scheme, _BARS["int8"])
    return {"scheme": scheme, "sqnr_db": sqnr_db, "sqnr_bar": sqnr_bar,
            "sqnr_pass": sqnr_db >= sqnr_bar, "cos": cos, "cos_bar": cos_bar,
            "cos_pass": cos >= cos_bar}


@dataclass
class Compressed:
    scheme: str
    shape: tuple
    dtype: torch.dtype
    group_size: int | None
    payload: torch.Tensor
    scales: torch.Tensor
    d: int


def compress_activation(x: torch.Tensor, scheme: str = "int8", group_size: int | None = None,
                        *, payload: torch.Tensor | None = None,
                        scales: torch.Tensor | None = None) -> Compressed:
    """Encode x [..., d] (rows = all leading dims). payload/scales may be preallocated on
    another GPU (peer stores)."""
    if group_size not in (None, 128):
        raise ValueError("the s8b codec groups int4 / nf4 scales by 128")
    d = x.shape[-1]
    rows = x.reshape(-1, d).contiguous()
    pay, sc = ops.codec_encode(rows, None, scheme, payload=payload, scales=scales)
    if scheme == "fp16":
        sc = sc[:0]
    return Compressed(scheme, tuple(x.shape), x.dtype, 128 if _grouped(scheme) else None,
                      pay, sc, d)


def decompress_activation(c: Compressed) -> torch.Tensor:
    T = 1
    for s in c.shape[:-1]:
        T *= s
    sc = c.scales if c.scales.numel() else torch.empty(1, dtype=torch.float32,
                                                       device=c.payload.device)
    out, _ = ops.codec_decode(c.payload, sc, T, c.d, 0, c.scheme, c.dtype)
    return out.reshape(c.shape)


@dataclass
class TransferHandle:
    src_device: int
    dst_device: int
    scheme: str
    shape: torch.Size
    dtype: torch.dtype
    group_size: int | None
    d_payload: torch.Tensor
    d_scales: torch.Tensor
    compress_elapsed_ms: float
    p2p_elapsed_ms: float
    decompress_elapsed_ms: float | None = None
    used_p2p: bool = False
    entropy_freqs: object | None = None
    entropy_n: int | None = None
    entropy_payload_dtype: torch.dtype | None = None
    entropy_payload_shape: tuple | None = None

    @property
    def on_wire_bytes(self) -> int:
        payload = self.d_payload.numel() * self.d_payload.element_size()
        scales = self.d_scales.numel() * self.d_scales.element_size()
        freq = 0 if self.entropy_freqs is None else int(len(self.entropy_freqs)) * 2
        return payload + scales + freq

    @property
    def theoretical_wire_ms(self) -> float:
        return self.on_wire_bytes / _WIRE_BYTES_PER_S * 1000.0


def _can_use_p2p(src: int, dst: int) -> bool:
    allowed, _ = peer_route_allowed(src, dst)
    return allowed


def send(x: torch.Tensor, dst: int, *, scheme: str = "int8", group_size: int | None = None,
         entropy: bool = False) -> TransferHandle:
    """Compress x on its GPU and deliver the codes to GPU ``dst``
    (``superl8serve/dist/__init__.py:163-265``)."""
    if not x.is_cuda:
        raise RuntimeError("send() takes a CUDA tensor")
    if entropy:
        return _send_entropy(x, dst, scheme, group_size)
    src = x.device.index
    d = x.shape[-1]
    T = x.numel() // d
    nbytes, nsc = ops.codec_sizes(T, d, scheme)
    use_p2p = _can_use_p2p(src, dst)
    with torch.cuda.device(src):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if use_p2p:
            from .._lib import call

            call("s8b_enable_peer_access", src, dst)
            payload = torch.empty(nbytes, dtype=torch.uint8, device=dst)
            scales = torch.empty(max(nsc, 1), dtype=torch.float32, device=dst)
            start.record()
            c = compress_activation(x, scheme, group_size, payload=payload, scales=scales)
            end.record()
            end.synchronize()
            compress_ms = start.elapsed_time(end)
            p2p_ms = compress_ms  # the codes crossed NVLink inside the encoder
        else:
            start.record()
            c = compress_activation(x, scheme, group_size)
            end.record()
            end.synchronize()
            compress_ms = start.elapsed_time(end)
    if not use_p2p:
        with torch.cuda.device(dst):
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            hp = torch.empty(c.payload.shape, dtype=c.payload.dtype, pin_memory=True)
            hs = torch.empty(c.scales.shape, dtype=c.scales.dtype, pin_memory=True)
            hp.copy_(c.payload)
            hs.copy_(c.scales)
            t0.record()
            payload = hp.to(dst, non_blocking=True)
            scales = hs.to(dst, non_blocking=True)
            t1.record()
            t1.synchronize()
            p2p_ms = t0.elapsed_time(t1)
    else:
        payload, scales = c.payload, c.scales
    if scheme == "fp16":
        scales = scales[:0]
    return TransferHandle(src, dst, scheme, torch.Size(c.shape), c.dtype, c.group_size,
                          payload, scales[: (nsc if nsc else 0)], compress_ms, p2p_ms,
                          used_p2p=use_p2p)


def _send_entropy(x: torch.Tensor, dst: int, scheme: str, group_size) -> TransferHandle:
    """``send(..., entropy=True)`` (``superl8serve/dist/__init__.py:191-205``): compress on
    the source GPU, rANS-code the payload's bytes there, copy the coded bytes and the scales
    to ``dst``. The handle carries the frequency table and the payload's dtype and shape."""
    from . import entropy as ent

    src = x.device.index
    with torch.cuda.device(src):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        c = compress_activation(x, scheme, group_size)
        raw = c.payload.contiguous().view(torch.uint8).reshape(-1)
        coded, freqs, _ = ent.encode(raw)
        end.record()
        end.synchronize()
        compress_ms = start.elapsed_time(end)
    with torch.cuda.device(dst):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        payload = coded.to(f"cuda:{dst}")
        scales = c.scales.to(f"cuda:{dst}")
        t1.record()
        t1.synchronize()
        p2p_ms = t0.elapsed_time(t1)
    _, nsc = ops.codec_sizes(x.numel() // x.shape[-1], x.shape[-1], scheme)
    return TransferHandle(src, dst, scheme, torch.Size(c.shape), c.dtype, c.group_size,
                          payload, scales[: (nsc if nsc else 0)], compress_ms, p2p_ms,
                          used_p2p=_can_use_p2p(src, dst), entropy_freqs=freqs,
                          entropy_n=int(raw.numel()), entropy_payload_dtype=c.payload.dtype,
                          entropy_payload_shape=tuple(c.payload.shape))


def recv(handle: TransferHandle) -> torch.Tensor:
    """Decode the transferred codes on the destination GPU (``:268-302``); an entropy-coded
    payload is first rANS-decoded there, back to the payload's own dtype and shape."""
    payload = handle.d_payload
    if handle.entropy_freqs is not None and handle.entropy_n is not None:
        from . import entropy as ent

        with torch.cuda.device(handle.dst_device):
            raw = ent.decode(payload, handle.entropy_freqs, handle.entropy_n)
        payload = raw.view(handle.entropy_payload_dtype or torch.uint8)
        if handle.entropy_payload_shape is not None:
            payload = payload.reshape(handle.entropy_payload_shape)
    c = Compressed(handle.scheme, tuple(handle.shape), handle.dtype, handle.group_size,
                   payload, handle.d_scales, handle.shape[-1])
    with torch.cuda.device(handle.dst_device):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        xr = decompress_activation(c)
        t1.record()
        t1.synchronize()
        handle.decompress_elapsed_ms = t0.elapsed_time(t1)
    return xr
