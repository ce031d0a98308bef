"""rANS entropy stage on the GPU, in the wire format of the reference's
``superl8serve/dist/entropy.py`` (static byte-level rANS, frequencies normalised to 2^12,
32-bit state, final state flushed as 4 bytes).

``encode`` counts the symbols on the GPU (``s8b_rans_histogram``), normalises the 256-entry
table on the host exactly as the reference does (``_normalize_freqs``, ``entropy.py:54-91``:
the drift spread in ``np.argsort(-counts)`` order, so tied counts resolve the same way), and
codes on the GPU (``s8b_rans_encode``). With one stream the bytes are the reference's
``encode`` output, decodable by its ``decode``. ``n_streams > 1`` cuts the payload into equal
chunks coded as independent streams, one GPU thread each, for throughput; that layout carries
one length per stream and is this build's own. ``decode`` inverts either form on the GPU.
"""

from __future__ import annotations

import numpy as np
import torch

from .._lib import call, ptr, stream

SCALE_BITS = 12
M = 1 << SCALE_BITS


def normalize_freqs(counts) -> np.ndarray:
    """Raw symbol counts -> int32[256] summing to 2^12, every present symbol >= 1."""
    counts = np.asarray(counts, np.int64)
    total = int(counts.sum())
    freqs = np.zeros(256, np.int64)
    if total == 0:
        return freqs.astype(np.int32)
    present = counts > 0
    freqs[present] = np.maximum(counts[present] * M // total, 1)
    drift = M - int(freqs.sum())
    ranked = np.argsort(-counts)
    n_present = int(present.sum())
    i = 0
    while drift:
        s = ranked[i % n_present]
        if drift > 0:
            freqs[s] += 1
            drift -= 1
        elif freqs[s] > 1:
            freqs[s] -= 1
            drift += 1
        i += 1
    return freqs.astype(np.int32)


def _lib_size(name: str, *args) -> int:
    from .._lib import load

    return int(getattr(load(), name)(*args))


def encode(data: torch.Tensor, n_streams: int = 1):
    """data: CUDA uint8 [n]. Returns (encoded CUDA uint8, freqs int32[256] numpy, stream
    lengths CUDA int64 [n_streams]). With one stream the encoded tensor is exactly the
    reference's byte stream (empty for an empty input)."""
    data = data.contiguous().view(torch.uint8).reshape(-1)
    n = data.numel()
    dev = data.device
    if n == 0:
        return (torch.zeros(0, dtype=torch.uint8, device=dev), np.zeros(256, np.int32),
                torch.zeros(1, dtype=torch.int64, device=dev))
    n_streams = max(1, min(n_streams, n))
    counts = torch.empty(256, dtype=torch.int32, device=dev)
    call("s8b_rans_histogram", ptr(data), n, ptr(counts), stream(dev))
    freqs = normalize_freqs(counts.cpu().numpy().astype(np.int64))
    f_dev = torch.from_numpy(freqs).to(dev)
    cap = _lib_size("s8b_rans_encoded_capacity", n, n_streams)
    out = torch.empty(cap, dtype=torch.uint8, device=dev)
    lens = torch.empty(n_streams, dtype=torch.int64, device=dev)  # -1: uncodable symbol
    call("s8b_rans_encode", ptr(data), n, ptr(f_dev), n_streams, ptr(out), cap, ptr(lens),
         stream(dev))
    host_lens = lens.cpu()
    if int(host_lens.min()) < 0 or int(host_lens.max()) > cap:
        raise RuntimeError("rANS encode: a symbol has no frequency")
    if n_streams == 1:
        return out[: int(host_lens[0])].clone(), freqs, lens
    return out, freqs, lens


def decode(enc: torch.Tensor, freqs, n: int, *, lengths: torch.Tensor | None = None,
           n_streams: int = 1) -> torch.Tensor:
    """Inverse of ``encode`` on enc's device. ``lengths`` (per-stream byte counts) is needed
    for more than one stream; one stream takes the whole tensor."""
    dev = enc.device
    if n == 0:
        return torch.zeros(0, dtype=torch.uint8, device=dev)
    f = np.asarray(freqs, np.int64)
    if f.shape != (256,) or int(f.sum()) != M or (f < 0).any():
        raise ValueError("rANS frequency table must hold 256 non-negative entries summing to 4096")
    if lengths is None:
        if n_streams != 1:
            raise ValueError("multi-stream decode needs the per-stream lengths")
        lengths = torch.tensor([enc.numel()], dtype=torch.int64, device=dev)
    n_streams = lengths.numel()
    if enc.numel() < _lib_size("s8b_rans_stream_offset", n, n_streams, n_streams - 1):
        raise ValueError("encoded buffer shorter than its stream layout")
    f_dev = torch.from_numpy(f.astype(np.int32)).to(dev)
    out = torch.empty(n, dtype=torch.uint8, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    lens = lengths.to(device=dev, dtype=torch.int64).contiguous()
    if n_streams > 1:
        # every stream's bytes must lie inside the buffer
        offs = [_lib_size("s8b_rans_stream_offset", n, n_streams, i) for i in range(n_streams)]
        ends = torch.tensor(offs, dtype=torch.int64) + lens.cpu()
        if int(ends.max()) > enc.numel():
            raise ValueError("rANS stream lengths run past the encoded buffer")
    elif int(lens[0].item()) > enc.numel():
        raise ValueError("rANS stream length runs past the encoded buffer")
    call("s8b_rans_decode", ptr(enc.contiguous()), ptr(lens), n_streams, ptr(f_dev), n, ptr(out),
         ptr(bad), stream(dev))
    if int(bad.item()):
        raise RuntimeError("rANS decode: stream ended early (corrupt payload or wrong table)")
    return out
