"""Fail-closed GPU peer-route selection, with the reference's API and policy
(``superl8serve/dist/peer_routes.py``).

A route (src, dst) may use P2P only when src != dst, the unordered pair is in the validated
set and ``cudaDeviceCanAccessPeer`` is true. The validated set comes from
``SUPERL8_P2P_VALIDATED_PAIRS`` (the name the reference's docs and tools use) or, if that is
unset, ``FNI8_P2P_VALIDATED_PAIRS`` (the name its code reads, ``:52``); format ``"0,1;1,2"``.
Unset/empty means no pair is validated. Malformed specs raise ``ValueError``.
"""

from __future__ import annotations

import os

import torch

VALIDATED_PAIRS_ENV = "SUPERL8_P2P_VALIDATED_PAIRS"
LEGACY_VALIDATED_PAIRS_ENV = "FNI8_P2P_VALIDATED_PAIRS"

_VALIDATED_CACHE: dict[str, frozenset[tuple[int, int]]] = {}

_ROUTE_P2P = "validated-p2p"
_ROUTE_SAME_DEVICE = "same-device"
_ROUTE_NOT_VALIDATED = "not-validated"
_ROUTE_NO_CAPABILITY = "no-peer-capability"


def _normalize_pair(a: int, b: int) -> tuple[int, int]:
    if a < 0 or b < 0:
        raise ValueError(f"GPU index must be >= 0: ({a}, {b})")
    if a == b:
        raise ValueError(f"a peer pair cannot reference the same GPU: ({a}, {b})")
    return (a, b) if a < b else (b, a)


def parse_validated_pairs(spec: str | None) -> frozenset[tuple[int, int]]:
    if not spec or not spec.strip():
        return frozenset()
    chunks = [c.strip() for c in spec.split(";")]
    if all(not c for c in chunks):
        return frozenset()
    if any(not c for c in chunks):
        raise ValueError("malformed P2P validated-pairs spec: empty ';'-separated element")
    pairs: set[tuple[int, int]] = set()
    for chunk in chunks:
        parts = [p.strip() for p in chunk.split(",")]
        if len(parts) != 2 or not all(parts):
            raise ValueError(f"malformed P2P validated pair {chunk!r}; expected 'src,dst'")
        try:
            a, b = int(parts[0]), int(parts[1])
        except ValueError as exc:
            raise ValueError(
                f"malformed P2P validated pair {chunk!r}; indices must be integers") from exc
        pairs.add(_normalize_pair(a, b))
    return frozenset(pairs)


def _env_spec() -> str:
    v = os.environ.get(VALIDATED_PAIRS_ENV)
    return v if v is not None else os.environ.get(LEGACY_VALIDATED_PAIRS_ENV, "")


def validated_pairs() -> frozenset[tuple[int, int]]:
    spec = _env_spec()
    if spec not in _VALIDATED_CACHE:
        _VALIDATED_CACHE[spec] = parse_validated_pairs(spec)
    return _VALIDATED_CACHE[spec]


def _torch_can_peer(src: int, dst: int) -> bool:
    return bool(torch.cuda.can_device_access_peer(src, dst))


def peer_capability(src: int, dst: int) -> bool:
    try:
        return _torch_can_peer(src, dst)
    except (RuntimeError, AttributeError, AssertionError):
        return False


def select_route(src: int, dst: int, *, validated: frozenset[tuple[int, int]],
                 capability: bool | None) -> tuple[bool, str]:
    if src == dst:
        return False, _ROUTE_SAME_DEVICE
    pair = _normalize_pair(src, dst)
    if pair not in validated:
        return False, _ROUTE_NOT_VALIDATED
    if capability is not True:
        return False, _ROUTE_NO_CAPABILITY
    return True, _ROUTE_P2P


def peer_route_allowed(src: int, dst: int, *, capability: bool | None = None) -> tuple[bool, str]:
    if capability is None:
        capability = peer_capability(src, dst)
    return select_route(src, dst, validated=validated_pairs(), capability=capability)


def all_pairs_spec(devices) -> str:
    """Validated-pairs spec naming every pair of `devices` (an NVSwitch box: every GPU reaches
    every other at full bandwidth), for operators who qualify the whole box at once."""
    d = list(devices)
    return ";".join(f"{a},{b}" for i, a in enumerate(d) for b in d[i + 1:])
