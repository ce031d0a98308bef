"""Which (src, dst) GPU pairs may use peer-to-peer stores: a fail-closed policy.

Interface of the reference's ``superl8serve/dist/peer_routes.py`` (function names, the four
reason strings, ``ValueError`` on malformed specs), re-designed here as an ordered chain of
checks: the first check that fails names the reason, and a route passes only when every
check does.

* ``same-device``: src == dst needs no peer route.
* ``not-validated``: the unordered pair is not in the operator's validated set.
* ``no-peer-capability``: the driver does not report peer access (unknown counts as no).

The validated set is read from ``SUPERL8_P2P_VALIDATED_PAIRS`` (the name the reference's
documentation and tools use), else from ``FNI8_P2P_VALIDATED_PAIRS`` (the name its code
reads, ``superl8serve/dist/peer_routes.py:52``). Spec grammar: pairs separated by ``;``,
each pair two GPU indices separated by ``,``, whitespace ignored, e.g. ``"0,1; 1,2"``.
An unset or blank spec (or one made only of separators) validates nothing; any other
malformed spec raises ``ValueError``, so a typo never silently opens a route.
"""

from __future__ import annotations

import functools
import os
from typing import NamedTuple

import torch

VALIDATED_PAIRS_ENV = "SUPERL8_P2P_VALIDATED_PAIRS"
LEGACY_VALIDATED_PAIRS_ENV = "FNI8_P2P_VALIDATED_PAIRS"

ROUTE_P2P = "validated-p2p"
ROUTE_SAME_DEVICE = "same-device"
ROUTE_NOT_VALIDATED = "not-validated"
ROUTE_NO_CAPABILITY = "no-peer-capability"

Pair = tuple[int, int]


class RouteDecision(NamedTuple):
    """(allowed, reason); compares equal to the reference's plain tuple."""

    allowed: bool
    reason: str


def canonical_pair(a: int, b: int) -> Pair:
    """The unordered pair {a, b} as (low, high); both indices >= 0 and distinct."""
    if a < 0 or b < 0:
        raise ValueError(f"P2P pair ({a}, {b}) holds a negative GPU index")
    if a == b:
        raise ValueError(f"P2P pair ({a}, {b}) names the same GPU twice")
    return (min(a, b), max(a, b))


def _pair_from_text(text: str) -> Pair:
    fields = text.split(",")
    if len(fields) != 2 or not all(f.strip() for f in fields):
        raise ValueError(f"P2P pair {text.strip()!r} is not two comma-separated GPU indices")
    try:
        a, b = (int(f) for f in fields)
    except ValueError:
        raise ValueError(f"P2P pair {text.strip()!r} holds a non-integer GPU index") from None
    return canonical_pair(a, b)


@functools.lru_cache(maxsize=64)
def parse_validated_pairs(spec: str | None) -> frozenset[Pair]:
    """Spec text -> the set of validated unordered pairs (see the module docstring)."""
    elements = (spec or "").split(";")
    blank = [not e.strip() for e in elements]
    if all(blank):
        return frozenset()
    if any(blank):
        raise ValueError(f"P2P validated-pairs spec {spec!r} has an empty element between ';'")
    return frozenset(_pair_from_text(e) for e in elements)


def validated_pairs() -> frozenset[Pair]:
    """The validated set named by the environment (the first of the two variables set)."""
    for name in (VALIDATED_PAIRS_ENV, LEGACY_VALIDATED_PAIRS_ENV):
        spec = os.environ.get(name)
        if spec is not None:
            return parse_validated_pairs(spec)
    return frozenset()


def peer_capability(src: int, dst: int) -> bool:
    """Whether the driver reports that src can access dst's memory; False when it cannot
    say (no CUDA, an index out of range)."""
    try:
        return bool(torch.cuda.can_device_access_peer(src, dst))
    except (RuntimeError, AttributeError, AssertionError, ValueError):
        return False


def select_route(src: int, dst: int, *, validated: frozenset[Pair],
                 capability: bool | None) -> RouteDecision:
    """The policy itself, on explicit inputs (no environment, no driver query)."""
    checks = (
        (lambda: src != dst, ROUTE_SAME_DEVICE),
        (lambda: canonical_pair(src, dst) in validated, ROUTE_NOT_VALIDATED),
        (lambda: capability is True, ROUTE_NO_CAPABILITY),
    )
    for passes, reason in checks:
        if not passes():
            return RouteDecision(False, reason)
    return RouteDecision(True, ROUTE_P2P)


def peer_route_allowed(src: int, dst: int, *, capability: bool | None = None) -> RouteDecision:
    """``peer_route_allowed`` (``superl8serve/dist/peer_routes.py:167-180``): the policy over
    the environment's validated set and (unless given) the driver's peer capability."""
    if capability is None:
        capability = peer_capability(src, dst)
    return select_route(src, dst, validated=validated_pairs(), capability=capability)


def all_pairs_spec(devices) -> str:
    """Validated-pairs spec naming every pair of `devices` (an NVSwitch box: every GPU reaches
    every other at full bandwidth), for operators who qualify the whole box at once."""
    d = list(devices)
    return ";".join(f"{a},{b}" for i, a in enumerate(d) for b in d[i + 1:])
