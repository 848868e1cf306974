"""Host-side fault injection and failure detection.

Failures are injected on the host only: a chosen rank raises an exception
at a named point (before a collective, during a checkpoint write, in the
middle of a prefill). No GPU is ever made to fault, trap or hang. Tests run
these as CPU ``gloo`` ranks and check that every rank ends with an error
(the process-group timeout bounds the wait of the surviving ranks) and that
no partial file is left behind.

Configuration (environment, read at each call so tests can set it late)::

    EB200_FAULT=<point>[,<point>...]     points that fail
    EB200_FAULT_RANK=<rank>              only this global rank fails (default: any)
    EB200_FAULT_AFTER=<count>            skip the first <count> hits of a point
"""
from __future__ import annotations

import os
from collections import Counter

_hits: Counter = Counter()


class InjectedFault(RuntimeError):
    """Raised at an injection point selected by ``EB200_FAULT``."""


def _rank() -> int:
    return int(os.environ.get("RANK", "0"))


def maybe_fail(point: str) -> None:
    spec = os.environ.get("EB200_FAULT", "")
    if not spec or point not in {p.strip() for p in spec.split(",")}:
        return
    wanted = os.environ.get("EB200_FAULT_RANK")
    if wanted is not None and int(wanted) != _rank():
        return
    _hits[point] += 1
    if _hits[point] <= int(os.environ.get("EB200_FAULT_AFTER", "0")):
        return
    raise InjectedFault(f"injected fault at {point!r} on rank {_rank()}")


def reset() -> None:
    _hits.clear()
