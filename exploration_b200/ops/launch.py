"""Record of the native kernel configurations used by this process.

The reference retried Triton launches on ``OutOfResources`` and kept a
report of the chosen tiles (st/ops/kernels/launch.py:20-98). sm_100a kernels
here have static tile configurations chosen at compile time, so there is
nothing to retry: a configuration either exists for a shape or the op
raises before launch. What remains useful is the report: which kernel ran,
with which tile, and its compiled resource use, read from
``cudaFuncGetAttributes`` by the extension.
"""
from __future__ import annotations

import threading

_lock = threading.Lock()
_records: dict = {}


def record(kernel: str, **config) -> None:
    """Remember one launch configuration (idempotent per configuration)."""
    key = (kernel, tuple(sorted(config.items())))
    with _lock:
        if key in _records:
            _records[key]["calls"] += 1
            return
        entry = {"kernel": kernel, "calls": 1, **config}
        _records[key] = entry
    try:
        from . import _native
        module = _native.load(required=False)
        if module is not None and hasattr(module, "kernel_attributes"):
            entry["attributes"] = module.kernel_attributes(kernel)
    except Exception as exc:  # reporting must never break a launch
        entry["attributes_error"] = str(exc)


def launch_report() -> list:
    with _lock:
        return [dict(v) for v in _records.values()]


def reset() -> None:
    with _lock:
        _records.clear()
