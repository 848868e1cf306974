"""``st``: the reference's package name, served by :mod:`exploration_b200`.

Every module of ``exploration_b200`` is also importable as ``st.<same path>``
(``st.models.stack``, ``st.ops.attention``, ...), and the reference's flat
legacy aliases (``st.blocks``, ``st.stack_model``, ``st.attention``, ...,
reference: st/__init__.py:20-30) point at the same module objects. No code
lives here; there is exactly one implementation.
"""
import importlib
import pkgutil
import sys

import exploration_b200 as _impl
from exploration_b200 import *  # noqa: F401,F403
from exploration_b200 import __all__, __version__  # noqa: F401

_LEGACY = {
    "blocks": "models.blocks", "stack_model": "models.stack", "baseline": "models.baseline",
    "attention": "ops.attention", "sparse": "ops.sparse", "flash": "ops.flash",
    "checkpoint": "runtime.checkpoint", "inference": "runtime.inference",
    "parallel": "parallel.context", "memory": "runtime.memory", "token_data": "data.tokens",
    "runtime.parallel": "parallel.context",
}


def _alias_all():
    prefix = _impl.__name__ + "."
    for info in pkgutil.walk_packages(_impl.__path__, prefix):
        if info.name.endswith("__main__"):
            continue
        module = importlib.import_module(info.name)
        sys.modules["st." + info.name[len(prefix):]] = module
    for alias, target in _LEGACY.items():
        sys.modules["st." + alias] = importlib.import_module(prefix + target)
    for name in ("models", "ops", "runtime", "data", "tools", "parallel", "cli", "config",
                 "api"):
        globals()[name] = sys.modules["st." + name]
    for alias in ("blocks", "stack_model", "baseline", "attention", "sparse", "flash", "checkpoint",
                  "inference", "memory", "token_data"):
        globals()[alias] = sys.modules["st." + alias]
    globals()["parallel"] = sys.modules["st.parallel"]


_alias_all()
from exploration_b200.cli import main  # noqa: E402,F401
