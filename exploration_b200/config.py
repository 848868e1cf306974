"""Serializable model and execution configuration.

Two frozen dataclasses describe everything needed to rebuild a model:

* ``ModelConfig`` is the architecture. It is stored in every checkpoint and
  is the only source of truth when a checkpoint is loaded.
* ``ExecutionConfig`` selects how a model executes (kernel backend, chunk
  sizes, recomputation). It never changes the function being computed.

Field names and defaults follow the reference contract
(st/config.py:5-69) so JSON configs and checkpoints written by either
framework load in the other.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, fields
from numbers import Integral

MODEL_KINDS = ("stack", "baseline")
# "cuda" is this framework's native sm_100a path. "triton" is accepted as a
# synonym so configs and command lines written for the reference keep
# working; no Triton code exists here.
BACKENDS = ("auto", "torch", "cuda", "triton")
SDPA_MODES = ("auto", "flash", "math")

_STACK_ONLY = ("arch", "block_size", "topk")
_BASELINE_ONLY = ("layers",)


def canonical_backend(name: str) -> str:
    """Map a user-facing backend name onto the two real code paths."""
    if name not in BACKENDS:
        raise ValueError(f"backend must be one of {BACKENDS}, got {name!r}")
    return "cuda" if name == "triton" else name


@dataclass(frozen=True)
class ModelConfig:
    model: str = "stack"
    vocab_size: int = 128
    dim: int = 256
    heads: int = 4
    block_size: int = 16
    topk: int = 64
    arch: str = "Lx2,G"
    ffn_ratio: float = 4.0
    layers: int = 3

    @classmethod
    def from_dict(cls, value) -> "ModelConfig":
        if isinstance(value, cls):
            return value
        known = {f.name for f in fields(cls)}
        extra = set(value) - known
        if extra:
            raise ValueError(f"unknown model configuration keys: {sorted(extra)}")
        return cls(**value)

    def to_dict(self) -> dict:
        """Drop the fields that do not apply to this model kind."""
        out = asdict(self)
        if self.model == "stack":
            for key in _BASELINE_ONLY:
                out.pop(key)
        elif self.model == "baseline":
            for key in _STACK_ONLY:
                out.pop(key)
        else:
            raise ValueError(f"model must be one of {MODEL_KINDS}")
        return out


def _positive_int(value) -> bool:
    return isinstance(value, Integral) and not isinstance(value, bool) and value >= 1


@dataclass(frozen=True)
class ExecutionConfig:
    backend: str = "auto"
    checkpoint_chunks: bool = True
    encoder_chunk: int = 1024
    query_chunk: int = 0          # 0: the model picks a memory-bounded tile
    loss_chunk: int = 128
    flash_attention: str = "auto"  # baseline SDPA selection
    attention_q_chunk: int = 128   # bounded torch-reference tiles
    attention_kv_chunk: int = 4096

    def __post_init__(self):
        canonical_backend(self.backend)
        if self.flash_attention not in SDPA_MODES:
            raise ValueError(f"flash_attention must be one of {SDPA_MODES}")
        for name in ("encoder_chunk", "loss_chunk", "attention_q_chunk", "attention_kv_chunk"):
            if not _positive_int(getattr(self, name)):
                raise ValueError("execution chunk sizes must be positive integers")
        q = self.query_chunk
        if not isinstance(q, Integral) or isinstance(q, bool) or q < 0:
            raise ValueError("query_chunk must be a non-negative integer (0 = auto)")

    def to_dict(self) -> dict:
        return asdict(self)
