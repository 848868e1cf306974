"""exploration_b200: a Blackwell (sm_100a)-native Stack framework.

Public API (reference parity: st/__init__.py:5-18)::

    from exploration_b200 import (StackModel, BaselineModel, ModelConfig, ExecutionConfig,
                                  build_model, load_model, InferenceSession, ParallelContext,
                                  TokenDataset, flash_attention, backend_info,
                                  MetricAccumulator, parse_bucket_edges, tail_mask)

The same package is importable as ``st`` (``python -m st ...``), the
reference's package name, so existing commands and imports keep working.
"""
from .api import build_model, load_model
from .config import ExecutionConfig, ModelConfig
from .data.tokens import TokenDataset
from .models.baseline import BaselineModel
from .models.stack import StackModel
from .ops.flash import backend_info, flash_attention
from .parallel.context import ParallelContext
from .runtime.inference import InferenceSession
from .runtime.metrics import MetricAccumulator, parse_bucket_edges, tail_mask

__version__ = "0.1.0"
__all__ = ["StackModel", "BaselineModel", "ModelConfig", "ExecutionConfig", "build_model",
           "load_model", "InferenceSession", "ParallelContext", "TokenDataset", "flash_attention",
           "backend_info", "MetricAccumulator", "parse_bucket_edges", "tail_mask"]
