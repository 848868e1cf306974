"""Public construction and loading API (independent of the CLI and tasks).

Reference parity: st/api.py:10-54.
"""
from __future__ import annotations

import torch

from .config import ExecutionConfig, ModelConfig
from .models.baseline import BaselineModel
from .models.stack import StackModel
from .runtime import checkpoint


def build_model(config=ModelConfig(), *, execution=ExecutionConfig(), device="cpu", dtype=None):
    """Build a Stack or baseline model directly on ``device`` (``"meta"`` allocates nothing)."""
    config = ModelConfig.from_dict(config)
    if isinstance(execution, dict):
        execution = ExecutionConfig(**execution)
    options = config.to_dict()
    kind = options.pop("model")
    with torch.device(device):
        if kind == "stack":
            model = StackModel(**options, backend=execution.backend,
                               checkpoint_chunks=execution.checkpoint_chunks,
                               encoder_chunk=execution.encoder_chunk, pos_chunk=execution.query_chunk,
                               loss_chunk=execution.loss_chunk,
                               attention_q_chunk=execution.attention_q_chunk,
                               attention_kv_chunk=execution.attention_kv_chunk)
        else:
            model = BaselineModel(**options, checkpoint_chunks=execution.checkpoint_chunks,
                                  loss_chunk=execution.loss_chunk, backend=execution.flash_attention)
    model.model_config = config
    if dtype is not None:
        model.to(dtype=dtype)
    return model


def load_model(path, *, device="cpu", dtype=None, execution=ExecutionConfig(), topk=None):
    """Weights of a trusted (new or legacy) checkpoint, in eval mode.

    The architecture always comes from the checkpoint; only the inference
    ``topk`` and execution settings may change.
    """
    state = checkpoint.load(path)
    options = dict(checkpoint.model_config(state))
    if topk is not None:
        if options.get("model", "stack") != "stack":
            raise ValueError("topk is a StackModel inference setting")
        options["topk"] = topk
    model = build_model(options, execution=execution, device=device)
    model.load_state_dict(state["model"], strict=True)
    if dtype is not None:
        model.to(dtype=dtype)
    return model.eval()
