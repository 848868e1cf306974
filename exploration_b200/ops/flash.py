"""Causal SDPA for the dense baseline Transformer.

The baseline is the comparator model, so it deliberately runs PyTorch's own
``scaled_dot_product_attention`` (FlashAttention / memory-efficient / math,
chosen by PyTorch) rather than kernels of this framework
(reference: st/ops/flash.py:34-70).
"""
from __future__ import annotations

from contextlib import nullcontext

import torch
from torch.nn import functional as F

MODES = ("auto", "flash", "math")


def _sdpa_context(mode: str):
    if mode == "auto":
        return nullcontext()
    if mode not in MODES:
        raise ValueError("attention mode must be auto, flash or math")
    from torch.nn.attention import SDPBackend, sdpa_kernel
    return sdpa_kernel(SDPBackend.FLASH_ATTENTION if mode == "flash" else SDPBackend.MATH)


def flash_attention(q, k, v, *, is_causal=False, attn_mask=None, dropout_p=0.0, mode="auto",
                    enable_gqa=False):
    """SDPA over ``[batch, heads, sequence, head_dim]`` tensors."""
    if dropout_p < 0:
        raise ValueError("dropout_p must be non-negative")
    with _sdpa_context(mode):
        return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, dropout_p=dropout_p,
                                              is_causal=is_causal, enable_gqa=enable_gqa)


def backend_info(device=None, dtype=None) -> dict:
    device = torch.device(device or "cpu")
    info = {"device": str(device), "dtype": None if dtype is None else str(dtype),
            "implementation": "torch-scaled-dot-product-attention"}
    if device.type == "cuda":
        info.update(flash_enabled=bool(torch.backends.cuda.flash_sdp_enabled()),
                    mem_efficient_enabled=bool(torch.backends.cuda.mem_efficient_sdp_enabled()),
                    math_enabled=bool(torch.backends.cuda.math_sdp_enabled()))
        try:
            info["flash_available"] = bool(torch.backends.cuda.is_flash_attention_available())
        except AttributeError:
            info["flash_available"] = None
    else:
        info.update(flash_enabled=False, mem_efficient_enabled=False, math_enabled=True,
                    flash_available=False)
    return info
