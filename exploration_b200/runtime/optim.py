"""Optimizers: fused multi-tensor AdamW for CUDA, ZeRO-1 sharding for DP.

``FusedAdamW`` keeps PyTorch's AdamW state layout (``step``, ``exp_avg``,
``exp_avg_sq`` per parameter and the standard ``param_groups``), so its state
dict is interchangeable with ``torch.optim.AdamW`` in checkpoints. On CUDA
one kernel of the extension (``csrc/fused/loss_optim.cu``) updates every fp32
master parameter of a group: decoupled weight decay, both moment updates,
bias correction and the optional gradient-clipping scale are one pass over
memory. CPU parameters use the same arithmetic in torch.

The engine uses ``torch.optim.AdamW`` on CPU, exactly like the reference
(st/runtime/engine.py:88-119), so CPU runs are the reference's numerics.
"""
from __future__ import annotations

import math

import torch
from torch.autograd.graph import increment_version
from torch.optim import Optimizer

from ..ops import _native
from ..ops.launch import record


class FusedAdamW(Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2):
        if lr < 0 or eps < 0 or not 0 <= betas[0] < 1 or not 0 <= betas[1] < 1:
            raise ValueError("invalid AdamW hyper-parameters")
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=False,
                        maximize=False, foreach=None, capturable=False, differentiable=False,
                        fused=None)
        super().__init__(params, defaults)
        self.grad_scale = 1.0     # multiplies every gradient inside the update (clipping)

    def _init_state(self, p):
        state = self.state[p]
        if not state:
            state["step"] = torch.tensor(0.0)
            state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
        return state

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group in self.param_groups:
            beta1, beta2 = group["betas"]
            by_step: dict = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("FusedAdamW does not support sparse gradients")
                state = self._init_state(p)
                state["step"] += 1
                key = (float(state["step"]), p.device)
                by_step.setdefault(key, []).append(p)
            for (step, device), params in by_step.items():
                bc1 = 1 - beta1 ** step
                bc2 = 1 - beta2 ** step
                if device.type == "cuda":
                    self._cuda_update(params, group, bc1, bc2)
                else:
                    self._torch_update(params, group, bc1, bc2)
        return loss

    def _torch_update(self, params, group, bc1, bc2):
        lr, wd, eps = group["lr"], group["weight_decay"], group["eps"]
        beta1, beta2 = group["betas"]
        for p in params:
            state = self.state[p]
            grad = p.grad * self.grad_scale if self.grad_scale != 1.0 else p.grad
            p.mul_(1 - lr * wd)
            state["exp_avg"].lerp_(grad, 1 - beta1)
            state["exp_avg_sq"].mul_(beta2).addcmul_(grad, grad, value=1 - beta2)
            denom = (state["exp_avg_sq"].sqrt() / math.sqrt(bc2)).add_(eps)
            p.addcdiv_(state["exp_avg"], denom, value=-lr / bc1)

    def _cuda_update(self, params, group, bc1, bc2):
        ext = _native.native(params[0])
        for p in params:
            if p.dtype != torch.float32 or not p.is_contiguous() or not p.grad.is_contiguous():
                raise ValueError("FusedAdamW expects contiguous fp32 master parameters and grads")
        beta1, beta2 = group["betas"]
        ext.adamw_step(params, [p.grad for p in params],
                       [self.state[p]["exp_avg"] for p in params],
                       [self.state[p]["exp_avg_sq"] for p in params],
                       float(group["lr"]), float(beta1), float(beta2), float(group["eps"]),
                       float(group["weight_decay"]), float(bc1), float(bc2), float(self.grad_scale))
        # The kernel writes through raw pointers; bump the version counters so
        # caches keyed on them (the bf16 weight copies) see the update.
        for p in params:
            increment_version(p)
        record("adamw_step", tensors=len(params))


def build_optimizer(model, args, parallel, device):
    """AdamW for the engine: fused on CUDA, torch on CPU, ZeRO-1 over DP when asked."""
    kwargs = dict(lr=args.lr, betas=(0.9, 0.95), weight_decay=args.weight_decay)
    if device.type == "cuda":
        cls = FusedAdamW
    else:
        cls = torch.optim.AdamW
        kwargs["foreach"] = False
    if args.optimizer_shard and parallel.world_size > 1:
        from torch.distributed.optim import ZeroRedundancyOptimizer
        return ZeroRedundancyOptimizer(model.parameters(), optimizer_class=cls, **kwargs)
    return cls(model.parameters(), **kwargs)
