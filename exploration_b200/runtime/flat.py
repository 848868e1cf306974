"""Flat parameter storage, flat AdamW and the CUDA-graph training step.

``FlatParameters`` moves every trainable parameter into one fp32 buffer
(parameters become views), gradients into a second one and keeps a bf16
shadow of the masters for the GEMMs. That makes three things one kernel or
one collective each: the gradient reduction across ranks (one NCCL
all-reduce, or reduce-scatter + all-gather under ZeRO-1), the gradient norm
and the AdamW update (``csrc/fused/flat_optim.cu``), which also refreshes
the bf16 shadow, so no per-step weight casts remain.

``GraphTrainer`` captures one whole training micro-step (input copies from
pinned memory, forward, backward, gradient reduction, clipping, AdamW and
the statistics copy back to pinned memory) in a CUDA graph after two eager
steps, then replays it. The step is host-sync free: the supervised width is
the full shard (no data-dependent ``width``), the non-finite check and the
clip coefficient are evaluated on the device (a non-finite step is skipped
by the optimizer kernel and reported after the replay, as the eager path
raises before applying it), and the learning rate and step count are read
from device memory refreshed by an in-graph copy.

Across GPUs of one node the gradient reduction runs over NVLink peer memory
(``PeerGradBuckets``, kernels in ``csrc/comm/grad_reduce.cu``): the flat
gradient and the bf16 shadow live in a symmetric heap, each bucket is
reduce-scattered by one kernel as soon as backward completes it (every rank
pulls its slice of the bucket from all peers; the gradient-norm partials
come out of the same pass), and the ZeRO-1 update writes the new bf16
weights straight into every rank's shadow. ``EB200_P2P_GRAD=0`` selects the
NCCL path (``GradBuckets``: bucketed all-reduce, then an all-gather of the
shadows).

The reference trains eagerly with DDP and torch AdamW
(st/runtime/engine.py:85-119,160-190); it has no graph capture.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops import _native, fused
from ..ops import gemm as G
from . import trace

ALIGN = 64            # elements: 256-byte aligned parameter views


class FlatParameters:
    """One fp32 buffer for the masters, one for gradients, a bf16 shadow.

    Layout: ``[replicated | sharded]``. Parameters the model reads in fp32
    (norms, biases, embeddings: anything that is not only a GEMM operand) come
    first and are updated on every rank; the GEMM weights follow and, under
    ZeRO-1, each rank updates only its equal slice of them, after which the
    bf16 shadows (all the forward pass reads of those weights) are
    all-gathered. Their fp32 masters are gathered only when a checkpoint
    needs them (``gather_masters``).
    """

    def __init__(self, model: torch.nn.Module, device: torch.device, shards: int = 1, peer_group=None):
        """``peer_group``: place the gradient and the shadow in a symmetric heap over
        that group (collective), so peer kernels can reach every rank's copy."""
        params = [p for p in model.parameters() if p.requires_grad]
        fp32_read = {id(m.weight) for m in model.modules() if isinstance(m, torch.nn.Embedding)}
        norm_ids = {id(t) for m in model.modules() if isinstance(m, torch.nn.LayerNorm)
                    for t in (m.weight, m.bias) if t is not None}
        norm_ids |= {id(m.bias) for m in model.modules() if isinstance(m, torch.nn.Linear) and m.bias is not None}
        small = [p for p in params if p.dim() < 2 or id(p) in fp32_read]
        big = [p for p in params if not (p.dim() < 2 or id(p) in fp32_read)]
        self.params = small + big
        quantum = ALIGN * max(1, shards)
        offsets, total = [], 0
        for i, p in enumerate(self.params):
            if i == len(small):
                total = -(-total // quantum) * quantum
            offsets.append(total)
            total += -(-p.numel() // ALIGN) * ALIGN
        if not big:
            total = -(-total // quantum) * quantum
        self.norm_ids = norm_ids
        self.split = offsets[len(small)] if big else total
        total = self.split + -(-(total - self.split) // quantum) * quantum
        self.total, self.offsets = total, offsets
        self.data = torch.zeros(total, device=device, dtype=torch.float32)
        self.heap = None
        if peer_group is not None:
            from ..parallel.symmetric import SymmetricHeap
            ext = _native.load(required=True)
            extra = ext.heap_signal_bytes() + ext.grad_flag_bytes() + 4096
            self.heap = SymmetricHeap(peer_group, device, total * 6 + extra)
            self.grad_offset = self.heap.alloc(total * 4)
            self.shadow_offset = self.heap.alloc(total * 2)
            self.grad = self.heap.tensor(self.grad_offset, [total], torch.float32)
            self.shadow = self.heap.tensor(self.shadow_offset, [total], torch.bfloat16)
            self.grad.zero_()
        else:
            self.grad = torch.zeros(total, device=device, dtype=torch.float32)
            self.shadow = torch.zeros(total, device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            for p, off in zip(self.params, offsets):
                view = self.data[off:off + p.numel()].view_as(p)
                view.copy_(p.detach())
                p.data = view
                p.grad = self.grad[off:off + p.numel()].view_as(p)
            self.shadow.copy_(self.data)
        for p, off in zip(self.params, offsets):
            fused.register_shadow(p, self.shadow[off:off + p.numel()].view_as(p))

    def zero_grad(self) -> None:
        self.grad.zero_()

    def sink_params(self):
        """Parameters whose gradients the native ops add straight into ``param.grad``: the
        GEMM weights (sharded region), the LayerNorm weights and biases and the linear
        layers' biases."""
        return [p for p, off in zip(self.params, self.offsets)
                if (off >= self.split and p.dim() == 2) or id(p) in self.norm_ids]

    def release(self) -> None:
        for p in self.params:
            fused._shadows.pop(id(p), None)
            G.remove_grad_sink(p)
            if self.heap is not None:
                p.grad = None                      # the heap memory goes away below
        if self.heap is not None:
            self.heap.close()                      # collective
            self.heap = None


def _bucket_bounds(flat: FlatParameters, bucket_bytes: int, split_boundary: bool):
    """Contiguous gradient buckets on parameter boundaries, and the bucket of each parameter."""
    limit = max(1, bucket_bytes // 4)
    bounds, owner, lo = [], {}, 0
    for p, off in zip(flat.params, flat.offsets):
        end = off + -(-p.numel() // ALIGN) * ALIGN
        if off > lo and (end - lo > limit or (split_boundary and off == flat.split)):
            bounds.append((lo, off))
            lo = off
        owner[id(p)] = len(bounds)
    if split_boundary and lo < flat.split < flat.total:
        bounds.append((lo, flat.split))
        lo = flat.split
    bounds.append((lo, flat.total))
    return bounds, owner


class ShardLayout:
    """Which rank updates which part of the sharded region under ZeRO-1.

    ``groups`` holds ``(lo, hi, q)``: rank ``r`` owns ``[lo + r*q, min(lo + (r+1)*q,
    hi))`` of every group. One group over the whole sharded region is the
    contiguous layout (one equal slice per rank); one group per gradient
    bucket is the layout of the peer-memory reduction, where every rank owns a
    slice of every bucket so that all ranks pull a bucket in parallel.
    """

    def __init__(self, groups, world: int, rank: int):
        self.groups, self.world, self.rank = list(groups), world, rank

    @staticmethod
    def part(group, r):
        lo, hi, q = group
        a = min(hi, lo + r * q)
        return a, min(hi, a + q) - a

    def owned(self):
        return [s for s in (self.part(g, self.rank) for g in self.groups) if s[1] > 0]

    def size(self) -> int:
        return sum(n for _, n in self.owned())

    def gather_(self, buf: torch.Tensor, group=None) -> None:
        """Collective: every rank's owned parts of the flat buffer ``buf`` reach all ranks."""
        for g in self.groups:
            lo, hi, q = g
            a, n = self.part(g, self.rank)
            if hi - lo == self.world * q:
                mine = buf[a:a + q]
                dist.all_gather_into_tensor(buf[lo:hi], mine if mine.is_cuda else mine.clone(), group=group)
                continue
            mine = buf.new_zeros(q)
            mine[:n] = buf[a:a + n]
            full = buf.new_zeros(self.world * q)
            dist.all_gather_into_tensor(full, mine, group=group)
            buf[lo:hi] = full[:hi - lo]


def bucket_layout(flat: FlatParameters, bounds, world: int, rank: int, shard: bool):
    """Per-bucket slices ``(q, all_reduce)`` and, when sharded, the ``ShardLayout`` they imply.

    Every bucket is cut into ``world`` slices of ``q`` elements (a multiple of
    ``ALIGN``); buckets of the replicated region, or all buckets when the
    optimizer is not sharded, are all-reduced.
    """
    quantum = ALIGN * world
    slices, groups = [], []
    for lo, hi in bounds:
        q = -(-(hi - lo) // quantum) * ALIGN
        all_reduce = hi <= flat.split or not shard
        slices.append((q, all_reduce))
        if not all_reduce:
            groups.append((lo, hi, q))
    return slices, (ShardLayout(groups, world, rank) if shard else None)


class _BucketCountdown:
    """Counts parameters down per bucket and launches complete buckets last to first.

    A parameter reports each gradient contribution through a post-accumulate
    hook or, for GEMM weights whose gradient the GEMM adds straight into
    ``param.grad``, through the grad-sink callback
    (``ops.gemm.register_grad_sink``). A parameter can receive several
    contributions per step (a tied embedding: the lookup and every loss
    chunk of the head; a weight applied per chunk), so the first step only
    counts them and reduces everything at ``finish()``; later steps launch a
    bucket once all of its contributions have arrived. Buckets are launched
    strictly from the last one down, so every rank issues the same sequence
    whatever order its hooks fire in; ``finish()`` launches what is left.
    Inside graph capture the hooks run once and the launches are recorded.
    """

    def __init__(self, flat: FlatParameters, bucket_bytes: int, split_boundary: bool = False):
        self.flat = flat
        self.bounds, self.owner = _bucket_bounds(flat, bucket_bytes, split_boundary)
        self.count = None                          # contributions per bucket, learned in the first step
        self.handles = [p.register_post_accumulate_grad_hook(self._hook) for p in flat.params]
        for p in flat.sink_params():
            G.register_grad_sink(p, self._hook)
        self.active = False

    def start(self) -> None:
        self.counting = self.count is None
        self.pending = [0] * len(self.bounds) if self.counting else list(self.count)
        self.ready = [not self.counting and c == 0 for c in self.pending]
        self.next = len(self.bounds) - 1
        self.active = True

    def _launch(self, index: int) -> None:
        raise NotImplementedError

    def _launch_ready(self) -> None:
        while self.next >= 0 and self.ready[self.next]:
            self._launch(self.next)
            self.next -= 1

    def _hook(self, param) -> None:
        if not self.active:
            return
        b = self.owner[id(param)]
        if self.counting:
            self.pending[b] += 1
            return
        self.pending[b] -= 1
        if self.pending[b] == 0:
            self.ready[b] = True
            self._launch_ready()

    def _flush(self) -> None:
        if self.counting:
            self.count = list(self.pending)
            self.counting = False
        self.ready = [True] * len(self.bounds)
        self._launch_ready()
        self.active = False

    def remove(self) -> None:
        for h in self.handles:
            h.remove()
        for p in self.flat.params:
            G.remove_grad_sink(p)


class GradBuckets(_BucketCountdown):
    """NCCL all-reduce of the flat gradient in contiguous buckets, overlapped with backward."""

    def __init__(self, flat: FlatParameters, group=None, bucket_bytes: int = 32 << 20):
        super().__init__(flat, bucket_bytes)
        self.group = group

    def start(self) -> None:
        super().start()
        self.works = []

    def _launch(self, index: int) -> None:
        lo, hi = self.bounds[index]
        self.works.append(dist.all_reduce(self.flat.grad[lo:hi], group=self.group, async_op=True))

    def finish(self, hyper=None) -> None:
        self._flush()
        for work in self.works:
            work.wait()
        self.works = []


class PeerGradBuckets(_BucketCountdown):
    """Gradient reduction over NVLink peer memory, one kernel per bucket during backward.

    Needs ``flat`` built with a ``peer_group`` (gradient and shadow in a
    symmetric heap). Bucket ``b`` = ``[lo, hi)`` is cut into one slice per
    rank (``q`` elements, a multiple of 64); ``grad_reduce_bucket`` on a side
    stream reduces this rank's slice from every rank as soon as the bucket is
    complete here, and waits on the device (bounded) for the peers to complete
    theirs. Buckets of the replicated region (and every bucket when the
    optimizer is not sharded) are all-reduced: the owner stores the sum into
    every rank's buffer. Sharded buckets are reduce-scattered: the owner keeps
    the sum, and ``layout`` (one group per bucket) tells the optimizer which
    slices this rank updates. ``finish(hyper)`` ends with the norm exchange,
    which leaves the global squared gradient norm in ``hyper[3]``.
    """

    CTAS = 64      # CTAs of 256 threads per bucket kernel (it shares the SMs with the backward)

    def __init__(self, flat: FlatParameters, shard: bool, bucket_bytes: int = 32 << 20):
        if flat.heap is None:
            raise ValueError("PeerGradBuckets needs the flat buffers in a symmetric heap")
        heap = flat.heap
        self.heap, self.ext = heap, heap.ext
        self.world, self.rank = heap.world, heap.rank
        max_buckets = self.ext.grad_reduce_max_buckets()
        bucket_bytes = max(bucket_bytes, -(-flat.total * 4 // (max_buckets - 4)))
        super().__init__(flat, bucket_bytes, split_boundary=True)
        self.slices, self.layout = bucket_layout(flat, self.bounds, self.world, self.rank, shard)
        self.flag_offset = heap.alloc(self.ext.grad_flag_bytes())
        self.grad_ptrs = heap.peer_ptrs(flat.grad_offset)
        self.flag_ptrs = heap.peer_ptrs(self.flag_offset)
        device = flat.grad.device
        self.partials = torch.zeros(len(self.bounds) * self.CTAS, device=device)
        self.stream = torch.cuda.Stream(device)
        from ..parallel.symmetric import barrier_timeout_s
        self.timeout = barrier_timeout_s()

    def _launch(self, index: int) -> None:
        lo, hi = self.bounds[index]
        q, all_reduce = self.slices[index]
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self.ext.grad_reduce_bucket(self.grad_ptrs, self.flag_ptrs, self.rank, index, lo, hi, q, all_reduce,
                                        1.0, self.partials[index * self.CTAS:(index + 1) * self.CTAS],
                                        self.timeout)

    def finish(self, hyper) -> None:
        self._flush()
        with torch.cuda.stream(self.stream):
            self.ext.grad_norm_exchange(self.partials, self.flag_ptrs, self.rank, hyper, self.timeout)
        torch.cuda.current_stream().wait_stream(self.stream)

    def shadow_ptrs(self, lo: int) -> list[int]:
        """Every rank's address of shadow element ``lo``."""
        return self.heap.peer_ptrs(self.flat.shadow_offset + lo * 2)

    def barrier(self) -> None:
        self.heap.barrier()


class FlatAdamW:
    """AdamW over a flat buffer; under ZeRO-1 over this rank's slice of the sharded region.

    Hyper-parameters that change per step live in ``hyper`` on the device:
    ``[lr, step, max_norm, grad_sq_norm]``.
    """

    def __init__(self, flat: FlatParameters, lr: float, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.0, max_norm: float = 0.0, group=None, shard: bool = False,
                 shadow_only: bool = False, layout: ShardLayout | None = None):
        """``shadow_only``: the model reads the sharded weights only through their bf16
        shadows (native bf16 path), so only the shadows are all-gathered each step.
        ``layout``: which slices of the sharded region this rank updates (default:
        one contiguous equal slice per rank)."""
        self.flat = flat
        self.shadow_only = shadow_only
        cuda = flat.data.is_cuda
        self.ext = _native.load(required=True) if cuda else _TorchFlat()
        self.lr, self.betas, self.eps, self.weight_decay, self.max_norm = lr, betas, eps, weight_decay, max_norm
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.shard = shard and self.world > 1 and flat.split < flat.total
        split = flat.split if self.shard else flat.total
        if self.shard and layout is None:
            layout = ShardLayout([(split, flat.total, (flat.total - split) // self.world)], self.world, self.rank)
        self.layout = layout if self.shard else None
        self.split = split
        self.segments = self.layout.owned() if self.shard else []
        owned = sum(n for _, n in self.segments)
        device = flat.data.device
        # Moments: the replicated region in full, then this rank's slices of the sharded one.
        self.exp_avg = torch.zeros(split + owned, device=device)
        self.exp_avg_sq = torch.zeros(split + owned, device=device)
        self.hyper = torch.zeros(4, device=device)
        self.hyper_small = torch.zeros(4, device=device)
        self.hyper_host = torch.zeros(4, pin_memory=cuda)
        self.step_count = 0

    def set_step(self, lr: float) -> None:
        """Host side of a step: refreshes the pinned hyper-parameters (copied in-graph)."""
        self.step_count += 1
        self.hyper_host[0] = lr
        self.hyper_host[1] = float(self.step_count)
        self.hyper_host[2] = float(self.max_norm)

    def load_hyper(self) -> None:
        self.hyper.copy_(self.hyper_host, non_blocking=True)

    def _regions(self):
        """(data, grad, exp_avg, exp_avg_sq, shadow) views: the replicated region, then owned slices."""
        f, a, b = self.flat, self.exp_avg, self.exp_avg_sq
        out = [(f.data[:self.split], f.grad[:self.split], a[:self.split], b[:self.split],
                f.shadow[:self.split])] if self.split else []
        off = self.split
        for lo, n in self.segments:
            out.append((f.data[lo:lo + n], f.grad[lo:lo + n], a[off:off + n], b[off:off + n],
                        f.shadow[lo:lo + n]))
            off += n
        return out

    def _adamw(self, region, loss_check) -> None:
        data, grad, m, v, shadow = region
        self.ext.flat_adamw(data, grad, m, v, shadow, self.hyper, loss_check,
                            self.betas[0], self.betas[1], self.eps, self.weight_decay)

    def reduce_and_step(self, loss_check: torch.Tensor | None = None, reduced: bool = False, peer=None) -> None:
        """``reduced``: the gradient was already all-reduced (bucketed during backward).
        ``peer``: a finished ``PeerGradBuckets`` (gradient reduced, ``hyper[3]`` set); the
        owned slices' shadows are then written to every rank by the update itself."""
        flat = self.flat
        regions = self._regions()
        if peer is not None:
            owned = regions[1:] if self.split else regions
            if self.split:
                self._adamw(regions[0], loss_check)
            for (data, grad, m, v, _), (lo, _) in zip(owned, self.segments):
                self.ext.flat_adamw_peer(data, grad, m, v, peer.shadow_ptrs(lo), peer.rank, self.hyper,
                                         loss_check, self.betas[0], self.betas[1], self.eps, self.weight_decay)
            if self.shard:
                peer.barrier()                       # every rank's shadow slices are in place
                if not self.shadow_only:
                    self.gather_masters()
            return
        if self.world > 1 and not reduced:
            dist.all_reduce(flat.grad, group=self.group)
        if self.shard:
            # |g|^2 = replicated part (same on every rank) + sum over ranks of their slices.
            self.hyper[3:4].zero_()
            for _, grad, _, _, _ in regions[1:] if self.split else regions:
                self.ext.flat_sq_norm(grad, self.hyper_small)
                self.hyper[3:4].add_(self.hyper_small[3:4])
            dist.all_reduce(self.hyper[3:4], group=self.group)
            if self.split:
                self.ext.flat_sq_norm(regions[0][1], self.hyper_small)
                self.hyper[3:4].add_(self.hyper_small[3:4])
        else:
            self.ext.flat_sq_norm(flat.grad, self.hyper)
        for region in regions:
            self._adamw(region, loss_check)
        if self.shard:
            self.layout.gather_(flat.shadow, self.group)
            if not self.shadow_only:
                self.gather_masters()

    def gather_masters(self) -> None:
        """Collective: make every rank's fp32 masters of the sharded region current."""
        if self.shard:
            self.layout.gather_(self.flat.data, self.group)

    def grad_norm(self) -> float:
        return float(self.hyper[3].sqrt())

    # -- checkpoints: torch.optim.AdamW layout (per-parameter state) ---------

    def _full_moments(self):
        if not self.shard:
            return self.exp_avg, self.exp_avg_sq
        full = []
        for moment in (self.exp_avg, self.exp_avg_sq):
            buf = torch.zeros(self.flat.total, device=moment.device)
            buf[:self.split].copy_(moment[:self.split])
            off = self.split
            for lo, n in self.segments:
                buf[lo:lo + n].copy_(moment[off:off + n])
                off += n
            self.layout.gather_(buf, self.group)
            full.append(buf)
        return tuple(full)

    def consolidate_state_dict(self, to: int = 0) -> None:
        """Collective under sharding (every rank calls it, like ZeRO's): moments and masters."""
        self.gather_masters()
        self._consolidated = self._full_moments()

    def state_dict(self) -> dict:
        moments = getattr(self, "_consolidated", None) or self._full_moments()
        self._consolidated = None
        m, v = moments
        state = {}
        for i, (p, off) in enumerate(zip(self.flat.params, self.flat.offsets)):
            state[i] = {"step": torch.tensor(float(self.step_count)),
                        "exp_avg": m[off:off + p.numel()].view_as(p).detach().cpu().clone(),
                        "exp_avg_sq": v[off:off + p.numel()].view_as(p).detach().cpu().clone()}
        group = {"lr": self.lr, "betas": self.betas, "eps": self.eps, "weight_decay": self.weight_decay,
                 "amsgrad": False, "maximize": False, "foreach": None, "capturable": False,
                 "differentiable": False, "fused": None, "params": list(range(len(self.flat.params)))}
        return {"state": state, "param_groups": [group]}

    def load_state_dict(self, sd: dict) -> None:
        device = self.exp_avg.device
        m = torch.zeros(self.flat.total, device=device)
        v = torch.zeros(self.flat.total, device=device)
        steps = set()
        for i, (p, off) in enumerate(zip(self.flat.params, self.flat.offsets)):
            entry = sd["state"].get(i) or sd["state"].get(str(i))
            if entry is None:
                continue
            m[off:off + p.numel()].copy_(entry["exp_avg"].reshape(-1))
            v[off:off + p.numel()].copy_(entry["exp_avg_sq"].reshape(-1))
            steps.add(int(float(entry["step"])))
        for full, mine in ((m, self.exp_avg), (v, self.exp_avg_sq)):
            mine[:self.split].copy_(full[:self.split])
            off = self.split
            for lo, n in self.segments:
                mine[off:off + n].copy_(full[lo:lo + n])
                off += n
        self.step_count = max(steps) if steps else 0

    def zero_grad(self, set_to_none: bool = True) -> None:
        """Gradients are cleared inside the captured step."""


class _TorchFlat:
    """CPU arithmetic of the flat kernels (same formulas; used by the gloo tests)."""

    @staticmethod
    def flat_sq_norm(grad, hyper):
        hyper[3] = grad.double().pow(2).sum().float()

    @staticmethod
    def flat_adamw(param, grad, exp_avg, exp_avg_sq, shadow, hyper, loss_check, beta1, beta2, eps, decay):
        lr, step, max_norm, sq = (float(x) for x in hyper[:4])
        check = float(loss_check) if loss_check is not None else 0.0
        if not (torch.isfinite(torch.tensor(sq)) and torch.isfinite(torch.tensor(check))):
            return
        scale = min(max_norm / (sq ** 0.5 + 1e-6), 1.0) if max_norm > 0 else 1.0
        g = grad * scale
        bc1, bc2 = 1 - beta1 ** step, 1 - beta2 ** step
        param.mul_(1 - lr * decay)
        exp_avg.lerp_(g, 1 - beta1)
        exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1 - beta2)
        param.addcdiv_(exp_avg, exp_avg_sq.sqrt() / bc2 ** 0.5 + eps, value=-lr / bc1)
        if shadow is not None:
            shadow.copy_(param)


def _no_signal(param) -> None:
    """Grad-sink callback when no bucket waits for the gradient."""


def peer_reduction_enabled(world: int) -> bool:
    """Gradient reduction over peer memory: CUDA ranks of one node, unless ``EB200_P2P_GRAD=0``."""
    if os.environ.get("EB200_P2P_GRAD", "1") == "0" or world > 8:
        return False
    return int(os.environ.get("LOCAL_WORLD_SIZE", world)) == world


class GraphTrainer:
    """One micro-step per optimizer step, captured in a CUDA graph after two eager steps."""

    EAGER_STEPS = 2

    def __init__(self, args, model, parallel, use_graph: bool = True, overlap: bool = True):
        if args.grad_accum != 1:
            raise ValueError("the graph trainer runs one micro-step per optimizer step")
        self.args, self.model, self.parallel = args, model, parallel
        self.device = next(model.parameters()).device
        group = None
        shards = parallel.world_size if args.optimizer_shard else 1
        self.cuda = self.device.type == "cuda"
        world = dist.get_world_size() if dist.is_initialized() else 1
        self.peer = self.cuda and world > 1 and overlap and peer_reduction_enabled(world)
        self.flat = FlatParameters(model, self.device, shards, peer_group=dist.group.WORLD if self.peer else None)
        layout = None
        if self.peer:
            self.buckets = PeerGradBuckets(self.flat, shard=args.optimizer_shard)
            layout = self.buckets.layout
        else:
            self.buckets = GradBuckets(self.flat) if world > 1 and overlap else None
        native_bf16 = (self.device.type == "cuda" and args.precision == "bf16"
                       and getattr(model, "backend", "auto") != "torch")
        self.optimizer = FlatAdamW(self.flat, args.lr, (0.9, 0.95), weight_decay=args.weight_decay,
                                   max_norm=args.clip_grad, group=group, shard=args.optimizer_shard,
                                   shadow_only=native_bf16, layout=layout)
        self.use_graph = use_graph and self.cuda
        if self.cuda and self.buckets is None:
            # One process: GEMM weight and LayerNorm gradients still go straight into the flat buffer.
            for p in self.flat.sink_params():
                G.register_grad_sink(p, _no_signal)
        self.graph = None
        self.graph_launches = 0
        self.calls = 0
        self.static = None

    def _buffers(self, ids, target, mask):
        pinned = [t.pin_memory() if self.cuda else t.clone() for t in (ids, target, mask)]
        device = [torch.empty_like(t, device=self.device) for t in pinned]
        stats_host = torch.zeros(6, dtype=torch.float64, pin_memory=self.cuda)
        return pinned, device, stats_host

    def _body(self):
        (ids_h, tgt_h, mask_h), (ids, tgt, mask), stats_host = self.static
        opt, parallel = self.optimizer, self.parallel
        opt.load_hyper()
        ids.copy_(ids_h, non_blocking=True)
        tgt.copy_(tgt_h, non_blocking=True)
        mask.copy_(mask_h, non_blocking=True)
        self.flat.zero_grad()
        amp = torch.autocast(self.device.type, dtype=torch.bfloat16, enabled=self.args.precision == "bf16",
                             cache_enabled=False)
        with amp, trace.phase("forward"):
            result = self.model.forward_loss(ids, tgt, sup=mask, parallel=parallel, offset=self.offset,
                                             static_width=True)
        totals = torch.stack((result["loss_sum"].detach().float(), result["count"].float()))
        if dist.is_initialized():
            dist.all_reduce(totals)
        loss = result["loss_sum"] / totals[1].clamp_min(1.0)
        if self.buckets is not None:
            self.buckets.start()
        with trace.phase("backward"):
            loss.backward()
        with trace.phase("gradient_reduction"):
            if self.buckets is not None:
                self.buckets.finish(opt.hyper)
        check = totals[0] / totals[1]               # non-finite (or 0/0 with no tokens) skips the update
        with trace.phase("optimizer"):
            opt.reduce_and_step(check, reduced=self.buckets is not None,
                                peer=self.buckets if self.peer else None)
        stats = torch.cat((torch.stack((result["loss_sum"].detach().double(), result["count"].double(),
                                        result["correct"].double(), opt.hyper[3].double())),
                           totals.double()))
        stats_host.copy_(stats, non_blocking=True)

    def step(self, ids, target, mask, lr: float):
        """One optimizer step; returns host ``(loss_sum, count, correct)`` float64 and the grad norm."""
        parallel = self.parallel
        ids, self.offset = parallel.shard(ids, self.model.block_size)
        target, _ = parallel.shard(target, self.model.block_size, -100)
        mask, _ = parallel.shard(mask, self.model.block_size, False)
        if self.static is None:
            self.static = self._buffers(ids, target, mask)
        (ids_h, tgt_h, mask_h), _, stats_host = self.static
        ids_h.copy_(ids)
        tgt_h.copy_(target)
        mask_h.copy_(mask)
        self.optimizer.set_step(lr)
        if not self.use_graph:
            self._body()
        elif self.calls < self.EAGER_STEPS:
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self._body()
            torch.cuda.current_stream().wait_stream(side)
        else:
            if self.graph is None:
                ext = _native.load(required=True)
                before = ext.launch_count()
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph):
                    self._body()
                self.graph_launches = ext.launch_count() - before   # native kernels per replay
            self.graph.replay()
        self.calls += 1
        if self.cuda:
            torch.cuda.current_stream().synchronize()
        stats = stats_host.clone()          # [loss_sum, count, correct, grad_sq_norm, global loss, global count]
        self.last_stats = stats
        if stats[5] == 0:
            self.optimizer.step_count -= 1
            raise ValueError("global batch has no supervised tokens")
        if not bool(torch.isfinite(stats[4])) or not bool(torch.isfinite(stats[3])):
            self.optimizer.step_count -= 1
            raise FloatingPointError("non-finite loss across ranks; optimizer step was not applied")
        return stats[:3], float(stats[3].sqrt())

    def close(self) -> None:
        """Release the graph before the process group goes away."""
        self.graph = None
        if self.buckets is not None:
            self.buckets.remove()
        self.flat.release()
