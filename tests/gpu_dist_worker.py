"""Worker for the multi-GPU tests: one process per GPU over NCCL (torchrun).

``parity``: one forward/backward of a small Stack model with context
parallelism, once through the NVLink-fused Ulysses exchange and once through
the NCCL all-to-all path, on identical weights and data; every rank compares
its loss and local parameter gradients and reports the largest differences.
``train``: a few optimizer steps through the engine with the fused exchange.
``graph``: graph-captured steps against eager steps. ``peer_grad``: the
peer-memory gradient reduction against the NCCL path.
"""
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from exploration_b200 import ExecutionConfig, ParallelContext, build_model  # noqa: E402
from exploration_b200.ops import _native  # noqa: E402


def _model(device):
    torch.manual_seed(0)
    options = {"model": "stack", "vocab_size": 256, "dim": 256, "heads": 8, "block_size": 16, "topk": 8,
               "arch": "Lx2,G", "ffn_ratio": 4.0}
    return build_model(options, execution=ExecutionConfig(backend="cuda"), device=device)


def _loss_and_grads(model, ids, targets, parallel, offset):
    model.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = model.forward_loss(ids, targets, parallel=parallel, offset=offset)
    out["loss_sum"].backward()
    grads = {n: p.grad.detach().float().clone() for n, p in model.named_parameters() if p.grad is not None}
    return float(out["loss_sum"]), grads


def parity(world, rank, device):
    parallel = ParallelContext.initialize(world, "cuda")
    model = _model(device)
    g = torch.Generator().manual_seed(7)
    length = 512 * world
    ids_full = torch.randint(0, 256, (1, length), generator=g)
    tgt_full = torch.randint(0, 256, (1, length), generator=g)
    ids, offset = parallel.shard(ids_full, model.block_size)
    tgt, _ = parallel.shard(tgt_full, model.block_size, -100)
    ids, tgt = ids.to(device), tgt.to(device)
    assert parallel.attach_fused(device)
    fused_loss, fused_grads = _loss_and_grads(model, ids, tgt, parallel, offset)
    exchange = parallel.ulysses
    parallel.ulysses = None
    nccl_loss, nccl_grads = _loss_and_grads(model, ids, tgt, parallel, offset)
    parallel.ulysses = exchange
    worst = 0.0
    for name, ref in nccl_grads.items():
        got = fused_grads[name]
        scale = max(ref.abs().max().item(), 1e-3)
        worst = max(worst, (got - ref).abs().max().item() / scale)
    errors = _native.load().device_errors(device.index)
    parallel.close()
    return {"fused_loss": fused_loss, "nccl_loss": nccl_loss, "worst_grad_rel": worst,
            "device_errors": list(errors), "heap_high_water": exchange.heap.high_water}


def train(world, rank, device):
    from exploration_b200.cli import parse_args
    from exploration_b200.runtime.engine import Trainer, make_batch
    args = parse_args(["train", "--dim", "256", "--heads", "8", "--block-size", "16", "--arch", "Lx2,G",
                       "--task", "random", "--length", str(512 * world), "--batch-size", "1",
                       "--precision", "bf16", "--backend", "cuda", "--context-parallel", str(world),
                       "--steps", "4", "--save", "", "--no-checkpoint-chunks"])
    parallel = ParallelContext.initialize(world, "cuda")
    model = _model(device)
    assert parallel.attach_fused(device)
    trainer = Trainer(args, model, parallel)
    gen = torch.Generator().manual_seed(100)
    losses = []
    for step in range(4):
        trainer.optimizer.zero_grad(set_to_none=True)
        trainer.set_lr(step)
        ids, target, mask, _ = make_batch(args, gen)
        stats = trainer.micro_step(ids, target, mask, last=True)
        trainer.finish_step()
        losses.append(float(stats[0] / stats[1]))
    errors = _native.load().device_errors(device.index)
    parallel.close()
    return {"losses": losses, "device_errors": list(errors)}


def graph(world, rank, device):
    """Graph-captured steps (fused exchange, bucketed all-reduce, ZeRO-1) against eager steps."""
    import copy
    from exploration_b200.cli import parse_args
    from exploration_b200.runtime.engine import Trainer, lr_factor, make_batch
    from exploration_b200.runtime.flat import GraphTrainer
    args = parse_args(["train", "--dim", "256", "--heads", "8", "--block-size", "16", "--arch", "Lx2,G",
                       "--task", "random", "--length", str(512 * world), "--batch-size", "1",
                       "--precision", "bf16", "--backend", "cuda", "--context-parallel", str(world),
                       "--steps", "5", "--save", "", "--no-checkpoint-chunks", "--optimizer-shard"])
    parallel = ParallelContext.initialize(world, "cuda")
    base = _model(device)
    eager_model, graph_model = copy.deepcopy(base), copy.deepcopy(base)
    assert parallel.attach_fused(device)
    eager = Trainer(args, eager_model, parallel)
    graphed = GraphTrainer(args, graph_model, parallel)
    gen_a, gen_b = torch.Generator().manual_seed(100), torch.Generator().manual_seed(100)
    diffs = []
    for step in range(args.steps):
        lr = args.lr * lr_factor(step, args.steps)
        eager.optimizer.zero_grad(set_to_none=True)
        eager.set_lr(step)
        ids, target, mask, _ = make_batch(args, gen_a)
        a = eager.micro_step(ids, target, mask, last=True).cpu()
        eager.finish_step()
        ids, target, mask, _ = make_batch(args, gen_b)
        b, _ = graphed.step(ids, target, mask, lr)
        diffs.append(abs(float(a[0] / a[1]) - float(b[0] / b[1])))
    captured = graphed.graph is not None
    graphed.close()
    errors = _native.load().device_errors(device.index)
    parallel.close()
    return {"loss_diffs": diffs, "captured": captured, "device_errors": list(errors)}


def peer_grad(world, rank, device):
    """Graph-captured steps with the peer-memory gradient reduction against the NCCL path.

    Two trainers on copies of one model and identical batches: ``EB200_P2P_GRAD=1``
    (per-bucket reduce-scatter kernels over NVLink, fused norm, shadows stored to
    every rank by the update) and ``EB200_P2P_GRAD=0`` (NCCL bucketed all-reduce,
    shadow all-gather). Both shard the optimizer (ZeRO-1) or both do not.
    """
    import copy
    from exploration_b200.cli import parse_args
    from exploration_b200.runtime.engine import lr_factor, make_batch
    from exploration_b200.runtime.flat import GraphTrainer
    shard = os.environ.get("TEST_SHARD", "1") == "1"
    args = parse_args(["train", "--dim", "256", "--heads", "8", "--block-size", "16", "--arch", "Lx2,G",
                       "--task", "random", "--length", str(512 * world), "--batch-size", "1",
                       "--precision", "bf16", "--backend", "cuda", "--context-parallel", str(world),
                       "--steps", "5", "--save", "", "--no-checkpoint-chunks", "--clip-grad", "0.5",
                       "--optimizer-shard" if shard else "--no-optimizer-shard"])
    parallel = ParallelContext.initialize(world, "cuda")
    base = _model(device)
    peer_model, nccl_model = copy.deepcopy(base), copy.deepcopy(base)
    os.environ["EB200_P2P_GRAD"] = "1"
    peer = GraphTrainer(args, peer_model, parallel)
    os.environ["EB200_P2P_GRAD"] = "0"
    nccl = GraphTrainer(args, nccl_model, parallel)
    assert peer.peer and not nccl.peer
    gen_a, gen_b = torch.Generator().manual_seed(100), torch.Generator().manual_seed(100)
    loss_diffs, norm_diffs = [], []
    for step in range(args.steps):
        lr = args.lr * lr_factor(step, args.steps)
        ids, target, mask, _ = make_batch(args, gen_a)
        a, norm_a = peer.step(ids, target, mask, lr)
        ids, target, mask, _ = make_batch(args, gen_b)
        b, norm_b = nccl.step(ids, target, mask, lr)
        loss_diffs.append(abs(float(a[0] / a[1]) - float(b[0] / b[1])))
        norm_diffs.append(abs(norm_a - norm_b) / max(norm_b, 1e-6))
    worst = 0.0
    for p, q in zip(peer_model.parameters(), nccl_model.parameters()):
        worst = max(worst, (p.detach() - q.detach()).abs().max().item())
    # Every rank's bf16 shadows agree after the peer stores (they are what the GEMMs read).
    shadow = peer.flat.shadow.float()
    gathered = [torch.empty_like(shadow) for _ in range(world)]
    dist.all_gather(gathered, shadow)
    shadows_equal = all(torch.equal(gathered[0], t) for t in gathered[1:])
    captured = peer.graph is not None
    peer.close()
    nccl.close()
    errors = _native.load().device_errors(device.index)
    parallel.close()
    return {"loss_diffs": loss_diffs, "norm_diffs": norm_diffs, "worst_param_diff": worst,
            "shadows_equal": shadows_equal, "captured": captured, "device_errors": list(errors)}


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    device = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(device)
    torch.backends.cuda.matmul.allow_tf32 = False
    result = {"parity": parity, "train": train, "graph": graph,
              "peer_grad": peer_grad}[sys.argv[1]](world, rank, device)
    gathered = [None] * world
    dist.all_gather_object(gathered, result)
    if rank == 0:
        print("RESULT " + json.dumps(gathered), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
