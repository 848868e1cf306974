"""Worker bodies for the CPU multi-process tests (gloo ranks)."""
import os
import traceback


def setup_env(rank, world, port, extra):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "LOCAL_WORLD_SIZE": str(world), "MASTER_ADDR": "127.0.0.1",
                       "MASTER_PORT": str(port)})
    os.environ.update(extra)


def run(target, rank, world, port, extra, results):
    setup_env(rank, world, port, extra)
    import torch
    torch.set_num_threads(1)
    try:
        out = globals()[target](rank, world)
        results.put((rank, "ok", out))
    except BaseException as exc:  # reported to the parent, which asserts on it
        results.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()[-1500:]}"))


def gradient_parity(rank, world):
    import torch.distributed as dist
    from exploration_b200.parallel.context import ParallelContext
    from exploration_b200.tools import validate
    cp = int(os.environ["TEST_CP"])
    parallel = ParallelContext.initialize(cp, "cpu")
    import torch
    try:
        records = [validate._gradient_parity(kind, mask, parallel, torch.device("cpu"))
                   for kind in ("stack", "baseline") for mask in ("full", "tail", "ragged")]
        return len(records)
    finally:
        dist.destroy_process_group()


def sparse_prefill(rank, world):
    import torch
    import torch.distributed as dist
    from exploration_b200.parallel.context import init_distributed
    from exploration_b200.tools import validate
    init_distributed("cpu")
    try:
        return validate._sparse_prefill_parity(torch.device("cpu"))["max_abs"]
    finally:
        dist.destroy_process_group()


def exchanges(rank, world):
    """Ulysses round trip and halo exchange values/gradients against direct formulas."""
    import torch
    import torch.distributed as dist
    from exploration_b200.parallel.context import ParallelContext
    parallel = ParallelContext.initialize(world, "cpu")
    try:
        torch.manual_seed(0)
        full = torch.randn(2, 8 * world, 4 * world, 3, dtype=torch.float64)
        local = full[:, rank * 8:(rank + 1) * 8].clone().requires_grad_()
        heads = parallel.to_heads(local)
        hc = 4
        torch.testing.assert_close(heads, full[:, :, rank * hc:(rank + 1) * hc])
        back = parallel.to_sequence(heads)
        torch.testing.assert_close(back, local)
        (heads * heads).sum().backward()
        torch.testing.assert_close(local.grad, 2 * local.detach())
        x = torch.arange(world * 6, dtype=torch.float64).reshape(1, world * 6, 1)
        mine = x[:, rank * 6:(rank + 1) * 6].clone().requires_grad_()
        halo = parallel.halo(mine, 2)
        expected = torch.zeros(1, 2, 1, dtype=torch.float64) if rank == 0 else \
            x[:, rank * 6 - 2:rank * 6]
        torch.testing.assert_close(halo, expected)
        halo.sum().backward()
        tail_grad = mine.grad[0, -2:, 0]
        want = torch.zeros(2, dtype=torch.float64) if rank == world - 1 else torch.ones(2, dtype=torch.float64)
        torch.testing.assert_close(tail_grad, want)
        return True
    finally:
        dist.destroy_process_group()


def train_with_fault(rank, world):
    """Engine training where one rank raises before backward; every rank must end in an error."""
    from exploration_b200.cli import main
    main(["train", "--task", "random", "--vocab-size", "31", "--dim", "16", "--heads", "2",
          "--block-size", "4", "--arch", "L,G", "--length", "32", "--batch-size", "1",
          "--encoder-chunk", "8", "--steps", "3", "--device", "cpu", "--backend", "torch",
          "--precision", "fp32", "--save", "", "--context-parallel", "2", "--log-every", "1"])
    return "finished"


def train_cp2(rank, world):
    from exploration_b200.cli import main
    main(["train", "--task", "mqar", "--length", "64", "--npairs", "4", "--nqueries", "2",
          "--vocab-size", "128", "--dim", "16", "--heads", "2", "--block-size", "4", "--arch", "L,G",
          "--batch-size", "2", "--encoder-chunk", "8", "--steps", "2", "--device", "cpu",
          "--backend", "torch", "--precision", "fp32", "--save", os.environ["TEST_SAVE"],
          "--context-parallel", os.environ["TEST_CP"], "--log-every", "1", "--grad-accum", "2"])
    return "finished"


def _flat_vs_eager(parallel, shard, layout="contiguous"):
    """Three steps of the flat (graph-ready) trainer against the eager trainer."""
    import copy
    import torch
    from exploration_b200 import ExecutionConfig, build_model
    from exploration_b200.cli import parse_args
    from exploration_b200.runtime.engine import Trainer, make_batch, lr_factor
    from exploration_b200.runtime.flat import GraphTrainer
    world = parallel.world_size
    args = parse_args(["train", "--dim", "64", "--heads", "4", "--block-size", "8", "--arch", "Lx1,G",
                       "--task", "random", "--length", str(64 * max(1, parallel.cp_size)),
                       "--batch-size", "1", "--precision", "fp32", "--device", "cpu", "--backend", "torch",
                       "--context-parallel", str(parallel.cp_size), "--steps", "3", "--save", "",
                       "--clip-grad", "0.05", "--weight-decay", "0.1"] +
                      (["--optimizer-shard"] if shard else ["--no-optimizer-shard"]))
    torch.manual_seed(0)
    options = {"model": "stack", "vocab_size": 256, "dim": 64, "heads": 4, "block_size": 8, "topk": 4,
               "arch": "Lx1,G", "ffn_ratio": 2.0}
    base = build_model(options, execution=ExecutionConfig(backend="torch"))
    eager_model, flat_model = copy.deepcopy(base), copy.deepcopy(base)
    eager = Trainer(args, eager_model, parallel)
    flat = GraphTrainer(args, flat_model, parallel, use_graph=False)
    if layout == "buckets":
        # The peer-reduction layout: a slice of every (small) bucket per rank.
        from exploration_b200.runtime.flat import FlatAdamW, _bucket_bounds, bucket_layout
        bounds, _ = _bucket_bounds(flat.flat, 4096, split_boundary=True)
        _, shard_layout = bucket_layout(flat.flat, bounds, world, parallel.rank, shard)
        assert shard_layout is None or len(shard_layout.groups) > 2
        opt = flat.optimizer
        flat.optimizer = FlatAdamW(flat.flat, args.lr, opt.betas, weight_decay=args.weight_decay,
                                   max_norm=args.clip_grad, shard=shard, layout=shard_layout)
    gen_a = torch.Generator().manual_seed(5 + parallel.dp_rank)
    gen_b = torch.Generator().manual_seed(5 + parallel.dp_rank)
    for step in range(3):
        lr = args.lr * lr_factor(step, args.steps)
        eager.optimizer.zero_grad(set_to_none=True)
        for group in eager.optimizer.param_groups:
            group["lr"] = lr
        ids, target, mask, _ = make_batch(args, gen_a)
        a = eager.micro_step(ids, target, mask, last=True)
        eager.finish_step()
        ids, target, mask, _ = make_batch(args, gen_b)
        b, _ = flat.step(ids, target, mask, lr)
        assert torch.allclose(a, b, rtol=1e-5, atol=1e-5), (step, a, b)
    for (name, p), q in zip(eager_model.named_parameters(), flat_model.parameters()):
        assert torch.allclose(p, q, rtol=1e-4, atol=1e-6), name
    # Optimizer state round trip through the torch.optim.AdamW layout (collective).
    state = flat.optimizer.state_dict()
    assert all(entry["exp_avg_sq"].abs().sum() > 0 for entry in state["state"].values())
    from exploration_b200.runtime.flat import FlatAdamW
    fresh = FlatAdamW(flat.flat, args.lr, shard=shard)
    fresh.load_state_dict(state)
    reloaded = fresh.state_dict()
    for i in state["state"]:
        assert torch.equal(reloaded["state"][i]["exp_avg"], state["state"][i]["exp_avg"])
        assert torch.equal(reloaded["state"][i]["exp_avg_sq"], state["state"][i]["exp_avg_sq"])
    flat.close()
    return world


def flat_trainer(rank, world):
    import torch.distributed as dist
    from exploration_b200.parallel.context import ParallelContext
    cp = int(os.environ["TEST_CP"])
    shard = os.environ.get("TEST_SHARD") == "1"
    layout = os.environ.get("TEST_LAYOUT", "contiguous")
    parallel = ParallelContext.initialize(cp, "cpu")
    try:
        return _flat_vs_eager(parallel, shard, layout)
    finally:
        dist.destroy_process_group()
