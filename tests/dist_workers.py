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
