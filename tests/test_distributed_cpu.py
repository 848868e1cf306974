"""Multi-process host logic on CPU gloo ranks: CP/DP parity, exchanges, faults."""
import multiprocessing as mp
import queue
import socket

import pytest

from tests import dist_workers


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(target, world, extra=None, timeout=180):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=dist_workers.run, args=(target, r, world, port, extra or {}, results))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            rank, status, payload = results.get(timeout=timeout)
            out[rank] = (status, payload)
    except queue.Empty:
        pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
            p.join()
    return out


@pytest.mark.parametrize("cp", [2, 1])
def test_gradient_parity_cp_and_dp(cp):
    out = launch("gradient_parity", 2, {"TEST_CP": str(cp)})
    assert len(out) == 2, out
    for rank, (status, payload) in out.items():
        assert status == "ok", payload


def test_distributed_sparse_prefill_parity():
    out = launch("sparse_prefill", 2)
    assert all(status == "ok" for status, _ in out.values()), out


def test_ulysses_and_halo_exchanges():
    out = launch("exchanges", 2)
    assert all(status == "ok" for status, _ in out.values()), out


def test_engine_cp2_with_accumulation_saves(tmp_path):
    path = str(tmp_path / "cp2.pt")
    out = launch("train_cp2", 2, {"TEST_CP": "2", "TEST_SAVE": path})
    assert all(status == "ok" for status, _ in out.values()), out
    from exploration_b200.runtime import checkpoint
    saved = checkpoint.load(path)
    assert saved["topology"] == {"world_size": 2, "cp_size": 2}
    assert len(saved["rng_by_rank"]) == 2


def test_injected_rank_failure_ends_every_rank():
    extra = {"EB200_FAULT": "before_backward", "EB200_FAULT_RANK": "1", "EB200_PG_TIMEOUT_S": "15"}
    out = launch("train_with_fault", 2, extra, timeout=120)
    assert out.get(1, ("missing",))[0] == "error" and "injected fault" in out[1][1]
    # The healthy rank must not finish training: its next collective fails or times out.
    assert out.get(0, ("error", "no report"))[0] == "error"


@pytest.mark.parametrize("cp,shard,layout", [(2, "0", "contiguous"), (1, "1", "contiguous"), (2, "1", "contiguous"),
                                             (2, "1", "buckets"), (1, "0", "buckets")])
def test_flat_trainer_matches_eager(cp, shard, layout):
    """``buckets``: the optimizer updates a slice of every gradient bucket per rank (the
    layout of the peer-memory reduction), including the checkpoint state round trip."""
    out = launch("flat_trainer", 2, {"TEST_CP": str(cp), "TEST_SHARD": shard, "TEST_LAYOUT": layout})
    assert len(out) == 2, out
    for rank, (status, payload) in out.items():
        assert status == "ok", payload
