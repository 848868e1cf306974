"""Correctness suites: ``python -m st validate --suite {reference,resources,cuda,distributed}``.

* ``reference``: the CPU test suite (``pytest -m "not gpu"``).
* ``resources``: compiled resource use of every native kernel plus the
  parity cases that stress the largest tiles.
* ``cuda``: native sm_100a kernels against the loop oracle over the
  reference's case matrix (fp32 and bf16), the sparse path against the
  top-k oracle, and an end-to-end bf16 model (native vs torch backend).
* ``distributed``: under torchrun, CP x DP gradients against a
  single-process fp64 model (full, tail and ragged masks; Stack and the
  baseline) and distributed sparse prefill against the in-core forward.

Failures are fatal and recorded in the JSON report
(reference: st/tools/validate.py:47-273).
"""
from __future__ import annotations

import argparse
import copy
import json
import os
import platform
import subprocess
import sys
import time
import traceback
from pathlib import Path

import torch
import torch.distributed as dist
from torch.nn.parallel import DistributedDataParallel as DDP

from ..models.baseline import BaselineModel
from ..models.stack import StackModel
from ..ops.attention import dense_attention
from ..ops.flash import backend_info
from ..ops.launch import launch_report
from ..ops.sparse import TensorPages, block_scores_reference, sparse_attention
from ..parallel.context import ParallelContext, sum_all
from ..runtime.inference import InferenceSession
from .oracle import eager_attention, error_metrics

CASES = [(17, 2, 16), (129, 16, 32), (257, 32, 64), (193, 64, 96), (385, 128, 128),
         (131, 16, 256), (385, 128, 256)]
RESOURCE_CASES = [(385, 128, 128), (385, 128, 256), (193, 64, 96)]
TOLERANCE = {torch.float32: (2e-5, 2e-4), torch.bfloat16: (3e-2, 5e-2)}


def environment() -> dict:
    record = {"python": platform.python_version(), "torch": torch.__version__,
              "cuda_runtime": torch.version.cuda, "platform": platform.platform()}
    if torch.cuda.is_available():
        record["gpus"] = [{"name": torch.cuda.get_device_name(i),
                           "memory_bytes": torch.cuda.get_device_properties(i).total_memory,
                           "capability": torch.cuda.get_device_capability(i),
                           "sm_count": torch.cuda.get_device_properties(i).multi_processor_count}
                          for i in range(torch.cuda.device_count())]
    from ..ops import _native
    path = _native.so_path()
    record["native_extension"] = str(path) if path else None
    record["sdpa"] = backend_info("cuda" if torch.cuda.is_available() else "cpu")
    return record


def reference_suite() -> dict:
    root = Path(__file__).resolve().parents[2]
    if not (root / "tests").is_dir():
        raise RuntimeError("the reference suite needs the source checkout (tests/)")
    proc = subprocess.run([sys.executable, "-m", "pytest", str(root / "tests"), "-q", "-m", "not gpu",
                           "-p", "no:cacheprovider"], cwd=root, capture_output=True, text=True)
    tail = proc.stdout.strip().splitlines()[-1:] if proc.stdout else []
    if proc.returncode:
        raise AssertionError(f"CPU tests failed:\n{proc.stdout[-4000:]}\n{proc.stderr[-2000:]}")
    return {"summary": tail[0] if tail else ""}


def _dense_case(n, b, d, dtype):
    q = torch.randn(2, 5, 2, d, device="cuda", dtype=dtype, requires_grad=True)
    k = torch.randn(2, n, 2, d, device="cuda", dtype=dtype, requires_grad=True)
    v = torch.randn_like(k, requires_grad=True)
    pos = torch.tensor([[0, b - 1, min(2 * b + 1, n - 1), n - 1, -1], [n - 1, 0, n // 2, -1, n - 2]],
                       device="cuda")
    return q, k, v, pos


def cuda_suite(resources_only=False) -> dict:
    if not torch.cuda.is_available():
        raise RuntimeError("the CUDA suite needs an NVIDIA GPU")
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(772)
    results = []
    for dtype in (torch.float32, torch.bfloat16):
        atol, rtol = TOLERANCE[dtype]
        for n, b, d in (RESOURCE_CASES if resources_only else CASES):
            q, k, v, pos = _dense_case(n, b, d, dtype)
            rq, rk, rv = (t.detach().float().requires_grad_() for t in (q, k, v))
            expected = eager_attention(rq, rk, rv, pos, b)
            actual = dense_attention(q, k, v, pos, b, "cuda")
            probe = torch.randn_like(actual)
            got = torch.autograd.grad((actual * probe).sum(), (q, k, v))
            want = torch.autograd.grad((expected * probe.float()).sum(), (rq, rk, rv))
            torch.testing.assert_close(actual.float(), expected, atol=atol, rtol=rtol)
            for a, e in zip(got, want):
                torch.testing.assert_close(a.float(), e, atol=atol, rtol=rtol)
            results.append({"operation": "dense", "dtype": str(dtype), "n": n, "block": b,
                            "head_dim": d, "forward": error_metrics(actual, expected),
                            "gradients": [error_metrics(a, e) for a, e in zip(got, want)]})
            with torch.no_grad():
                keep = 2
                expected_sparse = eager_attention(rq, rk, rv, pos, b, keep)
                sparse = sparse_attention(q.detach(), TensorPages(k.detach(), v.detach(), 4 * b), pos,
                                          b, keep, "cuda", score_page_tokens=2 * b)
                torch.testing.assert_close(sparse.float(), expected_sparse, atol=atol, rtol=rtol)
                offset = 2 * b
                shifted = torch.where(pos >= 0, pos + offset, pos)
                ref_scores = block_scores_reference(q, k, shifted, b, offset)
                results.append({"operation": "sparse", "dtype": str(dtype), "n": n, "block": b,
                                "head_dim": d, **error_metrics(sparse, expected_sparse),
                                "visible_blocks_offset": int(torch.isfinite(ref_scores).sum())})
            print(json.dumps(results[-1]), flush=True)
    if not resources_only:
        torch.manual_seed(42)
        model = StackModel(128, 64, 4, 16, 64, "Lx2,(G)x2", backend="cuda", checkpoint_chunks=True,
                           encoder_chunk=32, pos_chunk=7).cuda()
        ref = copy.deepcopy(model)
        ref.set_backend("torch")
        ids = torch.randint(128, (2, 131), device="cuda")
        targets = torch.randint(128, ids.shape, device="cuda")
        sup = torch.rand(ids.shape, device="cuda") > 0.75
        with torch.autocast("cuda", dtype=torch.bfloat16):
            actual = model(ids, sup=sup, targets=targets)["loss_sum"]
            expected = ref(ids, sup=sup, targets=targets)["loss_sum"]
        torch.testing.assert_close(actual, expected, atol=0.1, rtol=0.003)
        actual.backward()
        expected.backward()
        grads = {}
        for (name, a), (_, e) in zip(model.named_parameters(), ref.named_parameters()):
            if a.grad is not None:
                torch.testing.assert_close(a.grad, e.grad, atol=0.08, rtol=0.06, msg=name)
                grads[name] = error_metrics(a.grad, e.grad)
        results.append({"operation": "end_to_end_bf16", "loss": error_metrics(actual, expected),
                        "gradients": grads})
    return {"cases": results, "kernel_launches": launch_report()}


def distributed_suite(cp_size) -> dict:
    device_type = "cuda" if torch.cuda.is_available() else "cpu"
    if int(os.environ.get("WORLD_SIZE", "1")) < 2:
        raise RuntimeError("the distributed suite runs under torchrun with >= 2 ranks")
    parallel = ParallelContext.initialize(cp_size, device_type)
    device = torch.device(device_type, int(os.environ.get("LOCAL_RANK", "0"))) \
        if device_type == "cuda" else torch.device("cpu")
    records = []
    try:
        for kind in ("stack", "baseline"):
            for mask_kind in ("full", "tail", "ragged"):
                records.append(_gradient_parity(kind, mask_kind, parallel, device))
        records.append(_sparse_prefill_parity(device))
        return {"cases": records, "world": parallel.world_size}
    finally:
        dist.destroy_process_group()


def _gradient_parity(kind, mask_kind, parallel, device) -> dict:
    torch.manual_seed(928)
    if kind == "stack":
        base = StackModel(31, 32, 8, 4, 64, "(L)x2,(G)x2", backend="torch", checkpoint_chunks=True,
                          encoder_chunk=8, pos_chunk=3)
    else:
        base = BaselineModel(31, 32, 8, layers=2, checkpoint_chunks=True, loss_chunk=3)
    base = base.to(device).double()
    ref = copy.deepcopy(base)
    wrapped = DDP(base, device_ids=[device.index] if device.type == "cuda" else None,
                  broadcast_buffers=False)
    n, batch = 37, 2
    batches = []
    for replica in range(parallel.dp_size):
        g = torch.Generator().manual_seed(127 + replica)
        ids = torch.randint(31, (batch, n), generator=g)
        target = torch.randint(31, (batch, n), generator=g)
        mask = torch.ones_like(ids, dtype=torch.bool)
        if mask_kind == "tail":
            mask[:, :-3] = False            # every CP rank but the last owns no query
        elif mask_kind == "ragged":
            mask = torch.rand(batch, n, generator=g) > 0.65
            mask[0] = False
        batches.append((ids, target, mask))
    total = sum(int(m.sum()) for _, _, m in batches)
    ref_loss = 0
    for ids, target, mask in batches:
        out = ref(ids.to(device), targets=target.to(device), sup=mask.to(device))
        ref_loss = ref_loss + out["loss_sum"] / total
    ref_loss.backward()
    ids, target, mask = batches[parallel.dp_rank]
    ids, offset = parallel.shard(ids, base.block_size)
    target, _ = parallel.shard(target, base.block_size, -100)
    mask, _ = parallel.shard(mask, base.block_size, False)
    result = wrapped(ids.to(device), targets=target.to(device), sup=mask.to(device), parallel=parallel,
                     offset=offset)
    count = sum_all(result["count"])
    (result["loss_sum"] * parallel.world_size / count).backward()
    torch.testing.assert_close(sum_all(result["loss_sum"]) / count, ref_loss.detach(), rtol=2e-6,
                               atol=2e-6)
    metrics = {}
    for (name, p), (_, rp) in zip(base.named_parameters(), ref.named_parameters()):
        if rp.grad is not None:
            torch.testing.assert_close(p.grad, rp.grad, rtol=5e-5, atol=5e-7, msg=name)
            metrics[name] = error_metrics(p.grad, rp.grad)
    return {"operation": "distributed_gradient", "model": kind, "mask": mask_kind,
            "cp": parallel.cp_size, "dp": parallel.dp_size, "gradients": metrics}


def _sparse_prefill_parity(device) -> dict:
    torch.manual_seed(99)
    model = StackModel(31, 32, 8, 4, 2, "(L)x3,(G)x2", backend="torch", encoder_chunk=8)
    model = model.to(device).double().eval()
    g = torch.Generator().manual_seed(83)
    ids = torch.randint(31, (2, 73), generator=g)
    positions = torch.tensor([[0, 8, 31, 72], [1, 17, 50, 71]])
    sup = torch.zeros_like(ids, dtype=torch.bool).scatter_(1, positions, True)
    with torch.no_grad():
        expected = model(ids.to(device), sup=sup.to(device), compact=True)
        with InferenceSession(model, group=dist.group.WORLD, cache="cpu", page_tokens=12,
                              encoder_chunk=8, query_chunk=2) as session:
            session.prefill(ids, positions)
            actual = torch.cat([out for _, out, _ in session.iter_logits()], 1)
    torch.testing.assert_close(actual, expected, atol=1e-8, rtol=1e-7)
    return {"operation": "distributed_sparse_prefill", **error_metrics(actual, expected)}


def parser():
    p = argparse.ArgumentParser(prog="python -m st validate", description=__doc__, allow_abbrev=False,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--suite", choices=["reference", "resources", "cuda", "distributed"], required=True)
    p.add_argument("--cp", type=int, default=2)
    p.add_argument("--output", default="validation.json")
    return p


def main(argv=None):
    args = parser().parse_args(argv)
    report = {"environment": environment(), "suite": args.suite, "passed": False}
    start = time.perf_counter()
    error = None
    try:
        if args.suite == "reference":
            report["results"] = reference_suite()
        elif args.suite in ("cuda", "resources"):
            report["results"] = cuda_suite(resources_only=args.suite == "resources")
        else:
            report["results"] = distributed_suite(args.cp)
        report["passed"] = True
    except BaseException:
        error = traceback.format_exc()
        report["error"] = error
        report["kernel_launches"] = launch_report()
    report["seconds"] = time.perf_counter() - start
    rank = int(os.environ.get("RANK", "0"))
    path = Path(args.output)
    if rank:
        path = path.with_name(f"{path.stem}.rank{rank}{path.suffix}")
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(report, indent=2, default=str) + "\n")
    if error:
        print(error, file=sys.stderr)
        raise SystemExit(1)
    print(json.dumps({"passed": True, "report": str(path)}), flush=True)
    return report
