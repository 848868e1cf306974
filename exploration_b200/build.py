"""Ahead-of-time build of the sm_100a extension: ``python -m exploration_b200.build``.

Every CUDA source is compiled for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``; no PTX fallback for other
GPUs) with ``-lineinfo``. The shared object lands in
``exploration_b200/_build/`` next to the package, so it travels with the
source tree and is loaded from there at import time (nothing is compiled at
import). Passing the ``-gencode`` flag explicitly keeps PyTorch from adding
its own architecture list.
"""
from __future__ import annotations

import argparse
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
BUILD_DIR = ROOT / "_build"
NAME = "eb200_C"

SOURCES = [
    "bindings.cpp",
    "fused/norm_act.cu",
    "fused/loss_optim.cu",
    "fused/embedding.cu",
    "fused/flat_optim.cu",
    "attention/local_halo.cu",
    "attention/local_halo_b16.cu",
    "attention/local_tc.cu",
    "attention/gated_entry.cu",
    "attention/gated_simt.cu",
    "attention/gated_tc.cu",
    "attention/gated_tc_bwd.cu",
    "sparse/sparse_read.cu",
    "sparse/block_scores_tc.cu",
    "gemm/gemm_tc.cu",
    "comm/symm_heap.cu",
    "comm/grad_reduce.cu",
]

CUDA_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]


def sources():
    return [str(CSRC / s) for s in SOURCES]


def build(verbose: bool = False, ptxas_info: bool = False):
    """Compile (incrementally, via ninja) and return the loaded module."""
    from torch.utils import cpp_extension
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    flags = list(CUDA_FLAGS)
    if ptxas_info:
        flags.append("-Xptxas=-v")
    os.environ.setdefault("MAX_JOBS", str(max(1, min(8, os.cpu_count() or 1))))
    started = time.time()
    module = cpp_extension.load(
        name=NAME,
        sources=sources(),
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=flags,
        extra_include_paths=[str(CSRC)],
        build_directory=str(BUILD_DIR),
        with_cuda=True,
        verbose=verbose,
    )
    if verbose:
        print(f"built {NAME} in {time.time() - started:.1f}s -> {BUILD_DIR}", file=sys.stderr)
    return module


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas-info", action="store_true", help="print registers/smem per kernel")
    args = parser.parse_args(argv)
    build(verbose=args.verbose, ptxas_info=args.ptxas_info)
    print(f"ok: {BUILD_DIR}")


if __name__ == "__main__":
    main()
