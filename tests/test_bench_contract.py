"""bench.py pieces that run without a GPU: the clock sampler's timed window."""
import importlib.util
import time
from datetime import datetime
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _line(t, index, sm, hw="Not Active", power_cap="Not Active"):
    stamp = datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return f"{stamp}, {index}, {sm}, 1965, 900, 0x0, {hw}, Not Active, Not Active, {power_cap}"


def test_clock_sampler_keeps_the_timed_window():
    sampler = _bench().ClockSampler([0])
    now = time.time()
    sampler.lines = [_line(now - 0.1, 0, 1965), _line(now + 0.02, 0, 1800, power_cap="Active"),
                     _line(now + 0.04, 0, 1850), _line(now + 0.3, 0, 1000, hw="Active"),
                     _line(now + 0.03, 1, 500, hw="Active")]          # another GPU: ignored
    sampler.mark(now, now + 0.05)
    summary = sampler.summary()
    assert summary["window"] == "timed" and summary["samples"] == 2
    assert summary["sm_mhz"] == 1825 and summary["reasons"] == ["sw_power_cap"]


def test_clock_sampler_short_window_uses_adjacent_samples():
    sampler = _bench().ClockSampler([0])
    now = time.time()
    sampler.lines = [_line(now - 0.04, 0, 1965), _line(now + 0.06, 0, 1900)]
    sampler.mark(now, now + 0.01)
    summary = sampler.summary()
    assert summary["window"] == "adjacent" and summary["samples"] == 2


def test_clock_sampler_without_samples():
    sampler = _bench().ClockSampler([0])
    sampler.mark(0.0, 1.0)
    assert sampler.summary()["reasons"] == ["unsampled"]


def test_gemm_plan_splits_only_few_tile_shapes():
    """Weight-gradient shapes (few output tiles, K = tokens) split K; token-major GEMMs do not."""
    from exploration_b200.ops import _native
    ext = _native.load(required=False)
    if ext is None:
        import pytest
        pytest.skip("extension not built")
    assert ext.gemm_plain_plan(1024, 1024, 8192, 148)[1] > 1
    assert ext.gemm_plain_plan(256, 1024, 8192, 148)[1] > 1
    assert ext.gemm_plain_plan(8192, 1024, 3072, 148) == [3, 1]       # CTA-pair tiles, no split
    assert ext.gemm_plain_plan(4096, 1024, 8192, 148)[1] == 1
    bn, splits = ext.gemm_plain_plan(8192, 4096, 64, 148)
    assert splits == 1


def test_both_arms_describe_the_workload_with_the_same_keys():
    bench = _bench()

    class Args:
        config = str(ROOT / "configs" / "stack_100m.json")
        length = 8192
        recompute = False

    ours = bench.common_config(Args, 1, 2)
    assert set(ours) == {"model", "global_batch", "seq_len", "parallelism", "activation_recompute", "l2"}
    assert ours["parallelism"] == "cp2" and ours["model"] == "stack_100m"
    assert [bench.last_window(k) for k in (1, 10, 20, 25, 100)] == [1, 10, 10, 5, 10]


def test_step_profile_puts_kernels_in_phases():
    from exploration_b200.tools.step_profile import phase_of
    assert phase_of("void eb::(anonymous namespace)::gemm_tc_kernel<256, 0, 0, 6, 0, 1>(CUtensorMap_st)") == "ulysses_scatter"
    assert phase_of("void eb::(anonymous namespace)::gemm_tc_kernel<256, 0, 1, 4, 1, 1>(x)") == "ulysses_gather"
    assert phase_of("void eb::(anonymous namespace)::gemm_tc_kernel<256, 1, 1, 1, 0, 2>(x)") == "gemm"
    assert phase_of("eb::(anonymous namespace)::heap_barrier_kernel(int)") == "heap_barrier"
    assert phase_of("eb::(anonymous namespace)::grad_reduce_kernel(x)") == "grad_reduce"
    assert phase_of("void eb::(anonymous namespace)::gated_dkv_tc_kernel<64, 16, 2>(x)") == "gated_attention"
    assert phase_of("ncclDevKernel_AllReduce_Sum_f32_RING_LL(x)") == "nccl"
    assert phase_of("something_else") == "other"
    assert phase_of("void eb::(anonymous namespace)::gemm_tc_kernel<256, false, true, 0, false, 2>(x)") == "gemm"
    assert phase_of("void eb::(anonymous namespace)::gemm_tc_kernel<256, false, false, 6, false, 1>(x)") == "ulysses_scatter"
    assert phase_of("void eb::(anonymous namespace)::gemm_tc_kernel<256, false, true, 4, true, 1>(x)") == "ulysses_gather"
