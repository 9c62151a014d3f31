"""Host-side logic that needs no GPU: the chunk-length policy, argument
checks that run before any CUDA call, and the bench's per-stage tables."""
import importlib.util
import os

import pytest
import torch

from conftest import ROOT


def test_chunk_policy_exact_by_default():
    from gdn2_package import gdn2_fwd
    assert gdn2_fwd.EXACT_BT and not gdn2_fwd.MASKED_TAIL
    k = gdn2_fwd._kernel_chunk
    assert k(8192, 128, 128) == 128
    assert k(8192, 64, 128) == 64          # exact BT: the CUDA-core kernels
    assert k(8192, 256, 128) == 128        # BT = 256 runs as chunks of 128
    assert k(256, 64, 64) == 64
    with pytest.raises(AssertionError, match="divisible"):
        k(100, 64, 128)
    with pytest.raises(ValueError):
        k(96, 32, 128)                     # no kernel runs chunks of 32


def test_chunk_policy_tensor_core_opt_in():
    from gdn2_package import gdn2_fwd
    gdn2_fwd.EXACT_BT = False
    k = gdn2_fwd._kernel_chunk
    assert k(4096, 64, 128) == 128         # merged onto the tensor-core chunk
    assert k(192, 64, 128) == 64           # T not a multiple of 128
    assert k(256, 64, 64) == 64            # D = 64 has no tensor-core path


def test_decode_rejects_unsupported_head_dim_before_cuda():
    from gdn2_package import gdn2_decode
    x = torch.zeros(1, 2, 1, 96)
    with pytest.raises(ValueError, match="head dim"):
        gdn2_decode(x, x, x, x, x, x, 0.1)
    y = torch.zeros(1, 2, 1, 64)
    with pytest.raises(ValueError, match="shape"):
        gdn2_decode(x, y, y, y, y, y, 0.1)


def test_bench_tables_cover_every_profiled_stage():
    from gdn2_package import _lib
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    fl, by = bench.flops_per_chunk(128, 128), bench.bytes_per_chunk(128, 128)
    assert set(_lib.STAGES) == set(fl) == set(by)
    assert set(bench.NCU_TRAFFIC_PER_CHUNK) <= set(_lib.STAGES)
    work = {k for k in fl if k != "bwd_exact"}   # the guard launch does no work unless flagged
    assert all(fl[k] > 0 for k in work) and all(by[k] > 0 for k in work)
    assert fl["bwd_exact"] == 0 and by["bwd_exact"] == 0
    # step-level work: the benchmark spec's per token and head figures for config 1
    f, b = bench.step_work(bench.CONFIGS[1])
    assert abs(f - 2.19e11) / 2.19e11 < 0.01 and abs(b - 4.03e9) / 4.03e9 < 0.01
    assert bench.tensor_peak(bench.CONFIGS[1], 1659.4)[0] == 1659.4 / 6
    assert bench.tensor_peak(bench.CONFIGS[2], 1659.4)[0] == 1659.4 / 6   # paired BT = 64 tiles
    assert bench._shard(bench.CONFIGS[1], 8, 0, "strong") == (1, 6)
    assert bench._shard(bench.CONFIGS[1], 4, 0, "strong") == (2, 6)
    assert bench._shard(bench.CONFIGS[1], 8, 0, "weak") == (8, 6)


def test_clock_summary_reads_only_samples_after_startup():
    """The bench's clock record: median SM clock and the throttle reasons seen
    in the samples taken after nvidia-smi's first (start-up) line."""
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    clk = bench.ClockSampler(0)
    row = "0, {sm}, 1965, 700.0, 0x0, Not Active, Not Active, {thermal}, {cap}"
    clk.lines = [row.format(sm=345, thermal="Not Active", cap="Not Active"),   # idle, before the region
                 row.format(sm=1965, thermal="Not Active", cap="Not Active"),
                 row.format(sm=1965, thermal="Not Active", cap="Active"),
                 row.format(sm=1950, thermal="Active", cap="Not Active"),
                 "garbled"]
    clk.n0 = 1
    s = clk.summary()
    assert s["samples"] == 3 and s["sm_mhz"] == 1965 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]
    clk.n0 = len(clk.lines)   # no sample after start-up: fall back to every line
    assert clk.summary()["samples"] == 4
