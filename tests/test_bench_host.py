"""Host logic of bench.py that needs no GPU: the per-rank workload of the
multi-GPU runs and the clock sampler's fallback."""
import os
import sys

import numpy as np

from conftest import ROOT

sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tgai-go_b200"))
import bench  # noqa: E402


def test_weak_scaling_gives_every_rank_the_one_gpu_profile():
    wl = bench.WORKLOADS["cfg4"]
    one = bench.rank_lengths(wl, 0, 0, 1, False)
    assert len(one) == wl["n_seq"]
    assert wl["lmin"] <= one.min() and one.max() <= wl["lmax"]
    for world in (2, 4, 8):
        for rank in range(world):
            assert np.array_equal(bench.rank_lengths(wl, 0, rank, world, False), one)


def test_strong_scaling_splits_the_one_gpu_set_once():
    wl = bench.WORKLOADS["cfg4"]
    one = bench.rank_lengths(wl, 0, 0, 1, False)
    for world in (2, 4, 8):
        parts = [bench.rank_lengths(wl, 0, r, world, True) for r in range(world)]
        assert sorted(np.concatenate(parts).tolist()) == sorted(one.tolist())
        loads = [int(p.sum()) for p in parts]
        # LPT: no rank exceeds the mean by more than the longest sequence
        assert max(loads) - sum(loads) / world <= one.max()


def test_clock_sampler_reports_samples_or_nothing():
    """NVML where it answers, else nvidia-smi; on a box with neither, no record
    (the bench line then carries clocks: null) rather than an error."""
    c = bench.ClockSampler(0)
    c.start()
    r = c.stop()
    if r is not None:
        assert r["samples"] >= 1 and r["sm_max_mhz"] > 0
        assert set(r["reasons"]) <= {"hw_slowdown", "hw_thermal_slowdown",
                                     "sw_thermal_slowdown", "sw_power_cap"}
