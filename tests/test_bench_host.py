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


def test_both_arms_print_the_same_config():
    """The reference arm's config is built from the arguments alone, by the
    same function the GPU arm uses, for every N and mode."""
    import argparse
    args = argparse.Namespace(seqs=0, layers=0, seed=1, gather="fused", weak=False)
    for world in (1, 2, 4, 8):
        for name in ("cfg4", "cfg5"):
            mode = bench.decode_mode(name, world, False)
            assert mode == ("own" if world == 1 else ("lpt" if name == "cfg4" else "heads"))
            c = bench.decode_config(args, name, world, mode)
            assert c == bench.decode_config(args, name, world, mode)
            assert c["sequences"] == bench.WORKLOADS[name]["n_seq"]
    weak = bench.decode_config(args, "cfg4", 4, bench.decode_mode("cfg4", 4, True))
    assert weak["sequences"] == 4 * 64 and "own set per GPU" in weak["parallelism"]


def test_cpu_sample_spans_short_and_long_contexts():
    wl = bench.WORKLOADS["cfg4"]
    lens = bench.lengths_for(wl, 1, 0)
    items = bench.make_cpu_sample(wl, lens, 1, max_bytes=3e8)
    ls = [it[2] for it in items]
    assert min(ls) == lens.min()
    assert max(ls) > np.percentile(lens, 75)
    assert sum(2 * L * wl["nkv"] * wl["hd"] * 4 for L in ls) <= 3e8
