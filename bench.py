"""Benchmark of the KV-cache decode path (append + GQA decode attention).

Default workload ("cfg4"): 64 independent sequences
with context lengths U[1k, 32k], 32 layers, 32 query / 8 KV heads, head_dim
128, bf16 caches.  One step = for every layer, one batched decode call (append
of each sequence's new K/V row + split-sequence attention of its new query
over the whole cache).  The metric is decode tokens/s (one token per sequence
per step, all layers) and achieved HBM GB/s of the attention launches.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload cfg4|cfg5|cfg2|cfg3|fwd]

N > 1 runs under torchrun, one rank per GPU.  The cfg4 headline shards the one
set of 64 sequences over the ranks by longest-processing-time on length
(strong scaling, no collective on the data path).  Beside it the same line
carries `weak` (N > 1: every rank its own 64 sequences) and `cfg5`
(configs[4]: one 131072-token sequence; at N > 1 its KV-head groups are split
over the ranks and the attention kernel gathers the per-head outputs over
NVLink).  `--workload cfg5|cfg2` runs those alone.

Inputs are synthetic (seeded normal values; the reference names no dataset)
and larger than L2 (126 MB) between timed iterations.  `--impl reference`
times the reference algorithm's CPU path (the engine-order restatement of
src/tgai_engine.c:3943-4011 in oracle/, all host threads) on a bounded sample
of the same workload, extrapolated to the full step, with the same config.
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tgai-go_b200"))

HBM_FALLBACK_GBS = 6650.0
METRIC = "decode attn+KV-append tokens/s & HBM GB/s vs ~8 TB/s peak at 1/2/4/8 B200"

WORKLOADS = {
    # name: sequences per rank, layers, q heads, kv heads, head_dim, length range
    # (caches bf16 unless the entry says dtype "f32")
    "cfg1": dict(n_seq=1, layers=4, nh=8, nkv=8, hd=64, lmin=512, lmax=512, dtype="f32",
                 desc="configs[0] at its largest context: 1 seq, L=512, 4 layers, 8q/8kv, hd64, "
                      "fp32"),
    "cfg4": dict(n_seq=64, layers=32, nh=32, nkv=8, hd=128, lmin=1024, lmax=32768,
                 desc="configs[3]: 64 seqs, L~U[1k,32k], 32 layers, 32q/8kv, hd128, bf16"),
    "cfg5": dict(n_seq=1, layers=32, nh=32, nkv=8, hd=128, lmin=131072, lmax=131072,
                 desc="configs[4]: 1 seq, L=131072, 32 layers, 32q/8kv, hd128, bf16"),
    "cfg2": dict(n_seq=1, layers=24, nh=16, nkv=4, hd=128, lmin=4096, lmax=4096,
                 desc="configs[1] at its largest context: 1 seq, L=4096, 24 layers, 16q/4kv, hd128, bf16"),
    "cfg3": dict(n_seq=1, layers=24, nh=16, nkv=4, hd=128, lmin=64, lmax=512,
                 desc="configs[2]: multi-turn LCP reuse, keep U[50%,95%] of history, append a "
                      "U[64,512]-token suffix, causal suffix attention; 24 layers, 16q/4kv, hd128, bf16"),
}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


class NvmlSampler:
    """SM clock and clock-event reasons read through NVML every 10 ms from a
    thread during the timed region (read-only queries), so that a region of a
    few hundred milliseconds still gets tens of samples.  The device is found
    by the PCI address torch reports for the CUDA device, so the CUDA and NVML
    orders need not agree."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, cuda_dev):
        import pynvml
        self.nv = pynvml
        pynvml.nvmlInit()
        try:
            import torch
            pr = torch.cuda.get_device_properties(cuda_dev)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            self.h = pynvml.nvmlDeviceGetHandleByIndex(cuda_dev)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        self.sm, self.bits, self.stop_ev, self.th = [], 0, None, None

    def _run(self):
        nv = self.nv
        while not self.stop_ev.is_set():
            try:
                self.sm.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.bits |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            self.stop_ev.wait(0.01)

    def start(self):
        import threading
        self.stop_ev = threading.Event()
        self.th = threading.Thread(target=self._run, daemon=True)
        self.th.start()

    def stop(self):
        if not self.th:
            return None
        self.stop_ev.set()
        self.th.join(timeout=5)
        if not self.sm:
            return None
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": self.max_mhz,
                "samples": len(self.sm),
                "reasons": sorted(n for b, n in self.REASONS.items() if self.bits & b),
                "source": "nvml every 10 ms"}


def ClockSampler(cuda_dev):
    """The NVML sampler where pynvml is importable and answers, else nvidia-smi."""
    try:
        return NvmlSampler(cuda_dev)
    except Exception:
        return SmiClockSampler(cuda_dev)


class SmiClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons), "source": "nvidia-smi every 200 ms"}


def lengths_for(wl, seed, rank):
    rng = np.random.default_rng([seed, rank, 4])
    return rng.integers(wl["lmin"], wl["lmax"] + 1, wl["n_seq"]).astype(np.int64)


def rank_lengths(wl, seed, rank, world, shard_seqs):
    """Context lengths of this rank's sequences.  Weak scaling (default):
    every rank serves its own set (values seeded per rank) with the 1-GPU
    run's length profile, so per-GPU work is fixed as N grows.  shard_seqs
    (strong scaling): the 1-GPU set split over the ranks by LPT on length."""
    all_lens = lengths_for(wl, seed, 0)
    if not shard_seqs:
        return all_lens
    import shard
    return all_lens[shard.lpt_partition(all_lens, world)[rank]]


def cache_esize(wl):
    return 4 if wl.get("dtype") == "f32" else 2


def attn_bytes(lens_after, nh, nkv, hd, b=2):
    """Algorithmic bytes of one layer's decode call: K and V read once per KV
    head over L positions, the new row's append write, q read and out write."""
    L = np.asarray(lens_after, np.float64)
    return float((2 * L * nkv * hd * b + 2 * nkv * hd * b + nh * hd * 4 * 2).sum())


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    return world, rank, local


def make_cpu_sample(wl, lens, seed, max_bytes=1.5e9):
    """Whole sequences of one layer as fp32 caches (the reference has no bf16
    cache), within max_bytes of host memory, taken at evenly spaced ranks of
    the sorted lengths so that short and long contexts are both timed."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    nh, nkv, hd = wl["nh"], wl["nkv"], wl["hd"]
    order = np.argsort(lens, kind="stable")
    per_pos = 2 * nkv * hd * 4
    mean_b = float(np.mean(lens)) * per_pos
    k = int(max(1, min(len(lens), max_bytes // max(mean_b, 1.0))))
    picks = order[np.unique(np.round(np.linspace(0, len(lens) - 1, k)).astype(int))]
    items, used = [], 0
    for idx in picks:
        L = int(lens[idx])
        b = L * per_pos
        if items and used + b > max_bytes:
            continue
        items.append((O.normal(2 * L * nkv * hd, seed, int(idx), 9),
                      O.normal(nh * hd, seed, int(idx), 10), L))
        used += b
    return items


def time_cpu_sample(wl, lens, items, threads, budget_s):
    """Reference-order CPU decode (oracle/: the engine loop of
    src/tgai_engine.c:3943-4011, one query per sequence) over the sample until
    budget_s of CPU work; extrapolated by positions x layers to the full step.
    Returns (tokens/s, description, seconds timed)."""
    import oracle as O
    nh, nkv, hd = wl["nh"], wl["nkv"], wl["hd"]
    done, spent, n = 0, 0.0, 0
    while spent < budget_s or n < len(items):
        kvc, q, L = items[n % len(items)]
        t0 = time.perf_counter()
        O.decode_batch([kvc], [q], [L], nh, nkv, hd, threads=threads)
        spent += time.perf_counter() - t0
        done += L
        n += 1
    step_s = spent * float(np.sum(lens)) * wl["layers"] / done
    ls = sorted(it[2] for it in items)
    desc = (f"extrapolated: {n} single-layer sequence decodes over {len(items)} of the "
            f"{len(lens)} sequences (L={ls[0]}..{ls[-1]}, evenly spaced ranks of the sorted "
            f"lengths), fp32 cache, {spent:.1f}s of CPU work, scaled by positions x "
            f"{wl['layers']} layers to the full step")
    return len(lens) / step_s, desc, spent


def workload(args, name):
    wl = dict(WORKLOADS[name])
    if args.seqs:
        wl["n_seq"] = args.seqs
    if args.layers:
        wl["layers"] = args.layers
    if getattr(args, "kv_heads", 0):
        wl["nkv"] = args.kv_heads
    if getattr(args, "q_heads", 0):
        wl["nh"] = args.q_heads
    return wl


def decode_mode(name, world, weak):
    """How a decode workload spreads over `world` ranks: 'own' (every rank
    its own copy of the set: weak scaling), 'lpt' (the one set of sequences
    split by longest-processing-time: strong) or 'heads' (the KV heads of
    the set split into groups, outputs gathered: strong)."""
    if world == 1:
        return "own"
    if name == "cfg4":
        return "own" if weak else "lpt"
    return "heads"


def job_lengths(wl, seed, world, mode):
    """Context lengths of every sequence of the whole job (all ranks)."""
    one = lengths_for(wl, seed, 0)
    return np.tile(one, world) if mode == "own" else one


def decode_config(args, name, world, mode):
    """The `config` of a decode line: a function of the arguments only, so
    the reference arm prints the same one."""
    wl = workload(args, name)
    lens = job_lengths(wl, args.seed, world, mode)
    if mode == "heads":
        par = f"kv-head groups x{world} + " + ("in-kernel NVLink gather" if args.gather == "fused"
                                                else "NCCL all-gather")
    elif mode == "lpt":
        par = f"sequences x{world} (LPT split of one set), no collective"
    else:
        par = (f"sequences x{world} (own set per GPU), no collective" if world > 1 else
               "one GPU")
    return {"workload": name, "desc": wl["desc"], "layers": wl["layers"],
            "sequences": int(len(lens)),
            "kv_heads_per_gpu": wl["nkv"] // world if mode == "heads" else wl["nkv"],
            "context_mean": float(np.mean(lens)),
            "l2": "inputs larger than L2 (K/V read per step >> 126 MB)",
            "parallelism": par}


def run_reference(args):
    """--impl reference: the reference algorithm's CPU path, all host threads,
    on the same workload and config as this arm."""
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return
    name = args.workload
    wl = workload(args, name)
    mode = decode_mode(name, world, args.weak)
    lens = lengths_for(wl, args.seed, 0)     # the job repeats this set under 'own'
    threads = os.cpu_count() or 1
    items = make_cpu_sample(wl, lens, args.seed)
    budget = max(0.5, args.cpu_total_s / max(1, args.steps + args.warmup))
    vals, secs = [], []
    for i in range(args.warmup + args.steps):
        tok, desc, spent = time_cpu_sample(wl, lens, items, threads, budget)
        if i >= args.warmup:
            vals.append(tok)
            secs.append(spent)
    v = float(np.median(vals))
    njob = len(job_lengths(wl, args.seed, world, mode))
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        # what each timed step took: a bounded sample of the workload
        "ms_per_step": 1000.0 * float(np.median(secs)),
        "full_step_ms_extrapolated": 1000.0 * njob / v,
        "extrapolated": True,
        "higher_is_better": True, "scaling": "weak" if mode == "own" and world > 1 else "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": decode_config(args, name, world, mode),
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def decode_run(args, lib, name, world, rank, local, mode, cpu=False):
    """One decode workload: fill the caches, time `steps` decode steps on the
    device and again through host buffers, free everything.  Every rank
    returns the same summary (times are the max over ranks)."""
    import torch
    import torch.distributed as dist
    import tgkv
    import shard
    wl = workload(args, name)
    if mode == "heads":
        kv0, kv1, q0, q1 = shard.kv_head_shard(wl["nh"], wl["nkv"], world, rank)
        nkv, nh = kv1 - kv0, q1 - q0
    else:
        nkv, nh = wl["nkv"], wl["nh"]
    hd, layers = wl["hd"], wl["layers"]
    lens0 = rank_lengths(wl, args.seed, rank, world, mode == "lpt")
    n_seq = len(lens0)
    kvd = nkv * hd
    e2e_steps = 0 if args.no_e2e else args.steps
    e2e_warm = 0 if args.no_e2e else args.warmup
    total_steps = args.warmup + args.steps + e2e_warm + e2e_steps + 1
    stream = torch.cuda.current_stream()
    sh = tgkv.stream_handle(stream)

    # ---- caches: one per (layer, sequence), filled by the append kernel
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed * 1000 + rank)
    caches = [[None] * n_seq for _ in range(layers)]
    t_fill = time.time()
    for i in range(n_seq):
        L = int(lens0[i])
        for l in range(layers):
            c = lib.tg_kv_create_ex(L + total_steps, nkv, hd,
                                    tgkv.TG_KV_F32 if cache_esize(wl) == 4 else tgkv.TG_KV_BF16)
            tgkv.check(c, lib, "tg_kv_create_ex")
            k = torch.randn(L, kvd, device="cuda", generator=gen)
            v = torch.randn(L, kvd, device="cuda", generator=gen)
            tgkv.check(lib.tg_kv_append_dev(c, k.data_ptr(), v.data_ptr(), L, sh), lib,
                       "append_dev")
            caches[l][i] = c
    torch.cuda.synchronize()
    t_fill = time.time() - t_fill
    plans = []
    for l in range(layers):
        arr = (C.c_void_p * n_seq)(*caches[l])
        b = lib.tg_kv_batch_create(arr, n_seq, nh)
        tgkv.check(b, lib, "tg_kv_batch_create")
        plans.append(b)
    q = [torch.randn(n_seq, nh, hd, device="cuda", generator=gen) for _ in range(layers)]
    kn = [torch.randn(n_seq, kvd, device="cuda", generator=gen) for _ in range(layers)]
    vn = [torch.randn(n_seq, kvd, device="cuda", generator=gen) for _ in range(layers)]
    out = [torch.empty(n_seq, nh, hd, device="cuda") for _ in range(layers)]
    heads = mode == "heads"
    gathered = ([torch.empty(world, n_seq, nh, hd, device="cuda") for _ in range(layers)]
                if heads else None)
    # in-kernel gather over NVLink: every rank's attention stores its heads'
    # outputs into every rank's gathered buffer (CUDA IPC peer memory); one
    # gather object serves every layer and step
    fused = heads and args.gather == "fused"
    gather = None
    if fused:
        gather = lib.tg_kv_gather_create(world, rank, n_seq * nh * hd)
        tgkv.check(gather, lib, "tg_kv_gather_create")
        h = (C.c_uint8 * 64)()
        tgkv.check(lib.tg_kv_gather_export(gather, h), lib, "tg_kv_gather_export")
        allh = [None] * world
        dist.all_gather_object(allh, bytes(h))
        tgkv.check(lib.tg_kv_gather_import(gather, b"".join(allh)), lib, "tg_kv_gather_import")
    launches = [0]

    def step(events=None):
        for l in range(layers):
            if events is not None:
                events[l][0].record(stream)
            if fused:
                ok = lib.tg_kv_batch_decode_gather(plans[l], q[l].data_ptr(), kn[l].data_ptr(),
                                                   vn[l].data_ptr(), out[l].data_ptr(),
                                                   gather, sh)
            else:
                ok = lib.tg_kv_batch_decode(plans[l], q[l].data_ptr(), kn[l].data_ptr(),
                                            vn[l].data_ptr(), out[l].data_ptr(), sh)
            if not ok:
                raise RuntimeError(lib.tg_kv_last_error().decode())
            launches[0] += lib.tg_kv_batch_last_launches(plans[l])
            if events is not None:
                events[l][1].record(stream)
            if heads and not fused:
                dist.all_gather_into_tensor(gathered[l], out[l])

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x):
        return shard.max_over_ranks(x, world, device="cuda")

    for _ in range(args.warmup):
        step()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    ev = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
          for _ in range(layers * args.steps)]
    lens_step = np.array([lib.tg_kv_len(caches[0][i]) for i in range(n_seq)]) + 1
    launches[0] = 0
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    # Per-call events only where NCCL collectives share the step: otherwise the
    # step is nothing but the per-layer attention launches, back to back, and
    # events between them would break their programmatic-dependent overlap
    # (a 13 us cfg2 call measured 21 us with them).
    per_call_events = heads and not fused
    t0.record(stream)
    for s_ in range(args.steps):
        step(ev[s_ * layers:(s_ + 1) * layers] if per_call_events else None)
    t1.record(stream)
    barrier()
    clock = clocks.stop()
    timed_launches = launches[0]
    kid = lib.tg_cuda_kv_attn_last_kernel()
    ms = t0.elapsed_time(t1) / args.steps
    ms_max = max_over_ranks(ms)
    algo = sum(attn_bytes(lens_step + s_, nh, nkv, hd, cache_esize(wl))
               for s_ in range(args.steps)) * layers
    if per_call_events:
        call_ms = sum(a.elapsed_time(b) for a, b in ev)
    else:
        call_ms = ms * args.steps                      # the timed region is the calls
    kernel_gbs = algo / (call_ms / 1000.0) / 1e9
    # the slowest rank's achieved bandwidth and the least-loaded rank's
    gbs_min = -max_over_ranks(-kernel_gbs)
    per_launch_bytes = algo / (args.steps * layers)
    # tokens per step over all ranks: the whole sequence set once (sharded
    # heads or LPT-split sequences), else every rank's own sequences
    tokens = n_seq * world if mode == "own" else wl["n_seq"]

    # ---- end to end: host buffers, copies inside the timed region
    e2e = None
    if e2e_steps:
        qh = [torch.randn(n_seq, nh, hd, generator=torch.Generator().manual_seed(l)).pin_memory()
              for l in range(layers)]
        kh = [torch.randn(n_seq, kvd).pin_memory() for _ in range(layers)]
        vh = [torch.randn(n_seq, kvd).pin_memory() for _ in range(layers)]
        oh = [torch.empty((world if fused else 1) * n_seq, nh, hd).pin_memory()
              for _ in range(layers)]

        def step_host():
            for l in range(layers):
                if fused:       # out_host receives every rank's outputs
                    ok = lib.tg_kv_batch_decode_gather_host(
                        plans[l], qh[l].data_ptr(), kh[l].data_ptr(), vh[l].data_ptr(),
                        oh[l].data_ptr(), gather, sh)
                else:
                    ok = lib.tg_kv_batch_decode_host(plans[l], qh[l].data_ptr(),
                                                     kh[l].data_ptr(), vh[l].data_ptr(),
                                                     oh[l].data_ptr(), sh)
                if not ok:
                    raise RuntimeError(lib.tg_kv_last_error().decode())
                if heads and not fused:
                    dist.all_gather_into_tensor(gathered[l], out[l])

        for _ in range(e2e_warm):
            step_host()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            step_host()
        e1.record(stream)
        barrier()
        e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
        h2d = layers * (qh[0].numel() + 2 * kh[0].numel()) * 4
        d2h = layers * oh[0].numel() * 4
        e2e = {"value": tokens / (e_ms / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e_ms}

    err = lib.tg_cuda_kv_device_error()
    barrier()                     # no rank still writes into a peer's buffer
    if gather:
        lib.tg_kv_gather_destroy(gather)
    for b in plans:
        lib.tg_kv_batch_destroy(b)
    for row in caches:
        for c in row:
            lib.tg_kv_destroy(c)
    del q, kn, vn, out, gathered
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if err:
        raise RuntimeError(f"kernel bounded wait expired (code {err})")

    peak, peak_kind = measured_peak()
    traffic = None
    tp = os.path.join(ROOT, "profiles", "attention_dram_ratio.json")
    if os.path.exists(tp):
        try:
            # DRAM bytes / algorithmic bytes of the kernel that ran, from its ncu capture
            key = {1: "attention_kernel", 3: "attention_tc_kernel"}[kid]
            traffic = per_launch_bytes * float(json.load(open(tp))[key])
        except Exception:
            traffic = None
    cpu_line = None
    if cpu and rank == 0 and world == 1 and not args.no_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        items = make_cpu_sample(wl, lens0, args.seed)
        tok, desc, _ = time_cpu_sample(wl, lens0, items, 1, args.cpu_baseline_s)
        cpu_line = {"value": tok, "unit": "tokens/s", "cores": 1, "kind": "port",
                    "sample": desc}
    return {
        "value": tokens / (ms_max / 1000.0), "ms_per_step": ms_max, "tokens_per_step": tokens,
        "kernel_gbs": kernel_gbs, "algo": algo, "per_launch_bytes": per_launch_bytes,
        "roofline": {"bound": "hbm", "achieved": kernel_gbs, "peak": peak, "unit": "GB/s",
                     "frac": kernel_gbs / peak, "traffic": traffic, "peak_source": peak_kind,
                     "min_rank_frac": gbs_min / peak,
                     "kernel": ("tg_kv_batch_decode per layer (append fused into the "
                                "split-sequence attention launch): CUDA events on the launch "
                                "stream, " + ("around every call" if per_call_events else
                                              "around the timed region, which holds only "
                                              "these calls")),
                     "algorithmic_bytes_per_launch": per_launch_bytes},
        "hbm_gbs": algo / (ms * args.steps / 1000.0) / 1e9,
        "gpu_launches": timed_launches, "clocks": clock, "e2e": e2e, "cpu_baseline": cpu_line,
        "details": {"attention_kernel": {1: "attention_kernel (CUDA cores)",
                                         3: "attention_tc_kernel (tcgen05)"}.get(kid, "?"),
                    "sequences_per_gpu": n_seq, "query_heads_per_gpu": nh,
                    "fill_s": round(t_fill, 1)},
    }


def sub_record(args, name, world, mode, r):
    """A decode run beside the headline, in the same units."""
    return {"workload": name, "value": r["value"], "unit": "tokens/s",
            "ms_per_step": r["ms_per_step"],
            "scaling": "weak" if mode == "own" and world > 1 else "strong",
            "config": decode_config(args, name, world, mode),
            "roofline": r["roofline"], "e2e": r["e2e"], "gpu_launches": r["gpu_launches"],
            "clocks": r["clocks"], "details": r["details"]}


def run_ours(args):
    import torch
    import torch.distributed as dist
    import tgkv

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    lib = tgkv.load()
    tgkv.check(lib.tg_cuda_kv_set_device(local), lib, "set_device")
    tgkv.check(lib.tg_be_select(b"cuda"), lib, "tg_be_select")
    name = args.workload
    mode = decode_mode(name, world, args.weak)
    r = decode_run(args, lib, name, world, rank, local, mode, cpu=True)
    extra = {}
    if name == "cfg4" and not args.no_extra:
        # beside the headline: every GPU with its own 64 sequences (weak
        # scaling) at N > 1, and configs[4] (one 131072-token sequence; KV
        # heads split over the GPUs at N > 1)
        if world > 1 and mode != "own":
            extra["weak"] = sub_record(args, "cfg4", world, "own",
                                       decode_run(args, lib, "cfg4", world, rank, local, "own"))
        m5 = decode_mode("cfg5", world, False)
        extra["cfg5"] = sub_record(args, "cfg5", world, m5,
                                   decode_run(args, lib, "cfg5", world, rank, local, m5))
    if rank == 0:
        line = {
            "metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True,
            "scaling": "weak" if mode == "own" and world > 1 else "strong",
            "vs_baseline": None, "dtype": "f32" if cache_esize(WORKLOADS[name]) == 4 else "bf16",
            "data": "synthetic",
            "config": decode_config(args, name, world, mode),
            "hbm_gbs": r["hbm_gbs"],
            "roofline": r["roofline"],
            "gpu_launches": r["gpu_launches"],
            "clocks": r["clocks"],
            "e2e": r["e2e"],
            "cpu_baseline": r["cpu_baseline"],
            "details": r["details"],
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def turn_script(seed, n_turns, lmin, lmax, vocab=32000):
    """configs[2]'s turns: (lcp, suffix length) per turn.  Token ids only
    matter through the LCP (K/V are synthetic), so the script keeps lengths."""
    rng = np.random.default_rng([seed, 3])
    hist, out = 0, []
    for _ in range(n_turns):
        lcp = int(hist * rng.uniform(0.5, 0.95))
        n = int(rng.integers(lmin, lmax + 1))
        out.append((lcp, n))
        hist = lcp + n
    return out


def run_cfg3(args):
    """One step = one chat turn over all layers: truncate every layer's cache
    to the turn's LCP, append the suffix's K/V and attend the suffix queries
    causally (tg_kv_append_attention).  tokens/s counts suffix tokens through
    all layers."""
    import torch
    import tgkv
    lib = tgkv.load()
    tgkv.check(lib.tg_be_select(b"cuda"), lib, "tg_be_select")
    wl = WORKLOADS["cfg3"]
    nh, nkv, hd, layers = wl["nh"], wl["nkv"], wl["hd"], wl["layers"]
    kvd = nkv * hd
    turns = turn_script(args.seed, args.warmup + args.steps, wl["lmin"], wl["lmax"])
    max_len = max(l + n for l, n in turns)
    stream = torch.cuda.current_stream()
    sh = tgkv.stream_handle(stream)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed)
    caches = []
    for _ in range(layers):
        c = lib.tg_kv_create_ex(max_len, nkv, hd, tgkv.TG_KV_BF16)
        tgkv.check(c, lib, "tg_kv_create_ex")
        caches.append(c)
    nmax = wl["lmax"]
    q = [torch.randn(nmax, nh, hd, device="cuda", generator=gen) for _ in range(layers)]
    k = [torch.randn(nmax, kvd, device="cuda", generator=gen) for _ in range(layers)]
    v = [torch.randn(nmax, kvd, device="cuda", generator=gen) for _ in range(layers)]
    out = [torch.empty(nmax, nh, hd, device="cuda") for _ in range(layers)]

    launches = [0]
    fused = os.environ.get("TGKV_FUSE_SUFFIX", "") == "1"

    def turn(lcp, n):
        # truncate to the LCP, then the suffix's append + causal attention in
        # one call (one launch of the tensor-core suffix kernel where it applies)
        for l in range(layers):
            c = caches[l]
            tgkv.check(lib.tg_kv_truncate(c, min(lcp, lib.tg_kv_len(c))), lib, "truncate")
            tgkv.check(lib.tg_kv_append_attention(c, k[l].data_ptr(), v[l].data_ptr(),
                                                  q[l].data_ptr(), out[l].data_ptr(), nh, n, sh),
                       lib, "append + attention")
            # the attention's launches, and the append kernel's unless fused in
            launches[0] += lib.tg_cuda_kv_attn_last_launches() + (0 if fused else 1)

    for lcp, n in turns[:args.warmup]:
        turn(lcp, n)
    torch.cuda.synchronize()
    launches[0] = 0
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for lcp, n in turns[args.warmup:]:
        turn(lcp, n)
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    kernel = {1: "split-sequence", 2: "tcgen05 suffix"}.get(lib.tg_cuda_kv_attn_last_kernel(), "?")
    timed = turns[args.warmup:]
    tokens = sum(n for _, n in timed)
    # causal suffix attention FLOPs (QK^T + PV) over all layers
    flops = sum(4.0 * nh * hd * sum(l + j + 1 for j in range(n)) for l, n in timed) * layers

    # The appends alone: the same turns' truncate + append of every layer, no
    # attention, timed as one region (the append launches back to back).
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for lcp, n in timed:
        for l in range(layers):
            c = caches[l]
            tgkv.check(lib.tg_kv_truncate(c, min(lcp, lib.tg_kv_len(c))), lib, "truncate")
            tgkv.check(lib.tg_kv_append_dev(c, k[l].data_ptr(), v[l].data_ptr(), n, sh), lib,
                       "append")
    a1.record(stream)
    torch.cuda.synchronize()
    a_ms = a0.elapsed_time(a1)
    rows = sum(n for _, n in timed) * layers
    app_write = 2.0 * rows * kvd * 2          # K and V rows written, bf16
    app_read = 2.0 * rows * kvd * 4           # K and V rows read, fp32
    for c in caches:
        lib.tg_kv_destroy(c)
    line = {"metric": METRIC, "value": tokens / (ms / 1000.0), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": "cfg3", "desc": wl["desc"], "turns": timed,
                       "attention_kernel": kernel},
            "attention_tflops": flops / (ms / 1000.0) / 1e12,
            "gpu_launches": launches[0],
            "append": {"ms_per_turn": a_ms / len(timed),
                       "write_gbs": app_write / (a_ms / 1000.0) / 1e9,
                       "read_write_gbs": (app_write + app_read) / (a_ms / 1000.0) / 1e9,
                       "launches_per_turn": layers,
                       "bytes": "write: 2 x rows x kv_dim x 2 B (bf16); read: the fp32 rows"}}
    print(json.dumps(line), flush=True)


# ---- whole-model decode through the engine seam's forward (tg_fwd_*) ----
# A synthetic model shaped like the reference's headline whole-model number
# (README.md:279: "V2.7 3B BF16, 28-layer MoE", 11.2 tok/s on 8 CPU threads):
# 28 layers, d_model 1536, 12 query / 4 KV heads of 128, 8 experts top-2 with
# d_ff 2560 and a router bias, vocab 32000 (2.9 B parameters, fp32 here).
FWD = dict(arch=0, n_layers=28, d_model=1536, n_heads=12, n_kv_heads=4, d_ff=2560, vocab=32000,
           max_seq=4096, n_experts=8, n_activated=2, rope_theta=10000, unk=1, qkv_bias=False,
           qb_bias=True)
FWD_METRIC = "whole-model decode tokens/s (tg_engine_cuda_forward / tg_fwd_forward)"


def fwd_shapes(cfg):
    """name -> (rows, cols) of every tensor of the model."""
    d, dff, ne = cfg["d_model"], cfg["d_ff"], cfg["n_experts"]
    hd = d // cfg["n_heads"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    sh = {"token_embedding.weight": (cfg["vocab"], d), "final_norm.weight": (d, 1)}
    for l in range(cfg["n_layers"]):
        p = f"blocks.{l}."
        sh.update({p + "ln1.weight": (d, 1), p + "ln2.weight": (d, 1),
                   p + "attn.q_proj.weight": (qd, d), p + "attn.k_proj.weight": (kvd, d),
                   p + "attn.v_proj.weight": (kvd, d), p + "attn.out_proj.weight": (d, qd),
                   p + "moe.router.weight": (ne, d), p + "moe._qb_bias": (ne, 1)})
        for e in range(ne):
            sh[p + f"moe.experts.{e}.w1.weight"] = (dff, d)
            sh[p + f"moe.experts.{e}.w2.weight"] = (dff, d)
            sh[p + f"moe.experts.{e}.w3.weight"] = (d, dff)
    return sh


def fwd_tensor(seed, name, rows, cols):
    """Seeded uniform values of unit variance / sqrt(fan-in); norms near 1."""
    import zlib
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    a = rng.random((rows, cols) if cols > 1 else rows, dtype=np.float32) - np.float32(0.5)
    if name.endswith("norm.weight") or ".ln" in name:
        return np.float32(1.0) + np.float32(0.2) * a
    if name == "token_embedding.weight":
        return np.float32(np.sqrt(12.0)) * a
    return a * np.float32(np.sqrt(12.0 / max(cols, 1)))


def fwd_bytes_per_token(cfg, ctx):
    """Algorithmic HBM bytes of one decode token (fp32): every weight the token
    touches once (attention, router, the top-k experts, the LM head), the K/V
    of ctx positions read once per KV head and the new row written."""
    d, dff, ne, na = cfg["d_model"], cfg["d_ff"], cfg["n_experts"], cfg["n_activated"]
    hd = d // cfg["n_heads"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    per_layer = (2 * d + (qd + 2 * kvd) * d + d * qd + ne * d + ne + na * 3 * dff * d
                 + 2 * ctx * kvd + 2 * kvd)
    return 4.0 * (cfg["n_layers"] * per_layer + cfg["vocab"] * d + 2 * d)


def fwd_cpu_sample(cfg, seed, prefill, steps, threads):
    """The reference engine's own CPU forward (oracle/_ref build of
    src/tgai_engine.c) on the same model cut to 2 and 4 layers: decode
    seconds per token at each, extrapolated linearly in layers.  None when
    the reference build is absent."""
    so = os.path.join(ROOT, "oracle", "_ref", "libtgai_engine_ref.so")
    if not os.path.exists(so):
        return None
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import tempfile
    import fwd_model as FM
    eng = C.CDLL(so, mode=os.RTLD_LAZY)
    eng.tg_load.restype = C.c_void_p
    eng.tg_load.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_int)]
    eng.tg_kvcache_new.restype = C.c_void_p
    eng.tg_kvcache_new.argtypes = [C.c_void_p, C.c_int]
    eng.tg_kvcache_free.argtypes = [C.c_void_p]
    eng.tg_forward.restype = C.POINTER(C.c_float)
    eng.tg_forward.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_void_p, C.c_int]
    eng.tg_free.argtypes = [C.c_void_p]
    eng.tg_set_nthreads.argtypes = [C.c_int]
    eng.tg_set_nthreads(threads)
    ids = np.random.default_rng(seed).integers(0, cfg["vocab"], prefill + steps).astype(np.int32)
    per = {}
    for nl in (2, 4):
        c = dict(cfg, n_layers=nl)
        w = {n: fwd_tensor(seed, n, *rc) for n, rc in fwd_shapes(c).items()}
        with tempfile.TemporaryDirectory() as td:
            path = os.path.join(td, "m.TG")
            FM.write_tg(path, c, w)
            del w
            err = C.c_int(0)
            m = eng.tg_load(path.encode(), 1, C.byref(err))
            if not m:
                return None
            kv = eng.tg_kvcache_new(m, prefill + steps + 1)
            arr = (C.c_int32 * prefill)(*ids[:prefill].tolist())
            eng.tg_forward(m, arr, prefill, kv, 0)
            t0 = time.perf_counter()
            for i in range(steps):
                one = (C.c_int32 * 1)(int(ids[prefill + i]))
                eng.tg_forward(m, one, 1, kv, prefill + i)
            per[nl] = (time.perf_counter() - t0) / steps
            eng.tg_kvcache_free(kv)
            eng.tg_free(m)
    slope = (per[4] - per[2]) / 2.0
    t_tok = per[2] + slope * (cfg["n_layers"] - 2)
    desc = (f"reference engine tg_forward (oracle/_ref), fp32, {threads} threads: {steps} decode "
            f"tokens after a {prefill}-token prefill on the model cut to 2 and 4 layers "
            f"({per[2] * 1e3:.1f} / {per[4] * 1e3:.1f} ms per token), extrapolated linearly to "
            f"{cfg['n_layers']} layers")
    return 1.0 / t_tok, desc


def run_fwd(args):
    """One step = one decode token of one sequence through tg_fwd_forward
    (host token id in, host logits out, synchronous as a sampling loop
    needs), after a 512-token prefill."""
    world, rank, _ = dist_setup(args)
    cfg = dict(FWD)
    if args.layers:                  # a cut-down model for small profiling captures
        cfg["n_layers"] = args.layers
    prefill = 512
    threads = os.cpu_count() or 1
    if args.impl == "reference":
        if rank != 0:
            return
        r = fwd_cpu_sample(cfg, args.seed, prefill, max(args.steps, 3), threads)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref engine not built"}))
            return
        v, desc = r
        print(json.dumps({
            "impl": "reference", "metric": FWD_METRIC, "value": v, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 / v, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "fwd", "model": "V2.7-shaped 28-layer MoE (synthetic)"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads,
                             "kind": "reference", "sample": desc},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return
    import tgkv
    lib = tgkv.load()
    if world > 1:
        tgkv.check(lib.tg_cuda_kv_set_device(int(os.environ.get("LOCAL_RANK", "0"))), lib)
    tgkv.check(lib.tg_be_select(b"cuda"), lib, "tg_be_select")
    shapes = fwd_shapes(cfg)
    held = {}

    def get(ctx, name, shape):
        # tg_fwd_create reads a layer's tensors while it assembles that layer:
        # every array of the current layer stays alive until the next begins
        n = name.decode()
        rc = shapes.get(n)
        if rc is None:
            return None
        layer = n.split(".")[1] if n.startswith("blocks.") else None
        if layer is not None and held.get("_layer") != layer:
            held.clear()
            held["_layer"] = layer
        a = held[n] = fwd_tensor(args.seed, n, *rc)
        shape[0], shape[1] = rc
        return a.ctypes.data

    cb = tgkv.WEIGHT_FN(get)
    fc = tgkv.TGFwdConfig(n_layers=cfg["n_layers"], d_model=cfg["d_model"],
                          n_heads=cfg["n_heads"], n_kv_heads=cfg["n_kv_heads"], d_ff=cfg["d_ff"],
                          vocab_size=cfg["vocab"], max_seq_len=cfg["max_seq"],
                          n_experts=cfg["n_experts"], n_activated=cfg["n_activated"],
                          rope_theta=cfg["rope_theta"], unk_id=cfg["unk"])
    m = lib.tg_fwd_create(C.byref(fc), cb, None)
    held.clear()
    if not m:
        raise SystemExit("tg_fwd_create: " + lib.tg_fwd_last_error().decode())
    ids = np.random.default_rng([args.seed, rank]).integers(
        0, cfg["vocab"], prefill + args.warmup + args.steps).astype(np.int32)
    key = C.c_void_p(1)

    def fwd(tok, pos):
        p = lib.tg_fwd_forward(m, key, tok.ctypes.data_as(C.POINTER(C.c_int32)), len(tok), pos)
        if not p:
            raise SystemExit("tg_fwd_forward: " + lib.tg_fwd_last_error().decode())
        return p

    fwd(ids[:prefill], 0)
    # a warm prefill: the same 512 tokens again from position 0 (the slot's
    # workspaces and caches exist now; an LCP of 0 overwrites the cache)
    t_pf = time.perf_counter()
    fwd(ids[:prefill], 0)
    pf_s = time.perf_counter() - t_pf
    pf_launches = lib.tg_fwd_last_launches()
    for i in range(args.warmup):
        fwd(ids[prefill + i:prefill + i + 1], prefill + i)
    launches = lib.tg_fwd_last_launches()
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo")
        dist.barrier()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    clocks.start()
    t0 = time.perf_counter()
    pos0 = prefill + args.warmup
    for i in range(args.steps):
        fwd(ids[pos0 + i:pos0 + i + 1], pos0 + i)
    dt = time.perf_counter() - t0
    clk = clocks.stop()
    if world > 1:
        t = np.array([dt])
        import torch
        tt = torch.tensor(t)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dt = float(tt[0])
        dist.destroy_process_group()
    # several sequences at once, one thread each, as a server runs them: the
    # one-token forwards in flight together run as batches over the weights
    multi = None
    if not args.no_extra:
        import threading
        n_thr, mp = 8, 64
        keys = [C.c_void_p(1000 + i) for i in range(n_thr)]
        mids = np.random.default_rng([args.seed, rank, 7]).integers(
            0, cfg["vocab"], (n_thr, mp + args.warmup + args.steps)).astype(np.int32)
        go = threading.Barrier(n_thr + 1)
        fail = []

        def seq(i):
            try:
                def one(a, pos):
                    if not lib.tg_fwd_forward(m, keys[i], a.ctypes.data_as(C.POINTER(C.c_int32)),
                                              len(a), pos):
                        raise RuntimeError(lib.tg_fwd_last_error().decode())
                one(mids[i, :mp], 0)
                for t in range(args.warmup):
                    one(mids[i, mp + t:mp + t + 1], mp + t)
                go.wait()
                for t in range(args.warmup, args.warmup + args.steps):
                    one(mids[i, mp + t:mp + t + 1], mp + t)
                go.wait()
            except Exception as e:
                fail.append(repr(e))
                go.abort()

        tok0, bat0 = C.c_uint64(), C.c_uint64()
        lib.tg_fwd_batch_stats(m, C.byref(tok0), C.byref(bat0))
        th = [threading.Thread(target=seq, args=(i,)) for i in range(n_thr)]
        for t in th:
            t.start()
        go.wait()
        t0m = time.perf_counter()
        go.wait()
        dtm = time.perf_counter() - t0m
        for t in th:
            t.join()
        if fail:
            raise SystemExit("multi-sequence decode: " + fail[0])
        tok1, bat1 = C.c_uint64(), C.c_uint64()
        lib.tg_fwd_batch_stats(m, C.byref(tok1), C.byref(bat1))
        nb = bat1.value - bat0.value
        multi = {"sequences": n_thr, "tokens_per_s": n_thr * args.steps / dtm,
                 "ms_per_round": 1000.0 * dtm / args.steps,
                 "mean_batch": (tok1.value - tok0.value) / nb if nb else 1.0,
                 "how": f"{n_thr} threads, each its own sequence (a {mp}-token prefill, then "
                        f"one-token forwards): host clock over {args.steps} tokens per thread"}
    lib.tg_fwd_destroy(m)
    if rank != 0:
        return
    tok_s = world * args.steps / dt
    ctx = pos0 + args.steps / 2.0
    bpt = fwd_bytes_per_token(cfg, ctx)
    peak, src = measured_peak()
    achieved = bpt * args.steps / dt / 1e9
    line = {"metric": FWD_METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "fwd", "model": "V2.7-shaped 28-layer MoE (synthetic)",
                       "layers": cfg["n_layers"], "d_model": cfg["d_model"],
                       "heads": f"{cfg['n_heads']}q/{cfg['n_kv_heads']}kv x 128",
                       "experts": f"{cfg['n_experts']} top-{cfg['n_activated']}, d_ff {cfg['d_ff']}",
                       "vocab": cfg["vocab"], "context": f"{pos0}..{pos0 + args.steps}",
                       "parallelism": f"replicas x{world}",
                       "decode_path": ("per-layer launches (TGKV_FWD_STEP=0)"
                                       if os.environ.get("TGKV_FWD_STEP", "") == "0" else
                                       "one cooperative launch per token over all layers"),
                       "l2": "weights read per token (3.4 GB) >> 126 MB L2"},
            "roofline": {"bound": "hbm", "kernel": "whole decode step", "achieved": achieved,
                         "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": src, "traffic": None,
                         "bytes_per_token": bpt},
            "gpu_launches": launches * args.steps,
            "multi_sequence": multi,
            "prefill": {"tokens": prefill, "ms": 1000.0 * pf_s, "tokens_per_s": prefill / pf_s,
                        "launches": pf_launches,
                        "how": "host clock around one synchronous tg_fwd_forward of the "
                               "prompt (logits copied back), after a first prefill"},
            "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4 * cfg["vocab"]},
            "clocks": clk}
    if not args.no_cpu:
        r = fwd_cpu_sample(cfg, args.seed, prefill, 3, threads)
        if r:
            line["cpu_baseline"] = {"value": r[0], "unit": "tokens/s", "cores": threads,
                                    "kind": "reference", "sample": r[1]}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["fwd"], default="cfg4")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--seqs", type=int, default=0,
                    help="sequences per GPU (default: the workload's); for small profiling cases")
    ap.add_argument("--layers", type=int, default=0,
                    help="layers (default: the workload's); for small profiling cases")
    ap.add_argument("--kv-heads", type=int, default=0,
                    help="KV heads (default: the workload's); with --q-heads, e.g. one rank's "
                         "share of a KV-head split on one GPU")
    ap.add_argument("--q-heads", type=int, default=0, help="query heads (default: the workload's)")
    ap.add_argument("--weak", action="store_true",
                    help="cfg4 at N > 1: every GPU its own set of sequences (weak scaling) as "
                         "the headline, instead of the one set split over the GPUs (strong)")
    ap.add_argument("--no-extra", action="store_true",
                    help="cfg4: only the headline (no weak-scaling or cfg5 record beside it)")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="KV heads split over ranks (cfg5/cfg2 at N>1): outputs gathered by the "
                         "attention kernel over NVLink (fused) or by an NCCL all-gather")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-baseline-s", type=float, default=12.0)
    ap.add_argument("--cpu-total-s", type=float, default=120.0)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.workload == "fwd":
        run_fwd(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg3":
        run_cfg3(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
