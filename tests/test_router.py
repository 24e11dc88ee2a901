"""The KV-cache path router (tgai_gpu_dispatch.c) under TG_BACKEND.

The reference router reads TG_BACKEND once at init
(src/tgai_gpu_dispatch.c:467-492) and reports through tg_gpu_backend_name,
_reason, _device and _ready (:773-819).  Here "auto"/"cuda" (any case) bring
the CUDA path up; "cpu" and "vulkan" are refused with a reason and nothing
falls back; other values are refused as unknown.  Each setting runs in a
fresh process (tests/router_probe.py), since the router reads the variable
only while no backend is selected.

The refusals need no device and run everywhere; the bring-up and the
fallback counters over a configs[0] run are GPU tests.
"""
import ctypes as C
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle as O
import tgkv
from conftest import rel_head_err

PROBE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "router_probe.py")


def probe(value):
    env = dict(os.environ)
    env.pop("TG_BACKEND", None)
    if value is not None:
        env["TG_BACKEND"] = value
    r = subprocess.run([sys.executable, PROBE], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("value", ["vulkan", "cpu", "VULKAN", "Cpu"])
def test_cpu_and_vulkan_are_refused_without_fallback(value):
    d = probe(value)
    assert d["rc"] == 0 and d["ready"] == 0 and d["name"] == "none" and d["device"] == ""
    assert f"TG_BACKEND={value} refused" in d["reason"] and "no fallback" in d["reason"]
    assert not d["cache"] and "no backend selected" in d["cache_err"]
    assert d["fallbacks"] == 0


def test_unknown_backend_is_refused():
    d = probe("metal")
    assert d["rc"] == 0 and d["ready"] == 0 and d["name"] == "none"
    assert "TG_BACKEND=metal not recognised" in d["reason"]
    assert not d["cache"]


@pytest.mark.gpu
@pytest.mark.parametrize("value", [None, "auto", "cuda", "CUDA"])
def test_cuda_comes_up(value):
    d = probe(value)
    assert d["rc"] == 1 and d["ready"] == 1 and d["name"] == "cuda", d
    assert d["device"] and d["reason"] == "cuda: KV-cache path on " + d["device"]
    assert d["cache"], d["cache_err"]
    assert d["fallbacks"] == 0


@pytest.mark.gpu
def test_stats_count_a_cfg1_run_with_no_fallback(cuda, devbuf):
    """configs[0] through the routed calls: 4 layers of 8 = 8 heads of 64,
    fp32 caches, a 128-token prefill append, then 384 single-token appends +
    attention per layer.  Every routed call succeeds, none falls back, and
    the last step of every layer matches the engine-order oracle."""
    lib = cuda
    assert lib.tg_gpu_backend_init() == 1
    nh = nkv = 8
    hd, L, layers = 64, 512, 4
    calls0, ok0, fb0 = C.c_uint64(), C.c_uint64(), C.c_uint64()
    lib.tg_gpu_kv_stats(C.byref(calls0), C.byref(ok0), C.byref(fb0))
    for layer in range(layers):
        q = O.normal(L * nh * hd, 31, layer, 1).reshape(L, nh, hd)
        k = O.normal(L * nkv * hd, 31, layer, 2).reshape(L, nkv * hd)
        v = O.normal(L * nkv * hd, 31, layer, 3).reshape(L, nkv * hd)
        c = lib.tg_kv_create(L, nkv, hd)
        tgkv.check(c, lib)
        kd, vd, qd = devbuf(k), devbuf(v), devbuf(q)
        od = devbuf(nbytes=q.nbytes)
        tgkv.check(lib.tg_kv_append_dev(c, kd.ptr, vd.ptr, 128, None), lib)
        row_k, row_q = nkv * hd * 4, nh * hd * 4
        for t in range(128, L):
            tgkv.check(lib.tg_kv_append_dev(c, kd.ptr + t * row_k, vd.ptr + t * row_k, 1,
                                            None), lib)
            tgkv.check(lib.tg_kv_attention(c, qd.ptr + t * row_q, od.ptr + t * row_q, nh, 1,
                                           None), lib)
        assert lib.tg_cuda_kv_sync(None)
        out = od.get(np.float32, q.shape)
        kvc = np.zeros((2, L, nkv * hd), np.float32)
        kvc[0], kvc[1] = k, v
        eng = O.attention_engine(q[L - 1], kvc, nh, nkv, hd, 1, L - 1, L, L)
        assert rel_head_err(out[L - 1], eng[0]) < 1e-5, layer
        lib.tg_kv_destroy(c)
    calls, ok, fb = C.c_uint64(), C.c_uint64(), C.c_uint64()
    lib.tg_gpu_kv_stats(C.byref(calls), C.byref(ok), C.byref(fb))
    routed = calls.value - calls0.value
    assert routed >= layers * (1 + 2 * (L - 128)), routed
    assert ok.value - ok0.value == routed
    assert fb.value == 0
