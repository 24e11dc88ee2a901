"""The C-ABI library loads and exports every entry point include/*.h declares.

Runs without a GPU: only loading, symbol lookup and the host-side error paths
that stop before any device call.
"""
import ctypes as C
import glob
import os
import re
import subprocess

import pytest

from conftest import ROOT, PKG

DECL = re.compile(r"^[A-Za-z_][\w\s\*]*?\b(tg_\w+)\s*\(", re.M)
VAR = re.compile(r"^extern\s+\w+\s+(tg_\w+)\s*;", re.M)


def declared():
    funcs, vars_ = set(), set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        funcs |= set(DECL.findall(src))
        vars_ |= set(VAR.findall(src))
    return funcs, vars_


def exported():
    out = subprocess.run(["nm", "-D", "--defined-only", os.path.join(PKG, "libtgkv.so")],
                         capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_every_declared_symbol_is_exported():
    funcs, vars_ = declared()
    assert len(funcs) >= 60, sorted(funcs)
    missing = sorted((funcs | vars_) - exported())
    assert not missing, missing


def test_kernel_launchers_stay_internal():
    ex = exported()
    assert not [s for s in ex if s.startswith("tgkv_launch")]


def test_python_binding_declares_every_entry_point(lib):
    import tgkv
    funcs, _ = declared()
    assert funcs == set(tgkv.PROTOS), sorted(funcs ^ set(tgkv.PROTOS))


def test_build_targets_sm100a_only():
    mk = open(os.path.join(PKG, "Makefile")).read()
    arch = re.findall(r"arch=compute_\w+,code=\w+", mk)
    assert arch == ["arch=compute_100a,code=sm_100a"], arch


def test_create_without_backend_fails_cleanly(lib):
    lib.tg_be_shutdown()
    assert not lib.tg_kv_create(16, 2, 64)
    assert b"no backend selected" in lib.tg_kv_last_error()
    assert not lib.tg_kv_create(0, 2, 64)
    assert b"invalid argument" in lib.tg_kv_last_error()


def test_cpu_and_vulkan_are_not_compiled_in(lib):
    assert lib.tg_be_select(b"cpu") == 0
    assert lib.tg_be_select(b"vulkan") == 0
    assert lib.tg_be_select(b"metal") == 0
    names = lib.tg_be_list()
    got = []
    i = 0
    while names[i]:
        got.append(names[i])
        i += 1
    assert got == [b"cuda", b"vulkan", b"cpu"]
    assert lib.tg_be_probe() == 1


def test_null_handles_are_harmless(lib):
    assert lib.tg_kv_len(None) == 0 and lib.tg_kv_capacity(None) == 0
    assert not lib.tg_kv_device_handle(None)
    lib.tg_kv_reset(None)
    lib.tg_kv_advance(None, 3)
    lib.tg_kv_destroy(None)
    assert lib.tg_kv_append(None, None, None, 1) == 0
    assert lib.tg_kv_truncate(None, 0) == 0
    calls, ok, fb = C.c_uint64(), C.c_uint64(), C.c_uint64()
    lib.tg_gpu_kv_stats(C.byref(calls), C.byref(ok), C.byref(fb))
    assert fb.value == 0


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="CPU-only behaviour")
def test_cuda_backend_without_device_reports_reason(lib):
    assert lib.tg_be_select(b"cuda") == 0
    assert lib.tg_cuda_kv_last_error()
    assert lib.tg_gpu_backend_ready() == 0
    assert lib.tg_gpu_backend_name() == b"none"


def test_static_attention_rejects_bad_arguments_before_any_device_call(lib):
    """tg_kv_attention_static checks its arguments on the host first: each bad
    call returns 0 with a reason and touches no device (so this runs without a
    GPU).  Addresses are only compared for alignment, never dereferenced."""
    kvc, q, out = 0x10000, 0x20000, 0x30000
    cases = [
        ((None, 0, 64, 2, 64, 8, q, out, 4, 1), b"null pointer"),
        ((kvc, 0, 64, 2, 96, 8, q, out, 4, 1), b"no kernel for dtype 0 head_dim 96"),
        ((kvc, 1, 64, 4, 64, 8, q, out, 6, 1), b"not a multiple"),
        ((kvc, 0, 64, 2, 64, 8, q, out, 4, 9), b"need 1 <= n_q"),
        ((kvc, 0, 64, 2, 64, 65, q, out, 4, 1), b"need 1 <= n_q"),
        ((kvc, 0, 64, 2, 64, 8, q, out, 4, 0), b"need 1 <= n_q"),
        ((kvc, 0, 4096, 2, 64, 2048, q, out, 4, 1025), b"above the limit of 1024"),
        ((kvc + 8, 0, 64, 2, 64, 8, q, out, 4, 1), b"16-byte"),
        ((kvc, 0, 64, 2, 64, 8, q + 4, out, 4, 1), b"8-byte"),
    ]
    for args, why in cases:
        a = [C.c_void_p(x) if i in (0, 6, 7) else x for i, x in enumerate(args)]
        assert lib.tg_kv_attention_static(*a, None) == 0, args
        assert why in lib.tg_kv_last_error(), (args, lib.tg_kv_last_error())


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="CPU-only behaviour")
def test_static_error_reader_without_a_call(lib):
    """The static entry's error reader answers 0 where no static call was ever
    made (here: no device at all), and the stall hook only arms a counter."""
    lib.tg_kv_attention_static_inject_stall(0)
    assert lib.tg_kv_attention_static_error(None) == 0


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="CPU-only behaviour")
def test_forward_create_fails_cleanly(lib):
    import tgkv
    assert not lib.tg_fwd_create(None, tgkv.WEIGHT_FN(lambda *a: None), None)
    assert b"null argument" in lib.tg_fwd_last_error()
    cfg = tgkv.TGFwdConfig(n_layers=1, d_model=64, n_heads=2, n_kv_heads=1, head_dim=0, d_ff=64,
                           vocab_size=16, max_seq_len=8, n_experts=0, n_activated=0,
                           rope_theta=10000.0, unk_id=0)
    cb = tgkv.WEIGHT_FN(lambda *a: None)
    assert not lib.tg_fwd_create(C.byref(cfg), cb, None)
    assert lib.tg_fwd_last_error()
