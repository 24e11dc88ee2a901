"""Run in a fresh process by test_gpu_router.py: brings the router up under the
process's TG_BACKEND, tries to create a cache, prints one JSON line.

The router reads TG_BACKEND only when no backend has been selected yet, so
each setting needs a process of its own."""
import ctypes as C
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "tgai-go_b200"))
import tgkv  # noqa: E402

lib = tgkv.load()
rc = lib.tg_gpu_backend_init()
c = lib.tg_kv_create(64, 2, 64)
calls, ok, fb = C.c_uint64(), C.c_uint64(), C.c_uint64()
lib.tg_gpu_kv_stats(C.byref(calls), C.byref(ok), C.byref(fb))
print(json.dumps({
    "rc": rc, "ready": lib.tg_gpu_backend_ready(),
    "name": lib.tg_gpu_backend_name().decode(), "device": lib.tg_gpu_backend_device().decode(),
    "reason": lib.tg_gpu_backend_reason().decode(),
    "cache": bool(c), "cache_err": "" if c else lib.tg_kv_last_error().decode(),
    "calls": calls.value, "ok": ok.value, "fallbacks": fb.value}))
if c:
    lib.tg_kv_destroy(c)
lib.tg_gpu_backend_shutdown()
