"""Child process of tests/test_engine_dropin.py: the unmodified reference
engine built with its CUDA seam on (oracle/_ref/libtgai_engine_bridge.so,
linked against libtgkv.so) loads a .TG model with its own tg_load and runs
the script of tests/fwd_model.py through its own tg_forward.

    python engine_dropin_run.py <model name> <model.TG> <out.npz>

Writes the logits of every step, the bridge's reason string and its
call / fallback counters.  TGAI_USE_GPU in the environment decides whether
the engine's tg_load hands the model to the GPU forward."""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import fwd_model as FM  # noqa: E402


def main(name, path, out):
    so = os.path.join(HERE, "..", "oracle", "_ref", "libtgai_engine_bridge.so")
    eng = C.CDLL(so)
    eng.tg_load.restype = C.c_void_p
    eng.tg_load.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_int)]
    eng.tg_kvcache_new.restype = C.c_void_p
    eng.tg_kvcache_new.argtypes = [C.c_void_p, C.c_int]
    eng.tg_kvcache_free.argtypes = [C.c_void_p]
    eng.tg_forward.restype = C.POINTER(C.c_float)
    eng.tg_forward.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_void_p, C.c_int]
    eng.tg_free.argtypes = [C.c_void_p]
    eng.tg_engine_cuda_reason.restype = C.c_char_p
    eng.tg_engine_cuda_calls.restype = C.c_longlong
    eng.tg_engine_cuda_fallbacks.restype = C.c_longlong
    cfg = FM.CONFIGS[name]
    err = C.c_int(0)
    m = eng.tg_load(path.encode(), 0, C.byref(err))
    if not m:
        raise SystemExit(f"tg_load failed: {err.value}")
    reason = eng.tg_engine_cuda_reason().decode()
    caches, logits = {}, []
    for key, ids, pos in FM.script(cfg, FM.SEEDS[name]):
        if key not in caches:
            caches[key] = eng.tg_kvcache_new(m, cfg["max_seq"])
        arr = (C.c_int32 * len(ids))(*ids.tolist())
        lp = eng.tg_forward(m, arr, len(ids), caches[key], int(pos))
        if not lp:
            raise SystemExit("tg_forward failed")
        logits.append(np.ctypeslib.as_array(lp, shape=(cfg["vocab"],)).copy())
    calls, falls = eng.tg_engine_cuda_calls(), eng.tg_engine_cuda_fallbacks()
    for c in caches.values():
        eng.tg_kvcache_free(c)
    eng.tg_free(m)
    np.savez(out, logits=np.array(logits), reason=np.array(reason), calls=np.int64(calls),
             fallbacks=np.int64(falls))


if __name__ == "__main__":
    main(*sys.argv[1:4])
