"""ctypes binding of libtgkv.so -- the KV-cache path's C-ABI.

This mirrors how the reference's Python layer binds its engine
(python/tgai_go/_engine.py:344-347 declares tg_kvcache_new/free/reset and
tg_forward with ctypes): every entry point of include/tgai_kv_cache.h,
include/tgai_backend.h, include/tgai_gpu_dispatch.h, include/tgai_cuda_bridge.h
and include/tgai_engine_bridge.h gets argtypes/restype here.  Loading fails loudly if
the library is missing -- there is no Python or CPU fallback.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtgkv.so")

TG_KV_F32 = 0
TG_KV_BF16 = 1

u32, u64, i32 = C.c_uint32, C.c_uint64, C.c_int
vp, cp, fp = C.c_void_p, C.c_char_p, C.c_float
PF = C.POINTER(C.c_float)
PU32 = C.POINTER(C.c_uint32)


class TGBackendInfo(C.Structure):
    _fields_ = [("name", cp), ("device_name", cp), ("caps", u32), ("mem_bytes", u64),
                ("is_gpu", i32), ("is_uma", i32)]


class TGCudaCacheDesc(C.Structure):
    _fields_ = [("base", u64), ("max_seq", u32), ("pad", u32), ("tmap", u64), ("tmap_sw", u64)]


# struct TGBackend of include/tgai_backend.h (src/tgai_backend.h:55-94 order)
ATTN_FN = C.CFUNCTYPE(i32, vp, vp, vp, u32, u32, u32, u32, u32, u32)
ROPE_FN = C.CFUNCTYPE(i32, vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32)
UPLOAD_FN = C.CFUNCTYPE(i32, vp, vp, C.c_size_t)


class TGBackend(C.Structure):
    _fields_ = [("name", cp), ("caps", u32),
                ("init", vp), ("shutdown", vp), ("ready", vp), ("info", vp),
                ("last_error", vp),
                ("alloc", vp), ("free", vp), ("upload", UPLOAD_FN), ("download", UPLOAD_FN),
                ("map", vp),
                ("rmsnorm", vp), ("silu_mul", vp), ("softmax", vp), ("rope", ROPE_FN),
                ("mm_bf16", vp), ("attention", ATTN_FN), ("moe_router", vp), ("priv", vp)]


class TGFwdConfig(C.Structure):
    """TGFwdConfig of include/tgai_engine_bridge.h."""
    _fields_ = [("n_layers", u32), ("d_model", u32), ("n_heads", u32), ("n_kv_heads", u32),
                ("head_dim", u32), ("d_ff", u32), ("vocab_size", u32), ("max_seq_len", u32),
                ("n_experts", u32), ("n_activated", u32), ("rope_theta", C.c_float),
                ("unk_id", C.c_int32)]


# TGFwdWeightFn: const float* (*)(void* ctx, const char* name, uint32_t shape[2])
WEIGHT_FN = C.CFUNCTYPE(vp, vp, cp, PU32)


def current_backend(lib):
    """The selected TGBackend table (raises if none is selected)."""
    p = lib.tg_be_current()
    if not p:
        raise KvError("no backend selected")
    return C.cast(p, C.POINTER(TGBackend)).contents


# name: (restype, [argtypes]) for every exported entry point of include/*.h
PROTOS = {
    # tgai_kv_cache.h -- reference interface
    "tg_kv_create": (vp, [u32, u32, u32]),
    "tg_kv_destroy": (None, [vp]),
    "tg_kv_reset": (None, [vp]),
    "tg_kv_len": (u32, [vp]),
    "tg_kv_capacity": (u32, [vp]),
    "tg_kv_device_handle": (vp, [vp]),
    "tg_kv_host_ptr": (PF, [vp]),
    "tg_kv_append": (i32, [vp, vp, vp, u32]),
    "tg_kv_advance": (None, [vp, u32]),
    "tg_kv_last_error": (cp, []),
    # tgai_kv_cache.h -- additive
    "tg_kv_create_ex": (vp, [u32, u32, u32, i32]),
    "tg_kv_dtype": (i32, [vp]),
    "tg_kv_n_kv_heads": (u32, [vp]),
    "tg_kv_head_dim": (u32, [vp]),
    "tg_kv_truncate": (i32, [vp, u32]),
    "tg_kv_append_dev": (i32, [vp, vp, vp, u32, vp]),
    "tg_kv_attention": (i32, [vp, vp, vp, u32, u32, vp]),
    "tg_kv_bytes": (u64, [vp]),
    "tg_kv_download": (i32, [vp, vp]),
    "tg_kv_attention_static": (i32, [vp, i32, u32, u32, u32, u32, vp, vp, u32, u32, vp]),
    "tg_kv_append_attention": (i32, [vp, vp, vp, vp, vp, u32, u32, vp]),
    "tg_cuda_kv_attn_fuses_suffix": (i32, [vp]),
    "tg_kv_attention_static_error": (i32, [vp]),
    "tg_kv_attention_static_inject_stall": (None, [i32]),
    "tg_kv_rope_tables": (i32, [fp, u32, u32, u32, u32, u32, PF, PF, PF]),
    "tg_kv_set_attn_mscale": (None, [vp, fp]),
    "tg_kv_batch_create": (vp, [C.POINTER(vp), u32, u32]),
    "tg_kv_batch_destroy": (None, [vp]),
    "tg_kv_batch_decode": (i32, [vp, vp, vp, vp, vp, vp]),
    "tg_kv_batch_decode_host": (i32, [vp, vp, vp, vp, vp, vp]),
    "tg_kv_batch_last_launches": (u32, [vp]),
    "tg_kv_gather_create": (vp, [u32, u32, u64]),
    "tg_kv_gather_destroy": (None, [vp]),
    "tg_kv_gather_export": (i32, [vp, vp]),
    "tg_kv_gather_import": (i32, [vp, vp]),
    "tg_kv_gather_buffer": (vp, [vp]),
    "tg_kv_batch_decode_gather": (i32, [vp, vp, vp, vp, vp, vp, vp]),
    "tg_kv_batch_decode_gather_host": (i32, [vp, vp, vp, vp, vp, vp, vp]),
    # tgai_backend.h
    "tg_be_probe": (i32, []),
    "tg_be_select": (i32, [cp]),
    "tg_be_current": (vp, []),
    "tg_be_current_info": (i32, [C.POINTER(TGBackendInfo)]),
    "tg_be_shutdown": (None, []),
    "tg_be_list": (C.POINTER(cp), []),
    # tgai_gpu_dispatch.h
    "tg_gpu_backend_init": (i32, []),
    "tg_gpu_backend_ready": (i32, []),
    "tg_gpu_backend_name": (cp, []),
    "tg_gpu_backend_reason": (cp, []),
    "tg_gpu_backend_device": (cp, []),
    "tg_gpu_backend_shutdown": (None, []),
    "tg_gpu_kv_stats": (None, [C.POINTER(u64), C.POINTER(u64), C.POINTER(u64)]),
    "tg_gpu_kv_register": (None, [vp, i32, u32, u32, u32, vp]),
    "tg_gpu_kv_lookup_tmap": (vp, [vp, u32, u32, u32]),
    "tg_gpu_kv_unregister": (None, [vp]),
    "tg_gpu_kv_lookup_dtype": (i32, [vp]),
    "tg_gpu_kv_append_dev": (i32, [i32, vp, u32, u32, u32, vp, vp, u32, vp]),
    "tg_gpu_kv_attention": (i32, [i32, vp, u32, vp, vp, u32, u32, u32, vp, vp, PU32, u32, fp,
                                  vp, vp, vp]),
    "tg_gpu_kv_error": (cp, []),
    # tgai_cuda_bridge.h
    "tg_cuda_kv_init": (i32, []),
    "tg_cuda_kv_set_device": (i32, [i32]),
    "tg_cuda_kv_shutdown": (None, []),
    "tg_cuda_kv_ready": (i32, []),
    "tg_cuda_kv_last_error": (cp, []),
    "tg_cuda_kv_device_name": (cp, []),
    "tg_cuda_kv_device_mem": (u64, []),
    "tg_cuda_kv_sm_count": (i32, []),
    "tg_cuda_kv_malloc": (vp, [C.c_size_t]),
    "tg_cuda_kv_free": (None, [vp]),
    "tg_cuda_kv_h2d": (i32, [vp, vp, C.c_size_t, vp]),
    "tg_cuda_kv_h2d_async": (i32, [vp, vp, C.c_size_t, vp]),
    "tg_cuda_kv_d2h_async": (i32, [vp, vp, C.c_size_t, vp]),
    "tg_cuda_kv_stage_host": (i32, [vp, vp, C.c_size_t, vp, C.c_size_t, vp, C.c_size_t, vp]),
    "tg_cuda_kv_d2h": (i32, [vp, vp, C.c_size_t, vp]),
    "tg_cuda_kv_memset": (i32, [vp, i32, C.c_size_t, vp]),
    "tg_cuda_kv_sync": (i32, [vp]),
    "tg_cuda_kv_device_error": (i32, []),
    "tg_cuda_kv_inject_alloc_failures": (None, [i32]),
    "tg_cuda_kv_tmap_create": (vp, [i32, u64, u32, u32, u32]),
    "tg_cuda_kv_tmap_write": (i32, [i32, u64, u32, u32, u32, vp]),
    "tg_cuda_kv_tmap_sw_create": (vp, [u64, u32, u32]),
    "tg_cuda_kv_append": (i32, [i32, TGCudaCacheDesc, u32, u32, vp, vp, u32, vp]),
    "tg_cuda_kv_append_batch": (i32, [i32, vp, u32, PU32, u32, vp, vp, vp]),
    "tg_cuda_kv_attn_supported": (i32, [i32, u32]),
    "tg_cuda_kv_attn_scratch_bytes": (u64, [vp]),
    "tg_cuda_kv_attn_counters": (u64, [vp]),
    "tg_cuda_kv_attn_segments": (u64, [vp]),
    "tg_cuda_kv_attn_last_launches": (u32, []),
    "tg_cuda_kv_attn_last_kernel": (i32, []),
    "tg_cuda_kv_attn_last_split": (u32, []),
    "tg_cuda_kv_host_device_ptr": (vp, [vp]),
    "tg_cuda_kv_stream_create": (vp, []),
    "tg_cuda_kv_stream_destroy": (None, [vp]),
    "tg_cuda_kv_event_create": (vp, []),
    "tg_cuda_kv_event_destroy": (None, [vp]),
    "tg_cuda_kv_event_record": (i32, [vp, vp]),
    "tg_cuda_kv_stream_wait": (i32, [vp, vp]),
    "tg_cuda_kv_ipc_handle": (i32, [vp, vp]),
    "tg_cuda_kv_ipc_open": (vp, [vp]),
    "tg_cuda_kv_ipc_close": (None, [vp]),
    "tg_cuda_kv_gather_wait": (i32, [vp, u32, vp]),
    "tg_cuda_kv_attention": (i32, [vp, vp]),
    "tg_cuda_kv_rope_append": (i32, [i32, vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32,
                                     vp]),
    # tgai_engine_bridge.h -- the engine's CUDA seam (cuda/tgai_cuda_bridge.h:31-60)
    "tg_engine_cuda_init": (i32, [vp]),
    "tg_engine_cuda_forward": (i32, [vp, C.POINTER(C.c_int32), i32, vp, i32,
                                     C.POINTER(PF)]),
    "tg_engine_cuda_reset": (None, []),
    "tg_engine_cuda_reset_slot": (None, [vp]),
    "tg_engine_cuda_free_slot": (None, [vp]),
    "tg_engine_cuda_shutdown": (None, []),
    "tg_engine_cuda_ready": (i32, []),
    "tg_engine_cuda_reason": (cp, []),
    "tg_engine_cuda_calls": (C.c_longlong, []),
    "tg_engine_cuda_fallbacks": (C.c_longlong, []),
    "tg_gpu_kv_slot_of": (i32, [vp]),
    "tg_gpu_kv_slot_seq": (i32, [vp]),
    "tg_gpu_kv_slot_live": (i32, []),
    "tg_gpu_kv_slot_max": (i32, []),
    "tg_gpu_kv_slot_rejects": (C.c_longlong, []),
    "tg_gpu_cuda_calls": (C.c_longlong, []),
    "tg_gpu_cuda_fallbacks": (C.c_longlong, []),
    # tgai_engine_bridge.h -- neutral whole-forward API
    "tg_fwd_create": (vp, [C.POINTER(TGFwdConfig), WEIGHT_FN, vp]),
    "tg_fwd_destroy": (None, [vp]),
    "tg_fwd_forward": (PF, [vp, vp, C.POINTER(C.c_int32), u32, u32]),
    "tg_fwd_reset_slot": (i32, [vp, vp]),
    "tg_fwd_free_slot": (i32, [vp, vp]),
    "tg_fwd_reset_all": (None, [vp]),
    "tg_fwd_slot_count": (u32, [vp]),
    "tg_fwd_slot_last_pos": (i32, [vp, vp]),
    "tg_fwd_weight_bytes": (u64, [vp]),
    "tg_fwd_last_launches": (u32, []),
    "tg_fwd_last_error": (cp, []),
    "tg_fwd_gemm_f32": (i32, [u32, u32, u32, vp, u32, vp, u32, vp, u32, i32, vp]),
    "tg_fwd_batch_stats": (None, [vp, C.POINTER(u64), C.POINTER(u64)]),
}

_lib = None


def load(path=LIB_PATH):
    """Load libtgkv.so and declare every prototype; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"libtgkv.so not built at {path}: run __graft_entry__.build()")
    lib = C.CDLL(path)
    for name, (res, args) in PROTOS.items():
        fn = getattr(lib, name)          # AttributeError if an entry point is missing
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class KvError(RuntimeError):
    pass


class Forward:
    """A whole-model forward (tg_fwd_*) over fp32 host weights.

    weights: dict name -> float32 array (the engine's tensor names; Linear
    weights [out, in]).  forward(key, ids, pos) returns the logits row as a
    numpy copy; key is any hashable naming the sequence.
    """

    def __init__(self, lib, cfg, weights):
        import numpy as np
        self.lib = lib
        self._w = {k: np.ascontiguousarray(v, np.float32) for k, v in weights.items()}
        self._names = {}

        def get(ctx, name, shape):
            a = self._w.get(name.decode())
            if a is None:
                return None
            shape[0] = a.shape[0]
            shape[1] = int(a.size // a.shape[0]) if a.ndim > 1 else 1
            return a.ctypes.data

        self._cb = WEIGHT_FN(get)
        self.cfg = cfg
        self.m = lib.tg_fwd_create(C.byref(cfg), self._cb, None)
        if not self.m:
            raise KvError(f"tg_fwd_create: {lib.tg_fwd_last_error().decode(errors='replace')}")
        self._w = None                      # read during create only
        self._keys = {}

    def key(self, k):
        return self._keys.setdefault(k, len(self._keys) + 1)

    def forward(self, k, ids, pos):
        import numpy as np
        ids = np.ascontiguousarray(ids, np.int32)
        arr = ids.ctypes.data_as(C.POINTER(C.c_int32))
        p = self.lib.tg_fwd_forward(self.m, C.c_void_p(self.key(k)), arr, len(ids), pos)
        if not p:
            raise KvError(f"tg_fwd_forward: {self.lib.tg_fwd_last_error().decode(errors='replace')}")
        return np.ctypeslib.as_array(p, shape=(self.cfg.vocab_size,)).copy()

    def close(self):
        if self.m:
            self.lib.tg_fwd_destroy(self.m)
            self.m = None


def check(ok, lib=None, what="tg_kv"):
    """Raise KvError with tg_kv_last_error() when a C-ABI call returned 0/NULL."""
    if not ok:
        lib = lib or load()
        raise KvError(f"{what}: {lib.tg_kv_last_error().decode(errors='replace')}")
    return ok


def ptr(t):
    """Device/host address of a torch tensor or numpy array as c_void_p."""
    if hasattr(t, "data_ptr"):
        return C.c_void_p(t.data_ptr())
    return C.c_void_p(t.ctypes.data)


def stream_handle(stream=None):
    """cudaStream_t of a torch stream (the current one when None)."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)
