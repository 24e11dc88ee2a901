"""ctypes wrapper of oracle/liboracle.so -- TEST INFRASTRUCTURE ONLY.

The CPU restatement of the reference's KV-cache path (oracle/tgkv_oracle.c).
Only tests/, __graft_entry__.smoke() and bench.py's CPU legs may import this
module, as the checker or as the timed CPU baseline; the product library never
touches it.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
F32, BF16 = 0, 1

_P = C.POINTER(C.c_float)
_lib = None


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} missing: run `make -C oracle`")
    lib = C.CDLL(LIB_PATH)
    lib.orc_dot.restype = C.c_float
    lib.orc_dot.argtypes = [_P, _P, C.c_int]
    lib.orc_softmax.argtypes = [_P, C.c_int]
    lib.orc_rope.argtypes = [_P, _P] + [C.c_int] * 5 + [C.c_float]
    lib.orc_rope_tables.argtypes = [_P] + [C.c_int] * 4 + [_P, _P]
    lib.orc_f32_to_bf16.restype = C.c_uint16
    lib.orc_f32_to_bf16.argtypes = [C.c_float]
    lib.orc_kv_append.restype = C.c_int
    lib.orc_kv_append.argtypes = [C.c_void_p, C.c_int, C.c_uint32, C.c_uint32, C.c_uint32,
                                  _P, _P, C.c_uint32]
    lib.orc_kv_decode.argtypes = [C.c_void_p, C.c_int, C.c_uint32, C.c_uint32, _P]
    for n in ("orc_attention_engine", "orc_attention_f64", "orc_attention_weights_last"):
        getattr(lib, n).argtypes = [_P, _P, _P] + [C.c_int] * 7
    lib.orc_attention_engine_scaled.argtypes = [_P, _P, _P] + [C.c_int] * 7 + [C.c_float]
    lib.orc_decode_batch.argtypes = [C.POINTER(_P), C.POINTER(_P), C.POINTER(_P),
                                     C.POINTER(C.c_int), C.POINTER(C.c_int)] + [C.c_int] * 5
    lib.orc_normal.restype = C.c_float
    lib.orc_normal.argtypes = [C.c_uint64] * 5
    lib.orc_fill_normal.argtypes = [_P, C.c_size_t] + [C.c_uint64] * 4 + [C.c_float]
    _lib = lib
    return lib


def _f(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_P)


def normal(n, seed, k0=0, k1=0, k2=0, scale=1.0):
    """Seeded N(0,1)*scale float32 vector keyed by (seed, k0, k1, k2)."""
    out = np.empty(n, np.float32)
    load().orc_fill_normal(_f(out), n, seed, k0, k1, k2, scale)
    return out


def f32_to_bf16(x):
    """Round-to-nearest-even fp32 -> bf16 bits (uint16), vectorised in numpy with
    the same rule as orc_f32_to_bf16."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, ((u >> 16) | 0x40) & 0xFFFF, r)
    return r.astype(np.uint16)


def bf16_to_f32(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def dot(a, b):
    return load().orc_dot(_f(a), _f(b), a.size)


def softmax(x):
    y = np.ascontiguousarray(x, np.float32).copy()
    load().orc_softmax(_f(y), y.size)
    return y


def rope(q, k, n_heads, n_kv_heads, d_k, pos0, theta=10000.0):
    """Rotate copies of q [seq][nh][dk] and k [seq][nkv][dk]; returns (q, k)."""
    q = np.ascontiguousarray(q, np.float32).copy()
    k = np.ascontiguousarray(k, np.float32).copy()
    seq = q.size // (n_heads * d_k)
    load().orc_rope(_f(q), _f(k), seq, n_heads, n_kv_heads, d_k, pos0, theta)
    return q, k


def rope_tables(x, n_heads, d_k, pos0, cs, sn):
    """Rotate a copy of x [seq][nh][dk] with tables cs/sn [pos][dk/2]."""
    x = np.ascontiguousarray(x, np.float32).copy()
    seq = x.size // (n_heads * d_k)
    load().orc_rope_tables(_f(x), seq, n_heads, d_k, pos0,
                           _f(np.ascontiguousarray(cs, np.float32)),
                           _f(np.ascontiguousarray(sn, np.float32)))
    return x


def attention_engine(q, kvc, n_heads, n_kv_heads, head_dim, n_q, pos0, kv_len, max_seq,
                     mscale=1.0):
    """Engine-order attention (src/tgai_engine.c:3943-4011) over an fp32
    [2][max_seq][kv_dim] cache.  q: [n_q][nh][hd]; mscale: YaRN temperature."""
    q = np.ascontiguousarray(q, np.float32)
    kvc = np.ascontiguousarray(kvc, np.float32)
    out = np.zeros(n_q * n_heads * head_dim, np.float32)
    load().orc_attention_engine_scaled(_f(q), _f(kvc), _f(out), n_heads, n_kv_heads, head_dim,
                                       n_q, pos0, kv_len, max_seq, mscale)
    return out.reshape(n_q, n_heads, head_dim)


def attention_f64(q, kvc, n_heads, n_kv_heads, head_dim, n_q, pos0, kv_len, max_seq):
    q = np.ascontiguousarray(q, np.float32)
    kvc = np.ascontiguousarray(kvc, np.float32)
    out = np.zeros(n_q * n_heads * head_dim, np.float32)
    load().orc_attention_f64(_f(q), _f(kvc), _f(out), n_heads, n_kv_heads, head_dim, n_q, pos0,
                             kv_len, max_seq)
    return out.reshape(n_q, n_heads, head_dim)


def attention_weights_last(q, kvc, n_heads, n_kv_heads, head_dim, n_q, pos0, kv_len, max_seq):
    q = np.ascontiguousarray(q, np.float32)
    kvc = np.ascontiguousarray(kvc, np.float32)
    w = np.zeros(n_heads * kv_len, np.float32)
    load().orc_attention_weights_last(_f(q), _f(kvc), _f(w), n_heads, n_kv_heads, head_dim, n_q,
                                      pos0, kv_len, max_seq)
    return w.reshape(n_heads, kv_len)


def kv_append(cache, dtype, max_seq, kv_dim, length, k, v):
    """Write rows into a host cache array (fp32 or uint16 bf16 bits) in place."""
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    n = k.size // kv_dim
    return load().orc_kv_append(cache.ctypes.data, dtype, max_seq, kv_dim, length, _f(k), _f(v), n)


def decode_batch(kvcs, qs, lens, n_heads, n_kv_heads, head_dim, threads=1):
    """CPU baseline: one decode query per fp32 cache, engine order."""
    n = len(kvcs)
    outs = [np.zeros(n_heads * head_dim, np.float32) for _ in range(n)]
    arr = lambda xs: (_P * n)(*[_f(x) for x in xs])
    ml = (C.c_int * n)(*[int(k.size // (2 * n_kv_heads * head_dim)) for k in kvcs])
    ln = (C.c_int * n)(*[int(x) for x in lens])
    load().orc_decode_batch(arr(kvcs), arr(qs), arr(outs), ln, ml, n, n_heads, n_kv_heads,
                            head_dim, threads)
    return outs
