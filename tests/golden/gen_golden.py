"""Generate the golden vectors in tests/golden/ from the reference's own code.

Runs only where the reference checkout exists (the REF environment variable
names it; the default is the build container's checkout) and oracle/_ref/ has
been built (`make -C oracle ref`); the GPU box never runs this, it only reads
the committed .npz files.

  engine_pins.npz    tg_dot / softmax / rope of src/tgai_engine.c on seeded
                     random inputs (outputs of the reference build).
  engine_fixture.npz real forwards of tests/fixtures/mini_stream.TG through
                     tg_forward: the last layer's post-RoPE queries, its KV
                     cache rows and the softmax weights the engine dumps
                     (TGAI_DUMP_ATTN=1, c_attn<layer>.bin), for prefill,
                     decode, and LCP truncate + re-append steps.
  kvtest.npz         tests/test_kv_cache_gpu.c's scenario (srand(31415), NH=16,
                     HD=64, MAXSEQ=128, 32 appends): inputs from glibc rand(),
                     the cache bytes after the appends (reference CPU backend
                     of src/tgai_kv_cache.c), the capacity count, and the
                     double-precision cpu_attention output.
  attntest.npz       tests/test_vk_attn_moe.c's attention scenario (srand(777),
                     MAXSEQ=256, NKV=40, POS=39 and POS=10).
  forward.npz        whole-model logits of tg_forward (CPU engine) over the
                     seeded synthetic models of tests/fwd_model.py (a MoE and a
                     dense GQA model, written as .TG files), one row per step
                     of their scripts: prefill, decode, a second sequence,
                     LCP truncate + re-append.

Usage: python tests/golden/gen_golden.py
"""
import ctypes as C
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
REF = os.environ.get("REF", "/root/reference")
REF_LIB = os.path.join(ROOT, "oracle", "_ref")
P = C.POINTER(C.c_float)


def fptr(a):
    return a.ctypes.data_as(P)


def engine_pins(eng):
    eng.tgref_dot.restype = C.c_float
    eng.tgref_dot.argtypes = [P, P, C.c_int]
    eng.tgref_softmax.argtypes = [P, C.c_int]
    eng.tgref_rope.argtypes = [P, P] + [C.c_int] * 5 + [C.c_float]
    rng = np.random.default_rng(20261201)
    out = {}
    lens = np.array([1, 7, 8, 15, 16, 17, 31, 32, 33, 64, 100, 128, 256], np.int32)
    da, db, dr = [], [], []
    for n in lens:
        for _ in range(8):
            a = rng.standard_normal(n).astype(np.float32)
            b = rng.standard_normal(n).astype(np.float32)
            da.append(np.pad(a, (0, 256 - n)))
            db.append(np.pad(b, (0, 256 - n)))
            dr.append(eng.tgref_dot(fptr(a), fptr(b), int(n)))
    out["dot_len"] = np.repeat(lens, 8)
    out["dot_a"], out["dot_b"] = np.array(da), np.array(db)
    out["dot_out"] = np.array(dr, np.float32)
    sx, so = [], []
    for _ in range(16):
        x = (rng.standard_normal(300) * 4).astype(np.float32)
        x[rng.random(300) < 0.25] = -1e30
        y = x.copy()
        eng.tgref_softmax(fptr(y), y.size)
        sx.append(x)
        so.append(y)
    out["softmax_in"], out["softmax_out"] = np.array(sx), np.array(so)
    cases = [(3, 8, 8, 64, 0), (5, 16, 4, 128, 1000), (2, 6, 6, 32, 77), (1, 32, 8, 128, 131000)]
    for ci, (seq, nh, nkv, dk, pos) in enumerate(cases):
        q = rng.standard_normal(seq * nh * dk).astype(np.float32)
        k = rng.standard_normal(seq * nkv * dk).astype(np.float32)
        q2, k2 = q.copy(), k.copy()
        eng.tgref_rope(fptr(q2), fptr(k2), seq, nh, nkv, dk, pos, C.c_float(10000.0))
        out[f"rope{ci}_shape"] = np.array([seq, nh, nkv, dk, pos], np.int32)
        out[f"rope{ci}_q"], out[f"rope{ci}_k"] = q, k
        out[f"rope{ci}_qout"], out[f"rope{ci}_kout"] = q2, k2
    out["rope_cases"] = np.int32(len(cases))
    # context extension (NTK-by-parts + YaRN mscale), tgai_engine.c:3404-3460
    eng.tgref_rope_ext.restype = C.c_float
    eng.tgref_rope_ext.argtypes = [P, P] + [C.c_int] * 5 + [C.c_float, C.c_int, C.c_int]
    ext = [(4, 8, 2, 128, 16000, 10000.0, 32768, 8192), (3, 4, 4, 64, 5000, 500000.0, 16384, 4096),
           (2, 6, 6, 32, 100, 10000.0, 1024, 128)]
    for ci, (seq, nh, nkv, dk, pos, theta, ectx, msl) in enumerate(ext):
        q = rng.standard_normal(seq * nh * dk).astype(np.float32)
        k = rng.standard_normal(seq * nkv * dk).astype(np.float32)
        q2, k2 = q.copy(), k.copy()
        ms = eng.tgref_rope_ext(fptr(q2), fptr(k2), seq, nh, nkv, dk, pos, C.c_float(theta),
                                ectx, msl)
        out[f"ropex{ci}_shape"] = np.array([seq, nh, nkv, dk, pos, ectx, msl], np.int32)
        out[f"ropex{ci}_theta"] = np.float32(theta)
        out[f"ropex{ci}_q"], out[f"ropex{ci}_k"] = q, k
        out[f"ropex{ci}_qout"], out[f"ropex{ci}_kout"] = q2, k2
        out[f"ropex{ci}_mscale"] = np.float32(ms)
    out["ropex_cases"] = np.int32(len(ext))
    np.savez_compressed(os.path.join(HERE, "engine_pins.npz"), **out)


def engine_fixture(eng):
    model_path = os.path.join(REF, "tests", "fixtures", "mini_stream.TG")
    eng.tg_load.restype = C.c_void_p
    eng.tg_load.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_int)]
    eng.tg_kvcache_new.restype = C.c_void_p
    eng.tg_kvcache_new.argtypes = [C.c_void_p, C.c_int]
    eng.tg_kvcache_free.argtypes = [C.c_void_p]
    eng.tg_forward.restype = P
    eng.tg_forward.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_void_p, C.c_int]
    eng.tgref_work_q.restype = P
    eng.tgref_work_q.argtypes = [C.c_void_p]
    eng.tgref_cache_info.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
    eng.tgref_cache_k.restype = P
    eng.tgref_cache_k.argtypes = [C.c_void_p]
    eng.tgref_cache_v.restype = P
    eng.tgref_cache_v.argtypes = [C.c_void_p]
    eng.tg_dump_set_enabled.argtypes = [C.c_int]
    eng.tg_free.argtypes = [C.c_void_p]

    dump = tempfile.mkdtemp(prefix="tgdump")
    os.environ["TGAI_DUMP_DIR"] = dump
    os.environ["TGAI_DUMP_ATTN"] = "1"
    eng.tg_dump_set_enabled(1)
    err = C.c_int(0)
    m = eng.tg_load(model_path.encode(), 0, C.byref(err))
    if not m:
        raise RuntimeError(f"tg_load failed: {err.value}")
    max_seq = 64
    cache = eng.tg_kvcache_new(m, max_seq)
    info = (C.c_int * 5)()
    eng.tgref_cache_info(cache, info)
    msl, n_layers, nh, nkv, dk = list(info)
    rng = np.random.default_rng(7)
    ids = rng.integers(0, 8000, 24).astype(np.int32)
    ids2 = rng.integers(0, 8000, 8).astype(np.int32)
    # (tokens, cache_pos): prefill, decode x2, LCP truncate to 4 + re-append 3,
    # then a longer suffix after a /clear-style restart at 0.
    steps = [(ids[:8], 0), (ids[8:9], 8), (ids[9:10], 9), (ids2[:3], 4), (ids[:13], 0),
             (ids[13:14], 13)]
    out = {"geometry": np.array([msl, n_layers, nh, nkv, dk], np.int32),
           "n_steps": np.int32(len(steps))}
    last = n_layers - 1
    for si, (tok, pos) in enumerate(steps):
        arr = (C.c_int32 * len(tok))(*tok.tolist())
        lp = eng.tg_forward(m, arr, len(tok), cache, int(pos))
        if not lp:
            raise RuntimeError("tg_forward failed")
        seq = len(tok)
        kv_len = pos + seq
        q = np.ctypeslib.as_array(eng.tgref_work_q(m), shape=(seq * nh * dk,)).copy()
        kall = np.ctypeslib.as_array(eng.tgref_cache_k(cache), shape=(n_layers, nkv, msl, dk))
        vall = np.ctypeslib.as_array(eng.tgref_cache_v(cache), shape=(n_layers, nkv, msl, dk))
        # engine layout [layer][kvh][pos][dk] -> [2][max_seq][nkv*dk] of tgai_kv_cache.h
        kvc = np.zeros((2, msl, nkv * dk), np.float32)
        kvc[0] = kall[last].transpose(1, 0, 2).reshape(msl, nkv * dk)
        kvc[1] = vall[last].transpose(1, 0, 2).reshape(msl, nkv * dk)
        w = np.fromfile(os.path.join(dump, f"c_attn{last}.bin"), np.float32)
        assert w.size == nh * kv_len, (w.size, nh, kv_len)
        out[f"s{si}_meta"] = np.array([seq, pos, kv_len], np.int32)
        out[f"s{si}_q"] = q.reshape(seq, nh, dk)
        out[f"s{si}_kvc"] = kvc[:, :kv_len].copy()      # rows beyond kv_len are never read
        out[f"s{si}_w"] = w.reshape(nh, kv_len)
    eng.tg_kvcache_free(cache)
    eng.tg_free(m)
    np.savez_compressed(os.path.join(HERE, "engine_fixture.npz"), **out)


def glibc_rand_values(libc, n):
    """((rand() % 2000) - 1000) / 1000.0f, n times, as the reference tests do."""
    out = np.empty(n, np.float32)
    for i in range(n):
        out[i] = np.float32((libc.rand() % 2000) - 1000) / np.float32(1000.0)
    return out


def kvtest(ref, libc):
    ref.tg_be_select.argtypes = [C.c_char_p]
    ref.tg_kv_create.restype = C.c_void_p
    ref.tg_kv_create.argtypes = [C.c_uint32] * 3
    ref.tg_kv_append.argtypes = [C.c_void_p, P, P, C.c_uint32]
    ref.tg_kv_host_ptr.restype = P
    ref.tg_kv_host_ptr.argtypes = [C.c_void_p]
    ref.tg_kv_reset.argtypes = [C.c_void_p]
    ref.tg_kv_len.restype = C.c_uint32
    ref.tg_kv_len.argtypes = [C.c_void_p]
    ref.tg_kv_last_error.restype = C.c_char_p
    ref.tg_kv_destroy.argtypes = [C.c_void_p]
    ref.tgref_cpu_attention_kvtest.argtypes = [P, P, P] + [C.c_int] * 6
    NH = NKVH = 16
    HD, MAXSEQ, NTOK = 64, 128, 32
    KVDIM = NKVH * HD
    libc.srand(31415)
    kall = np.empty(NTOK * KVDIM, np.float32)
    vall = np.empty(NTOK * KVDIM, np.float32)
    for i in range(NTOK * KVDIM):
        kall[i] = np.float32((libc.rand() % 2000) - 1000) / np.float32(1000.0)
        vall[i] = np.float32((libc.rand() % 2000) - 1000) / np.float32(1000.0)
    q = glibc_rand_values(libc, NH * HD)
    assert ref.tg_be_select(b"cpu")
    kv = ref.tg_kv_create(MAXSEQ, NKVH, HD)
    for t in range(NTOK):
        assert ref.tg_kv_append(kv, fptr(kall[t * KVDIM:]), fptr(vall[t * KVDIM:]), 1)
    host = np.ctypeslib.as_array(ref.tg_kv_host_ptr(kv), shape=(2, MAXSEQ, KVDIM)).copy()
    assert not host[:, NTOK:].any()
    oref = np.zeros(NH * HD, np.float32)
    ref.tgref_cpu_attention_kvtest(fptr(q), fptr(np.ascontiguousarray(host)), fptr(oref),
                                   NH, NKVH, HD, NTOK, NTOK - 1, MAXSEQ)
    ref.tg_kv_reset(kv)
    len_after_reset = ref.tg_kv_len(kv)
    n = 0
    while ref.tg_kv_append(kv, fptr(kall), fptr(vall), 1):
        n += 1
    extra = ref.tg_kv_append(kv, fptr(kall), fptr(vall), 1)
    ref.tg_kv_destroy(kv)
    np.savez_compressed(os.path.join(HERE, "kvtest.npz"),
                        geometry=np.array([NH, NKVH, HD, MAXSEQ, NTOK], np.int32),
                        kall=kall.reshape(NTOK, KVDIM), vall=vall.reshape(NTOK, KVDIM), q=q,
                        cache_rows=host[:, :NTOK], out=oref,
                        len_after_reset=np.int32(len_after_reset), fill_count=np.int32(n),
                        extra_append=np.int32(extra))


def attntest(ref, libc):
    ref.tgref_cpu_attention_attntest.argtypes = [P, P, P] + [C.c_int] * 6
    NH = NKVH = 16
    HD, MAXSEQ, NKV, POS = 64, 256, 40, 39
    KVDIM = NKVH * HD
    libc.srand(777)
    q = glibc_rand_values(libc, NH * HD)
    kvc = glibc_rand_values(libc, 2 * MAXSEQ * KVDIM).reshape(2, MAXSEQ, KVDIM)
    kvc[:, NKV:] = 0.0
    outs = {}
    for pos in (POS, 10):
        o = np.zeros(NH * HD, np.float32)
        ref.tgref_cpu_attention_attntest(fptr(q), fptr(np.ascontiguousarray(kvc)), fptr(o),
                                         NH, NKVH, HD, NKV, pos, MAXSEQ)
        outs[pos] = o
    np.savez_compressed(os.path.join(HERE, "attntest.npz"),
                        geometry=np.array([NH, NKVH, HD, MAXSEQ, NKV, POS], np.int32),
                        q=q, kv_rows=kvc[:, :NKV].copy(), out_pos39=outs[39], out_pos10=outs[10])


def forward_golden(eng):
    sys.path.insert(0, os.path.dirname(HERE))
    import fwd_model as FM
    eng.tg_load.restype = C.c_void_p
    eng.tg_load.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_int)]
    eng.tg_kvcache_new.restype = C.c_void_p
    eng.tg_kvcache_new.argtypes = [C.c_void_p, C.c_int]
    eng.tg_kvcache_free.argtypes = [C.c_void_p]
    eng.tg_forward.restype = P
    eng.tg_forward.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.c_int, C.c_void_p, C.c_int]
    eng.tg_free.argtypes = [C.c_void_p]
    out = {}
    for name, cfg in FM.CONFIGS.items():
        seed = FM.SEEDS[name]
        w = FM.weights(cfg, seed)
        with tempfile.TemporaryDirectory() as td:
            path = os.path.join(td, f"{name}.TG")
            FM.write_tg(path, cfg, w)
            err = C.c_int(0)
            m = eng.tg_load(path.encode(), 0, C.byref(err))
            if not m:
                raise RuntimeError(f"tg_load({name}) failed: {err.value}")
            caches = {}
            logits = []
            for seq_name, ids, pos in FM.script(cfg, seed):
                if seq_name not in caches:
                    caches[seq_name] = eng.tg_kvcache_new(m, cfg["max_seq"])
                arr = (C.c_int32 * len(ids))(*ids.tolist())
                lp = eng.tg_forward(m, arr, len(ids), caches[seq_name], int(pos))
                if not lp:
                    raise RuntimeError("tg_forward failed")
                logits.append(np.ctypeslib.as_array(lp, shape=(cfg["vocab"],)).copy())
            for c in caches.values():
                eng.tg_kvcache_free(c)
            eng.tg_free(m)
        out[f"{name}_logits"] = np.array(logits, np.float32)
        out[f"{name}_seed"] = np.int32(seed)
    np.savez_compressed(os.path.join(HERE, "forward.npz"), **out)


def main():
    if not os.path.isdir(REF) or not os.path.exists(os.path.join(REF_LIB, "libtgkv_ref.so")):
        sys.exit("reference checkout or oracle/_ref missing: run `make -C oracle ref` first")
    eng = C.CDLL(os.path.join(REF_LIB, "libtgai_engine_ref.so"), mode=os.RTLD_LAZY)
    ref = C.CDLL(os.path.join(REF_LIB, "libtgkv_ref.so"), mode=os.RTLD_LAZY)
    libc = C.CDLL("libc.so.6")
    engine_pins(eng)
    engine_fixture(eng)
    kvtest(ref, libc)
    attntest(ref, libc)
    forward_golden(eng)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main()
