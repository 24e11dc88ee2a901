"""Parity of the CUDA path (through the C-ABI) with the reference and the oracle.

Bit-exact: cache contents after append / truncate / re-append (fp32 copies,
bf16 round-to-nearest-even).  Attention: within 1e-5 of each head's output
scale for fp32 caches and 1e-2 for bf16 caches (rel_head_err in conftest),
against the engine-order oracle run on the same (decoded) cache.
"""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
import tgkv
from conftest import GOLDEN, attn_tol, rel_head_err

pytestmark = pytest.mark.gpu

TOL_F32 = 1e-5
TOL_BF16 = 1e-2


@pytest.fixture(autouse=True, params=["auto", "tc", "tc-steal"])
def decode_kernel(request, monkeypatch):
    """Every test three times: with the library's own choice of decode
    kernel; with every bf16 head_dim-128 call forced onto the tensor-core
    decode kernel (which the library otherwise keeps for launches of at
    least 131072 position x head rows); and the same with its opt-in tile
    stealing.  Both
    split-sequence kernels and both tensor-core schedules meet every case."""
    if request.param.startswith("tc"):
        monkeypatch.setenv("TGKV_DECODE_TC", "1")
    if request.param == "tc-steal":
        monkeypatch.setenv("TGKV_STEAL", "1")
    return request.param


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def download(lib, c):
    n = lib.tg_kv_bytes(c)
    buf = np.empty(n, np.uint8)
    tgkv.check(lib.tg_kv_download(c, buf.ctypes.data), lib)
    return buf


def cache_rows(lib, c, dtype, max_seq, kv_dim):
    raw = download(lib, c)
    if dtype == tgkv.TG_KV_F32:
        return raw.view(np.float32).reshape(2, max_seq, kv_dim)
    return raw.view(np.uint16).reshape(2, max_seq, kv_dim)


def attend(lib, devbuf, c, q, n_heads, n_q):
    """tg_kv_attention of q ([n_q][nh][hd] fp32) -> host array."""
    qd = devbuf(np.ascontiguousarray(q, np.float32))
    od = devbuf(nbytes=q.nbytes)
    tgkv.check(lib.tg_kv_attention(c, qd.ptr, od.ptr, n_heads, n_q, None), lib)
    assert lib.tg_cuda_kv_sync(None)
    return od.get(np.float32, np.asarray(q).shape)


def test_reference_kv_cache_test_sequence(cuda, devbuf):
    """tests/test_kv_cache_gpu.c with tg_be_select("cuda"): create, 32 appends,
    attention through TGBackend.attention on the cache's device handle, reset,
    fill to capacity."""
    lib = cuda
    z = golden("kvtest.npz")
    nh, nkvh, hd, ms, nt = (int(v) for v in z["geometry"])
    kvd = nkvh * hd
    c = lib.tg_kv_create(ms, nkvh, hd)
    tgkv.check(c, lib)
    assert lib.tg_kv_capacity(c) == ms and lib.tg_kv_len(c) == 0
    assert lib.tg_kv_device_handle(c) and not lib.tg_kv_host_ptr(c)
    kall, vall = z["kall"], z["vall"]
    for t in range(nt):
        tgkv.check(lib.tg_kv_append(c, kall[t].ctypes.data, vall[t].ctypes.data, 1), lib)
    assert lib.tg_kv_len(c) == nt
    rows = cache_rows(lib, c, 0, ms, kvd)
    assert np.array_equal(rows[:, :nt].view(np.uint32), z["cache_rows"].view(np.uint32))
    assert not rows[:, nt:].any()

    be = tgkv.current_backend(lib)
    qd = devbuf(z["q"])
    od = devbuf(nbytes=nh * hd * 4)
    assert be.attention(qd.ptr, lib.tg_kv_device_handle(c), od.ptr, nh, nkvh, hd, nt, nt - 1, ms)
    got = od.get(np.float32, (nh * hd,))
    ref = z["out"]
    den = np.maximum(np.abs(ref), 1e-6)
    assert (np.abs(got - ref) / den <= 0.01).all()          # the reference test's criterion
    kvc = rows.astype(np.float32)
    eng = O.attention_engine(z["q"], kvc, nh, nkvh, hd, 1, nt - 1, nt, ms)
    assert rel_head_err(got.reshape(1, nh, hd), eng) < TOL_F32

    lib.tg_kv_reset(c)
    assert lib.tg_kv_len(c) == 0
    n = 0
    while lib.tg_kv_append(c, kall[0].ctypes.data, vall[0].ctypes.data, 1):
        n += 1
        assert n <= ms
    assert n == int(z["fill_count"]) == ms
    assert lib.tg_kv_append(c, kall[0].ctypes.data, vall[0].ctypes.data, 1) == 0
    assert b"capacity" in lib.tg_kv_last_error()
    lib.tg_kv_destroy(c)


def test_reference_attention_test_sequence(cuda, devbuf):
    """tests/test_vk_attn_moe.c's attention case (NKV=40, pos 39 and pos 10)."""
    lib = cuda
    z = golden("attntest.npz")
    nh, nkvh, hd, ms, nkv, pos = (int(v) for v in z["geometry"])
    kvd = nkvh * hd
    full = np.zeros((2, ms, kvd), np.float32)
    full[:, :nkv] = z["kv_rows"]
    kb = devbuf(full)
    qd = devbuf(z["q"])
    od = devbuf(nbytes=nh * hd * 4)
    be = tgkv.current_backend(lib)
    for p, key in ((pos, "out_pos39"), (10, "out_pos10")):
        assert be.attention(qd.ptr, kb.ptr, od.ptr, nh, nkvh, hd, nkv, p, ms)
        got = od.get(np.float32, (nh * hd,))
        ref = z[key]
        assert (np.abs(got - ref) / np.maximum(np.abs(ref), 1e-6) <= 0.01).all(), p
        eng = O.attention_engine(z["q"], full, nh, nkvh, hd, 1, p, min(nkv, p + 1), ms)
        assert rel_head_err(got.reshape(1, nh, hd), eng) < TOL_F32, p


def test_engine_fixture_forwards(cuda, devbuf):
    """q and K/V captured from the reference engine's real forwards of its
    fixture model (head_dim 32, 6 heads): causal multi-token and decode steps."""
    lib = cuda
    z = golden("engine_fixture.npz")
    msl, _, nh, nkv, dk = (int(v) for v in z["geometry"])
    kvd = nkv * dk
    for si in range(int(z["n_steps"])):
        seq, pos, kvl = (int(v) for v in z[f"s{si}_meta"])
        c = lib.tg_kv_create(msl, nkv, dk)
        rows = z[f"s{si}_kvc"]
        tgkv.check(lib.tg_kv_append(c, np.ascontiguousarray(rows[0]).ctypes.data,
                                    np.ascontiguousarray(rows[1]).ctypes.data, kvl), lib)
        got = attend(lib, devbuf, c, z[f"s{si}_q"], nh, seq)
        kvc = np.zeros((2, msl, kvd), np.float32)
        kvc[:, :kvl] = rows
        eng = O.attention_engine(z[f"s{si}_q"], kvc, nh, nkv, dk, seq, pos, kvl, msl)
        assert rel_head_err(got, eng) < TOL_F32, si
        lib.tg_kv_destroy(c)


def make_cache(lib, devbuf, max_seq, nkv, hd, dtype, k, v):
    """Cache of max_seq rows with k, v ([n][kv_dim] fp32) appended from device."""
    c = lib.tg_kv_create_ex(max_seq, nkv, hd, dtype)
    tgkv.check(c, lib)
    if len(k):
        kd, vd = devbuf(np.ascontiguousarray(k, np.float32)), devbuf(np.ascontiguousarray(v, np.float32))
        tgkv.check(lib.tg_kv_append_dev(c, kd.ptr, vd.ptr, len(k), None), lib)
    assert lib.tg_cuda_kv_sync(None)
    return c


def host_cache(lib, c, dtype, max_seq, kv_dim):
    rows = cache_rows(lib, c, dtype, max_seq, kv_dim)
    return rows if dtype == 0 else O.bf16_to_f32(rows)


@pytest.mark.parametrize("dtype", [0, 1])
def test_append_bits(cuda, devbuf, dtype):
    """Stored bits equal the host rule (fp32 copy / bf16 RNE), including ties,
    infinities, NaN, denormals and signed zero."""
    lib = cuda
    nkv, hd, ms = 2, 64, 40
    kvd = nkv * hd
    rng = np.random.default_rng(11)
    k = rng.standard_normal((33, kvd)).astype(np.float32) * 100
    v = rng.standard_normal((33, kvd)).astype(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-39, 3.39e38,
                        1.0 + 2**-8, 1.0 + 3 * 2**-8, -(1.0 + 2**-8), 65504.0], np.float32)
    k[0, :special.size] = special
    v[1, :special.size] = special[::-1]
    c = make_cache(lib, devbuf, ms, nkv, hd, dtype, k[:20], v[:20])
    tgkv.check(lib.tg_kv_append(c, k[20:].ctypes.data, v[20:].ctypes.data, 13), lib)
    rows = cache_rows(lib, c, dtype, ms, kvd)
    if dtype == 0:
        assert np.array_equal(rows[0, :33].view(np.uint32), k.view(np.uint32))
        assert np.array_equal(rows[1, :33].view(np.uint32), v.view(np.uint32))
    else:
        assert np.array_equal(rows[0, :33], O.f32_to_bf16(k))
        assert np.array_equal(rows[1, :33], O.f32_to_bf16(v))
    assert not rows[:, 33:].any()
    lib.tg_kv_destroy(c)


def synth_qkv(seed, n, nh, nkv, hd, scale=1.0):
    q = O.normal(n * nh * hd, seed, 1, nh, hd, scale).reshape(n, nh, hd)
    k = O.normal(n * nkv * hd, seed, 2, nkv, hd, scale).reshape(n, nkv * hd)
    v = O.normal(n * nkv * hd, seed, 3, nkv, hd, scale).reshape(n, nkv * hd)
    return q, k, v


def test_cfg1_prefill_then_decode_fp32(cuda, devbuf):
    """configs[0] shape: 8 q = 8 kv heads, head_dim 64, fp32, RoPE (theta 1e4)
    applied on the host before append; 128-token causal prefill, then
    single-token append + attention steps (sampled) up to L = 512."""
    lib = cuda
    nh = nkv = 8
    hd, ms, L = 64, 512, 512
    q, k, v = synth_qkv(101, L, nh, nkv, hd)
    qr, kr = O.rope(q.ravel(), k.ravel(), nh, nkv, hd, 0)
    qr = qr.reshape(L, nh, hd)
    kr = kr.reshape(L, nkv * hd)
    c = make_cache(lib, devbuf, ms, nkv, hd, 0, kr[:128], v[:128])
    got = attend(lib, devbuf, c, qr[:128], nh, 128)
    kvc = host_cache(lib, c, 0, ms, nkv * hd)
    eng = O.attention_engine(qr[:128], kvc, nh, nkv, hd, 128, 0, 128, ms)
    assert rel_head_err(got, eng) < TOL_F32
    kd, vd = devbuf(kr), devbuf(v)
    qd, od = devbuf(qr), devbuf(nbytes=qr.nbytes)
    row_k = kr.shape[1] * 4
    row_q = nh * hd * 4
    for t in range(128, L):
        tgkv.check(lib.tg_kv_append_dev(c, kd.ptr + t * row_k, vd.ptr + t * row_k, 1, None), lib)
        tgkv.check(lib.tg_kv_attention(c, qd.ptr + t * row_q, od.ptr + t * row_q, nh, 1, None), lib)
    assert lib.tg_cuda_kv_sync(None)
    out = od.get(np.float32, qr.shape)
    kvc = host_cache(lib, c, 0, ms, nkv * hd)
    assert np.array_equal(kvc[0].view(np.uint32), kr.view(np.uint32))
    for t in (128, 129, 200, 255, 256, 257, 383, 511):
        eng = O.attention_engine(qr[t], kvc, nh, nkv, hd, 1, t, t + 1, ms)
        assert rel_head_err(out[t], eng[0]) < TOL_F32, t
    lib.tg_kv_destroy(c)


@pytest.mark.parametrize("L", [1, 2, 31, 32, 33, 127, 128, 129, 1000, 4096])
def test_cfg2_gqa_bf16_lengths(cuda, devbuf, L):
    """configs[1] shape: 16 q / 4 kv heads, head_dim 128, bf16, inputs scaled
    by 1/sqrt(128); attention of the newest token over L positions."""
    lib = cuda
    nh, nkv, hd = 16, 4, 128
    q, k, v = synth_qkv(202 + L, L, nh, nkv, hd, 128 ** -0.5)
    c = make_cache(lib, devbuf, 4096, nkv, hd, 1, k, v)
    got = attend(lib, devbuf, c, q[-1:], nh, 1)
    kvc = host_cache(lib, c, 1, 4096, nkv * hd)
    eng = O.attention_engine(q[-1:], kvc, nh, nkv, hd, 1, L - 1, L, 4096)
    err = rel_head_err(got, eng)
    assert err < TOL_BF16
    assert err < 1e-5          # fp32 arithmetic on bf16-decoded rows: tighter in fact
    lib.tg_kv_destroy(c)


@pytest.mark.parametrize("nh,nkv,hd,dtype", [(8, 8, 32, 0), (8, 8, 128, 0), (12, 4, 64, 1),
                                             (16, 2, 64, 0), (32, 4, 128, 1), (4, 1, 256, 1),
                                             (6, 3, 32, 1), (64, 8, 64, 1)])
def test_head_geometries(cuda, devbuf, nh, nkv, hd, dtype):
    """Head dims 32..256, group sizes 1..8 (group 8 runs as two head subsets),
    MQA, both storage types, with a causal multi-token query block."""
    lib = cuda
    L, nq = 300, 5
    q, k, v = synth_qkv(303 + nh + hd, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, 320, nkv, hd, dtype, k, v)
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    kvc = host_cache(lib, c, dtype, 320, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, 320)
    assert rel_head_err(got, eng) < (TOL_F32 if dtype == 0 else TOL_BF16)
    if dtype == 1:
        assert rel_head_err(got, eng) < attn_tol(lib)
    lib.tg_kv_destroy(c)


def test_cfg4_batched_decode_ragged(cuda, devbuf):
    """configs[3] shape at reduced count: 12 sequences of ragged lengths,
    32 q / 8 kv heads, head_dim 128, bf16; two batched decode steps
    (append + attention per sequence in one call each)."""
    lib = cuda
    nh, nkv, hd = 32, 8, 128
    kvd = nkv * hd
    lens = [1, 2, 33, 100, 511, 1000, 1024, 1025, 2047, 3000, 4096, 5000]
    caches = []
    for i, L in enumerate(lens):
        _, k, v = synth_qkv(400 + i, L, nh, nkv, hd)
        caches.append(make_cache(lib, devbuf, L + 4, nkv, hd, 1, k, v))
    arr = (C.c_void_p * len(caches))(*caches)
    b = lib.tg_kv_batch_create(arr, len(caches), nh)
    tgkv.check(b, lib)
    for step in range(2):
        q = O.normal(len(lens) * nh * hd, 77 + step, 5).reshape(len(lens), nh, hd)
        kn = O.normal(len(lens) * kvd, 78 + step, 6).reshape(len(lens), kvd)
        vn = O.normal(len(lens) * kvd, 79 + step, 7).reshape(len(lens), kvd)
        qd, kd, vd = devbuf(q), devbuf(kn), devbuf(vn)
        od = devbuf(nbytes=q.nbytes)
        tgkv.check(lib.tg_kv_batch_decode(b, qd.ptr, kd.ptr, vd.ptr, od.ptr, None), lib)
        assert lib.tg_cuda_kv_sync(None)
        out = od.get(np.float32, q.shape)
        for i, c in enumerate(caches):
            L = lens[i] + step + 1
            assert lib.tg_kv_len(c) == L
            rows = cache_rows(lib, c, 1, lens[i] + 4, kvd)
            assert np.array_equal(rows[0, L - 1], O.f32_to_bf16(kn[i]))
            assert np.array_equal(rows[1, L - 1], O.f32_to_bf16(vn[i]))
            kvc = O.bf16_to_f32(rows)
            eng = O.attention_engine(q[i], kvc, nh, nkv, hd, 1, L - 1, L, lens[i] + 4)
            assert rel_head_err(out[i], eng[0]) < 1e-5, (i, L)
    lib.tg_kv_batch_destroy(b)
    for c in caches:
        lib.tg_kv_destroy(c)


@pytest.mark.parametrize("dtype,nh,nkv,hd", [(0, 16, 2, 64), (1, 16, 2, 64), (1, 8, 8, 32)])
def test_batched_decode_fused_append_geometries(cuda, devbuf, dtype, nh, nkv, hd):
    """The decode append runs inside the attention launch: with group 8 two head
    subsets write the same new row; fp32 and bf16; several consecutive steps
    (back-to-back launches on one stream)."""
    lib = cuda
    kvd = nkv * hd
    lens = [1, 40, 300, 2000]
    caches = []
    for i, L in enumerate(lens):
        _, k, v = synth_qkv(900 + i, L, nh, nkv, hd)
        caches.append(make_cache(lib, devbuf, L + 8, nkv, hd, dtype, k, v))
    b = lib.tg_kv_batch_create((C.c_void_p * len(caches))(*caches), len(caches), nh)
    tgkv.check(b, lib)
    steps = 5
    q = O.normal(steps * len(lens) * nh * hd, 31, 5).reshape(steps, len(lens), nh, hd)
    kn = O.normal(steps * len(lens) * kvd, 32, 6).reshape(steps, len(lens), kvd)
    vn = O.normal(steps * len(lens) * kvd, 33, 7).reshape(steps, len(lens), kvd)
    qd, kd, vd = devbuf(q), devbuf(kn), devbuf(vn)
    od = devbuf(nbytes=q.nbytes)
    qrow, krow = len(lens) * nh * hd * 4, len(lens) * kvd * 4
    for st in range(steps):
        tgkv.check(lib.tg_kv_batch_decode(b, qd.ptr + st * qrow, kd.ptr + st * krow,
                                          vd.ptr + st * krow, od.ptr + st * qrow, None), lib)
        assert lib.tg_kv_batch_last_launches(b) == 1
    assert lib.tg_cuda_kv_sync(None)
    out = od.get(np.float32, q.shape)
    for i, c in enumerate(caches):
        ms = lens[i] + 8
        rows = cache_rows(lib, c, dtype, ms, kvd)
        kvc = rows if dtype == 0 else O.bf16_to_f32(rows)
        for st in range(steps):
            L = lens[i] + st + 1
            want_k = kn[st, i] if dtype == 0 else O.bf16_to_f32(O.f32_to_bf16(kn[st, i]))
            assert np.array_equal(kvc[0, L - 1], want_k), (i, st)
            eng = O.attention_engine(q[st, i], kvc, nh, nkv, hd, 1, L - 1, L, ms)
            assert rel_head_err(out[st, i], eng[0]) < 1e-5, (i, st)
    lib.tg_kv_batch_destroy(b)
    for c in caches:
        lib.tg_kv_destroy(c)


@pytest.mark.parametrize("n_seq", [3, 24])
def test_batch_decode_pinned_host_buffers_on_a_stream(cuda, devbuf, n_seq):
    """tg_kv_batch_decode_host with page-locked buffers on a non-default
    stream, several steps back to back: uploads go through the plan's two
    staging slots on its copy stream, outputs straight from the kernel into
    the pinned out buffers (3 and 24 sequences)."""
    import torch
    lib = cuda
    nh, nkv, hd, steps = 16, 4, 128, 5
    kvd = nkv * hd
    caches = []
    lens = [[33, 1500, 4000][i % 3] + 7 * i for i in range(n_seq)]
    for i, L in enumerate(lens):
        _, k, v = synth_qkv(520 + i, L, nh, nkv, hd)
        caches.append(make_cache(lib, devbuf, 4400, nkv, hd, 1, k, v))
    n = n_seq
    b = lib.tg_kv_batch_create((C.c_void_p * n)(*caches), n, nh)
    qs = [torch.from_numpy(O.normal(n * nh * hd, 30 + s).reshape(n, nh, hd)).pin_memory()
          for s in range(steps)]
    ks = [torch.from_numpy(O.normal(n * kvd, 40 + s).reshape(n, kvd)).pin_memory()
          for s in range(steps)]
    vs = [torch.from_numpy(O.normal(n * kvd, 50 + s).reshape(n, kvd)).pin_memory()
          for s in range(steps)]
    outs = [torch.zeros(n, nh, hd).pin_memory() for _ in range(steps)]
    assert lib.tg_cuda_kv_host_device_ptr(outs[0].data_ptr())
    assert not lib.tg_cuda_kv_host_device_ptr(np.zeros(4, np.float32).ctypes.data)
    stream = lib.tg_cuda_kv_stream_create()
    assert stream
    for s in range(steps):
        tgkv.check(lib.tg_kv_batch_decode_host(b, qs[s].data_ptr(), ks[s].data_ptr(),
                                               vs[s].data_ptr(), outs[s].data_ptr(), stream), lib)
    assert lib.tg_cuda_kv_sync(stream)
    assert lib.tg_cuda_kv_device_error() == 0
    for i, c in enumerate(caches):
        L = lib.tg_kv_len(c)
        rows = cache_rows(lib, c, 1, 4400, kvd)
        kvc = O.bf16_to_f32(rows)
        for s in range(steps):
            m = L - steps + s + 1           # positions step s attended
            assert np.array_equal(rows[0, m - 1], O.f32_to_bf16(ks[s][i].numpy()))
            eng = O.attention_engine(qs[s][i].numpy(), kvc, nh, nkv, hd, 1, m - 1, m, 4400)
            assert rel_head_err(outs[s][i].numpy(), eng[0]) < 1e-5, (i, s)
    lib.tg_cuda_kv_stream_destroy(stream)
    lib.tg_kv_batch_destroy(b)
    for c in caches:
        lib.tg_kv_destroy(c)


def test_batch_decode_host_buffers(cuda, devbuf):
    """tg_kv_batch_decode_host: the same step from host buffers."""
    lib = cuda
    nh, nkv, hd = 8, 2, 128
    kvd = nkv * hd
    caches = []
    for i, L in enumerate([5, 700]):
        _, k, v = synth_qkv(500 + i, L, nh, nkv, hd)
        caches.append(make_cache(lib, devbuf, 800, nkv, hd, 1, k, v))
    b = lib.tg_kv_batch_create((C.c_void_p * 2)(*caches), 2, nh)
    q = O.normal(2 * nh * hd, 9).reshape(2, nh, hd)
    kn = O.normal(2 * kvd, 10).reshape(2, kvd)
    vn = O.normal(2 * kvd, 11).reshape(2, kvd)
    out = np.zeros_like(q)
    tgkv.check(lib.tg_kv_batch_decode_host(b, q.ctypes.data, kn.ctypes.data, vn.ctypes.data,
                                           out.ctypes.data, None), lib)
    assert lib.tg_cuda_kv_sync(None)
    for i, c in enumerate(caches):
        L = lib.tg_kv_len(c)
        kvc = O.bf16_to_f32(cache_rows(lib, c, 1, 800, kvd))
        eng = O.attention_engine(q[i], kvc, nh, nkv, hd, 1, L - 1, L, 800)
        assert rel_head_err(out[i], eng[0]) < 1e-5
    lib.tg_kv_batch_destroy(b)
    for c in caches:
        lib.tg_kv_destroy(c)


def test_cfg5_long_context_131072(cuda, devbuf):
    """configs[4] shape for one layer: L = 131072, 32 q / 8 kv, head_dim 128,
    bf16 ~N(0,1): split-sequence attention with the in-kernel combine."""
    lib = cuda
    nh, nkv, hd, L = 32, 8, 128, 131072
    q = O.normal(nh * hd, 606, 1).reshape(1, nh, hd)
    k = O.normal(L * nkv * hd, 606, 2).reshape(L, nkv * hd)
    v = O.normal(L * nkv * hd, 606, 3).reshape(L, nkv * hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 1, k, v)
    del k, v
    got = attend(lib, devbuf, c, q[-1:], nh, 1)
    kvc = host_cache(lib, c, 1, L, nkv * hd)
    eng = O.attention_engine(q[-1:], kvc, nh, nkv, hd, 1, L - 1, L, L)
    assert rel_head_err(got, eng) < TOL_BF16
    # At 131072 positions the engine order's sequential float sums carry
    # ~1e-5 of rounding themselves; the double-accumulation oracle is the
    # sharper reference: the CUDA-core kernel stays within 1e-5 of it, the
    # tensor-core one (fp32 accumulation inside the MMAs over ~1000 tiles)
    # within TC_TOL (measured 1.5e-5).
    tol = attn_tol(lib)
    f64 = O.attention_f64(q[-1:], kvc, nh, nkv, hd, 1, L - 1, L, L)
    assert rel_head_err(got, f64) < tol
    assert rel_head_err(eng, f64) < 1e-4
    lib.tg_kv_destroy(c)


@pytest.mark.parametrize("merge2", ["1", "0"])
def test_one_kv_head_of_131072_positions(cuda, devbuf, merge2, monkeypatch):
    """configs[4] with its KV heads split over 8 GPUs: each GPU attends one KV
    head (4 query heads) over 131072 positions, one segment of hundreds of
    chunks.  Such segments merge in two levels (groups of 16 chunks, then the
    groups); TGKV_MERGE2=0 merges in one CTA.  Both against the double oracle,
    twice in a row (the counters reset themselves)."""
    monkeypatch.setenv("TGKV_MERGE2", merge2)
    lib = cuda
    nh, nkv, hd, L = 4, 1, 128, 131072
    q = O.normal(nh * hd, 707, 1).reshape(1, nh, hd)
    k = O.normal(L * hd, 707, 2).reshape(L, hd)
    v = O.normal(L * hd, 707, 3).reshape(L, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 1, k, v)
    del k, v
    kvc = host_cache(lib, c, 1, L, hd)
    f64 = O.attention_f64(q, kvc, nh, nkv, hd, 1, L - 1, L, L)
    for _ in range(2):
        got = attend(lib, devbuf, c, q, nh, 1)
        assert rel_head_err(got, f64) < attn_tol(lib)
    assert lib.tg_cuda_kv_device_error() == 0
    lib.tg_kv_destroy(c)


def token_kv(tok, pos, layer, kvd):
    """K/V of a token as a pure function of (token id, position, layer)."""
    k = O.normal(kvd, 31337, int(tok), int(pos), int(layer) * 2)
    v = O.normal(kvd, 31337, int(tok), int(pos), int(layer) * 2 + 1)
    return k, v


def test_cfg3_lcp_truncate_reappend_bitexact(cuda, devbuf):
    """configs[2] semantics: 8 turns; each keeps an LCP of 50-95 % of the history,
    truncates there (python/tgai_go/_session.py:137-163) and appends a
    64-512-token suffix; /undo truncates to the previous turn boundary and
    /clear to 0.  After every turn, each layer's cache equals, bit for bit, a
    cache built from scratch from the final token sequence."""
    lib = cuda
    nh, nkv, hd, layers = 16, 4, 128, 3
    kvd = nkv * hd
    ms = 4096
    rng = np.random.default_rng(8)
    caches = [make_cache(lib, devbuf, ms, nkv, hd, 1, [], []) for _ in range(layers)]
    hist = []
    bounds = [0]
    for turn in range(8):
        if turn == 5:                            # /undo: back to the previous boundary
            lcp = bounds[-2]
        elif turn == 6:                          # /clear
            lcp = 0
        else:
            lcp = int(len(hist) * rng.uniform(0.5, 0.95))
        suffix = rng.integers(0, 32000, int(rng.integers(64, 513))).tolist()
        hist = hist[:lcp] + suffix
        for li, c in enumerate(caches):
            tgkv.check(lib.tg_kv_truncate(c, lcp), lib)
            ks, vs = zip(*[token_kv(t, lcp + j, li, kvd) for j, t in enumerate(suffix)])
            ks, vs = np.stack(ks), np.stack(vs)
            tgkv.check(lib.tg_kv_append(c, ks.ctypes.data, vs.ctypes.data, len(suffix)), lib)
            assert lib.tg_kv_len(c) == len(hist)
        bounds.append(len(hist))
        li = turn % layers
        rows = cache_rows(lib, caches[li], 1, ms, kvd)
        ks, vs = zip(*[token_kv(t, j, li, kvd) for j, t in enumerate(hist)])
        assert np.array_equal(rows[0, :len(hist)], O.f32_to_bf16(np.stack(ks))), turn
        assert np.array_equal(rows[1, :len(hist)], O.f32_to_bf16(np.stack(vs))), turn
        # suffix attention (causal block) over the re-appended cache
        nq = min(len(suffix), 64)
        q = O.normal(nq * nh * hd, 900 + turn).reshape(nq, nh, hd)
        got = attend(lib, devbuf, caches[li], q, nh, nq)
        kvc = O.bf16_to_f32(rows)
        eng = O.attention_engine(q, kvc, nh, nkv, hd, nq, len(hist) - nq, len(hist), ms)
        assert rel_head_err(got, eng) < attn_tol(lib)
    assert lib.tg_kv_truncate(caches[0], lib.tg_kv_len(caches[0]) + 1) == 0
    for c in caches:
        lib.tg_kv_destroy(c)


@pytest.mark.parametrize("chunk", ["32", "64", "96", "128", "4096"])
def test_split_chunk_boundaries(cuda, devbuf, chunk, monkeypatch):
    """Forced chunk lengths put split boundaries on, before and after tiles,
    and make some CTAs' chunks shorter than a warp's rows."""
    lib = cuda
    monkeypatch.setenv("TGKV_CHUNK", chunk)
    nh, nkv, hd = 8, 2, 64
    for L in (1, 31, 32, 33, 95, 97, 1000):
        q, k, v = synth_qkv(700 + L, L, nh, nkv, hd)
        for dtype in (0, 1):
            c = make_cache(lib, devbuf, L, nkv, hd, dtype, k, v)
            got = attend(lib, devbuf, c, q[-3:] if L >= 3 else q[-1:], nh, min(3, L))
            kvc = host_cache(lib, c, dtype, L, nkv * hd)
            nq = min(3, L)
            eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L)
            assert rel_head_err(got, eng) < 1e-5, (L, dtype)
            lib.tg_kv_destroy(c)


def test_many_items_split_launches(cuda, devbuf):
    """More than 1024 query rows in one call: several launches, each with its
    own CTA table and shared scratch."""
    lib = cuda
    nh, nkv, hd, L = 4, 1, 64, 1500
    q, k, v = synth_qkv(808, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 0, k, v)
    got = attend(lib, devbuf, c, q, nh, L)
    kvc = host_cache(lib, c, 0, L, nkv * hd)
    for t in (0, 1, 700, 1023, 1024, 1025, 1499):
        eng = O.attention_engine(q[t], kvc, nh, nkv, hd, 1, t, t + 1, L)
        assert rel_head_err(got[t], eng[0]) < 1e-5, t
    lib.tg_kv_destroy(c)


@pytest.mark.parametrize("dtype", [0, 1])
def test_rope_append_matches_engine_rope(cuda, devbuf, dtype):
    """TGBackend.rope (shaders/rope.comp semantics) with cos/sin tables of the
    engine's formula: rotated K in the cache and rotated Q are bit-identical to
    the engine's rope() (src/tgai_engine.c:3404-3490), V is copied."""
    lib = cuda
    nh, nkv, hd, ms, n, pos0 = 8, 2, 64, 64, 5, 17
    half = hd // 2
    ang = np.zeros((ms, half), np.float32)
    lib_o = O.load()
    # table entries exactly as the engine computes them: powf, float angle, cosf/sinf
    import ctypes
    libm = ctypes.CDLL("libm.so.6")
    for fn in ("powf", "cosf", "sinf"):
        getattr(libm, fn).restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    libm.cosf.argtypes = libm.sinf.argtypes = [ctypes.c_float]
    cs = np.zeros((ms, half), np.float32)
    sn = np.zeros((ms, half), np.float32)
    for i in range(half):
        freq = np.float32(1.0) / np.float32(libm.powf(10000.0, float(np.float32(2 * i) / np.float32(hd))))
        for p in range(ms):
            a = np.float32(p) * freq
            cs[p, i], sn[p, i] = libm.cosf(float(a)), libm.sinf(float(a))
    rng = np.random.default_rng(12)
    qkv = rng.standard_normal((n, nh * hd + 2 * nkv * hd)).astype(np.float32)
    c = make_cache(lib, devbuf, ms, nkv, hd, dtype, [], [])
    qd, csd, snd = devbuf(qkv), devbuf(cs), devbuf(sn)
    qo = devbuf(nbytes=n * nh * hd * 4)
    be = tgkv.current_backend(lib)
    assert be.rope(qd.ptr, csd.ptr, snd.ptr, lib.tg_kv_device_handle(c), qo.ptr, n, nh, nkv, hd,
                   pos0, ms)
    q_ref, k_ref = O.rope(qkv[:, :nh * hd].copy(), qkv[:, nh * hd:nh * hd + nkv * hd].copy(),
                          nh, nkv, hd, pos0)
    q_got = qo.get(np.float32, (n, nh * hd))
    assert np.array_equal(q_got.view(np.uint32), q_ref.reshape(n, -1).view(np.uint32))
    rows = cache_rows(lib, c, dtype, ms, nkv * hd)
    v_src = qkv[:, nh * hd + nkv * hd:]
    if dtype == 0:
        assert np.array_equal(rows[0, pos0:pos0 + n].view(np.uint32),
                              k_ref.reshape(n, -1).view(np.uint32))
        assert np.array_equal(rows[1, pos0:pos0 + n].view(np.uint32), v_src.view(np.uint32))
    else:
        assert np.array_equal(rows[0, pos0:pos0 + n], O.f32_to_bf16(k_ref.reshape(n, -1)))
        assert np.array_equal(rows[1, pos0:pos0 + n], O.f32_to_bf16(v_src))
    lib.tg_kv_destroy(c)


@pytest.mark.parametrize("dtype", [0, 1])
def test_rope_append_with_context_extension(cuda, devbuf, dtype):
    """TGBackend.rope with tg_kv_rope_tables' NTK-by-parts tables writes the
    engine's extended-context K (golden vectors from the compiled engine) into
    the cache, and attention with the engine's YaRN temperature
    (tg_kv_set_attn_mscale) matches the oracle at that scale."""
    lib = cuda
    z = golden("engine_pins.npz")
    seq, nh, nkv, dk, pos, ectx, msl = (int(v) for v in z["ropex0_shape"])
    n = pos + seq
    cs = np.zeros((n, dk // 2), np.float32)
    sn = np.zeros_like(cs)
    ms = C.c_float()
    assert lib.tg_kv_rope_tables(float(z["ropex0_theta"]), dk, 0, n, ectx, msl,
                                 cs.ctypes.data_as(tgkv.PF), sn.ctypes.data_as(tgkv.PF),
                                 C.byref(ms))
    kvd = nkv * dk
    rng = np.random.default_rng(99)
    v = rng.standard_normal((seq, kvd)).astype(np.float32)
    qkv = np.concatenate([z["ropex0_q"].reshape(seq, nh * dk), z["ropex0_k"].reshape(seq, kvd), v],
                         axis=1)
    # fill positions [0, pos) so attention has a context, then rope-append seq rows
    k_ctx = O.normal(pos * kvd, 4, 1).reshape(pos, kvd)
    v_ctx = O.normal(pos * kvd, 4, 2).reshape(pos, kvd)
    c = make_cache(lib, devbuf, n, nkv, dk, dtype, k_ctx, v_ctx)
    qd, csd, snd = devbuf(np.ascontiguousarray(qkv)), devbuf(cs), devbuf(sn)
    qo = devbuf(nbytes=seq * nh * dk * 4)
    be = tgkv.current_backend(lib)
    assert be.rope(qd.ptr, csd.ptr, snd.ptr, lib.tg_kv_device_handle(c), qo.ptr, seq, nh, nkv, dk,
                   pos, n)
    lib.tg_kv_advance(c, seq)
    rows = cache_rows(lib, c, dtype, n, kvd)
    kref = z["ropex0_kout"].reshape(seq, kvd)
    if dtype == 0:
        assert np.array_equal(rows[0, pos:n].view(np.uint32), kref.view(np.uint32))
    else:
        assert np.array_equal(rows[0, pos:n], O.f32_to_bf16(kref))
    q_rot = qo.get(np.float32, (seq, nh, dk))
    assert np.array_equal(q_rot.reshape(-1).view(np.uint32),
                          z["ropex0_qout"].reshape(-1).view(np.uint32))
    lib.tg_kv_set_attn_mscale(c, ms.value)
    got = attend(lib, devbuf, c, q_rot, nh, seq)
    kvc = host_cache(lib, c, dtype, n, kvd)
    eng = O.attention_engine(q_rot, kvc, nh, nkv, dk, seq, pos, n, n, mscale=ms.value)
    assert rel_head_err(got, eng) < attn_tol(lib)
    plain = O.attention_engine(q_rot, kvc, nh, nkv, dk, seq, pos, n, n)
    assert rel_head_err(got, plain) > 1e-3          # the temperature did change the result
    lib.tg_kv_destroy(c)


def test_error_paths(cuda, devbuf):
    lib = cuda
    c = make_cache(lib, devbuf, 8, 2, 64, 0, np.zeros((4, 128), np.float32),
                   np.zeros((4, 128), np.float32))
    q = devbuf(nbytes=8 * 64 * 4 * 8)
    assert lib.tg_kv_attention(c, q.ptr, q.ptr, 8, 5, None) == 0        # n_q > len
    assert b"n_q" in lib.tg_kv_last_error()
    assert lib.tg_kv_attention(c, q.ptr, q.ptr, 3, 1, None) == 0        # 3 % 2 != 0
    assert lib.tg_kv_attention(c, q.ptr, q.ptr, 8, 0, None) == 0
    big = np.zeros((5, 128), np.float32)
    assert lib.tg_kv_append(c, big.ctypes.data, big.ctypes.data, 5) == 0
    assert b"capacity" in lib.tg_kv_last_error()
    assert lib.tg_kv_len(c) == 4
    lib.tg_kv_advance(c, 100)
    assert lib.tg_kv_len(c) == 8                                         # clamped
    lib.tg_kv_destroy(c)
    odd = lib.tg_kv_create_ex(16, 1, 48, 0)                               # no kernel for hd 48
    tgkv.check(odd, lib)
    lib.tg_kv_advance(odd, 4)
    assert lib.tg_kv_attention(odd, q.ptr, q.ptr, 1, 1, None) == 0
    assert b"head_dim" in lib.tg_kv_last_error()
    lib.tg_kv_destroy(odd)
    lib.tg_cuda_kv_inject_alloc_failures(1)
    assert not lib.tg_kv_create(16, 2, 64)
    assert b"allocation" in lib.tg_kv_last_error()
    assert lib.tg_kv_create_ex(16, 2, 64, 7) is None


def test_no_bounded_wait_expired(cuda):
    """No kernel in this session hit its bounded-wait limit."""
    assert cuda.tg_cuda_kv_device_error() == 0
    calls, ok, fb = C.c_uint64(), C.c_uint64(), C.c_uint64()
    cuda.tg_gpu_kv_stats(C.byref(calls), C.byref(ok), C.byref(fb))
    assert calls.value > 0 and fb.value == 0
