"""A chat turn's suffix in one call: tg_kv_append_attention.

The engine writes a turn's K/V rows and then attends the turn's queries over
the cache (src/tgai_engine.c:3923-4011).  tg_kv_append_attention does both in
one call: by default the append kernel then the attention; with
TGKV_FUSE_SUFFIX=1, on a bf16 head_dim-128 cache, one launch of the
tensor-core suffix kernel whose clusters store the new rows they are about to
read (CTAs of different row blocks store the same bytes for shared rows).
These tests run configs[2]'s turn script -- LCP truncate, /undo, /clear,
64-512-token suffixes -- through the fused call and check:
  * the cache bytes equal, bit for bit, a cache built by the append kernel
    (the same rounding, every stale row of a truncated turn overwritten);
  * the outputs meet the engine-order oracle on the cache as stored;
  * the fused route is one launch of the suffix kernel; geometries it does
    not take (fp32 caches, too few rows) run the two launches with the same
    results.  Both routes are run.
"""
import numpy as np
import pytest

import oracle as O
import tgkv
from conftest import TC_TOL, rel_head_err
from test_gpu_parity import cache_rows, make_cache, token_kv

pytestmark = pytest.mark.gpu


def _turns(seed, n_turns):
    rng = np.random.default_rng(seed)
    hist, bounds, out = [], [0], []
    for turn in range(n_turns):
        if turn == 5:
            lcp = bounds[-2]                     # /undo
        elif turn == 6:
            lcp = 0                              # /clear
        else:
            lcp = int(len(hist) * rng.uniform(0.5, 0.95))
        suffix = rng.integers(0, 32000, int(rng.integers(64, 513))).tolist()
        hist = hist[:lcp] + suffix
        bounds.append(len(hist))
        out.append((lcp, suffix, list(hist)))
    return out


@pytest.mark.parametrize("fuse", ["1", "0"])     # in-kernel append, or the append kernel first
@pytest.mark.parametrize("nh", [16, 32])          # groups of 4 and 8 query heads
def test_fused_turns_match_separate_append_and_oracle(cuda, devbuf, nh, fuse, monkeypatch):
    lib = cuda
    monkeypatch.setenv("TGKV_FUSE_SUFFIX", fuse)
    nkv, hd, ms, layer = 4, 128, 4096, 1
    kvd = nkv * hd
    fused = make_cache(lib, devbuf, ms, nkv, hd, 1, [], [])
    plain = make_cache(lib, devbuf, ms, nkv, hd, 1, [], [])
    for turn, (lcp, suffix, hist) in enumerate(_turns(20 + nh, 8)):
        n = len(suffix)
        ks, vs = zip(*[token_kv(t, lcp + j, layer, kvd) for j, t in enumerate(suffix)])
        ks, vs = np.stack(ks), np.stack(vs)
        q = O.normal(n * nh * hd, 700 + turn).reshape(n, nh, hd)
        kd, vd, qd = devbuf(ks), devbuf(vs), devbuf(q)
        of, op = devbuf(nbytes=q.nbytes), devbuf(nbytes=q.nbytes)
        # the fused call on one cache ...
        tgkv.check(lib.tg_kv_truncate(fused, lcp), lib)
        tgkv.check(lib.tg_kv_append_attention(fused, kd.ptr, vd.ptr, qd.ptr, of.ptr, nh, n,
                                              None), lib)
        assert lib.tg_cuda_kv_attn_last_kernel() == 2          # the tensor-core suffix kernel
        assert lib.tg_cuda_kv_attn_last_launches() == 1
        assert lib.tg_kv_len(fused) == len(hist)
        monkeypatch.setenv("TGKV_FUSE_SUFFIX", "0")            # the reference side: two launches
        # ... and the append kernel + the attention on the other
        tgkv.check(lib.tg_kv_truncate(plain, lcp), lib)
        tgkv.check(lib.tg_kv_append_dev(plain, kd.ptr, vd.ptr, n, None), lib)
        tgkv.check(lib.tg_kv_attention(plain, qd.ptr, op.ptr, nh, n, None), lib)
        assert lib.tg_cuda_kv_sync(None)
        rf = cache_rows(lib, fused, 1, ms, kvd)
        rp = cache_rows(lib, plain, 1, ms, kvd)
        assert np.array_equal(rf[:, :len(hist)], rp[:, :len(hist)]), turn
        # every row of the history is the token's K/V, rounded once
        hk, hv = zip(*[token_kv(t, j, layer, kvd) for j, t in enumerate(hist)])
        assert np.array_equal(rf[0, :len(hist)], O.f32_to_bf16(np.stack(hk))), turn
        assert np.array_equal(rf[1, :len(hist)], O.f32_to_bf16(np.stack(hv))), turn
        got = of.get(np.float32, q.shape)
        eng = O.attention_engine(q, O.bf16_to_f32(rf), nh, nkv, hd, n, len(hist) - n,
                                 len(hist), ms)
        assert rel_head_err(got, eng) < TC_TOL, turn
        assert rel_head_err(got, op.get(np.float32, q.shape)) < TC_TOL, turn
        monkeypatch.setenv("TGKV_FUSE_SUFFIX", fuse)
    assert lib.tg_cuda_kv_device_error() == 0
    lib.tg_kv_destroy(fused)
    lib.tg_kv_destroy(plain)


@pytest.mark.parametrize("dtype,nh,nkv,hd,n", [
    (0, 16, 4, 128, 200),       # fp32 cache: not the suffix kernel
    (1, 16, 4, 128, 20),        # 80 (row, head) pairs: below the suffix kernel's 128
    (1, 8, 2, 64, 150),         # head_dim 64
])
def test_other_geometries_take_two_launches(cuda, devbuf, dtype, nh, nkv, hd, n):
    lib = cuda
    kvd, ms, L0 = nkv * hd, 1024, 300
    k0 = O.normal(L0 * kvd, 51, 2).reshape(L0, kvd)
    v0 = O.normal(L0 * kvd, 51, 3).reshape(L0, kvd)
    c = make_cache(lib, devbuf, ms, nkv, hd, dtype, k0, v0)
    ks = O.normal(n * kvd, 52, 2).reshape(n, kvd)
    vs = O.normal(n * kvd, 52, 3).reshape(n, kvd)
    q = O.normal(n * nh * hd, 53, 1).reshape(n, nh, hd)
    kd, vd, qd, od = devbuf(ks), devbuf(vs), devbuf(q), devbuf(nbytes=q.nbytes)
    tgkv.check(lib.tg_kv_append_attention(c, kd.ptr, vd.ptr, qd.ptr, od.ptr, nh, n, None), lib)
    assert lib.tg_cuda_kv_sync(None)
    assert lib.tg_kv_len(c) == L0 + n
    rows = cache_rows(lib, c, dtype, ms, kvd)
    want_k = np.concatenate([k0, ks])
    want_v = np.concatenate([v0, vs])
    if dtype == 1:
        assert np.array_equal(rows[0, :L0 + n], O.f32_to_bf16(want_k))
        assert np.array_equal(rows[1, :L0 + n], O.f32_to_bf16(want_v))
        kvc = O.bf16_to_f32(rows)
    else:
        assert np.array_equal(rows[0, :L0 + n].view(np.uint32), want_k.view(np.uint32))
        assert np.array_equal(rows[1, :L0 + n].view(np.uint32), want_v.view(np.uint32))
        kvc = rows
    eng = O.attention_engine(q, kvc, nh, nkv, hd, n, L0, L0 + n, ms)
    assert rel_head_err(od.get(np.float32, q.shape), eng) < TC_TOL
    lib.tg_kv_destroy(c)


def test_fused_call_rejects_before_launching(cuda, devbuf):
    lib = cuda
    c = make_cache(lib, devbuf, 256, 4, 128, 1, [], [])
    b = devbuf(nbytes=1 << 20)
    assert lib.tg_kv_append_attention(c, b.ptr, b.ptr, b.ptr, b.ptr, 16, 257, None) == 0
    assert b"capacity" in lib.tg_kv_last_error()
    assert lib.tg_kv_append_attention(c, b.ptr, b.ptr, b.ptr, b.ptr, 6, 10, None) == 0
    assert lib.tg_kv_append_attention(c, b.ptr, b.ptr, b.ptr, b.ptr, 16, 0, None) == 0
    assert lib.tg_kv_len(c) == 0
    lib.tg_kv_destroy(c)
