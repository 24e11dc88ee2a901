"""The tensor-core (tcgen05) suffix attention against the oracle.

Blocks of at least 128 (query row, head) pairs over a bf16 head_dim-128 cache
run on tgkv_prefill.cu: the suffix attention of an LCP re-append.  Checked
against the engine-order oracle on the bf16-decoded cache, and against the
split-sequence kernel (TGKV_PREFILL=0), for every group size the kernel takes,
partial and multiple 128-row tiles, the causal diagonal inside and across
128-position tiles, and contexts that are not multiples of the tile.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import tgkv
from conftest import TC_TOL, rel_head_err
from test_gpu_parity import attend, host_cache, make_cache, synth_qkv

pytestmark = pytest.mark.gpu

SPLIT, TENSOR, DECODE_TC, BLOCK32 = 1, 2, 3, 4   # tg_cuda_kv_attn_last_kernel() families
BF16_TOL = 1e-2            # the bf16-cache tolerance of the path
# TC_TOL: emulating the hi + lo split exactly on the CPU gives 6.5e-6 on the
# cfg3 shape; the tensor cores' fp32 accumulation adds about as much again.


@pytest.mark.parametrize("nh,nkv,nq,L", [
    (16, 4, 32, 32),        # one tile, the whole suffix is the causal diagonal
    (16, 4, 64, 1000),      # cfg3 shape, two row tiles, context not a multiple of 128
    (16, 4, 512, 1500),     # cfg3's largest suffix: 16 row tiles per KV head
    (8, 8, 128, 300),       # G = 1: 128 tokens per tile
    (16, 8, 100, 129),      # G = 2, ragged last tile
    (32, 4, 40, 4096),      # G = 8: 16 tokens per tile, long context
    (32, 8, 33, 200),       # cfg4/5 head layout
])
def test_prefill_matches_oracle(cuda, devbuf, nh, nkv, nq, L):
    lib = cuda
    hd = 128
    q, k, v = synth_qkv(1200 + nq + L, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L + 7, nkv, hd, 1, k, v)
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_launches() == 1
    assert lib.tg_cuda_kv_attn_last_kernel() == TENSOR
    kvc = host_cache(lib, c, 1, L + 7, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L + 7)
    err = rel_head_err(got, eng)
    print(f"prefill nh={nh} nkv={nkv} nq={nq} L={L}: rel err {err:.3g}")
    assert err < BF16_TOL
    assert err < TC_TOL
    assert lib.tg_cuda_kv_device_error() == 0
    lib.tg_kv_destroy(c)


def test_prefill_equals_split_sequence_kernel(cuda, devbuf, monkeypatch):
    lib = cuda
    nh, nkv, hd, nq, L = 16, 4, 128, 300, 2100
    q, k, v = synth_qkv(777, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 1, k, v)
    tc = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == TENSOR
    monkeypatch.setenv("TGKV_PREFILL", "0")
    monkeypatch.setenv("TGKV_DECODE_TC", "0")
    cc = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == SPLIT
    assert rel_head_err(tc, cc) < TC_TOL
    lib.tg_kv_destroy(c)


def test_prefill_with_temperature(cuda, devbuf):
    lib = cuda
    nh, nkv, hd, nq, L = 16, 4, 128, 64, 700
    q, k, v = synth_qkv(4321, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 1, k, v)
    lib.tg_kv_set_attn_mscale(c, C.c_float(1.25))
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == TENSOR
    kvc = host_cache(lib, c, 1, L, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L, mscale=1.25)
    assert rel_head_err(got, eng) < TC_TOL
    lib.tg_kv_destroy(c)


@pytest.mark.parametrize("dtype,hd,nh,nkv,nq", [
    (0, 128, 16, 4, 64),     # fp32 cache
    (1, 64, 16, 4, 64),      # head_dim 64
    (1, 128, 16, 4, 16),     # 64 (row, head) pairs < 128
    (1, 128, 12, 4, 64),     # group of 3
])
def test_ineligible_calls_stay_on_split_kernel(cuda, devbuf, dtype, hd, nh, nkv, nq):
    """Not for the suffix kernel: a split-sequence kernel takes them -- the
    CUDA-core one, or for the group of 3 (64 rows x ~270 positions x 12 head
    subsets, about 206K streamed rows, above the 131072-row threshold) the
    tensor-core decode kernel -- except the fp32 cache, whose block of rows
    goes to the fp32 block kernel (tgkv_prefill_f32.cu)."""
    lib = cuda
    L = 300
    q, k, v = synth_qkv(99 + nh + hd, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, dtype, k, v)
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    want = (BLOCK32 if dtype == 0 else
            DECODE_TC if (dtype, hd, nh // nkv) == (1, 128, 3) else SPLIT)
    assert lib.tg_cuda_kv_attn_last_kernel() == want
    kvc = host_cache(lib, c, dtype, L, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L)
    assert rel_head_err(got, eng) < 1e-5
    lib.tg_kv_destroy(c)


def test_prefill_ignores_stale_rows_after_truncate(cuda, devbuf):
    """Rows past the length (a truncated turn) may hold anything, infinities
    included; the suffix attention never lets them into the output."""
    lib = cuda
    nh, nkv, hd, L, nq = 16, 4, 128, 450, 200
    kvd = nkv * hd
    q, k, v = synth_qkv(2468, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L + 300, nkv, hd, 1, k, v)
    junk_k = np.full((300, kvd), np.inf, np.float32)
    junk_v = np.full((300, kvd), -np.inf, np.float32)
    junk_v[::3] = np.nan
    kd, vd = devbuf(junk_k), devbuf(junk_v)
    tgkv.check(lib.tg_kv_append_dev(c, kd.ptr, vd.ptr, 300, None), lib)
    tgkv.check(lib.tg_kv_truncate(c, L), lib)
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == TENSOR
    assert np.isfinite(got).all()
    kvc = host_cache(lib, c, 1, L + 300, kvd)
    kvc[:, L:] = 0.0            # what the reference never reads
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L + 300)
    assert rel_head_err(got, eng) < TC_TOL
    assert lib.tg_cuda_kv_device_error() == 0
    lib.tg_kv_destroy(c)


def test_multi_turn_lcp_reuse(cuda, devbuf):
    """The chat-turn flow the suffix kernel serves: truncate to the common
    prefix, append the new suffix, attend it causally; every turn checked."""
    lib = cuda
    nh, nkv, hd = 16, 4, 128
    kvd = nkv * hd
    turns = [(0, 320), (250, 130), (370, 511), (600, 64), (100, 257)]
    ms = max(l + n for l, n in turns)
    c = lib.tg_kv_create_ex(ms, nkv, hd, 1)
    tgkv.check(c, lib)
    for i, (lcp, n) in enumerate(turns):
        tgkv.check(lib.tg_kv_truncate(c, min(lcp, lib.tg_kv_len(c))), lib)
        base = lib.tg_kv_len(c)
        q, k, v = synth_qkv(5000 + i, n, nh, nkv, hd)
        kd, vd = devbuf(np.ascontiguousarray(k)), devbuf(np.ascontiguousarray(v))
        tgkv.check(lib.tg_kv_append_dev(c, kd.ptr, vd.ptr, n, None), lib)
        got = attend(lib, devbuf, c, q, nh, n)
        assert lib.tg_cuda_kv_attn_last_kernel() == TENSOR
        L = base + n
        kvc = host_cache(lib, c, 1, ms, kvd)
        eng = O.attention_engine(q, kvc, nh, nkv, hd, n, L - n, L, ms)
        err = rel_head_err(got, eng)
        print(f"turn {i} lcp={lcp} n={n}: rel err {err:.3g}")
        assert err < TC_TOL, (i, lcp, n)
    assert lib.tg_cuda_kv_device_error() == 0
    lib.tg_kv_destroy(c)


@pytest.mark.parametrize("split", [1, 2, 3, 5, 8])
def test_kv_split_across_cluster(cuda, devbuf, monkeypatch, split):
    """The KV tiles of a row block divided among `split` CTAs of a cluster and
    merged over distributed shared memory give the oracle's result for every
    split count."""
    lib = cuda
    nh, nkv, hd, nq, L = 16, 4, 128, 200, 2000
    q, k, v = synth_qkv(8080, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 1, k, v)
    monkeypatch.setenv("TGKV_PF_SPLIT", str(split))
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == TENSOR
    assert lib.tg_cuda_kv_attn_last_split() == split
    kvc = host_cache(lib, c, 1, L, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L)
    err = rel_head_err(got, eng)
    print(f"split {split}: rel err {err:.3g}")
    assert err < TC_TOL
    assert lib.tg_cuda_kv_device_error() == 0
    lib.tg_kv_destroy(c)


def test_split_with_rows_masked_out_of_a_split(cuda, devbuf, monkeypatch):
    """G = 1, rows at positions 100..227 over two tiles split in two: the
    second CTA's tile [128, 256) holds nothing the first 28 rows may see."""
    lib = cuda
    nh = nkv = 8
    hd, nq, L = 128, 128, 228
    q, k, v = synth_qkv(9191, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 1, k, v)
    monkeypatch.setenv("TGKV_PF_SPLIT", "2")
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == TENSOR
    assert lib.tg_cuda_kv_attn_last_split() == 2
    kvc = host_cache(lib, c, 1, L, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L)
    assert rel_head_err(got, eng) < TC_TOL
    lib.tg_kv_destroy(c)


def test_split_is_planned_to_fill_the_gpu(cuda, devbuf):
    """Left to the planner, a cfg3-sized turn (300 new tokens after 900 kept)
    is split so that the launch covers most of the SMs in one wave."""
    lib = cuda
    nh, nkv, hd, nq, L = 16, 4, 128, 300, 1200
    q, k, v = synth_qkv(4242, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 1, k, v)
    attend(lib, devbuf, c, q[-nq:], nh, nq)
    ns = lib.tg_cuda_kv_attn_last_split()
    blocks = -(-nq // 32) * nkv
    assert ns > 1 and blocks * ns <= lib.tg_cuda_kv_sm_count()
    lib.tg_kv_destroy(c)
