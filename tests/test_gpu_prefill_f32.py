"""The fp32 block kernel (tgkv_prefill_f32.cu) against the oracle.

Blocks of at least 32 (query row, head) pairs over one fp32 cache -- the
whole-model forward's prefill, whose caches are fp32 like the engine's -- run
on a CUDA-core kernel that stages a row block of up to 64 query vectors and
deals its K/V tiles (up to the block's causal limit) to splits that one CTA
each streams, the last split to finish merging them.  Checked against the engine-order
oracle (src/tgai_engine.c:3943-4011 semantics) at the split-sequence kernel's
fp32 bar, for every group size and head_dim the kernel takes, row counts that
are not multiples of a block's rows, one split and many, a fresh prefill from
position 0, a continuation far into the context, stale rows past the length,
and against the split-sequence kernel (TGKV_PREFILL=0) on the same call.
"""
import numpy as np
import pytest

import oracle as O
import tgkv
from conftest import rel_head_err
from test_gpu_parity import attend, host_cache, make_cache, synth_qkv

pytestmark = pytest.mark.gpu

SPLIT, BLOCK32 = 1, 4          # tg_cuda_kv_attn_last_kernel() families
F32_TOL = 1e-5                 # the fp32 split-sequence kernel's bar


@pytest.mark.parametrize("hd,nh,nkv,L,nq", [
    (128, 12, 4, 600, 512),     # the V2.7-shaped forward's prefill (G = 3), after 88 kept
    (128, 12, 4, 512, 512),     # a fresh prefill from position 0
    (128, 16, 4, 300, 64),      # G = 4
    (64, 8, 8, 100, 37),        # G = 1, rows not a multiple of the CTA's 32
    (32, 16, 2, 1000, 40),      # G = 8: 4 rows a CTA
    (128, 8, 4, 2048, 33),      # G = 2, far into the context, a last block of one row
    (32, 16, 2, 40, 40),        # two tiles in all: one split, rows written directly
])
def test_block_matches_oracle(cuda, devbuf, hd, nh, nkv, L, nq):
    lib = cuda
    q, k, v = synth_qkv(7000 + hd + nh + L + nq, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 0, k, v)
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == BLOCK32
    kvc = host_cache(lib, c, 0, L, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L)
    assert rel_head_err(got, eng) < F32_TOL
    assert lib.tg_cuda_kv_device_error() == 0
    lib.tg_kv_destroy(c)


def test_block_equals_split_sequence_kernel(cuda, devbuf, monkeypatch):
    """The same call on both kernels (TGKV_PREFILL=0 keeps the split one)."""
    lib = cuda
    nh, nkv, hd, L, nq = 12, 4, 128, 700, 300
    q, k, v = synth_qkv(4242, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 0, k, v)
    a = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == BLOCK32
    monkeypatch.setenv("TGKV_PREFILL", "0")
    b = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == SPLIT
    assert rel_head_err(a, b) < F32_TOL
    lib.tg_kv_destroy(c)


def test_block_ignores_stale_rows_after_truncate(cuda, devbuf):
    """Rows past the length may hold infinities and NaN; the block kernel's
    tiles zero them instead of reading them."""
    lib = cuda
    nh, nkv, hd, L, nq = 12, 4, 128, 450, 200
    kvd = nkv * hd
    q, k, v = synth_qkv(1357, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L + 300, nkv, hd, 0, k, v)
    junk_k = np.full((300, kvd), np.inf, np.float32)
    junk_v = np.full((300, kvd), -np.inf, np.float32)
    junk_v[::3] = np.nan
    kd, vd = devbuf(junk_k), devbuf(junk_v)
    tgkv.check(lib.tg_kv_append_dev(c, kd.ptr, vd.ptr, 300, None), lib)
    tgkv.check(lib.tg_kv_truncate(c, L), lib)
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == BLOCK32
    assert np.isfinite(got).all()
    kvc = host_cache(lib, c, 0, L + 300, kvd)
    kvc[:, L:] = 0.0
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L + 300)
    assert rel_head_err(got, eng) < F32_TOL
    lib.tg_kv_destroy(c)


def test_small_blocks_stay_on_split_kernel(cuda, devbuf):
    """Fewer than 32 (row, head) pairs: the split-sequence kernel."""
    lib = cuda
    nh, nkv, hd, L, nq = 8, 2, 64, 200, 7          # 28 pairs
    q, k, v = synth_qkv(99, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 0, k, v)
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert lib.tg_cuda_kv_attn_last_kernel() == SPLIT
    kvc = host_cache(lib, c, 0, L, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L)
    assert rel_head_err(got, eng) < F32_TOL
    lib.tg_kv_destroy(c)
