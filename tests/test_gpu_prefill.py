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
from conftest import rel_head_err
from test_gpu_parity import attend, host_cache, make_cache, synth_qkv

pytestmark = pytest.mark.gpu


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
    kvc = host_cache(lib, c, 1, L + 7, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L + 7)
    err = rel_head_err(got, eng)
    assert err < 1e-2          # the bf16-cache tolerance
    assert err < 1e-5          # q and P split into bf16 hi + lo keep it near fp32
    assert lib.tg_cuda_kv_device_error() == 0
    lib.tg_kv_destroy(c)


def test_prefill_equals_split_sequence_kernel(cuda, devbuf, monkeypatch):
    lib = cuda
    nh, nkv, hd, nq, L = 16, 4, 128, 300, 2100
    q, k, v = synth_qkv(777, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 1, k, v)
    tc = attend(lib, devbuf, c, q[-nq:], nh, nq)
    monkeypatch.setenv("TGKV_PREFILL", "0")
    cc = attend(lib, devbuf, c, q[-nq:], nh, nq)
    assert rel_head_err(tc, cc) < 1e-5
    lib.tg_kv_destroy(c)


def test_prefill_with_temperature(cuda, devbuf):
    lib = cuda
    nh, nkv, hd, nq, L = 16, 4, 128, 64, 700
    q, k, v = synth_qkv(4321, L, nh, nkv, hd)
    c = make_cache(lib, devbuf, L, nkv, hd, 1, k, v)
    lib.tg_kv_set_attn_mscale(c, C.c_float(1.25))
    got = attend(lib, devbuf, c, q[-nq:], nh, nq)
    kvc = host_cache(lib, c, 1, L, nkv * hd)
    eng = O.attention_engine(q[-nq:], kvc, nh, nkv, hd, nq, L - nq, L, L, mscale=1.25)
    assert rel_head_err(got, eng) < 1e-5
    lib.tg_kv_destroy(c)
