"""tg_kv_attention_static -- attention for callers that cannot allocate.

Some callers may not call cudaMalloc when they need attention. Examples are code
running inside a host allocator hook, a decode thread under a fixed
device-memory budget, and an engine that owns every buffer and hands over only
raw addresses. For them the library offers one entry point whose scratch is a
static device array inside the library. These tests check it through the C-ABI
against the engine-order CPU oracle (on the cache bytes as stored, so bf16
caches are decoded first) and against tg_kv_attention, the allocating entry
point, on the same cache and queries. Each case makes two calls in a row,
because the second call finds the first call's scratch contents still there.
The tolerance is the one the parity tests use.

The kernel's waits are bounded. A failure-injection hook holds back the loads
of one call, so that its waits run out; the tests check that the code reaches
tg_kv_attention_static_error, that a later call does not wipe it before it is
read, and that the next call after the read is correct again.

This file sorts last, so a run that stops at the first failure has already run
every other test.
"""
import numpy as np
import pytest

import oracle as O
import tgkv
from conftest import rel_head_err

pytestmark = pytest.mark.gpu


def _cache_with_rows(lib, devbuf, max_seq, nkv, hd, dtype, L, seed):
    kvd = nkv * hd
    k = O.normal(L * kvd, seed, 2).reshape(L, kvd)
    v = O.normal(L * kvd, seed, 3).reshape(L, kvd)
    c = lib.tg_kv_create_ex(max_seq, nkv, hd, dtype)
    tgkv.check(c, lib)
    kd, vd = devbuf(k), devbuf(v)
    tgkv.check(lib.tg_kv_append_dev(c, kd.ptr, vd.ptr, L, None), lib)
    assert lib.tg_cuda_kv_sync(None)
    return c


def _cache_as_f32(lib, c, dtype, max_seq, kvd):
    """The cache bytes as the GPU holds them, as fp32 (bf16 decoded)."""
    raw = np.empty(lib.tg_kv_bytes(c), np.uint8)
    assert lib.tg_kv_download(c, raw.ctypes.data)
    if dtype == 1:
        return O.bf16_to_f32(raw.view(np.uint16).reshape(2, max_seq, kvd))
    return raw.view(np.float32).reshape(2, max_seq, kvd)


@pytest.mark.parametrize("dtype,nh,nkv,hd,L,nq,max_seq", [
    (1, 32, 8, 128, 20000, 1, 20480),     # long context: many chunks, in-kernel combine
    (1, 16, 4, 128, 4096, 3, 4096),       # cfg2 shape, causal block of 3
    (0, 8, 2, 64, 300, 5, 320),           # fp32 cache, single chunk per row
    (0, 6, 6, 32, 1000, 16, 1024),        # head_dim 32, MHA, 16 query rows
])
def test_static_matches_oracle_and_allocating_entry(cuda, devbuf, dtype, nh, nkv, hd, L, nq,
                                                    max_seq):
    lib = cuda
    assert lib.tg_kv_attention_static_error(None) == 0
    c = _cache_with_rows(lib, devbuf, max_seq, nkv, hd, dtype, L, 4242 + L)
    q = O.normal(nq * nh * hd, 99 + L, 1).reshape(nq, nh, hd)
    qd = devbuf(q)
    ref_d = devbuf(nbytes=q.nbytes)
    tgkv.check(lib.tg_kv_attention(c, qd.ptr, ref_d.ptr, nh, nq, None), lib)
    assert lib.tg_cuda_kv_sync(None)
    alloc = ref_d.get(np.float32, q.shape)
    kvc_f32 = _cache_as_f32(lib, c, dtype, max_seq, nkv * hd)
    eng = O.attention_engine(q, kvc_f32, nh, nkv, hd, nq, L - nq, L, max_seq)
    kvc = lib.tg_kv_device_handle(c)
    for call in range(2):                  # two calls in a row share the static scratch
        out_d = devbuf(nbytes=q.nbytes)
        ok = lib.tg_kv_attention_static(kvc, dtype, max_seq, nkv, hd, L, qd.ptr, out_d.ptr,
                                        nh, nq, None)
        assert ok, lib.tg_kv_last_error().decode()
        assert lib.tg_kv_attention_static_error(None) == 0
        got = out_d.get(np.float32, q.shape)
        # the oracle, on the cache as stored: the split-sequence kernel's bar
        assert rel_head_err(got, eng) < 1e-5, call
        # the allocating entry runs the same kernel over the same plan
        assert rel_head_err(got, alloc) < 1e-5, call
    assert lib.tg_cuda_kv_device_error() == 0
    lib.tg_kv_destroy(c)


def test_static_on_caller_owned_buffer(cuda, devbuf):
    """The cache buffer does not have to come from tg_kv_create: a raw device
    buffer in the [2][max_seq][kv_dim] layout works the same way."""
    lib = cuda
    nh, nkv, hd, L, ms = 8, 2, 64, 777, 800
    kvc = np.zeros((2, ms, nkv * hd), np.float32)
    kvc[:, :L] = O.normal(2 * L * nkv * hd, 5150, 4).reshape(2, L, nkv * hd)
    kb = devbuf(kvc)
    q = O.normal(nh * hd, 5151, 1).reshape(1, nh, hd)
    qd, od = devbuf(q), devbuf(nbytes=q.nbytes)
    eng = O.attention_engine(q, kvc, nh, nkv, hd, 1, L - 1, L, ms)
    for _ in range(2):
        assert lib.tg_kv_attention_static(kb.ptr, 0, ms, nkv, hd, L, qd.ptr, od.ptr, nh, 1,
                                          None), lib.tg_kv_last_error().decode()
        assert lib.tg_kv_attention_static_error(None) == 0
        got = od.get(np.float32, q.shape)
        assert rel_head_err(got, eng) < 1e-5


def test_static_wait_timeout_is_reported(cuda, devbuf):
    """A call whose K/V loads are held back (failure injection; nothing is in
    flight) waits out its bound of about 2 s. Its code stays in the error word
    through a later good call, is returned once by the reader, and the calls
    after that are correct again."""
    lib = cuda
    nh, nkv, hd, L, ms = 8, 2, 64, 500, 512      # 1 query row: a handful of CTAs, one wave
    kvc = np.zeros((2, ms, nkv * hd), np.float32)
    kvc[:, :L] = O.normal(2 * L * nkv * hd, 6160, 4).reshape(2, L, nkv * hd)
    kb = devbuf(kvc)
    q = O.normal(nh * hd, 6161, 1).reshape(1, nh, hd)
    qd, od = devbuf(q), devbuf(nbytes=q.nbytes)
    eng = O.attention_engine(q, kvc, nh, nkv, hd, 1, L - 1, L, ms)

    def call():
        assert lib.tg_kv_attention_static(kb.ptr, 0, ms, nkv, hd, L, qd.ptr, od.ptr, nh, 1,
                                          None), lib.tg_kv_last_error().decode()

    assert lib.tg_kv_attention_static_error(None) == 0
    lib.tg_kv_attention_static_inject_stall(1)
    call()                                       # its waits run out
    call()                                       # a good call does not clear the code
    assert lib.tg_cuda_kv_sync(None)
    assert rel_head_err(od.get(np.float32, q.shape), eng) < 1e-5
    code = lib.tg_kv_attention_static_error(None)
    assert code == 1, code                       # a K/V stage never arrived
    assert lib.tg_kv_attention_static_error(None) == 0      # cleared once returned
    for _ in range(2):
        call()
        assert lib.tg_kv_attention_static_error(None) == 0
        assert rel_head_err(od.get(np.float32, q.shape), eng) < 1e-5
    # the library's own error word is separate and untouched
    assert lib.tg_cuda_kv_device_error() == 0


def test_static_rejects_beyond_limit(cuda, devbuf):
    """Scratch beyond the static 4 MiB is refused before anything is launched.
    The split partials stay below 2.2 MiB (at most two per CTA of one
    persistent wave), so the case that overflows is the arrival counters of
    very many (query row, KV head) pairs: 1024 rows x 1024 KV heads."""
    lib = cuda
    nh = nkv = 1024
    hd, L = 32, 1024
    c = lib.tg_kv_create_ex(L, nkv, hd, 0)
    tgkv.check(c, lib)
    q = devbuf(nbytes=4096)
    kvc = lib.tg_kv_device_handle(c)
    assert lib.tg_kv_attention_static(kvc, 0, L, nkv, hd, L, q.ptr, q.ptr, nh, 1024, None) == 0
    msg = lib.tg_kv_last_error()
    assert b"4 MiB" in msg and b"bytes of scratch" in msg, msg
    assert lib.tg_kv_attention_static(kvc, 0, L, nkv, hd, L, q.ptr, q.ptr, nh, 1025, None) == 0
    assert b"1024" in lib.tg_kv_last_error()
    assert lib.tg_kv_attention_static(kvc, 0, L, nkv, hd, L + 1, q.ptr, q.ptr, nh, 1, None) == 0
    lib.tg_kv_destroy(c)
