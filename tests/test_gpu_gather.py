"""Decode attention with the output gather over NVLink (tg_kv_batch_decode_gather).

With the KV heads of one long context split over the GPUs of a node, the
attention kernel stores every finished output element into every rank's
gathered buffer (peer memory) and counts arrivals there; the stream then waits
for all ranks.  One rank (world 1) runs the same kernel path on one GPU; the
two-rank test needs two GPUs and is skipped otherwise.
"""
import ctypes as C
import os

import numpy as np
import pytest

import oracle as O
import tgkv
from conftest import rel_head_err
from test_gpu_parity import host_cache, synth_qkv

pytestmark = pytest.mark.gpu


def _plan(lib, devbuf, n_seq, L, nkv, hd, nh, seed):
    """n_seq bf16 caches holding L-1 rows, and a batch plan over them."""
    caches, rows = [], []
    for i in range(n_seq):
        q, k, v = synth_qkv(seed + i, L, nh, nkv, hd)
        c = lib.tg_kv_create_ex(L + 8, nkv, hd, 1)
        tgkv.check(c, lib)
        kd, vd = devbuf(np.ascontiguousarray(k[:L - 1])), devbuf(np.ascontiguousarray(v[:L - 1]))
        tgkv.check(lib.tg_kv_append_dev(c, kd.ptr, vd.ptr, L - 1, None), lib)
        caches.append(c)
        rows.append((q[L - 1], k[L - 1], v[L - 1]))
    arr = (C.c_void_p * n_seq)(*caches)
    b = lib.tg_kv_batch_create(arr, n_seq, nh)
    tgkv.check(b, lib)
    return caches, b, rows


@pytest.mark.parametrize("kernel", ["auto", "tc"])
def test_single_rank_gather_equals_plain_decode(cuda, devbuf, monkeypatch, kernel):
    lib = cuda
    if kernel == "tc":                       # the tensor-core decode kernel's gather stores
        monkeypatch.setenv("TGKV_DECODE_TC", "1")
    n_seq, L, nkv, hd, nh = 3, 2500, 4, 128, 16
    caches, b, rows = _plan(lib, devbuf, n_seq, L, nkv, hd, nh, 6100)
    elems = n_seq * nh * hd
    g = lib.tg_kv_gather_create(1, 0, elems)
    tgkv.check(g, lib)
    q = devbuf(np.stack([r[0] for r in rows]).astype(np.float32))
    kn = devbuf(np.stack([r[1] for r in rows]).astype(np.float32))
    vn = devbuf(np.stack([r[2] for r in rows]).astype(np.float32))
    out = devbuf(nbytes=elems * 4)
    for step in range(3):                       # arrivals accumulate across steps
        tgkv.check(lib.tg_kv_batch_decode_gather(b, q.ptr, kn.ptr, vn.ptr, out.ptr, g, None), lib)
        assert lib.tg_kv_batch_last_launches(b) == 2      # attention + the wait
    assert lib.tg_cuda_kv_sync(None)
    assert lib.tg_cuda_kv_device_error() == 0
    got = out.get(np.float32, (n_seq, nh, hd))
    gath = np.zeros(elems, np.float32)
    assert lib.tg_cuda_kv_d2h(gath.ctypes.data, lib.tg_kv_gather_buffer(g), elems * 4, None)
    assert np.array_equal(gath.view(np.uint32), got.ravel().view(np.uint32))
    for i, c in enumerate(caches):
        Lc = lib.tg_kv_len(c)
        kvc = host_cache(lib, c, 1, L + 8, nkv * hd)
        eng = O.attention_engine(rows[i][0], kvc, nh, nkv, hd, 1, Lc - 1, Lc, L + 8)
        assert rel_head_err(got[i], eng[0]) < 1e-5
    lib.tg_kv_gather_destroy(g)
    lib.tg_kv_batch_destroy(b)
    for c in caches:
        lib.tg_kv_destroy(c)


def test_gather_rejects_mismatched_shape(cuda, devbuf):
    lib = cuda
    caches, b, rows = _plan(lib, devbuf, 2, 300, 2, 64, 8, 6200)
    g = lib.tg_kv_gather_create(1, 0, 123)
    q = devbuf(nbytes=2 * 8 * 64 * 4)
    assert lib.tg_kv_batch_decode_gather(b, q.ptr, q.ptr, q.ptr, q.ptr, g, None) == 0
    assert b"gather" in lib.tg_kv_last_error()
    assert not lib.tg_kv_gather_create(9, 0, 10)
    assert not lib.tg_kv_gather_create(2, 2, 10)
    lib.tg_kv_gather_destroy(g)
    lib.tg_kv_batch_destroy(b)
    for c in caches:
        lib.tg_kv_destroy(c)


def _rank_main(rank, world, port, result_dir):
    """One rank: its KV-head group of a shared synthetic context, decode with
    the gather, then the gathered outputs of all heads against the oracle."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.join(here, "..", "oracle"), os.path.join(here, "..", "tgai-go_b200")]
    import torch.distributed as dist
    import oracle as O
    import shard
    import tgkv
    from conftest import rel_head_err
    from test_gpu_parity import synth_qkv
    lib = tgkv.load()
    tgkv.check(lib.tg_cuda_kv_set_device(rank), lib)
    tgkv.check(lib.tg_be_select(b"cuda"), lib)
    import datetime
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    nh, nkv, hd, L = 16, 4, 128, 3000
    kv0, kv1, q0, q1 = shard.kv_head_shard(nh, nkv, world, rank)
    q, k, v = synth_qkv(7100, L, nh, nkv, hd)               # the full model's tensors
    kl = np.ascontiguousarray(k.reshape(L, nkv, hd)[:, kv0:kv1].reshape(L, -1))
    vl = np.ascontiguousarray(v.reshape(L, nkv, hd)[:, kv0:kv1].reshape(L, -1))
    ql = np.ascontiguousarray(q[L - 1, q0:q1])
    nkl, nhl = kv1 - kv0, q1 - q0
    c = lib.tg_kv_create_ex(L + 8, nkl, hd, 1)
    tgkv.check(c, lib)

    def dev(a):
        p = lib.tg_cuda_kv_malloc(a.nbytes)
        assert p and lib.tg_cuda_kv_h2d(p, a.ctypes.data, a.nbytes, None)
        return p
    kd, vd = dev(kl[:L - 1]), dev(vl[:L - 1])
    tgkv.check(lib.tg_kv_append_dev(c, kd, vd, L - 1, None), lib)
    b = lib.tg_kv_batch_create((C.c_void_p * 1)(c), 1, nhl)
    tgkv.check(b, lib)
    elems = nhl * hd
    g = lib.tg_kv_gather_create(world, rank, elems)
    tgkv.check(g, lib)
    h = (C.c_uint8 * 64)()
    tgkv.check(lib.tg_kv_gather_export(g, h), lib)
    allh = [None] * world
    dist.all_gather_object(allh, bytes(h))
    tgkv.check(lib.tg_kv_gather_import(g, b"".join(allh)), lib)
    qd, knd, vnd = dev(ql), dev(np.ascontiguousarray(kl[L - 1:L])), dev(np.ascontiguousarray(vl[L - 1:L]))
    out = lib.tg_cuda_kv_malloc(elems * 4)
    tgkv.check(lib.tg_kv_batch_decode_gather(b, qd, knd, vnd, out, g, None), lib)
    assert lib.tg_cuda_kv_sync(None)
    err = lib.tg_cuda_kv_device_error()
    gath = np.zeros(world * elems, np.float32)
    assert lib.tg_cuda_kv_d2h(gath.ctypes.data, lib.tg_kv_gather_buffer(g), gath.nbytes, None)
    # every head of the full model, in rank order = head order
    kvc = np.zeros((2, L, nkv * hd), np.float32)
    kvc[0] = O.bf16_to_f32(O.f32_to_bf16(k))
    kvc[1] = O.bf16_to_f32(O.f32_to_bf16(v))
    eng = O.attention_engine(q[L - 1:L], kvc, nh, nkv, hd, 1, L - 1, L, L)[0]
    e = rel_head_err(gath.reshape(nh, hd), eng)
    dist.barrier()
    lib.tg_kv_gather_destroy(g)
    lib.tg_kv_batch_destroy(b)
    lib.tg_kv_destroy(c)
    dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{e} {err}\n")


@pytest.mark.parametrize("kernel", ["auto", "tc"])
def test_two_rank_gather_over_nvlink(tmp_path, monkeypatch, kernel):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if kernel == "tc":                       # inherited by the spawned ranks
        monkeypatch.setenv("TGKV_DECODE_TC", "1")
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        e, err = open(tmp_path / f"rank{r}.txt").read().split()
        assert int(err) == 0
        assert float(e) < 1e-5, (r, e)
