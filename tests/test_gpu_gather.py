"""Decode attention with the output gather over NVLink (tg_kv_batch_decode_gather).

With the KV heads of one long context split over the GPUs of a node, the
attention kernel stores every finished output element into every rank's
gathered buffer (peer memory) and counts arrivals there; the stream then waits
for all ranks.  One rank (world 1) runs the same kernel path on one GPU; the
two-rank tests need two GPUs and are skipped otherwise.  One of them reuses a
single gather object for 128 calls with a slow consumer on one rank: a gather
object alternates between two buffers, so a call's outputs stay intact until
the call after next whatever the other rank does meanwhile.
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


@pytest.mark.parametrize("pinned", [True, False])
def test_single_rank_gather_from_host_buffers(cuda, devbuf, pinned):
    """tg_kv_batch_decode_gather_host on one rank: inputs from page-locked
    memory go up through the staging kernel, from pageable memory through
    copies; the gathered rows come back to out_host; five calls in a row on
    one gather object, each against the oracle."""
    import torch
    lib = cuda
    n_seq, L, nkv, hd, nh = 2, 1800, 4, 128, 16
    caches, b, rows = _plan(lib, devbuf, n_seq, L, nkv, hd, nh, 6300)
    elems = n_seq * nh * hd
    g = lib.tg_kv_gather_create(1, 0, elems)
    tgkv.check(g, lib)
    alloc = (lambda *s: torch.empty(*s).pin_memory()) if pinned else (lambda *s: torch.empty(*s))
    qh, kh, vh = alloc(n_seq, nh, hd), alloc(n_seq, nkv * hd), alloc(n_seq, nkv * hd)
    oh = alloc(elems)
    for step in range(5):
        q = O.normal(n_seq * nh * hd, 6400 + step, 1).reshape(n_seq, nh, hd)
        kn = O.normal(n_seq * nkv * hd, 6400 + step, 2).reshape(n_seq, nkv * hd)
        vn = O.normal(n_seq * nkv * hd, 6400 + step, 3).reshape(n_seq, nkv * hd)
        qh.numpy()[:] = q
        kh.numpy()[:] = kn
        vh.numpy()[:] = vn
        tgkv.check(lib.tg_kv_batch_decode_gather_host(b, qh.data_ptr(), kh.data_ptr(),
                                                      vh.data_ptr(), oh.data_ptr(), g, None), lib)
        assert lib.tg_cuda_kv_sync(None)
        got = oh.numpy().reshape(n_seq, nh, hd).copy()
        for i, c in enumerate(caches):
            Lc = lib.tg_kv_len(c)
            kvc = host_cache(lib, c, 1, L + 8, nkv * hd)
            eng = O.attention_engine(q[i:i + 1], kvc, nh, nkv, hd, 1, Lc - 1, Lc, L + 8)
            assert rel_head_err(got[i], eng[0]) < 1e-5, (step, i)
    assert lib.tg_cuda_kv_device_error() == 0
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


def _rank_reuse_main(rank, world, port, result_dir, n_dev_calls, n_host_calls):
    """One rank of a two-layer model decoding over ONE gather object for every
    layer and step.  Rank 1 is a slow consumer: in the first phase it holds
    its stream in a sleep kernel before copying each call's gathered outputs
    out, in the second it sleeps on the host between host-buffer calls.  Every
    call's gathered outputs (all heads) are checked against the oracle."""
    import sys
    import time
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [here, os.path.join(here, "..", "oracle"), os.path.join(here, "..", "tgai-go_b200")]
    import datetime
    import torch
    import torch.distributed as dist
    import oracle as O
    import shard
    import tgkv
    from conftest import rel_head_err
    torch.cuda.set_device(rank)
    lib = tgkv.load()
    tgkv.check(lib.tg_cuda_kv_set_device(rank), lib)
    tgkv.check(lib.tg_be_select(b"cuda"), lib)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=120))
    nh, nkv, hd, layers = 16, 4, 128, 2
    L0 = [700, 1300]
    n_seq = len(L0)
    n_calls = n_dev_calls + n_host_calls
    steps = (n_calls + layers - 1) // layers
    ms = max(L0) + steps + 8
    kv0, kv1, q0, q1 = shard.kv_head_shard(nh, nkv, world, rank)
    nkl, nhl = kv1 - kv0, q1 - q0
    kvd, kvdl = nkv * hd, nkl * hd

    def dev(a):
        a = np.ascontiguousarray(a, np.float32)
        p = lib.tg_cuda_kv_malloc(a.nbytes)
        assert p and lib.tg_cuda_kv_h2d(p, a.ctypes.data, a.nbytes, None)
        return p

    # the full model's K/V history per (layer, sequence), bf16-rounded, as the oracle sees it
    full = [[np.zeros((2, ms, kvd), np.float32) for _ in range(n_seq)] for _ in range(layers)]
    plans, caches = [], []
    for l in range(layers):
        row = []
        for i in range(n_seq):
            k = O.normal(L0[i] * kvd, 8100 + l, i, 2).reshape(L0[i], kvd)
            v = O.normal(L0[i] * kvd, 8100 + l, i, 3).reshape(L0[i], kvd)
            full[l][i][0, :L0[i]] = O.bf16_to_f32(O.f32_to_bf16(k))
            full[l][i][1, :L0[i]] = O.bf16_to_f32(O.f32_to_bf16(v))
            c = lib.tg_kv_create_ex(ms, nkl, hd, 1)
            tgkv.check(c, lib)
            kd = dev(k.reshape(L0[i], nkv, hd)[:, kv0:kv1].reshape(L0[i], kvdl))
            vd = dev(v.reshape(L0[i], nkv, hd)[:, kv0:kv1].reshape(L0[i], kvdl))
            tgkv.check(lib.tg_kv_append_dev(c, kd, vd, L0[i], None), lib)
            row.append(c)
        caches.append(row)
        b = lib.tg_kv_batch_create((C.c_void_p * n_seq)(*row), n_seq, nhl)
        tgkv.check(b, lib)
        plans.append(b)
    elems = n_seq * nhl * hd
    g = lib.tg_kv_gather_create(world, rank, elems)
    tgkv.check(g, lib)
    h = (C.c_uint8 * 64)()
    tgkv.check(lib.tg_kv_gather_export(g, h), lib)
    allh = [None] * world
    dist.all_gather_object(allh, bytes(h))
    tgkv.check(lib.tg_kv_gather_import(g, b"".join(allh)), lib)
    assert lib.tg_cuda_kv_sync(None)
    dist.barrier()

    qd, kd, vd = (lib.tg_cuda_kv_malloc(n_seq * nhl * hd * 4), lib.tg_cuda_kv_malloc(n_seq * kvdl * 4),
                  lib.tg_cuda_kv_malloc(n_seq * kvdl * 4))
    out = lib.tg_cuda_kv_malloc(elems * 4)
    qh = torch.empty(n_seq, nhl, hd).pin_memory()
    kh = torch.empty(n_seq, kvdl).pin_memory()
    vh = torch.empty(n_seq, kvdl).pin_memory()
    oh = torch.empty(world * elems).pin_memory()
    worst, n_checked = 0.0, 0
    for n in range(n_calls):
        l, s = n % layers, n // layers
        qf = O.normal(n_seq * nh * hd, 8200 + l, s, 1).reshape(n_seq, nh, hd)
        kf = O.normal(n_seq * kvd, 8200 + l, s, 2).reshape(n_seq, kvd)
        vf = O.normal(n_seq * kvd, 8200 + l, s, 3).reshape(n_seq, kvd)
        ql = np.ascontiguousarray(qf[:, q0:q1])
        kl = np.ascontiguousarray(kf.reshape(n_seq, nkv, hd)[:, kv0:kv1].reshape(n_seq, kvdl))
        vl = np.ascontiguousarray(vf.reshape(n_seq, nkv, hd)[:, kv0:kv1].reshape(n_seq, kvdl))
        gath = np.zeros(world * elems, np.float32)
        if n < n_dev_calls:
            for buf, a in ((qd, ql), (kd, kl), (vd, vl)):
                assert lib.tg_cuda_kv_h2d(buf, a.ctypes.data, a.nbytes, None)
            tgkv.check(lib.tg_kv_batch_decode_gather(plans[l], qd, kd, vd, out, g, None), lib)
            if rank == 1:
                torch.cuda._sleep(400000)         # a slow consumer holds its stream
            assert lib.tg_cuda_kv_d2h(gath.ctypes.data, lib.tg_kv_gather_buffer(g),
                                      gath.nbytes, None)
        else:
            qh.numpy()[:] = ql
            kh.numpy()[:] = kl
            vh.numpy()[:] = vl
            tgkv.check(lib.tg_kv_batch_decode_gather_host(plans[l], qh.data_ptr(), kh.data_ptr(),
                                                          vh.data_ptr(), oh.data_ptr(), g, None),
                       lib)
            assert lib.tg_cuda_kv_sync(None)
            gath[:] = oh.numpy()
            if rank == 1:
                time.sleep(0.003)                 # ... and is slow on the host
        got = gath.reshape(world, n_seq, nhl, hd).transpose(1, 0, 2, 3).reshape(n_seq, nh, hd)
        for i in range(n_seq):
            pos = L0[i] + s
            full[l][i][0, pos] = O.bf16_to_f32(O.f32_to_bf16(kf[i]))
            full[l][i][1, pos] = O.bf16_to_f32(O.f32_to_bf16(vf[i]))
            eng = O.attention_engine(qf[i:i + 1], full[l][i], nh, nkv, hd, 1, pos, pos + 1, ms)[0]
            worst = max(worst, rel_head_err(got[i], eng))
            n_checked += 1
    assert lib.tg_cuda_kv_sync(None)
    err = lib.tg_cuda_kv_device_error()
    dist.barrier()
    lib.tg_kv_gather_destroy(g)
    for b in plans:
        lib.tg_kv_batch_destroy(b)
    for row in caches:
        for c in row:
            lib.tg_kv_destroy(c)
    dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{worst} {err} {n_checked}\n")


def test_two_rank_gather_reused_with_slow_consumer(tmp_path):
    """One gather object over 128 calls (two layers, alternating) on two GPUs;
    rank 1 reads every call's gathered outputs late.  Each call must still
    deliver exactly its own outputs, for every head, on both ranks."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_rank_reuse_main, args=(2, port, str(tmp_path), 64, 64), nprocs=2,
                       join=True, start_method="spawn")
    for r in range(2):
        e, err, n = open(tmp_path / f"rank{r}.txt").read().split()
        assert int(err) == 0
        assert int(n) == 128 * 2
        assert float(e) < 1e-5, (r, e)
