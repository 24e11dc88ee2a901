"""The multi-rank host logic on CPU: world_size 2 over gloo.

The GPU runs shard a single long sequence by KV-head groups and all-gather the
per-head outputs (NCCL), or give whole sequences to ranks.  Here two CPU ranks
run the same partitioning with the oracle's attention in place of the kernel
and gloo in place of NCCL, and the gathered result must equal the unsharded
computation bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import sys
    for p in (os.path.join(ROOT, "tgai-go_b200"), os.path.join(ROOT, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))


def _head_sharded_rank(rank, world, port, result_dir):
    _init(rank, world, port)
    import oracle as O
    import shard
    nh, nkv, hd, L = 16, 4, 64, 333
    kvd = nkv * hd
    # the same synthetic cache and query on every rank
    kvc = O.normal(2 * L * kvd, 77, 1).reshape(2, L, kvd)
    q = O.normal(nh * hd, 77, 2).reshape(1, nh, hd)
    kv0, kv1, q0, q1 = shard.kv_head_shard(nh, nkv, world, rank)
    # this rank's cache holds only its KV heads; its queries only its heads
    local_kvc = np.ascontiguousarray(kvc.reshape(2, L, nkv, hd)[:, :, kv0:kv1].reshape(2, L, -1))
    local_q = np.ascontiguousarray(q[:, q0:q1])
    local = O.attention_engine(local_q, local_kvc, q1 - q0, kv1 - kv0, hd, 1, L - 1, L, L)
    full = shard.gather_heads(torch.from_numpy(np.ascontiguousarray(local)), world)
    t = shard.max_over_ranks(float(rank + 1), world)
    if rank == 0:
        ref = O.attention_engine(q, kvc, nh, nkv, hd, 1, L - 1, L, L)
        np.save(os.path.join(result_dir, "full.npy"), full.numpy())
        np.save(os.path.join(result_dir, "ref.npy"), ref)
        np.save(os.path.join(result_dir, "tmax.npy"), np.array([t]))
    dist.barrier()
    dist.destroy_process_group()


def _seq_sharded_rank(rank, world, port, result_dir):
    _init(rank, world, port)
    import oracle as O
    import shard
    nh, nkv, hd = 8, 2, 64
    lens = np.array([50, 700, 20, 300, 300, 90, 1000, 5])
    parts = shard.lpt_partition(lens, world)
    outs = {}
    for i in parts[rank]:
        L = int(lens[i])
        kvc = O.normal(2 * L * nkv * hd, 5, i).reshape(2, L, nkv * hd)
        q = O.normal(nh * hd, 6, i).reshape(1, nh, hd)
        outs[i] = O.attention_engine(q, kvc, nh, nkv, hd, 1, L - 1, L, L).ravel()
    # no collective on the data path; the test gathers once to check
    gathered = [None] * world
    dist.all_gather_object(gathered, outs)
    if rank == 0:
        merged = {}
        for d in gathered:
            merged.update(d)
        np.save(os.path.join(result_dir, "seq.npy"),
                np.stack([merged[i] for i in range(len(lens))]))
    dist.barrier()
    dist.destroy_process_group()


def test_kv_head_groups_gather_equals_unsharded(tmp_path):
    mp.spawn(_head_sharded_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    full = np.load(tmp_path / "full.npy")
    ref = np.load(tmp_path / "ref.npy")
    assert full.shape == ref.shape
    assert np.array_equal(full.view(np.uint32), ref.view(np.uint32))
    assert float(np.load(tmp_path / "tmax.npy")[0]) == 2.0


def test_sequence_sharding_covers_every_sequence(tmp_path):
    import oracle as O
    mp.spawn(_seq_sharded_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    got = np.load(tmp_path / "seq.npy")
    lens = [50, 700, 20, 300, 300, 90, 1000, 5]
    for i, L in enumerate(lens):
        kvc = O.normal(2 * L * 2 * 64, 5, i).reshape(2, L, 128)
        q = O.normal(8 * 64, 6, i).reshape(1, 8, 64)
        ref = O.attention_engine(q, kvc, 8, 2, 64, 1, L - 1, L, L).ravel()
        assert np.array_equal(got[i], ref)


def test_lpt_balances_kv_bytes():
    import shard
    rng = np.random.default_rng(4)
    lens = rng.integers(1024, 32769, 64)
    for world in (2, 4, 8):
        parts = shard.lpt_partition(lens, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [int(lens[p].sum()) for p in parts]
        assert max(loads) - min(loads) <= int(lens.max())
        assert max(loads) / (lens.sum() / world) < 1.05


def test_kv_head_shard_ranges():
    import shard
    assert shard.kv_head_shard(32, 8, 8, 3) == (3, 4, 12, 16)
    assert shard.kv_head_shard(32, 8, 2, 1) == (4, 8, 16, 32)
    with pytest.raises(ValueError):
        shard.kv_head_shard(32, 8, 3, 0)
