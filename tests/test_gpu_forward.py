"""Whole-model forward on the GPU (include/tgai_engine_bridge.h) against the
reference engine's own logits.

tests/golden/forward.npz holds tg_forward's logits (CPU engine,
src/tgai_engine.c built in oracle/_ref) for the seeded MoE and dense models of
tests/fwd_model.py over their scripts: prefill, decode, a second sequence on
its own KV, LCP truncate + re-append.  The CUDA forward computes in fp32
(tensor-core GEMMs at fp32-product accuracy, fp32 KV cache) in a different
summation order, so the bar is a relative error (max |diff| / max |logit|)
of 1e-4.
"""
import ctypes as C
import os

import numpy as np
import pytest

import fwd_model as FM
import fwd_oracle
import tgkv
from conftest import GOLDEN, ROOT

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4


def fwd_config(cfg, max_seq=None):
    return tgkv.TGFwdConfig(n_layers=cfg["n_layers"], d_model=cfg["d_model"],
                            n_heads=cfg["n_heads"], n_kv_heads=cfg["n_kv_heads"], head_dim=0,
                            d_ff=cfg["d_ff"], vocab_size=cfg["vocab"],
                            max_seq_len=max_seq or cfg["max_seq"], n_experts=cfg["n_experts"],
                            n_activated=cfg["n_activated"], rope_theta=cfg["rope_theta"],
                            unk_id=cfg["unk"])


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "forward.npz"))


@pytest.mark.parametrize("name", sorted(FM.CONFIGS))
def test_forward_matches_engine(cuda, golden, name, monkeypatch):
    """Every token through the per-layer launches (five per layer)."""
    monkeypatch.setenv("TGKV_FWD_STEP", "0")
    cfg = FM.CONFIGS[name]
    f = tgkv.Forward(cuda, fwd_config(cfg), FM.weights(cfg, FM.SEEDS[name]))
    try:
        gold = golden[f"{name}_logits"]
        for i, (key, ids, pos) in enumerate(FM.script(cfg, FM.SEEDS[name])):
            lg = f.forward(key, ids, pos)
            assert cuda.tg_fwd_last_launches() > 3 * cfg["n_layers"]
            e = rel(lg, gold[i])
            assert e < FWD_TOL, (name, i, e)
        assert cuda.tg_fwd_slot_count(f.m) == 2
        assert cuda.tg_fwd_slot_last_pos(f.m, C.c_void_p(f.key("a"))) == 12 + 7 + 1
    finally:
        f.close()
    assert cuda.tg_cuda_kv_device_error() == 0


@pytest.mark.parametrize("experts", ["tensor-core GEMM", "CUDA-core kernels"])
def test_long_prefill_and_decode_against_oracle(cuda, decode_path, experts, monkeypatch):
    """A 200-token prefill (longer than the workspaces' first size) and decode
    steps near the capacity, checked against the float64 oracle.  The
    prefill's experts run as grouped tensor-core GEMMs (the default) or on the
    CUDA-core expert kernels (TGKV_MOE_GEMM=0, read at model creation)."""
    monkeypatch.setenv("TGKV_MOE_GEMM", "0" if experts == "CUDA-core kernels" else "1")
    cfg = dict(FM.CONFIGS["moe"])
    w = FM.weights(cfg, 77)
    f = tgkv.Forward(cuda, fwd_config(cfg), w)
    o = fwd_oracle.Forward(cfg, w)
    rng = np.random.default_rng(5)
    ids = rng.integers(0, cfg["vocab"], 256).astype(np.int32)
    try:
        for pos, n in ((0, 200), (200, 1), (201, 54), (255, 1)):
            e = rel(f.forward("s", ids[pos:pos + n], pos), o.forward("s", ids[pos:pos + n], pos))
            assert e < FWD_TOL, (pos, n, e)
        with pytest.raises(tgkv.KvError, match="exceed max_seq_len"):
            f.forward("s", ids[:2], 255)
    finally:
        f.close()


@pytest.fixture(params=["launches", "one-launch step"])
def decode_path(request, monkeypatch):
    """Decode tokens through the per-layer launches, or through the
    one-launch decode step (all layers in one cooperative launch)."""
    monkeypatch.setenv("TGKV_FWD_STEP", "0" if request.param == "launches" else "1")
    return request.param


@pytest.mark.parametrize("name", sorted(FM.CONFIGS))
def test_decode_step_matches_engine(cuda, golden, name, monkeypatch):
    """The engine's scripts with every one-token decode on the one-launch
    step: a handful of launches per token instead of five per layer."""
    monkeypatch.setenv("TGKV_FWD_STEP", "1")
    cfg = FM.CONFIGS[name]
    f = tgkv.Forward(cuda, fwd_config(cfg), FM.weights(cfg, FM.SEEDS[name]))
    try:
        gold = golden[f"{name}_logits"]
        steps = 0
        for i, (key, ids, pos) in enumerate(FM.script(cfg, FM.SEEDS[name])):
            lg = f.forward(key, ids, pos)
            if len(ids) == 1:
                assert cuda.tg_fwd_last_launches() < 3 * cfg["n_layers"]
                steps += 1
            e = rel(lg, gold[i])
            assert e < FWD_TOL, (name, i, e)
        assert steps >= 3
    finally:
        f.close()
    assert cuda.tg_cuda_kv_device_error() == 0


def run_against_oracle(cuda, cfg, w, steps):
    f = tgkv.Forward(cuda, fwd_config(cfg), w)
    o = fwd_oracle.Forward(cfg, w)
    rng = np.random.default_rng(8)
    ids = rng.integers(0, cfg["vocab"], 64).astype(np.int32)
    try:
        for pos, n in steps:
            e = rel(f.forward("s", ids[pos:pos + n], pos), o.forward("s", ids[pos:pos + n], pos))
            assert e < FWD_TOL, (pos, n, e)
    finally:
        f.close()
    assert cuda.tg_cuda_kv_device_error() == 0


# a prefill (grouped expert kernels, one thread per token routes) and decode
# steps of 1-4 tokens (routing by one warp of every expert CTA)
STEPS = ((0, 6), (6, 1), (7, 1), (8, 3), (11, 4))


def test_v27_shape_against_oracle(cuda, decode_path):
    """The bench model's attention shape -- 12 query / 4 KV heads of 128 (a
    group of 3), 4 experts top-2, cut to 2 layers: the 100-token prefill on
    the fp32 block attention and the GEMMs, one-token steps on the
    one-launch step (or the per-layer launches), 3-token steps and a second
    prefill chunk on the per-layer kernels, against the float64 oracle."""
    cfg = dict(FM.CONFIGS["moe"], n_layers=2, d_model=1536, n_heads=12, n_kv_heads=4,
               d_ff=512, n_experts=4, n_activated=2)
    w = FM.weights(cfg, 2718)
    f = tgkv.Forward(cuda, fwd_config(cfg), w)
    o = fwd_oracle.Forward(cfg, w)
    rng = np.random.default_rng(27)
    ids = rng.integers(0, cfg["vocab"], 200).astype(np.int32)
    try:
        for pos, n in ((0, 100), (100, 1), (101, 1), (102, 3), (105, 40), (145, 1)):
            e = rel(f.forward("s", ids[pos:pos + n], pos), o.forward("s", ids[pos:pos + n], pos))
            assert e < FWD_TOL, (pos, n, e)
    finally:
        f.close()
    assert cuda.tg_cuda_kv_device_error() == 0


def test_router_ties_follow_the_engine(cuda, decode_path):
    """Equal router logits: the engine's top-k takes the lowest expert index
    among equals, never one already chosen (strict greater from -1e30,
    src/tgai_engine.c:4166-4192).  Zero routers make the logits the bias:
    layer 0 ties three experts for the maximum, layer 1 all four, layer 2 the
    first and the last."""
    cfg = FM.CONFIGS["moe"]
    w = FM.weights(cfg, 13)
    ties = ([0.5, 1.0, 1.0, 1.0], [0.0, 0.0, 0.0, 0.0], [1.0, 0.0, 0.0, 1.0])
    for l in range(cfg["n_layers"]):
        w[f"blocks.{l}.moe.router.weight"] = np.zeros_like(w[f"blocks.{l}.moe.router.weight"])
        w[f"blocks.{l}.moe._qb_bias"] = np.array(ties[l], np.float32)
    run_against_oracle(cuda, cfg, w, STEPS)


def test_odd_top_k_against_oracle(cuda, decode_path):
    """Top-3 of 8 experts: the decode W3 launch pairs choices (0, 1) and
    takes choice 2 alone."""
    cfg = dict(FM.CONFIGS["moe"], n_experts=8, n_activated=3)
    run_against_oracle(cuda, cfg, FM.weights(cfg, 14), STEPS)


def test_position_gap_clears_the_slot(cuda):
    """cache_pos past the slot's last position clears its KV first
    (cuda/tgai_cuda.cu:1703-1711): the result equals a fresh slot started at
    that position over an all-zero cache."""
    cfg = FM.CONFIGS["dense"]
    f = tgkv.Forward(cuda, fwd_config(cfg), FM.weights(cfg, 3))
    ids = np.arange(20, dtype=np.int32) * 7 % cfg["vocab"]
    try:
        f.forward("a", ids[:5], 0)
        gap = f.forward("a", ids[10:14], 10)
        fresh = f.forward("b", ids[10:14], 10)
        assert np.array_equal(gap, fresh)
        assert cuda.tg_fwd_slot_last_pos(f.m, C.c_void_p(f.key("a"))) == 14
        # reset_slot then a forward at 0 equals a new sequence
        assert cuda.tg_fwd_reset_slot(f.m, C.c_void_p(f.key("a")))
        assert cuda.tg_fwd_slot_last_pos(f.m, C.c_void_p(f.key("a"))) == -1
        assert np.array_equal(f.forward("a", ids[:6], 0), f.forward("c", ids[:6], 0))
    finally:
        f.close()


def test_slot_limit_and_release(cuda, monkeypatch):
    cfg = FM.CONFIGS["dense"]
    monkeypatch.setenv("TGAI_CUDA_KV_SLOTS", "2")
    f = tgkv.Forward(cuda, fwd_config(cfg, max_seq=64), FM.weights(cfg, 4))
    ids = np.array([1, 2, 3], np.int32)
    try:
        f.forward("a", ids, 0)
        f.forward("b", ids, 0)
        with pytest.raises(tgkv.KvError, match="no free slot"):
            f.forward("c", ids, 0)
        assert cuda.tg_fwd_free_slot(f.m, C.c_void_p(f.key("a")))
        assert cuda.tg_fwd_slot_count(f.m) == 1
        f.forward("c", ids, 0)
        assert cuda.tg_fwd_slot_count(f.m) == 2
    finally:
        f.close()


def test_create_rejects_bad_models(cuda):
    cfg = FM.CONFIGS["moe"]
    w = FM.weights(cfg, 9)
    bad = fwd_config(cfg)
    bad.n_activated = 9
    with pytest.raises(tgkv.KvError, match="top-1..8"):
        tgkv.Forward(cuda, bad, w)
    w2 = dict(w)
    del w2["blocks.1.moe.experts.2.w3.weight"]
    with pytest.raises(tgkv.KvError, match="missing weight blocks.1.moe.experts.2.w3.weight"):
        tgkv.Forward(cuda, fwd_config(cfg), w2)
    w3 = dict(w)
    w3["blocks.0.attn.k_proj.weight"] = w3["blocks.0.attn.q_proj.weight"]
    with pytest.raises(tgkv.KvError, match="k_proj.weight has shape"):
        tgkv.Forward(cuda, fwd_config(cfg), w3)


ENGINE_SO = os.path.join(ROOT, "oracle", "_ref", "libtgai_engine_ref.so")


def test_engine_seam(cuda, golden, tmp_path, monkeypatch):
    """tg_engine_cuda_* on a model the reference engine loaded (tg_load of a
    .TG file), with the engine's own TGKVCache objects as slot keys."""
    if not os.path.exists(ENGINE_SO):
        pytest.skip("oracle/_ref/libtgai_engine_ref.so not built")
    eng = C.CDLL(ENGINE_SO, mode=os.RTLD_LAZY | os.RTLD_GLOBAL)
    eng.tg_load.restype = C.c_void_p
    eng.tg_load.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_int)]
    eng.tg_kvcache_new.restype = C.c_void_p
    eng.tg_kvcache_new.argtypes = [C.c_void_p, C.c_int]
    eng.tg_kvcache_free.argtypes = [C.c_void_p]
    eng.tg_free.argtypes = [C.c_void_p]
    name = "moe"
    cfg = FM.CONFIGS[name]
    path = tmp_path / "m.TG"
    FM.write_tg(str(path), cfg, FM.weights(cfg, FM.SEEDS[name]))
    err = C.c_int(0)
    m = eng.tg_load(str(path).encode(), 0, C.byref(err))
    assert m, err.value
    lib = cuda
    caches = {}
    try:
        monkeypatch.delenv("TGAI_USE_GPU", raising=False)
        lib.tg_engine_cuda_shutdown()
        assert lib.tg_engine_cuda_init(m) == 0                 # not enabled: CPU path
        assert b"TGAI_USE_GPU" in lib.tg_engine_cuda_reason()
        lib.tg_engine_cuda_shutdown()
        monkeypatch.setenv("TGAI_USE_GPU", "1")
        assert lib.tg_engine_cuda_init(m) == 1, lib.tg_engine_cuda_reason()
        assert lib.tg_engine_cuda_init(m) == 1                 # idempotent
        assert lib.tg_engine_cuda_ready() == 1
        calls0, falls0 = lib.tg_engine_cuda_calls(), lib.tg_engine_cuda_fallbacks()
        gold = golden[f"{name}_logits"]
        for i, (key, ids, pos) in enumerate(FM.script(cfg, FM.SEEDS[name])):
            if key not in caches:
                caches[key] = eng.tg_kvcache_new(m, cfg["max_seq"])
            arr = (C.c_int32 * len(ids))(*ids.tolist())
            out = tgkv.PF()
            assert lib.tg_engine_cuda_forward(m, arr, len(ids), caches[key], int(pos),
                                              C.byref(out)) == 1
            lg = np.ctypeslib.as_array(out, shape=(cfg["vocab"],)).copy()
            e = rel(lg, gold[i])
            assert e < FWD_TOL, (i, e)
        n = len(FM.script(cfg, FM.SEEDS[name]))
        assert lib.tg_engine_cuda_calls() - calls0 == n
        assert lib.tg_engine_cuda_fallbacks() == falls0
        assert lib.tg_gpu_kv_slot_live() == 2 and lib.tg_gpu_kv_slot_max() == 16
        assert lib.tg_gpu_kv_slot_seq(caches["a"]) == 20
        assert lib.tg_gpu_kv_slot_of(caches["b"]) >= 0
        assert lib.tg_gpu_kv_slot_of(None) == -1
        # another model handle is not taken: 0, not counted as a fallback
        out = tgkv.PF()
        assert lib.tg_engine_cuda_forward(C.c_void_p(1), (C.c_int32 * 1)(1), 1, caches["a"], 0,
                                          C.byref(out)) == 0
        assert lib.tg_engine_cuda_fallbacks() == falls0
        lib.tg_engine_cuda_free_slot(caches["b"])
        assert lib.tg_gpu_kv_slot_live() == 1
        lib.tg_engine_cuda_reset_slot(caches["a"])
        assert lib.tg_gpu_kv_slot_seq(caches["a"]) == -1
    finally:
        lib.tg_engine_cuda_shutdown()
        assert lib.tg_engine_cuda_ready() == 0
        for c in caches.values():
            eng.tg_kvcache_free(c)
        eng.tg_free(m)


@pytest.mark.parametrize("name", sorted(FM.CONFIGS))
def test_concurrent_sequences_batch_across_slots(cuda, name):
    """Eight sequences decoded at once from eight threads, as a server does:
    one-token forwards that are in flight together run as batches over the
    weights (tg_fwd_batch_stats counts them), and every sequence's logits, at
    every step, match the float64 oracle at the forward's tolerance."""
    import threading
    cfg = dict(FM.CONFIGS[name])
    w = FM.weights(cfg, 91)
    f = tgkv.Forward(cuda, fwd_config(cfg), w)
    n_seq, prefill, steps = 8, 12, 20
    rng = np.random.default_rng(13)
    ids = rng.integers(0, cfg["vocab"], (n_seq, prefill + steps)).astype(np.int32)
    for i in range(n_seq):
        f.key(f"t{i}")                      # keys registered before the threads start
    out = [[None] * (steps + 1) for _ in range(n_seq)]
    errors = []
    start = threading.Barrier(n_seq)

    def worker(i):
        try:
            out[i][0] = f.forward(f"t{i}", ids[i, :prefill], 0)
            start.wait()
            for t in range(steps):
                out[i][t + 1] = f.forward(f"t{i}", ids[i, prefill + t:prefill + t + 1],
                                          prefill + t)
        except Exception as e:              # reported below, on the test's thread
            errors.append(f"{i}: {e!r}")

    tokens, batches = C.c_uint64(), C.c_uint64()
    try:
        th = [threading.Thread(target=worker, args=(i,)) for i in range(n_seq)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        assert not errors, errors
        cuda.tg_fwd_batch_stats(f.m, C.byref(tokens), C.byref(batches))
    finally:
        f.close()
    assert batches.value > 0 and tokens.value >= 2 * batches.value, (tokens.value, batches.value)
    for i in range(n_seq):
        o = fwd_oracle.Forward(cfg, w)
        e = rel(out[i][0], o.forward("s", ids[i, :prefill], 0))
        assert e < FWD_TOL, (i, "prefill", e)
        for t in range(steps):
            ref = o.forward("s", ids[i, prefill + t:prefill + t + 1], prefill + t)
            e = rel(out[i][t + 1], ref)
            assert e < FWD_TOL, (i, t, e)
    assert cuda.tg_cuda_kv_device_error() == 0
