"""The CPU oracle against golden vectors made by the reference's own code.

tests/golden/gen_golden.py produced these vectors by compiling and running the
reference (src/tgai_engine.c, src/tgai_kv_cache.c + the CPU backend of
src/tgai_backend.c, tests/test_kv_cache_gpu.c and tests/test_vk_attn_moe.c).
Every comparison here is bit-exact.
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_dot_matches_engine_tg_dot():
    z = load("engine_pins.npz")
    for n, a, b, r in zip(z["dot_len"], z["dot_a"], z["dot_b"], z["dot_out"]):
        got = O.dot(np.ascontiguousarray(a[:n]), np.ascontiguousarray(b[:n]))
        assert np.float32(got).view(np.uint32) == np.float32(r).view(np.uint32), n


def test_softmax_matches_engine():
    z = load("engine_pins.npz")
    for x, y in zip(z["softmax_in"], z["softmax_out"]):
        assert np.array_equal(bits(O.softmax(x)), bits(y))


def test_rope_matches_engine():
    z = load("engine_pins.npz")
    for ci in range(int(z["rope_cases"])):
        seq, nh, nkv, dk, pos = (int(v) for v in z[f"rope{ci}_shape"])
        q, k = O.rope(z[f"rope{ci}_q"], z[f"rope{ci}_k"], nh, nkv, dk, pos)
        assert np.array_equal(bits(q), bits(z[f"rope{ci}_qout"]))
        assert np.array_equal(bits(k), bits(z[f"rope{ci}_kout"]))


def fixture_steps():
    z = load("engine_fixture.npz")
    msl, _, nh, nkv, dk = (int(v) for v in z["geometry"])
    for si in range(int(z["n_steps"])):
        seq, pos, kvl = (int(v) for v in z[f"s{si}_meta"])
        kvc = np.zeros((2, msl, nkv * dk), np.float32)
        kvc[:, :kvl] = z[f"s{si}_kvc"]
        yield dict(q=z[f"s{si}_q"], kvc=kvc, w=z[f"s{si}_w"], seq=seq, pos=pos, kvl=kvl,
                   msl=msl, nh=nh, nkv=nkv, dk=dk)


def test_attention_weights_match_engine_forward():
    """Softmax weights of the engine's real forwards (prefill, decode, LCP
    truncate + re-append) equal the oracle's on the engine's own q and K."""
    n = 0
    for s in fixture_steps():
        w = O.attention_weights_last(s["q"], s["kvc"], s["nh"], s["nkv"], s["dk"], s["seq"],
                                     s["pos"], s["kvl"], s["msl"])
        assert np.array_equal(bits(w), bits(s["w"])), (s["seq"], s["pos"])
        n += 1
    assert n == 6


def test_f64_attention_matches_reference_kv_test():
    z = load("kvtest.npz")
    nh, nkvh, hd, ms, nt = (int(v) for v in z["geometry"])
    kvc = np.zeros((2, ms, nkvh * hd), np.float32)
    kvc[:, :nt] = z["cache_rows"]
    out = O.attention_f64(z["q"], kvc, nh, nkvh, hd, 1, nt - 1, nt, ms).ravel()
    assert np.array_equal(bits(out), bits(z["out"]))


def test_f64_attention_matches_reference_attn_test():
    z = load("attntest.npz")
    nh, nkvh, hd, ms, nkv, pos = (int(v) for v in z["geometry"])
    kvc = np.zeros((2, ms, nkvh * hd), np.float32)
    kvc[:, :nkv] = z["kv_rows"]
    for p, key in ((pos, "out_pos39"), (10, "out_pos10")):
        out = O.attention_f64(z["q"], kvc, nh, nkvh, hd, 1, p, nkv, ms).ravel()
        assert np.array_equal(bits(out), bits(z[key])), p


def test_append_layout_matches_reference_cpu_backend():
    """orc_kv_append writes the same bytes as src/tgai_kv_cache.c with the
    reference CPU backend (32 single-token appends)."""
    z = load("kvtest.npz")
    nh, nkvh, hd, ms, nt = (int(v) for v in z["geometry"])
    kvd = nkvh * hd
    cache = np.zeros((2, ms, kvd), np.float32)
    for t in range(nt):
        assert O.kv_append(cache, O.F32, ms, kvd, t, z["kall"][t], z["vall"][t]) == 1
    assert np.array_equal(bits(cache[:, :nt]), bits(z["cache_rows"]))
    assert not cache[:, nt:].any()
    # capacity rule: exactly max_seq appends fit, the next one fails
    filled = sum(O.kv_append(cache, O.F32, ms, kvd, t, z["kall"][0], z["vall"][0])
                 for t in range(ms))
    assert filled == int(z["fill_count"]) == ms
    assert O.kv_append(cache, O.F32, ms, kvd, ms, z["kall"][0], z["vall"][0]) == 0
    assert int(z["extra_append"]) == 0 and int(z["len_after_reset"]) == 0


def test_bf16_rule_round_to_nearest_even():
    lib = O.load()
    vals = np.array([0.0, -0.0, 1.0, 1.00390625, 1.01171875, 3.4e38, -3.4e38, np.inf, -np.inf,
                     1e-40, -1e-40, 65504.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8], np.float32)
    rnd = np.random.default_rng(3).standard_normal(4096).astype(np.float32)
    for x in np.concatenate([vals, rnd]):
        assert lib.orc_f32_to_bf16(float(x)) == int(O.f32_to_bf16(np.array([x]))[0])
    # ties go to even: 1 + 2^-8 is halfway between bf16 1.0 and 1.0078125
    assert O.f32_to_bf16(np.array([1.0 + 2**-8], np.float32))[0] == 0x3F80
    assert O.f32_to_bf16(np.array([1.0 + 3 * 2**-8], np.float32))[0] == 0x3F82
    nan = np.array([np.nan], np.float32)
    assert O.bf16_to_f32(O.f32_to_bf16(nan))[0] != O.bf16_to_f32(O.f32_to_bf16(nan))[0]


def test_engine_order_close_to_f64():
    """Float engine order vs double accumulation on the reference test data:
    the two reference CPU implementations agree to 1e-5 of each head's scale."""
    from conftest import rel_head_err
    z = load("kvtest.npz")
    nh, nkvh, hd, ms, nt = (int(v) for v in z["geometry"])
    kvc = np.zeros((2, ms, nkvh * hd), np.float32)
    kvc[:, :nt] = z["cache_rows"]
    eng = O.attention_engine(z["q"], kvc, nh, nkvh, hd, 1, nt - 1, nt, ms)
    assert rel_head_err(eng, z["out"].reshape(1, nh, hd)) < 1e-5


@pytest.mark.parametrize("seed", [1, 2])
def test_decode_batch_equals_engine_loop(seed):
    rng = np.random.default_rng(seed)
    nh, nkv, hd = 8, 2, 64
    kvcs, qs, lens = [], [], []
    for L in (1, 17, 64):
        kvc = rng.standard_normal((2, 80, nkv * hd)).astype(np.float32)
        kvcs.append(np.ascontiguousarray(kvc.ravel()))
        qs.append(rng.standard_normal(nh * hd).astype(np.float32))
        lens.append(L)
    outs = O.decode_batch(kvcs, qs, lens, nh, nkv, hd, threads=2)
    for kvc, q, L, o in zip(kvcs, qs, lens, outs):
        ref = O.attention_engine(q, kvc, nh, nkv, hd, 1, L - 1, L, 80).ravel()
        assert np.array_equal(bits(o), bits(ref))


def test_rope_tables_with_context_extension_match_engine(lib):
    """tg_kv_rope_tables (host code of the product, no GPU needed) builds the
    tables the engine's rope() evaluates inline -- NTK-by-parts frequencies and
    the YaRN temperature included (src/tgai_engine.c:3404-3460); rotating with
    them reproduces the engine's bits."""
    import ctypes as C
    import tgkv
    z = load("engine_pins.npz")
    for ci in range(int(z["ropex_cases"])):
        seq, nh, nkv, dk, pos, ectx, msl = (int(v) for v in z[f"ropex{ci}_shape"])
        n = pos + seq
        cs = np.zeros((n, dk // 2), np.float32)
        sn = np.zeros_like(cs)
        ms = C.c_float()
        assert lib.tg_kv_rope_tables(float(z[f"ropex{ci}_theta"]), dk, 0, n, ectx, msl,
                                     cs.ctypes.data_as(tgkv.PF), sn.ctypes.data_as(tgkv.PF),
                                     C.byref(ms))
        q = O.rope_tables(z[f"ropex{ci}_q"], nh, dk, pos, cs, sn)
        k = O.rope_tables(z[f"ropex{ci}_k"], nkv, dk, pos, cs, sn)
        assert np.array_equal(bits(q), bits(z[f"ropex{ci}_qout"])), ci
        assert np.array_equal(bits(k), bits(z[f"ropex{ci}_kout"])), ci
        assert np.float32(ms.value) == z[f"ropex{ci}_mscale"]
    # without extension the tables reproduce the plain rope() pins as well
    for ci in range(int(z["rope_cases"])):
        seq, nh, nkv, dk, pos = (int(v) for v in z[f"rope{ci}_shape"])
        n = pos + seq
        cs = np.zeros((n, dk // 2), np.float32)
        sn = np.zeros_like(cs)
        assert lib.tg_kv_rope_tables(10000.0, dk, 0, n, 0, 0, cs.ctypes.data_as(tgkv.PF),
                                     sn.ctypes.data_as(tgkv.PF), None)
        q = O.rope_tables(z[f"rope{ci}_q"], nh, dk, pos, cs, sn)
        assert np.array_equal(bits(q), bits(z[f"rope{ci}_qout"])), ci
