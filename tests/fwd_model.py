"""Seeded synthetic models for the whole-forward tests, and a .TG writer.

The weights are a pure function of (config name, seed): numpy's PCG64
standard normals, scaled per tensor.  The golden generator writes them into a
.TG file (the layout of the reference's src/tgai_format.h: 128-byte header,
52-byte weight entries keyed by the 64-bit FNV-1a hash of the tensor name,
fp32 data) for the reference engine to load; the GPU tests rebuild the same
arrays and hand them to tg_fwd_create directly, or write the same file for
the engine-facing test.
"""
import struct

import numpy as np

CONFIGS = {
    # TGAI-native MoE (arch 0): router bias, GQA 8 q heads over 2 KV heads, head_dim 32
    "moe": dict(arch=0, n_layers=3, d_model=256, n_heads=8, n_kv_heads=2, d_ff=384,
                vocab=512, max_seq=256, n_experts=4, n_activated=2, rope_theta=10000,
                unk=1, qkv_bias=False, qb_bias=True),
    # Llama-style dense SwiGLU (arch 1) with Q/K/V biases, head_dim 64
    "dense": dict(arch=1, n_layers=3, d_model=256, n_heads=4, n_kv_heads=2, d_ff=512,
                  vocab=512, max_seq=256, n_experts=0, n_activated=0, rope_theta=10000,
                  unk=1, qkv_bias=True, qb_bias=False),
}

SEEDS = {"moe": 41, "dense": 42}


def fnv1a64(name):
    h = 0xcbf29ce484222325
    for b in name.encode():
        h ^= b
        h = (h * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
    return h


def weights(cfg, seed):
    """name -> float32 array ([out, in] for Linear weights)."""
    rng = np.random.default_rng(seed)
    d, nh, nkv, dff = cfg["d_model"], cfg["n_heads"], cfg["n_kv_heads"], cfg["d_ff"]
    hd = d // nh
    qd, kvd = nh * hd, nkv * hd

    def lin(o, i):
        return (rng.standard_normal((o, i)) / np.sqrt(i)).astype(np.float32)

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    w = {"token_embedding.weight": rng.standard_normal((cfg["vocab"], d)).astype(np.float32)}
    for l in range(cfg["n_layers"]):
        p = f"blocks.{l}."
        w[p + "ln1.weight"] = norm(d)
        w[p + "ln2.weight"] = norm(d)
        w[p + "attn.q_proj.weight"] = lin(qd, d)
        w[p + "attn.k_proj.weight"] = lin(kvd, d)
        w[p + "attn.v_proj.weight"] = lin(kvd, d)
        if cfg["qkv_bias"]:
            for n, o in (("q", qd), ("k", kvd), ("v", kvd)):
                w[p + f"attn.{n}_proj.bias"] = (0.1 * rng.standard_normal(o)).astype(np.float32)
        w[p + "attn.out_proj.weight"] = lin(d, qd)
        if cfg["n_experts"] == 0:
            w[p + "ffn.w1.weight"] = lin(dff, d)
            w[p + "ffn.w2.weight"] = lin(dff, d)
            w[p + "ffn.w3.weight"] = lin(d, dff)
        else:
            ne = cfg["n_experts"]
            w[p + "moe.router.weight"] = lin(ne, d)
            if cfg["qb_bias"]:
                w[p + "moe._qb_bias"] = (0.2 * rng.standard_normal(ne)).astype(np.float32)
            for e in range(ne):
                w[p + f"moe.experts.{e}.w1.weight"] = lin(dff, d)
                w[p + f"moe.experts.{e}.w2.weight"] = lin(dff, d)
                w[p + f"moe.experts.{e}.w3.weight"] = lin(d, dff)
    w["final_norm.weight"] = norm(d)
    return w


def write_tg(path, cfg, w):
    """A version-1 .TG file: header, weight table, fp32 data, no tokenizer."""
    names = list(w)
    table_off = 128
    data_off = (table_off + 52 * len(names) + 63) // 64 * 64
    entries, blobs, off = [], [], 0
    for n in names:
        a = np.ascontiguousarray(w[n], np.float32)
        shape = list(a.shape) + [0] * (4 - a.ndim)
        entries.append(struct.pack("<QQQII4II", fnv1a64(n), off, a.nbytes, 0, a.ndim, *shape, 0))
        blobs.append(a.tobytes())
        off += (a.nbytes + 63) // 64 * 64
    data_len = off
    hdr = struct.pack("<16I6Q4I", 0x49414754, 1, 0, cfg["n_layers"], cfg["d_model"],
                      cfg["n_heads"], cfg["d_ff"], cfg["vocab"], cfg["max_seq"],
                      cfg["n_experts"], cfg["n_activated"], cfg["rope_theta"], 0, 2, 3,
                      cfg["unk"], 0, 0, table_off, len(names), data_off, data_len,
                      cfg["arch"], cfg["n_kv_heads"], 0, 0)
    assert len(hdr) == 128
    with open(path, "wb") as f:
        f.write(hdr)
        for e in entries:
            f.write(e)
        f.write(b"\0" * (data_off - table_off - 52 * len(names)))
        for b in blobs:
            f.write(b)
            f.write(b"\0" * ((len(b) + 63) // 64 * 64 - len(b)))


# Forward scripts: (sequence, ids, cache_pos).  Sequence "a" prefills, decodes,
# truncates to an LCP and re-appends, decodes again; "b" runs in between on its
# own KV.  Token ids include out-of-vocabulary ones (-> unk).
def script(cfg, seed):
    rng = np.random.default_rng(seed + 1000)
    v = cfg["vocab"]

    def toks(n):
        return rng.integers(0, v, n).astype(np.int32)

    a = toks(24)
    steps = [("a", a[:20], 0), ("a", a[20:21], 20), ("a", a[21:22], 21)]
    b = toks(9)
    b[3] = v + 7                                  # out of range -> unk
    steps += [("b", b[:8], 0), ("a", a[22:23], 22), ("b", b[8:9], 8)]
    lcp = 12
    re = toks(7)
    steps += [("a", re, lcp), ("a", toks(1), lcp + 7), ("b", toks(3), 9)]
    return steps
