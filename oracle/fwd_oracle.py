"""CPU restatement of the engine's whole-model forward, in float64 numpy.

TEST INFRASTRUCTURE ONLY: the tests compare the CUDA forward (libtgkv.so,
tg_fwd_* / tg_engine_cuda_*) with it; nothing in the library imports it.

Pinned: on the seeded models of tests/fwd_model.py it reproduces the logits
that the reference engine's own tg_forward (built from src/tgai_engine.c into
oracle/_ref) wrote to tests/golden/forward.npz to ~1e-7 relative
(tests/test_fwd_oracle.py).

It follows src/tgai_engine.c:
  embedding with out-of-range ids -> unk             :4396-4412
  rmsnorm  x * (1/sqrt(mean(x^2) + 1e-6)) * w        :2729-2784
  Q/K/V projections, optional biases                 :3865-3911
  interleaved-pair RoPE, freq_i = theta^(-i/dk)      :3404-3490
  KV write at cache_pos + t                          :3927-3941
  causal GQA attention, kvh = h*nkv/nh, -1e30 mask   :3947-4011
  out projection + residual                          :4020-4050
  dense FFN: clamp(+-88) SiLU(W1 x) * W2 x -> W3     :4108-4128
  MoE: router (+ _qb_bias), strict-greater top-k,
       max-shifted softmax over the k, experts
       W3 (SiLU(W1 x) * W2 x), k-ordered sum         :4130-4340
  final norm of the last row, tied-embedding head    :4455-4498
"""
import numpy as np


def rmsnorm(x, w):
    ss = (x ** 2).mean(-1, keepdims=True)
    return x / np.sqrt(ss + 1e-6) * w


def rope(x, pos0, theta, hd):
    """x [seq, heads, hd]: pairs (2i, 2i+1) rotated by (pos0 + t) * theta^(-2i/hd)."""
    seq = x.shape[0]
    i = np.arange(0, hd, 2)
    freq = 1.0 / float(theta) ** (i / hd)
    ang = np.arange(pos0, pos0 + seq)[:, None] * freq[None, :]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    a, b = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = a * c - b * s
    out[..., 1::2] = a * s + b * c
    return out


class Forward:
    """cfg: the keys of tests/fwd_model.CONFIGS; w: name -> array."""

    def __init__(self, cfg, w):
        self.c = cfg
        self.w = {k: np.asarray(v, np.float64) for k, v in w.items()}
        self.kv = {}

    def forward(self, key, ids, pos):
        c, w = self.c, self.w
        d, nh, nkv = c["d_model"], c["n_heads"], c["n_kv_heads"]
        hd = d // nh
        if key not in self.kv:
            self.kv[key] = [(np.zeros((c["max_seq"], nkv, hd)), np.zeros((c["max_seq"], nkv, hd)))
                            for _ in range(c["n_layers"])]
        kvs = self.kv[key]
        ids = np.asarray(ids)
        ids = np.where((ids < 0) | (ids >= c["vocab"]), c["unk"], ids)
        x = w["token_embedding.weight"][ids]
        seq = len(ids)
        for l in range(c["n_layers"]):
            p = f"blocks.{l}."
            ln = rmsnorm(x, w[p + "ln1.weight"])
            q = ln @ w[p + "attn.q_proj.weight"].T
            k = ln @ w[p + "attn.k_proj.weight"].T
            v = ln @ w[p + "attn.v_proj.weight"].T
            if p + "attn.q_proj.bias" in w:
                q = q + w[p + "attn.q_proj.bias"]
            if p + "attn.k_proj.bias" in w:
                k = k + w[p + "attn.k_proj.bias"]
            if p + "attn.v_proj.bias" in w:
                v = v + w[p + "attn.v_proj.bias"]
            q = rope(q.reshape(seq, nh, hd), pos, c["rope_theta"], hd)
            k = rope(k.reshape(seq, nkv, hd), pos, c["rope_theta"], hd)
            K, V = kvs[l]
            K[pos:pos + seq] = k
            V[pos:pos + seq] = v.reshape(seq, nkv, hd)
            att = np.zeros((seq, nh, hd))
            for t in range(seq):
                for h in range(nh):
                    kh = h * nkv // nh
                    sc = K[:pos + seq, kh] @ q[t, h] / np.sqrt(hd)
                    sc[pos + t + 1:] = -1e30
                    e = np.exp(sc - sc.max())
                    att[t, h] = (e / e.sum()) @ V[:pos + seq, kh]
            x = x + att.reshape(seq, -1) @ w[p + "attn.out_proj.weight"].T
            ln = rmsnorm(x, w[p + "ln2.weight"])
            if c["n_experts"] == 0:
                a = np.clip(ln @ w[p + "ffn.w1.weight"].T, -88, 88)
                b = ln @ w[p + "ffn.w2.weight"].T
                x = x + ((a / (1 + np.exp(-a))) * b) @ w[p + "ffn.w3.weight"].T
                continue
            r = ln @ w[p + "moe.router.weight"].T
            if p + "moe._qb_bias" in w:
                r = r + w[p + "moe._qb_bias"]
            out = np.zeros_like(x)
            for t in range(seq):
                top = np.argsort(-r[t], kind="stable")[: c["n_activated"]]
                e = np.exp(r[t][top] - r[t][top].max())
                e /= e.sum()
                for kk, ex in enumerate(top):
                    pe = p + f"moe.experts.{ex}."
                    a = w[pe + "w1.weight"] @ ln[t]
                    b = w[pe + "w2.weight"] @ ln[t]
                    out[t] += e[kk] * (w[pe + "w3.weight"] @ ((a / (1 + np.exp(-a))) * b))
            x = x + out
        xl = rmsnorm(x[-1:], w["final_norm.weight"])
        return (xl @ w["token_embedding.weight"].T)[0]
