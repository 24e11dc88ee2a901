/* tgkv_oracle.c -- CPU restatement of the reference's KV-cache path.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and the
 * CPU legs of bench.py as the checker / timed CPU baseline.  Never linked into
 * the product library.  Parity: pinned against the reference's own compiled
 * code through the vectors in tests/golden/ (see tgkv_oracle.h).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).  Fused
 * multiply-adds are written explicitly with fmaf() wherever the reference's
 * build fuses them, so the result does not depend on compiler contraction.
 */
#include "tgkv_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---- src/tgai_engine.c:580-603 (avx2_dot) --------------------------------
 * Two 8-lane fused accumulators over 16-element steps, an optional 8-element
 * step into the first accumulator, lane-wise add of the two accumulators,
 * low half + high half, then two pairwise horizontal adds; leftover elements
 * are added one by one as a rounded product then a rounded sum (the
 * reference build does not fuse this scalar tail). */
/* Hot loops get an x86-64-v3 clone (hardware FMA, chosen at run time) and a
 * portable default; fmaf() gives identical results in both. */
#if defined(__x86_64__) && defined(__GNUC__)
#define ORC_HOT __attribute__((target_clones("arch=x86-64-v3", "default")))
#else
#define ORC_HOT
#endif

static inline float dot_impl(const float* a, const float* b, int n) {
    float acc0[8] = {0}, acc1[8] = {0};
    int i = 0;
    for (; i + 16 <= n; i += 16) {
        for (int l = 0; l < 8; l++) {
            acc0[l] = fmaf(a[i + l], b[i + l], acc0[l]);
            acc1[l] = fmaf(a[i + 8 + l], b[i + 8 + l], acc1[l]);
        }
    }
    if (i + 8 <= n) {
        for (int l = 0; l < 8; l++) acc0[l] = fmaf(a[i + l], b[i + l], acc0[l]);
        i += 8;
    }
    float s8[8], s4[4];
    for (int l = 0; l < 8; l++) s8[l] = acc0[l] + acc1[l];
    for (int l = 0; l < 4; l++) s4[l] = s8[l] + s8[l + 4];
    float s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
    for (; i < n; i++) s += a[i] * b[i];
    return s;
}

ORC_HOT float orc_dot(const float* a, const float* b, int n) { return dot_impl(a, b, n); }

/* ---- src/tgai_engine.c:3493-3503 (softmax) ------------------------------- */
void orc_softmax(float* x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float s = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        s += x[i];
    }
    float inv = 1.0f / s;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* ---- src/tgai_engine.c:3404-3490 (rope, extend_ctx = 0) -------------------
 * freq = 1/powf(theta, i/d_k) for even i; angle = pos*freq; the pair (x0, x1)
 * becomes (x0*c - x1*s, x0*s + x1*c).  Q is rotated over n_heads heads and K
 * over n_kv_heads heads, each head once.  The reference's gcc -mfma build
 * fuses the second product of each line: x0*c - x1*s == fmaf(x0, c, -(x1*s)),
 * x0*s + x1*c == fmaf(x0, s, x1*c); the golden vectors pin this. */
static void rope_rows(float* x, int seq, int nh, int d_k, int pos0, float theta) {
    for (int t = 0; t < seq; t++) {
        int pos = pos0 + t;
        for (int h = 0; h < nh; h++) {
            float* xh = x + ((size_t)t * nh + h) * d_k;
            for (int i = 0; i < d_k; i += 2) {
                float freq = 1.0f / powf(theta, (float)i / d_k);
                float angle = (float)pos * freq;
                float c = cosf(angle), s = sinf(angle);
                float x0 = xh[i], x1 = xh[i + 1];
                xh[i]     = fmaf(x0, c, -(x1 * s));
                xh[i + 1] = fmaf(x0, s, x1 * c);
            }
        }
    }
}

void orc_rope_tables(float* x, int seq, int nh, int d_k, int pos0, const float* cs,
                     const float* sn) {
    const int half = d_k / 2;
    for (int t = 0; t < seq; t++)
        for (int h = 0; h < nh; h++) {
            float* xh = x + ((size_t)t * nh + h) * d_k;
            for (int i = 0; i < d_k; i += 2) {
                const float c = cs[(size_t)(pos0 + t) * half + i / 2];
                const float s = sn[(size_t)(pos0 + t) * half + i / 2];
                const float x0 = xh[i], x1 = xh[i + 1];
                xh[i]     = fmaf(x0, c, -(x1 * s));
                xh[i + 1] = fmaf(x0, s, x1 * c);
            }
        }
}

void orc_rope(float* q, float* k, int seq, int n_heads, int n_kv_heads, int d_k,
              int pos0, float theta) {
    if (q) rope_rows(q, seq, n_heads, d_k, pos0, theta);
    if (k) rope_rows(k, seq, n_kv_heads, d_k, pos0, theta);
}

/* ---- bf16 storage rule (the reference has no bf16 cache; this build names
 * round-to-nearest-even as the rule and the CUDA append kernel uses it). --- */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu))
        return (uint16_t)((u >> 16) | 0x0040u);           /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* ---- src/tgai_kv_cache.c:90-110 (append byte layout) --------------------- */
int orc_kv_append(void* cache, int dtype, uint32_t max_seq, uint32_t kv_dim,
                  uint32_t len, const float* k, const float* v, uint32_t n_tokens) {
    if ((uint64_t)len + n_tokens > max_seq) return 0;
    size_t kbase = (size_t)len * kv_dim;
    size_t vbase = (size_t)max_seq * kv_dim + kbase;
    size_t cnt = (size_t)n_tokens * kv_dim;
    if (dtype == ORC_F32) {
        float* c = (float*)cache;
        memcpy(c + kbase, k, cnt * 4);
        memcpy(c + vbase, v, cnt * 4);
    } else {
        uint16_t* c = (uint16_t*)cache;
        for (size_t i = 0; i < cnt; i++) {
            c[kbase + i] = orc_f32_to_bf16(k[i]);
            c[vbase + i] = orc_f32_to_bf16(v[i]);
        }
    }
    return 1;
}

void orc_kv_decode(const void* cache, int dtype, uint32_t max_seq, uint32_t kv_dim,
                   float* out) {
    size_t cnt = 2ull * max_seq * kv_dim;
    if (dtype == ORC_F32) {
        memcpy(out, cache, cnt * 4);
    } else {
        const uint16_t* c = (const uint16_t*)cache;
        for (size_t i = 0; i < cnt; i++) out[i] = orc_bf16_to_f32(c[i]);
    }
}

/* ---- src/tgai_engine.c:3943-4011 (attention loop) read through the
 * [2][max_seq][kv_dim] layout of src/tgai_kv_cache.h:15-21. -------------- */
ORC_HOT static void engine_head(const float* qh, const float* kvc, float* oh, float* sc,
                        int kvh, int head_dim, int kv_dim, int cur_abs, int kv_len,
                        int max_seq, float inv_sqrt) {
    const float* kb = kvc + (size_t)kvh * head_dim;
    const float* vb = kvc + (size_t)max_seq * kv_dim + (size_t)kvh * head_dim;
    for (int ki = 0; ki < kv_len; ki++)
        sc[ki] = dot_impl(qh, kb + (size_t)ki * kv_dim, head_dim) * inv_sqrt;
    for (int ki = 0; ki < kv_len; ki++)
        if (ki > cur_abs) sc[ki] = -1e30f;
    orc_softmax(sc, kv_len);
    for (int i = 0; i < head_dim; i++) oh[i] = 0.0f;
    for (int ki = 0; ki < kv_len; ki++) {
        const float* vh = vb + (size_t)ki * kv_dim;
        float w = sc[ki];
        for (int i = 0; i < head_dim; i++) oh[i] = fmaf(w, vh[i], oh[i]);
    }
}

void orc_attention_engine_scaled(const float* q, const float* kvc, float* out,
                                 int n_heads, int n_kv_heads, int head_dim,
                                 int n_q, int pos0, int kv_len, int max_seq, float mscale) {
    int kv_dim = n_kv_heads * head_dim;
    float inv_sqrt = (1.0f / sqrtf((float)head_dim)) * mscale;
    float* sc = (float*)malloc(sizeof(float) * (kv_len > 0 ? kv_len : 1));
    for (int t = 0; t < n_q; t++)
        for (int h = 0; h < n_heads; h++) {
            int kvh = h * n_kv_heads / n_heads;
            engine_head(q + ((size_t)t * n_heads + h) * head_dim, kvc,
                        out + ((size_t)t * n_heads + h) * head_dim, sc, kvh,
                        head_dim, kv_dim, pos0 + t, kv_len, max_seq, inv_sqrt);
        }
    free(sc);
}

void orc_attention_engine(const float* q, const float* kvc, float* out,
                          int n_heads, int n_kv_heads, int head_dim,
                          int n_q, int pos0, int kv_len, int max_seq) {
    orc_attention_engine_scaled(q, kvc, out, n_heads, n_kv_heads, head_dim, n_q, pos0, kv_len,
                                max_seq, 1.0f);
}

void orc_attention_weights_last(const float* q, const float* kvc, float* w,
                                int n_heads, int n_kv_heads, int head_dim,
                                int n_q, int pos0, int kv_len, int max_seq) {
    int kv_dim = n_kv_heads * head_dim;
    float inv_sqrt = 1.0f / sqrtf((float)head_dim);
    int t = n_q - 1;
    for (int h = 0; h < n_heads; h++) {
        int kvh = h * n_kv_heads / n_heads;
        const float* qh = q + ((size_t)t * n_heads + h) * head_dim;
        float* sc = w + (size_t)h * kv_len;
        const float* kb = kvc + (size_t)kvh * head_dim;
        for (int ki = 0; ki < kv_len; ki++)
            sc[ki] = dot_impl(qh, kb + (size_t)ki * kv_dim, head_dim) * inv_sqrt;
        for (int ki = 0; ki < kv_len; ki++)
            if (ki > pos0 + t) sc[ki] = -1e30f;
        orc_softmax(sc, kv_len);
    }
}

/* ---- tests/test_kv_cache_gpu.c:21-54 (double-precision cpu_attention),
 * kvh = h / (nh / nkvh), generalised to n_q causal query tokens. ---------- */
void orc_attention_f64(const float* q, const float* kvc, float* out,
                       int n_heads, int n_kv_heads, int head_dim,
                       int n_q, int pos0, int kv_len, int max_seq) {
    int kv_dim = n_kv_heads * head_dim;
    float scale = 1.0f / sqrtf((float)head_dim);
    int grp = n_heads / n_kv_heads;
    if (grp < 1) grp = 1;
    float* sc = (float*)malloc(sizeof(float) * (kv_len > 0 ? kv_len : 1));
    for (int t = 0; t < n_q; t++) {
        int pos = pos0 + t;
        for (int h = 0; h < n_heads; h++) {
            int kvh = h / grp;
            const float* qh = q + ((size_t)t * n_heads + h) * head_dim;
            float* oh = out + ((size_t)t * n_heads + h) * head_dim;
            float mx = -3.4e38f;
            for (int j = 0; j < kv_len; j++) {
                if (j > pos) { sc[j] = -3.4e38f; continue; }
                double dot = 0;
                for (int d = 0; d < head_dim; d++)
                    dot += (double)qh[d] * kvc[(size_t)j * kv_dim + kvh * head_dim + d];
                sc[j] = (float)(dot * scale);
                if (sc[j] > mx) mx = sc[j];
            }
            double sum = 0;
            for (int j = 0; j < kv_len; j++) {
                if (j > pos) { sc[j] = 0; continue; }
                sc[j] = expf(sc[j] - mx);
                sum += sc[j];
            }
            float inv = (sum > 0) ? (float)(1.0 / sum) : 0.0f;
            for (int d = 0; d < head_dim; d++) {
                double acc = 0;
                for (int j = 0; j < kv_len; j++) {
                    if (j > pos) continue;
                    acc += (double)sc[j] * inv *
                           kvc[(size_t)max_seq * kv_dim + (size_t)j * kv_dim + kvh * head_dim + d];
                }
                oh[d] = (float)acc;
            }
        }
    }
    free(sc);
}

/* ---- CPU baseline: one decode token per cache, engine order. ------------ */
void orc_decode_batch(const float* const* kvcs, const float* const* qs,
                      float* const* outs, const int* lens, const int* max_seqs,
                      int n_items, int n_heads, int n_kv_heads, int head_dim,
                      int threads) {
    int kv_dim = n_kv_heads * head_dim;
    float inv_sqrt = 1.0f / sqrtf((float)head_dim);
    int maxlen = 1;
    for (int i = 0; i < n_items; i++) if (lens[i] > maxlen) maxlen = lens[i];
    long total = (long)n_items * n_heads;
#ifdef _OPENMP
    if (threads < 1) threads = 1;
    #pragma omp parallel num_threads(threads)
#endif
    {
        float* sc = (float*)malloc(sizeof(float) * maxlen);
#ifdef _OPENMP
        #pragma omp for schedule(dynamic, 1)
#endif
        for (long w = 0; w < total; w++) {
            int it = (int)(w / n_heads), h = (int)(w % n_heads);
            int kvh = h * n_kv_heads / n_heads;
            int L = lens[it];
            engine_head(qs[it] + (size_t)h * head_dim, kvcs[it],
                        outs[it] + (size_t)h * head_dim, sc, kvh, head_dim, kv_dim,
                        L - 1, L, max_seqs[it], inv_sqrt);
        }
        free(sc);
    }
}

/* ---- counter-based N(0,1) ----------------------------------------------- */
static uint64_t splitmix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

float orc_normal(uint64_t seed, uint64_t k0, uint64_t k1, uint64_t k2, uint64_t idx) {
    uint64_t h = splitmix64(seed);
    h = splitmix64(h ^ k0);
    h = splitmix64(h ^ k1);
    h = splitmix64(h ^ k2);
    h = splitmix64(h ^ idx);
    double u1 = ((double)((h >> 40) & 0xffffff) + 1.0) / 16777217.0;   /* (0,1) */
    double u2 = (double)((h >> 8) & 0xffffff) / 16777216.0;           /* [0,1) */
    return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}

void orc_fill_normal(float* out, size_t n, uint64_t seed, uint64_t k0, uint64_t k1,
                     uint64_t k2, float scale) {
    for (size_t i = 0; i < n; i++) out[i] = orc_normal(seed, k0, k1, k2, i) * scale;
}
