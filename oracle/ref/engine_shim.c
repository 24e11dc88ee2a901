/* engine_shim.c -- builds the reference engine (src/tgai_engine.c) UNMODIFIED
 * into oracle/_ref/libtgai_engine_ref.so and exposes a few of its static
 * functions for pinning the oracle.  TEST INFRASTRUCTURE ONLY; compiled only
 * where the reference sources exist (oracle/Makefile target "ref").
 *
 * tgai_engine.c uses tg_dot_q4 before defining it (tgai_engine.c:901 vs 904),
 * which gcc rejects as an implicit declaration; the prototype below fixes that
 * without editing the file.  `__declspec(x)` is defined away on the command
 * line for the same reason (tgai_engine.c:3662-3748). */
#include <stdint.h>
static inline float tg_dot_q4(const float*, const uint8_t*, const float*,
                              const int16_t*, int);
#include "tgai_engine.c"

/* tg_dot: tgai_engine.c:767-785 (AVX2 path, tgai_engine.c:580-603) */
float tgref_dot(const float* a, const float* b, int n) { return tg_dot(a, b, n); }

/* softmax: tgai_engine.c:3493-3503 */
void tgref_softmax(float* x, int n) { softmax(x, n); }

/* rope without context extension: tgai_engine.c:3404-3490 */
void tgref_rope(float* q, float* k, int seq, int nh, int nkv, int dk, int pos0,
                float theta) {
    rope(q, k, seq, nh, nkv, dk, pos0, theta, 0, 0, NULL);
}

/* rope with NTK-by-parts / YaRN context extension (extend_ctx > max_seq_len);
 * returns the attention temperature mscale it reports. */
float tgref_rope_ext(float* q, float* k, int seq, int nh, int nkv, int dk, int pos0,
                     float theta, int extend_ctx, int max_seq_len) {
    float ms = 0.0f;
    rope(q, k, seq, nh, nkv, dk, pos0, theta, extend_ctx, max_seq_len, &ms);
    return ms;
}

/* After tg_forward: the last layer's post-RoPE queries [seq][nh][dk]. */
const float* tgref_work_q(TGModel* m) { return m->work_q; }

/* Geometry and storage of the engine's own KV cache (tgai_engine.c:1356-1364):
 * out[0..4] = max_seq_len, n_layers, n_heads, n_kv_heads, d_k. */
void tgref_cache_info(const TGKVCache* c, int* out) {
    out[0] = c->max_seq_len; out[1] = c->n_layers; out[2] = c->n_heads;
    out[3] = c->n_kv_heads;  out[4] = c->d_k;
}
const float* tgref_cache_k(const TGKVCache* c) { return c->k; }
const float* tgref_cache_v(const TGKVCache* c) { return c->v; }
const int*   tgref_cache_pos(const TGKVCache* c) { return c->pos; }
