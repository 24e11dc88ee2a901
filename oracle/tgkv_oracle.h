/* tgkv_oracle.h -- CPU oracle for the KV-cache path (TEST INFRASTRUCTURE ONLY).
 *
 * This library restates, in plain C, the reference engine's arithmetic for the
 * KV-cache path so that tests can check the CUDA path against it.  Only files
 * under tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load it, and only as the checker or the timed CPU baseline.  The
 * product library (libtgkv.so) never links or calls it.
 *
 * Parity status: pinned.  tests/golden/ holds vectors produced by the
 * reference's own code compiled from its sources (oracle/Makefile, target
 * "ref"): the engine's tg_dot/softmax/rope, the engine's softmax weights
 * dumped during real forwards of the reference fixture model, and the
 * double-precision cpu_attention of the reference's KV-cache test.
 */
#ifndef TGKV_ORACLE_H
#define TGKV_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Cache element types: same codes as TG_KV_F32 / TG_KV_BF16 of the product. */
#define ORC_F32  0
#define ORC_BF16 1

/* Dot product in the engine's AVX2 summation order (2 x 8 fused lanes, then
 * a pairwise horizontal add, then a scalar tail). src/tgai_engine.c:580-603. */
float orc_dot(const float* a, const float* b, int n);

/* In-place softmax exactly as src/tgai_engine.c:3493-3503. */
void orc_softmax(float* x, int n);

/* Interleaved-pair RoPE, non-extended path, src/tgai_engine.c:3404-3490.
 * q: [seq][n_heads][d_k], k: [seq][n_kv_heads][d_k], both rotated in place. */
void orc_rope(float* q, float* k, int seq, int n_heads, int n_kv_heads, int d_k,
              int pos0, float theta);

/* The same rotation with caller-given tables cs/sn [positions][d_k/2]
 * (absolute position pos0 + t), e.g. tables with context extension. */
void orc_rope_tables(float* x, int seq, int nh, int d_k, int pos0, const float* cs,
                     const float* sn);

/* fp32 -> bf16 bits, round to nearest even (NaN kept quiet). */
uint16_t orc_f32_to_bf16(float f);
float    orc_bf16_to_f32(uint16_t h);

/* Append n_tokens rows of K and V (fp32 source, [n][kv_dim]) at row `len` of
 * a cache laid out [2][max_seq][kv_dim] in `dtype`.  Mirrors the byte layout
 * of src/tgai_kv_cache.c:90-110 (K half then V half).  Returns 1, or 0 when
 * len + n_tokens > max_seq (capacity rule of src/tgai_kv_cache.c:95-98). */
int orc_kv_append(void* cache, int dtype, uint32_t max_seq, uint32_t kv_dim,
                  uint32_t len, const float* k, const float* v, uint32_t n_tokens);

/* Decode one cache (any dtype) to fp32 [2][max_seq][kv_dim]. */
void orc_kv_decode(const void* cache, int dtype, uint32_t max_seq, uint32_t kv_dim,
                   float* out);

/* Attention of n_q query tokens over a [2][max_seq][kv_dim] fp32 cache, in the
 * engine's order (src/tgai_engine.c:3943-4011): kvh = h*nkv/nh, scores =
 * orc_dot * (1/sqrtf(d_k)), mask ki > pos0+t to -1e30, orc_softmax over
 * kv_len, PV accumulated in float with ki ascending.
 * q, out: [n_q][n_heads][head_dim]. */
void orc_attention_engine(const float* q, const float* kvc, float* out,
                          int n_heads, int n_kv_heads, int head_dim,
                          int n_q, int pos0, int kv_len, int max_seq);

/* orc_attention_engine with the engine's YaRN temperature: scores scaled by
 * (1/sqrtf(d_k)) * mscale (src/tgai_engine.c:3947). */
void orc_attention_engine_scaled(const float* q, const float* kvc, float* out,
                                 int n_heads, int n_kv_heads, int head_dim,
                                 int n_q, int pos0, int kv_len, int max_seq, float mscale);

/* Same inputs, double accumulation, following the reference tests'
 * cpu_attention (tests/test_kv_cache_gpu.c:21-54) extended to n_q tokens:
 * query t sees positions j <= pos0 + t and j < kv_len. */
void orc_attention_f64(const float* q, const float* kvc, float* out,
                       int n_heads, int n_kv_heads, int head_dim,
                       int n_q, int pos0, int kv_len, int max_seq);

/* Softmax weights of the last query token, [n_heads][kv_len], from the
 * engine-order computation (what the engine dumps as c_attn<layer>). */
void orc_attention_weights_last(const float* q, const float* kvc, float* w,
                                int n_heads, int n_kv_heads, int head_dim,
                                int n_q, int pos0, int kv_len, int max_seq);

/* Batched decode step for the CPU baseline: for each of n_items caches,
 * attention of one query token (pos = len-1) over fp32 caches, engine order.
 * Parallel over (item, head) with `threads` OpenMP threads (1 = the
 * reference's single-threaded loop). */
void orc_decode_batch(const float* const* kvcs, const float* const* qs,
                      float* const* outs, const int* lens, const int* max_seqs,
                      int n_items, int n_heads, int n_kv_heads, int head_dim,
                      int threads);

/* Counter-based N(0,1) generator: value for (seed, key0..key3, index).
 * splitmix64 mixing of the key tuple, two 24-bit uniforms, Box-Muller. */
float orc_normal(uint64_t seed, uint64_t k0, uint64_t k1, uint64_t k2, uint64_t idx);
void  orc_fill_normal(float* out, size_t n, uint64_t seed, uint64_t k0, uint64_t k1,
                      uint64_t k2, float scale);

#ifdef __cplusplus
}
#endif
#endif
