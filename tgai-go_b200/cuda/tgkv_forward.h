/* tgkv_forward.h -- launchers of the whole-forward kernels (tgkv_forward.cu),
 * internal to libtgkv.so.  Every launcher queues on `stream` and returns a
 * cudaError_t value (0 = launched). */
#ifndef TGKV_FORWARD_H
#define TGKV_FORWARD_H

#include <stddef.h>
#include <stdint.h>
#include <cuda.h>                 /* CUtensorMap */

#ifdef __cplusplus
extern "C" {
#endif

/* x[t] = emb[ids[t]] (ids outside [0, rows) read row unk). */
int tgkv_fwd_embed(float* x, const float* emb, const int32_t* ids, uint32_t seq, uint32_t d,
                   uint32_t rows, int32_t unk, void* stream);

/* out[r] = x[r] * (1 / sqrt(mean(x[r]^2) + eps)) * w, for rows r < n_rows
 * (row strides in elements).  out may equal x. */
int tgkv_fwd_rmsnorm(float* out, const float* x, const float* w, uint32_t n_rows, uint32_t d,
                     uint64_t out_stride, uint64_t x_stride, float eps, void* stream);

/* y[r][c] += b[c]. */
int tgkv_fwd_bias(float* y, const float* b, uint32_t rows, uint32_t cols, void* stream);

/* h[r][j] = silu(a) * b with a = ab[r][j], b = ab[r][dff + j]; a is first
 * clamped to [-88, 88] when clamp != 0 (the dense FFN does, the experts do not). */
int tgkv_fwd_silu_mul(float* h, const float* ab, uint32_t rows, uint32_t dff, int clamp,
                      void* stream);

/* Router: logits [seq][ne] (+ bias [ne] when not NULL), top-na experts by
 * value, softmax over them.  top_ids/top_w [seq][na]; counts[ne] must be
 * zero on entry and receive, per expert, how many (token, k) pairs chose it;
 * lists[e * seq * na + i] holds those pairs (t * na + k), in no fixed order. */
int tgkv_fwd_route(const float* logits, const float* bias, int32_t* top_ids, float* top_w,
                   uint32_t* counts, uint32_t* lists, uint32_t seq, uint32_t ne, uint32_t na,
                   void* stream);

/* Expert FFN, grouped by expert.  Phase 1: for every pair p of expert e,
 * h[p][j] = silu(W1[e][j] . x[p / na]) * (W2[e][j] . x[p / na]) with
 * w12 = [ne][2 * dff][d] (W1 rows, then W2 rows).  Phase 2:
 * y[p][i] = W3[e][i] . h[p] with w3 = [ne][d][dff].  d and dff multiples of 4. */
int tgkv_fwd_expert_w12(const float* w12, const float* x, float* h, const uint32_t* counts,
                        const uint32_t* lists, uint32_t seq, uint32_t ne, uint32_t na,
                        uint32_t d, uint32_t dff, void* stream);
int tgkv_fwd_expert_w3(const float* w3, const float* h, float* y, const uint32_t* counts,
                       const uint32_t* lists, uint32_t seq, uint32_t ne, uint32_t na,
                       uint32_t d, uint32_t dff, void* stream);

/* x[t] += sum over k of top_w[t][k] * y[t * na + k] (k in order, invalid
 * experts skipped). */
int tgkv_fwd_moe_combine(float* x, const float* y, const int32_t* top_ids, const float* top_w,
                         uint32_t seq, uint32_t d, uint32_t ne, uint32_t na, void* stream);

/* Decode steps (at most tgkv_fwd_decode_rows() token rows), fused kernels,
 * launched as programmatic dependents (TGKV_PDL=0: plain launches).  pf /
 * pf_n (floats), when pf is not NULL, name weights of a later launch on the
 * stream that the kernel prefetches into L2 (w3_pf: the expert W3 tensor
 * [ne][d][dff], of which the routed experts are prefetched).
 * dec_gemv: out[r][n] for r < R, n < N from W [N][K] (mode 1: += ; mode 2:
 * SwiGLU over W = [W1; W2] of 2N rows, a clamped to +-88 when clamp != 0),
 * the input rows RMS-normalised with g first when g is not NULL, bias [N]
 * added in mode 0 when not NULL.  K and ldx multiples of 4. */
uint32_t tgkv_fwd_decode_rows(void);
int tgkv_fwd_dec_gemv(int mode, const float* w, const float* x, uint64_t ldx, const float* g,
                      const float* bias, float* out, uint64_t ldo, uint32_t R, uint32_t N,
                      uint32_t K, int clamp, const float* pf, uint64_t pf_n, void* stream);
/* Q/K/V rows of R tokens from rmsnorm(x, g) . W^T (+ bias), RoPE with the
 * cs/sn tables [max_seq][hd/2] at positions pos0 + r, queries to q_out
 * [R][q_dim], keys/values into the fp32 cache kvc [2][max_seq][kv_dim]. */
int tgkv_fwd_dec_qkv_rope(const float* w, const float* x, const float* g, const float* bias,
                          const float* cs, const float* sn, float* q_out, float* kvc, uint32_t R,
                          uint32_t d, uint32_t q_dim, uint32_t kv_dim, uint32_t hd, uint32_t pos0,
                          uint32_t max_seq, const float* pf, uint64_t pf_n, void* stream);
/* The same for R token rows of different sequences: row r at position
 * pos_rows[r] (device [R]); the rotated K rows and the V rows go to k_out /
 * v_out [R][kv_dim] (for the batched attention, which appends them). */
int tgkv_fwd_dec_qkv_rows(const float* w, const float* x, const float* g, const float* bias,
                          const float* cs, const float* sn, float* q_out, float* k_out,
                          float* v_out, uint32_t R, uint32_t d, uint32_t q_dim, uint32_t kv_dim,
                          uint32_t hd, const uint32_t* pos_rows, uint32_t max_seq,
                          const float* pf, uint64_t pf_n, void* stream);
/* Router and experts W1/W2 in one launch: for every pair p = (r, k),
 * ln = rmsnorm(x[r], g), the router's top-na of ln . router^T (+ bias) with
 * softmax weights, and h[p] = silu(W1[e_k] ln) * (W2[e_k] ln); top_ids /
 * top_w [R][na] written for tgkv_fwd_dec_w3_combine. */
int tgkv_fwd_dec_moe_w12(const float* x, const float* g, const float* router, const float* bias,
                         const float* w12, int32_t* top_ids, float* top_w, float* h, uint32_t R,
                         uint32_t d, uint32_t dff, uint32_t ne, uint32_t na, const float* w3_pf,
                         void* stream);
/* x[r] += sum_k top_w[r][k] * W3[e_k] . h[r * na + k]  (w3 = [ne][d][dff]). */
int tgkv_fwd_dec_w3_combine(const float* w3, const float* h, const int32_t* top_ids,
                            const float* top_w, float* x, uint32_t R, uint32_t d, uint32_t dff,
                            uint32_t ne, uint32_t na, const float* pf, uint64_t pf_n,
                            void* stream);

/* One decode token through all layers as ONE cooperative launch
 * (tgkv_decode_step.cu): one CTA per SM, the five phases of a layer (Q/K/V +
 * RoPE + append, split attention, out projection, router + experts W1/W2 or
 * the dense W1/W2, W3 + combine) separated by bounded grid barriers.  x [d]
 * holds the embedded token on entry and the last layer's output on return;
 * the caller zeroes state [kTgStepStateWords] (barrier count, error word,
 * attention tasks finished per head) before each launch and reads state[1]
 * after it (0, or 6 when a barrier timed out). */
enum { kTgStepMaxTasks = 128 };     /* attention partials per KV head */
enum { kTgStepStateWords = 2 + 128 };/* barrier count, error word, a task count per head */
typedef struct {
    const float *ln1, *ln2, *wqkv, *bqkv, *wo, *w12, *w3, *router, *qb;
} TGFwdStepLayer;
typedef struct {
    const TGFwdStepLayer* layers;   /* device [n_layers] */
    float* const* kvc;              /* device [n_layers]: fp32 caches [2][max_seq][kv_dim] */
    float *x, *q, *attn, *h, *part; /* [d], [q_dim], [q_dim], [na or 1][dff], partials */
    uint32_t* state;                /* barrier count, error word */
    const float *cs, *sn;           /* RoPE tables [max_seq][head_dim / 2] */
    uint32_t n_layers, d, n_heads, n_kv_heads, head_dim, dff, ne, na, pos, max_seq;
    uint32_t sx_floats;             /* max(d, q_dim) */
    float scale;                    /* score scale: 1/sqrt(head_dim) times the YaRN mscale */
} TGFwdStepParams;
int tgkv_fwd_step_supported(uint32_t d, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                            uint32_t dff, uint32_t ne, uint32_t na);
size_t tgkv_fwd_step_smem(uint32_t d, uint32_t q_dim, uint32_t dff, uint32_t ne, uint32_t na);
size_t tgkv_fwd_step_part_floats(uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim);
/* 0 launched; -1 the device cannot hold the grid resident (no cooperative
 * launch, or too few SMs for this process): nothing was queued; else a CUDA
 * error code. */
int tgkv_fwd_decode_step(const TGFwdStepParams* p, void* stream);

/* fp32 GEMM on the tensor cores (tgkv_gemm.cu): out[M][N] (row stride ldo)
 * = A[M][K] . W[N][K]^T, or += with accumulate, at fp32-product accuracy.
 * Each operand is given as its tf32-rounded part and the exact remainder
 * (tgkv_split_tf32); the kernel sums A_big.W_big + A_big.W_small +
 * A_small.W_big.  K, lda and ldw multiples of 4 (16-byte rows for TMA). */
typedef struct {
    CUtensorMap a_big, a_small;     /* [M][K], box 32 x 128, 128-byte swizzle */
    CUtensorMap w_big, w_small;     /* [N][K], box 32 x BN */
    float* out;
    uint64_t ldo;
    uint32_t M, N, K;
    int accumulate;
    int32_t* err;                   /* device error word: set when a bounded wait runs out */
    /* Grouped (one GEMM per MoE expert in one launch): group g multiplies
     * A rows [group_off[g], + group_count[g]) (device arrays, read in the
     * kernel) by W rows [g * N, (g + 1) * N); grid z = groups, y covers
     * max_rows rows.  out_rows (or NULL): the output row of packed A row r. */
    const uint32_t* group_count;
    const uint32_t* group_off;
    const uint32_t* out_rows;
    uint32_t groups, max_rows;
} TGGemmParams;
/* Fill p (host only; 0 on unsupported shapes or a failed tensor-map encode). */
int tgkv_gemm_encode(TGGemmParams* p, const float* a_big, const float* a_small, uint64_t lda,
                     const float* w_big, const float* w_small, uint64_t ldw, float* out,
                     uint64_t ldo, uint32_t M, uint32_t N, uint32_t K, int accumulate,
                     int32_t* err);
/* The grouped form: A = a_big/a_small [a_rows][K] (packed rows of every
 * group), W = w_big/w_small [groups * N][K]; M is each group's count from
 * the device. */
int tgkv_gemm_encode_grouped(TGGemmParams* p, const float* a_big, const float* a_small,
                             uint32_t a_rows, const float* w_big, const float* w_small,
                             uint32_t groups, uint32_t N, uint32_t K, float* out, uint64_t ldo,
                             const uint32_t* group_count, const uint32_t* group_off,
                             const uint32_t* out_rows, uint32_t max_rows, int32_t* err);
/* The MoE prefill's operands.  pack: from the router's counts[ne] and
 * lists[e * seq * na + i] (pairs t * na + k), the pairs of expert e become
 * rows off[e] .. off[e] + counts[e] - 1 (off = the prefix sums, written to
 * offs[ne]) of A (x's row t, split into tf32 part and remainder), and
 * rows[r] = the pair of packed row r.  silu_split: h = silu(ab[r][j]) *
 * ab[r][dff + j] for the first sum(counts) rows, split likewise. */
int tgkv_moe_pack_split(const uint32_t* counts, const uint32_t* lists, const float* x, uint32_t d,
                        uint32_t seq, uint32_t ne, uint32_t na, float* a_big, float* a_small,
                        uint32_t* offs, uint32_t* rows, void* stream);
int tgkv_moe_silu_split(const float* ab, const uint32_t* counts, uint32_t ne, uint32_t max_rows,
                        uint32_t dff, float* h_big, float* h_small, void* stream);
/* Output tile width the launch uses for an M x N product (64 or 128). */
uint32_t tgkv_gemm_bn(uint32_t M, uint32_t N);
int tgkv_gemm_launch(const TGGemmParams* p, void* stream);
/* big = x rounded to tf32 (nearest, ties away), small = x - big (exact), for
 * rows x cols (row strides ldx, ldo in elements). */
int tgkv_split_tf32(const float* x, uint64_t ldx, float* big, float* small, uint64_t ldo,
                    uint32_t rows, uint32_t cols, void* stream);

/* The bridge's device error word (tgai_cuda_bridge.c), which
 * tg_cuda_kv_device_error reads: kernels outside the bridge record their
 * bounded-wait expiries there too. */
int32_t* tgkv_bridge_err_word(void);

/* Page-locked host memory (NULL on failure). */
void* tgkv_fwd_host_alloc(size_t bytes);
void  tgkv_fwd_host_free(void* p);

#ifdef __cplusplus
}
#endif
#endif /* TGKV_FORWARD_H */
