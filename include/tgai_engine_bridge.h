/* tgai_engine_bridge.h -- whole-model forward on a B200 behind the engine's
 * CUDA seam.
 *
 * Two layers:
 *
 *  1. The engine-facing entry points, with the signatures and contract of the
 *     reference's cuda/tgai_cuda_bridge.h:31-60.  tgai_engine.c built with
 *     TG_ENGINE_HAS_CUDA_BRIDGE calls tg_engine_cuda_forward first in
 *     tg_forward (src/tgai_engine.c:4373-4378) and runs its CPU path only when
 *     it returns 0.  tg_engine_cuda_init reads the model through the engine's
 *     own exported accessors (tg_config, find_weight, get_cached_weight;
 *     src/tgai_engine.h:70-76), looked up in the running process, so this
 *     library needs no engine headers or link-time dependency.
 *
 *  2. A neutral C-ABI (tg_fwd_*) that takes the configuration and an fp32
 *     weight getter, for callers that hold weights without the engine.
 *
 * Model scope (what init accepts; anything else returns 0 with a reason and
 * the engine keeps its CPU path, the reference bridge's contract):
 * RMSNorm pre-norm blocks, Q/K/V projections with optional biases, GQA
 * (n_heads % n_kv_heads == 0), interleaved-pair RoPE, causal attention over
 * the layer's KV cache, out projection, and either the dense SwiGLU FFN
 * (n_experts == 0) or the routed MoE FFN (1..16 experts, top-1..8, optional
 * per-expert router bias); final RMSNorm and the tied-embedding LM head.
 * head_dim 32, 64 or 128.  QK-Norm and block AttnRes models are refused.
 *
 * Sequences ("slots") are keyed by the caller's pointer (the engine's
 * TGKVCache*, cuda/tgai_cuda.cu:1656-1672); each slot owns one KV cache per
 * layer, a stream and its workspaces, so different slots may run
 * concurrently from different threads.  One slot must not be used by two
 * threads at once.
 *
 * Errors: functions return 0 / NULL and set a thread-local message
 * (tg_fwd_last_error).  Nothing falls back to a CPU computation.
 */
#ifndef TGAI_ENGINE_BRIDGE_H
#define TGAI_ENGINE_BRIDGE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- engine-facing entry points (cuda/tgai_cuda_bridge.h:31-60) -------- */
typedef struct TGModel TGModel;        /* the engine's model (opaque here) */
typedef struct TGKVCache TGKVCache;    /* the engine's KV cache: the slot key */

/* Idempotent.  1 = the GPU forward has taken over this model; 0 = keep the
 * CPU path (not an error; tg_engine_cuda_reason says why). */
int  tg_engine_cuda_init(TGModel* m);

/* One forward of seq_len tokens at positions cache_pos .. cache_pos+seq_len-1
 * of the sequence keyed by `cache`.  Returns 1 and sets *out_logits (host
 * memory owned by the slot, [vocab], valid until that slot's next forward),
 * or 0 (counted in tg_engine_cuda_fallbacks). */
int  tg_engine_cuda_forward(TGModel* m, const int32_t* input_ids, int seq_len,
                            TGKVCache* cache, int cache_pos,
                            const float** out_logits);

void tg_engine_cuda_reset(void);                   /* clear every slot's KV */
void tg_engine_cuda_reset_slot(TGKVCache* cache);  /* clear one sequence's KV */
void tg_engine_cuda_free_slot(TGKVCache* cache);   /* release one sequence */
void tg_engine_cuda_shutdown(void);                /* release the model */

int         tg_engine_cuda_ready(void);            /* 1 = taken over */
const char* tg_engine_cuda_reason(void);
long long   tg_engine_cuda_calls(void);            /* successful GPU forwards */
long long   tg_engine_cuda_fallbacks(void);        /* forwards that returned 0 */

/* Slot introspection exported by the reference bridge
 * (cuda/tgai_cuda_bridge.c, tg_gpu_kv_slot_*): -1 before take-over.
 * slot_of: slot index of a sequence; slot_seq: positions it holds;
 * slot_live / slot_max: slots in use / allowed (TGAI_CUDA_KV_SLOTS, default
 * 16); slot_rejects: requests refused for want of a slot. */
int       tg_gpu_kv_slot_of(void* cache);
int       tg_gpu_kv_slot_seq(void* cache);
int       tg_gpu_kv_slot_live(void);
int       tg_gpu_kv_slot_max(void);
long long tg_gpu_kv_slot_rejects(void);
long long tg_gpu_cuda_calls(void);
long long tg_gpu_cuda_fallbacks(void);

/* ---- neutral C-ABI ------------------------------------------------------ */
typedef struct TGFwdModel TGFwdModel;

typedef struct {
    uint32_t n_layers;
    uint32_t d_model;
    uint32_t n_heads;
    uint32_t n_kv_heads;       /* 0 = n_heads */
    uint32_t head_dim;         /* 0 = d_model / n_heads */
    uint32_t d_ff;
    uint32_t vocab_size;
    uint32_t max_seq_len;      /* KV capacity per slot */
    uint32_t n_experts;        /* 0 = dense SwiGLU FFN */
    uint32_t n_activated;      /* top-k of the MoE router */
    float    rope_theta;
    int32_t  unk_id;           /* out-of-range token ids map here */
} TGFwdConfig;

/* Weight getter: the fp32 host copy of tensor `name` (row-major, the
 * engine's names, e.g. "blocks.3.attn.q_proj.weight"), with its shape in
 * shape[0..1] (rows, columns; 1-D tensors report columns = 1), or NULL when
 * the model has no such tensor.  The pointer is read during tg_fwd_create
 * only. */
typedef const float* (*TGFwdWeightFn)(void* ctx, const char* name, uint32_t shape[2]);

/* Uploads every weight to the current CUDA device.  NULL on error. */
TGFwdModel* tg_fwd_create(const TGFwdConfig* cfg, TGFwdWeightFn get, void* ctx);
void        tg_fwd_destroy(TGFwdModel* m);

/* Forward of the sequence keyed by `key` (any pointer; NULL is slot 0).
 * Returns the slot's host logits [vocab] or NULL. */
const float* tg_fwd_forward(TGFwdModel* m, const void* key, const int32_t* ids,
                            uint32_t seq_len, uint32_t cache_pos);

int      tg_fwd_reset_slot(TGFwdModel* m, const void* key);   /* 1 if it existed */
int      tg_fwd_free_slot(TGFwdModel* m, const void* key);    /* 1 if it existed */
void     tg_fwd_reset_all(TGFwdModel* m);
uint32_t tg_fwd_slot_count(const TGFwdModel* m);
/* Last position written + 1 for the slot, or -1 when it has none. */
int      tg_fwd_slot_last_pos(const TGFwdModel* m, const void* key);
uint64_t tg_fwd_weight_bytes(const TGFwdModel* m);
/* Kernel launches and GEMM calls issued by the last forward of this thread. */
uint32_t tg_fwd_last_launches(void);

/* One-token forwards of different sequences that are in flight at the same
 * time (from several threads) run as one pass over the weights, up to 4 at a
 * time: the reference bridge's per-slot streams (cuda/tgai_cuda_bridge.c:
 * 147-162) each read every weight.  Tokens decoded in such batches of two or
 * more so far, and the number of those batches.  TGKV_FWD_BATCH=0 turns the
 * batching off. */
void tg_fwd_batch_stats(const TGFwdModel* m, uint64_t* tokens, uint64_t* batches);

/* The fp32 GEMM the forward's prefill runs, as a standalone call on device
 * buffers: out[M][N] (row stride ldo) = x[M][K] . w[N][K]^T (row strides ldx,
 * ldw), or += with accumulate, on the sm_100a tensor cores at fp32-product
 * accuracy (each operand split into its tf32 part and exact remainder, three
 * products summed).  K, ldx and ldw multiples of 4.  Allocates the split
 * operands for the call and waits for `stream`.  1 = done, 0 = failed (reason
 * in tg_fwd_last_error).  Replaces the reference bridge's gemm_f32 /
 * cublasSgemm (cuda/tgai_cuda.cu:473-479). */
int tg_fwd_gemm_f32(uint32_t M, uint32_t N, uint32_t K, const float* x, uint32_t ldx,
                    const float* w, uint32_t ldw, float* out, uint32_t ldo, int accumulate,
                    void* stream);
const char* tg_fwd_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* TGAI_ENGINE_BRIDGE_H */
