/* tgai_kv_cache.h -- per-layer KV cache on a B200, behind TGAI GO's KV-cache API.
 *
 * The first block keeps the reference interface of src/tgai_kv_cache.h:41-76
 * (same names, argument meaning, return values and error behaviour) so that
 * existing callers link unchanged.  The cache layout is the reference's
 * (src/tgai_kv_cache.h:15-21): one device buffer [2][max_seq][kv_dim],
 * kv_dim = n_kv_heads * head_dim, the K half first and the V half at element
 * offset max_seq * kv_dim, positions [0, len) valid.
 *
 * Everything after "Additive extensions" is new API; the reference has no
 * counterpart unless one is cited.
 *
 * Threading: a cache must not be used from two threads at once (as in the
 * reference).  tg_kv_last_error() is thread-local here (the reference keeps
 * one process-global buffer, src/tgai_kv_cache.c:22-26).
 */
#ifndef TGAI_KV_CACHE_H
#define TGAI_KV_CACHE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct TGKvCache TGKvCache;

/* ---- Reference interface (src/tgai_kv_cache.h:41-76) ------------------- */

/* Replaces tg_kv_create (src/tgai_kv_cache.h:41, .c:28-69).  fp32 storage.
 * Uses the selected backend (tg_be_select("cuda") first); NULL on failure with
 * the reason in tg_kv_last_error().  The buffer is zero-filled once. */
TGKvCache* tg_kv_create(uint32_t max_seq, uint32_t n_kv_heads, uint32_t head_dim);

/* Replaces tg_kv_destroy (src/tgai_kv_cache.h:43, .c:71-76). */
void tg_kv_destroy(TGKvCache* c);

/* Replaces tg_kv_reset (src/tgai_kv_cache.h:46, .c:78-83): len = 0; memory kept. */
void tg_kv_reset(TGKvCache* c);

/* Replaces tg_kv_len / tg_kv_capacity (src/tgai_kv_cache.h:49-52). */
uint32_t tg_kv_len(const TGKvCache* c);
uint32_t tg_kv_capacity(const TGKvCache* c);

/* Replaces tg_kv_device_handle (src/tgai_kv_cache.h:56): here the raw device
 * address of the [2][max_seq][kv_dim] buffer (what TGBackend.attention takes
 * as `kvc`). */
void* tg_kv_device_handle(TGKvCache* c);

/* Replaces tg_kv_host_ptr (src/tgai_kv_cache.h:60): always NULL, the cache
 * lives in HBM and is not host-mappable. */
float* tg_kv_host_ptr(TGKvCache* c);

/* Replaces tg_kv_append (src/tgai_kv_cache.h:67-70, .c:90-110): append
 * n_tokens rows of K and V from HOST memory ([n_tokens][kv_dim] fp32 each).
 * Returns 1, or 0 with "capacity exceeded" when len + n_tokens > max_seq, or
 * on NULL arguments.  n_tokens == 0 returns 1.  Blocks until the rows are in
 * the cache; bf16 caches store round-to-nearest-even. */
int tg_kv_append(TGKvCache* c, const float* k_src, const float* v_src,
                 uint32_t n_tokens);

/* Replaces tg_kv_advance (src/tgai_kv_cache.h:73, .c:112-116): len += n,
 * clamped to capacity. */
void tg_kv_advance(TGKvCache* c, uint32_t n_tokens);

/* Replaces tg_kv_last_error (src/tgai_kv_cache.h:76). */
const char* tg_kv_last_error(void);

/* ---- Additive extensions ------------------------------------------------ */

/* Storage element types. */
#define TG_KV_F32  0
#define TG_KV_BF16 1

/* tg_kv_create with a storage type (TG_KV_F32 or TG_KV_BF16). */
TGKvCache* tg_kv_create_ex(uint32_t max_seq, uint32_t n_kv_heads, uint32_t head_dim,
                           int dtype);

int      tg_kv_dtype(const TGKvCache* c);
uint32_t tg_kv_n_kv_heads(const TGKvCache* c);
uint32_t tg_kv_head_dim(const TGKvCache* c);

/* Truncate to n positions (n <= len), the LCP prefix-reuse step of
 * python/tgai_go/_session.py:137-163.  Same effect as tg_kv_reset followed by
 * tg_kv_advance(n); rows [0, n) are untouched.  /clear is n = 0.
 * Returns 0 with an error if n > len. */
int tg_kv_truncate(TGKvCache* c, uint32_t n);

/* Append n_tokens rows from DEVICE memory (fp32 [n_tokens][kv_dim] each),
 * asynchronously on `stream` (a cudaStream_t; NULL = legacy default stream).
 * Same capacity rule as tg_kv_append; len advances at once on the host. */
int tg_kv_append_dev(TGKvCache* c, const float* k_dev, const float* v_dev,
                     uint32_t n_tokens, void* stream);

/* Causal attention of the last n_q cached positions' queries over the cache,
 * asynchronously on `stream`.  q_dev, out_dev: fp32 [n_q][n_heads][head_dim]
 * in device memory.  Query t sits at position p = len - n_q + t and sees
 * positions [0, p]; q head h reads KV head h * n_kv_heads / n_heads
 * (src/tgai_engine.c:3951).  Scores are scaled by 1/sqrt(head_dim).
 * Requires n_heads % n_kv_heads == 0 and 1 <= n_q <= len. */
int tg_kv_attention(TGKvCache* c, const float* q_dev, float* out_dev,
                    uint32_t n_heads, uint32_t n_q, void* stream);

/* Score scale used by tg_kv_attention and the batch calls of this cache:
 * (1/sqrt(head_dim)) * mscale, with mscale the engine's YaRN temperature
 * (src/tgai_engine.c:3947; tg_kv_rope_tables reports it).  Default 1. */
void tg_kv_set_attn_mscale(TGKvCache* c, float mscale);

/* Copy the whole [2][max_seq][kv_dim] buffer (raw storage bytes) to host
 * memory `dst` of tg_kv_bytes(c) bytes.  Blocks. */
uint64_t tg_kv_bytes(const TGKvCache* c);
int      tg_kv_download(const TGKvCache* c, void* dst);

/* RoPE tables for TGBackend.rope: cos/sin of positions pos0 .. pos0+n_pos-1,
 * host arrays [n_pos][head_dim/2], from the engine's formula
 * (src/tgai_engine.c:3404-3460): freq_i = 1/theta^(i/head_dim), and when
 * extend_ctx > max_seq_len the NTK-by-parts interpolation between the
 * extrapolated and interpolated frequencies.  *mscale_out (optional) gets the
 * YaRN attention temperature the engine multiplies into 1/sqrt(head_dim)
 * (1 without extension).  Rotating with these tables gives the engine's
 * bits.  Returns 0 on bad arguments. */
int tg_kv_rope_tables(float theta, uint32_t head_dim, uint32_t pos0, uint32_t n_pos,
                      uint32_t extend_ctx, uint32_t max_seq_len, float* cos_out,
                      float* sin_out, float* mscale_out);

/* A turn's suffix in one call: append n rows of K and V (fp32 device
 * [n][kv_dim], as tg_kv_append_dev) at positions len .. len + n - 1, then
 * the causal attention of their n queries (as tg_kv_attention with n_q = n);
 * len grows by n.  The engine writes a turn's K/V and then attends it
 * (src/tgai_engine.c:3923-4011): the pair in one call, the append kernel then
 * the attention.  With TGKV_FUSE_SUFFIX=1, on a bf16 head_dim-128 cache with
 * at least 128 (row, head) pairs and 16-byte aligned pointers, it is ONE
 * launch of the tensor-core suffix kernel, which stores the new rows itself
 * before it reads them (slower on the measured turn shapes, hence opt-in).
 * Returns 0 on capacity or argument errors (nothing launched). */
int tg_kv_append_attention(TGKvCache* c, const float* k_dev, const float* v_dev,
                           const float* q_dev, float* out_dev, uint32_t n_heads, uint32_t n,
                           void* stream);

/* Attention without any allocation.  No counterpart in the reference.
 *
 * For callers that cannot allocate device memory at this point: code running
 * inside a host allocator hook or under a fixed device-memory budget, or an
 * engine that owns every buffer itself and hands this library only raw
 * addresses.  Same semantics as tg_kv_attention over a caller-owned cache
 * buffer `kvc` ([2][max_seq][n_kv_heads*head_dim], dtype TG_KV_F32/BF16) whose
 * first kv_len rows are valid: the last n_q positions' queries (q, out: fp32
 * [n_q][n_heads][head_dim], device) attend causally; async on `stream`.
 *
 * Scratch comes from a static 4 MiB device array inside the library, which
 * every GPU that loads the library keeps until exit; calls that need more are
 * rejected (return 0, reason in tg_kv_last_error()), as are n_q > 1024.  The
 * function calls no cudaMalloc/cudaFree.  The first call on each device does a
 * one-time set-up (the array's device address) and should come before any
 * stream capture.  All calls share the array: calls that overlap on the GPU
 * (other streams, other threads) race; order them on one stream.
 *
 * Its kernel's waits are bounded (about 2 s).  A wait that runs out leaves
 * that call's output undefined and records a code in the array's error word,
 * which later calls do not clear: read it with tg_kv_attention_static_error. */
int tg_kv_attention_static(const void* kvc, int dtype, uint32_t max_seq, uint32_t n_kv_heads,
                           uint32_t head_dim, uint32_t kv_len, const float* q, float* out,
                           uint32_t n_heads, uint32_t n_q, void* stream);

/* The error word of tg_kv_attention_static on the current device, after
 * waiting for `stream`: 0 if every call since the last read finished its
 * waits, else the code of a wait that ran out (1: a K/V stage never arrived,
 * 2: a stage was never released); the word is cleared once returned.  -1 if
 * the word could not be read (reason in tg_kv_last_error()).  Allocates
 * nothing.  No counterpart in the reference. */
int tg_kv_attention_static_error(void* stream);

/* Failure injection for tests: the next n_calls calls of
 * tg_kv_attention_static launch with their K/V loads held back, so their
 * waits run out (about 2 s each) and report through
 * tg_kv_attention_static_error.  0 cancels.  No counterpart in the reference. */
void tg_kv_attention_static_inject_stall(int n_calls);

/* ---- Batched decode over many caches (one layer of many sequences) ------- */

typedef struct TGKvBatch TGKvBatch;

/* A plan over n caches of equal n_kv_heads, head_dim and dtype (up to 1024
 * per plan), for n_heads query heads.  The plan owns its split-sequence
 * scratch and device descriptor table.  NULL on failure. */
TGKvBatch* tg_kv_batch_create(TGKvCache* const* caches, uint32_t n, uint32_t n_heads);
void       tg_kv_batch_destroy(TGKvBatch* b);

/* One decode step for every cache i of the plan: append row i of k_new/v_new
 * (fp32 [n][kv_dim], device) at position len_i, then attend query row i of q
 * (fp32 [n][n_heads][head_dim], device) over positions [0, len_i] into row i
 * of out (same shape).  Each cache's len grows by one.  Async on `stream`;
 * one kernel launch per 1024 caches (the append is fused into the attention).
 * Returns 0 (nothing launched) if any cache is full. */
int tg_kv_batch_decode(TGKvBatch* b, const float* q, const float* k_new,
                       const float* v_new, float* out, void* stream);

/* The same step from HOST buffers: copies q/k_new/v_new in (pinned host memory
 * gives async copies), runs the step and copies out back, all on `stream`.
 * The caller synchronises `stream` before reading out_host. */
int tg_kv_batch_decode_host(TGKvBatch* b, const float* q_host, const float* k_host,
                            const float* v_host, float* out_host, void* stream);

/* Number of kernel launches the last tg_kv_batch_decode made (for reports). */
uint32_t tg_kv_batch_last_launches(const TGKvBatch* b);

/* ---- Output gather over NVLink (KV heads split over the GPUs of a node) --
 *
 * With the KV heads of one long context split into groups, one per GPU (one
 * process each), every rank attends its own heads and all ranks need every
 * head's output.  The attention kernel itself stores each finished output
 * element into every rank's gathered buffer (peer memory over NVLink) and
 * counts arrivals there, replacing a separate all-gather.  Without a GPU
 * fault nobody waits forever: the wait is bounded (~2 s) and reports through
 * tg_cuda_kv_device_error. */

typedef struct TGKvGather TGKvGather;

/* This rank's side of a gather among `world` ranks (<= 8): one device
 * allocation holding two buffers of gathered outputs [world][elems] fp32
 * (rank r's at [r*elems, (r+1)*elems)), used by alternate calls, and an
 * arrival counter for each.  NULL on failure. */
TGKvGather* tg_kv_gather_create(uint32_t world, uint32_t rank, uint64_t elems);
/* Closes the peers' buffers and frees this rank's.  Call on every rank after
 * all ranks have finished their last gathered step (a barrier). */
void        tg_kv_gather_destroy(TGKvGather* g);
/* This rank's 64-byte IPC handle. */
int tg_kv_gather_export(const TGKvGather* g, void* handle64);
/* Open the other ranks' allocations: `world` handles of 64 bytes in rank
 * order (this rank's own entry is not opened).  Every rank exports before any
 * rank imports. */
int tg_kv_gather_import(TGKvGather* g, const void* handles);
/* Device address of the gathered outputs [world][elems] of the last call on
 * this object (the first buffer before any call). */
float* tg_kv_gather_buffer(const TGKvGather* g);

/* tg_kv_batch_decode whose outputs also land in every rank's gathered buffer
 * (this rank's slice: elems = n * n_heads * head_dim), followed by a wait on
 * `stream` until every rank's outputs of this step have arrived here.  All
 * ranks make the same sequence of calls with plans of the same shape.
 *
 * One gather object can serve every layer and step.  A call's gathered
 * outputs (tg_kv_gather_buffer right after it) stay valid until the call after
 * next on the object, on every rank: queue their consumers on `stream` before
 * this rank's next call on the object (or order them before it with an
 * event); the next call's stores then go to the other buffer, and no rank's
 * call after that starts storing before this rank's next call has run. */
int tg_kv_batch_decode_gather(TGKvBatch* b, const float* q, const float* k_new,
                              const float* v_new, float* out, TGKvGather* g, void* stream);
/* The same from host buffers; out_host receives the whole gathered
 * [world][n][n_heads][head_dim]. */
int tg_kv_batch_decode_gather_host(TGKvBatch* b, const float* q_host, const float* k_host,
                                   const float* v_host, float* out_host, TGKvGather* g,
                                   void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TGAI_KV_CACHE_H */
