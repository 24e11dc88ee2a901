/* tgai_cuda_bridge.h -- the thin C-ABI layer between TGAI GO's host C code and
 * the CUDA kernels of the KV-cache path.
 *
 * Replaces the role of cuda/tgai_cuda_bridge.{h,c} (cuda/tgai_cuda_bridge.h:
 * 31-60) for this path: host C code (the KV-cache API, the backend table, the
 * GPU dispatch router) reaches CUDA only through these functions.  Plain C
 * types only; device memory is passed as addresses, streams as void*
 * (cudaStream_t, NULL = legacy default stream).
 *
 * Return convention (as the reference bridge): int 1 = done, 0 = failed with
 * the reason in tg_cuda_kv_last_error().  No function falls back to the CPU.
 *
 * The whole-forward entry points of the reference bridge (tg_engine_cuda_init
 * / forward / reset_slot / free_slot / shutdown, cuda/tgai_cuda_bridge.h:
 * 31-53) need the model's projections and FFN and are not part of this path.
 */
#ifndef TGAI_CUDA_BRIDGE_H
#define TGAI_CUDA_BRIDGE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- device and memory -------------------------------------------------- */
int         tg_cuda_kv_init(void);              /* idempotent; 1 = a CUDA device is usable */
/* Make `device` this thread's device for the library (one process per GPU
 * calls this before anything else; default: the runtime's current device). */
int         tg_cuda_kv_set_device(int device);
void        tg_cuda_kv_shutdown(void);
int         tg_cuda_kv_ready(void);
const char* tg_cuda_kv_last_error(void);        /* thread-local */
const char* tg_cuda_kv_device_name(void);
uint64_t    tg_cuda_kv_device_mem(void);
int         tg_cuda_kv_sm_count(void);

void* tg_cuda_kv_malloc(size_t bytes);          /* zero-filled; NULL on failure */
void  tg_cuda_kv_free(void* p);
int   tg_cuda_kv_h2d(void* dst, const void* src, size_t bytes, void* stream);
/* Host to device on `stream`, asynchronous also when stream is NULL (the
 * legacy default stream), where tg_cuda_kv_h2d copies synchronously.  A
 * pageable source may be reused as soon as this returns. */
int   tg_cuda_kv_h2d_async(void* dst, const void* src, size_t bytes, void* stream);
/* Device to host on `stream`, asynchronous also when stream is NULL (for a
 * page-locked destination; a pageable one is copied before the call returns). */
int   tg_cuda_kv_d2h_async(void* dst, const void* src, size_t bytes, void* stream);
/* dst (device) = a | b | c, read by one small kernel from page-locked host
 * memory (a, b, c: device pointers of such memory, tg_cuda_kv_host_device_ptr;
 * sizes and addresses multiples of 16 bytes).  Queued as a programmatic
 * dependent: it overlaps the previous kernel on `stream` and completes after
 * it. */
int   tg_cuda_kv_stage_host(void* dst, const void* a, size_t na, const void* b, size_t nb,
                            const void* c, size_t nc, void* stream);
int   tg_cuda_kv_d2h(void* dst, const void* src, size_t bytes, void* stream);
int   tg_cuda_kv_memset(void* dst, int value, size_t bytes, void* stream);
/* The h2d/d2h/memset calls block when stream is NULL; otherwise they are
 * queued on stream and tg_cuda_kv_sync(stream) waits for them. */
int   tg_cuda_kv_sync(void* stream);

/* Read and clear the device error word set by kernels whose bounded waits
 * expired (0 = none).  Blocks on the whole device. */
int   tg_cuda_kv_device_error(void);

/* Streams and events, for overlapping host<->device copies with kernels.
 * Streams are non-blocking (no implicit order with the legacy default stream,
 * NULL); order them with events. */
void* tg_cuda_kv_stream_create(void);
void  tg_cuda_kv_stream_destroy(void* stream);
void* tg_cuda_kv_event_create(void);
void  tg_cuda_kv_event_destroy(void* event);
int   tg_cuda_kv_event_record(void* event, void* stream);
/* Later work on `stream` waits for `event`'s last record. */
int   tg_cuda_kv_stream_wait(void* stream, void* event);

/* The device address of page-locked host memory (the host address itself
 * under unified addressing), or NULL for pageable memory: kernels can write
 * results straight into it over PCIe. */
void* tg_cuda_kv_host_device_ptr(const void* host);

/* CUDA IPC between the processes of one node (one per GPU): the 64-byte
 * handle of a tg_cuda_kv_malloc'ed buffer, a peer's buffer opened from its
 * handle (peer access enabled; NULL on failure), and closing it again. */
int   tg_cuda_kv_ipc_handle(const void* dev, void* handle64);
void* tg_cuda_kv_ipc_open(const void* handle64);
void  tg_cuda_kv_ipc_close(void* dev);

/* Queue a wait on stream until the 32-bit counter at flag (device memory)
 * reaches target (wrap-safe compare; acquire at system scope).  Bounded: after
 * ~2 s the device error word is set and the stream moves on. */
int   tg_cuda_kv_gather_wait(const uint32_t* flag, uint32_t target, void* stream);

/* Testing hook: make the next `n` tg_cuda_kv_malloc calls fail (0 = off).
 * Also set at start-up from TGKV_FAIL_ALLOC. */
void  tg_cuda_kv_inject_alloc_failures(int n);

/* ---- kernels ------------------------------------------------------------ */

/* Cache descriptor as the kernels read it (same layout as TGKvCacheDesc). */
typedef struct {
    uint64_t base;
    uint32_t max_seq;
    uint32_t pad;
    uint64_t tmap;               /* from tg_cuda_kv_tmap_create / _write */
    uint64_t tmap_sw;            /* bf16 head_dim 128 caches: tg_cuda_kv_tmap_sw_create, or 0 */
} TGCudaCacheDesc;

/* TMA tensor map of a cache buffer for the attention kernel, in device memory
 * (128 bytes).  create: allocates it (free with tg_cuda_kv_free); write:
 * encodes into existing device memory.  Blocks. */
void* tg_cuda_kv_tmap_create(int dtype, uint64_t base, uint32_t max_seq, uint32_t n_kv_heads,
                             uint32_t head_dim);
int   tg_cuda_kv_tmap_write(int dtype, uint64_t base, uint32_t max_seq, uint32_t n_kv_heads,
                            uint32_t head_dim, void* tmap_dev);
/* The second map of a bf16 head_dim-128 cache for the tensor-core suffix
 * kernel: 128-byte swizzle, box (64 dims, 128 positions, 1). */
void* tg_cuda_kv_tmap_sw_create(uint64_t base, uint32_t max_seq, uint32_t n_kv_heads);

/* Append rows (fp32 device sources [n_rows][kv_dim]) into one cache starting at
 * row `row0`, storing dtype (0 = fp32, 1 = bf16 round-to-nearest-even). */
int tg_cuda_kv_append(int dtype, TGCudaCacheDesc cache, uint32_t kv_dim, uint32_t row0,
                      const float* k, const float* v, uint32_t n_rows, void* stream);

/* Append one row per item i into cache table[i] at position pos[i] (host
 * array).  k, v: fp32 device [n_items][kv_dim]. */
int tg_cuda_kv_append_batch(int dtype, const TGCudaCacheDesc* table_dev, uint32_t kv_dim,
                            const uint32_t* pos, uint32_t n_items,
                            const float* k, const float* v, void* stream);

/* One attention call: item i attends positions [0, n_pos[i]) of its cache
 * with query row i of q (fp32 [n_items][n_heads][head_dim]) into row i of out.
 * Items use table_dev[i] when table_dev is set, else `cache`. */
typedef struct {
    int      dtype;
    uint32_t n_heads, n_kv_heads, head_dim;
    TGCudaCacheDesc        cache;
    const TGCudaCacheDesc* table_dev;
    const float*    q;
    float*          out;
    const float*    k_new;          /* optional fp32 [n_items][kv_dim]: written as row */
    const float*    v_new;          /*   n_pos[i]-1 of item i's cache before attending */
    const uint32_t* n_pos;          /* host array [n_items], each >= 1 */
    uint32_t        n_items;
    float           scale;          /* softmax scale (1/sqrt(head_dim)) */
    void*           scratch;        /* device, >= tg_cuda_kv_attn_scratch_bytes() */
    uint32_t*       counters;       /* device, zeroed, >= tg_cuda_kv_attn_counters() */
    /* Optional output gather over NVLink (gather_world 0 = off; at most 8):
     * every output element is also stored at gather_out[r][gather_base + its
     * index in out] on each rank r, and each finished (item, KV head, head
     * subset) adds 1 to every rank's *gather_flag[r].  Peer pointers come from
     * tg_cuda_kv_ipc_open; index gather_world-1 may be this rank's own. */
    float*          gather_out[8];
    uint32_t*       gather_flag[8];
    uint64_t        gather_base;
    uint32_t        gather_world;
} TGCudaAttnCall;

int      tg_cuda_kv_attn_supported(int dtype, uint32_t head_dim);
uint64_t tg_cuda_kv_attn_scratch_bytes(const TGCudaAttnCall* c);
uint64_t tg_cuda_kv_attn_counters(const TGCudaAttnCall* c);
/* (item, KV head, head subset) segments of a split-sequence call: each is
 * finished once, so a gather receives this many arrivals per rank. */
uint64_t tg_cuda_kv_attn_segments(const TGCudaAttnCall* c);
/* 1 if the call (with k_new/v_new: a suffix's new rows) runs as one launch
 * of the tensor-core suffix kernel with the append fused in. */
int tg_cuda_kv_attn_fuses_suffix(const TGCudaAttnCall* c);
/* Launches made by the last tg_cuda_kv_attention on this thread. */
uint32_t tg_cuda_kv_attn_last_launches(void);
/* Kernel family of this thread's last tg_cuda_kv_attention call:
 * 0 none, 1 split-sequence on CUDA cores (tgkv_kernels.cu), 2 tensor-core
 * suffix (tgkv_prefill.cu), 3 tensor-core split-sequence decode
 * (tgkv_decode_tc.cuh; bf16 head_dim-128 caches, TGKV_DECODE_TC=0 turns it
 * off), 4 causal block of query rows over an fp32 cache on CUDA cores
 * (tgkv_prefill_f32.cu; TGKV_PREFILL=0 turns it off). */
int tg_cuda_kv_attn_last_kernel(void);
/* CTAs per row block (KV split) of the last tensor-core suffix launch. */
uint32_t tg_cuda_kv_attn_last_split(void);
int      tg_cuda_kv_attention(const TGCudaAttnCall* c, void* stream);

/* RoPE + KV write, shaders/rope.comp semantics (see TGBackend.rope). */
int tg_cuda_kv_rope_append(int dtype, const float* qkv, const float* cs, const float* sn,
                           void* kvc, float* qout, uint32_t n_tokens, uint32_t n_heads,
                           uint32_t n_kv_heads, uint32_t head_dim, uint32_t start_pos,
                           uint32_t max_seq, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TGAI_CUDA_BRIDGE_H */
