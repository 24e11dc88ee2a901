/* tgkv_launch.h -- kernel parameter blocks shared by the C bridge
 * (tgai_cuda_bridge.c) and the CUDA kernels (tgkv_kernels.cu).  Plain C.
 *
 * The bridge plans a launch on the host (lengths, split-sequence chunking,
 * scratch slots) and fills one of these structs; the kernels receive it by
 * value in parameter space, so a launch carries every per-item length and
 * needs no host-to-device copy of its own.
 */
#ifndef TGKV_LAUNCH_H
#define TGKV_LAUNCH_H
#include <stdint.h>
#include <cuda.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TGKV_MAX_ITEMS 1024      /* items (query rows / caches) per launch */
#define TGKV_MAX_RANKS 8         /* GPUs of one node in an output gather */
#define TGKV_TILE      32        /* positions per pipeline stage */

/* One cache buffer [2][max_seq][kv_dim] in device memory, with the device
 * address of its TMA tensor map: a 3-D map over (kv_dim, max_seq, 2) whose box
 * is (head_dim, TGKV_TILE, 1) -- one KV head's rows of one tile of K or V. */
typedef struct {
    uint64_t base;               /* device address */
    uint32_t max_seq;
    uint32_t pad;
    uint64_t tmap;               /* device address of a 64-byte aligned CUtensorMap */
    uint64_t tmap_sw;            /* bf16, head_dim 128: 128B-swizzled map, box (64,128,1), or 0 */
} TGKvCacheDesc;

/* Split-sequence decode attention.
 * For each item i (a query row) and each (head subset sub, KV head kvh) of it
 * there is one segment: the n_pos[i] positions that row attends.  Every
 * segment is cut into chunks of `chunk` positions (a multiple of the TMA tile,
 * the last chunk shorter); chunks are numbered item-major, then
 * seg = sub*n_kv_heads + kvh, then chunk index, so chunk_prefix[i] is item i's
 * first chunk and a segment's chunks are consecutive.  CTA b streams chunk b
 * (one CTA per chunk, about eight waves, balanced by the hardware block
 * scheduler).  A one-chunk segment is finished by the CTA that streams it;
 * otherwise each chunk leaves a partial in slot <chunk number> and the last
 * chunk to finish merges the segment.  GT query heads (kvh*G + sub*GT ..)
 * share each staged K/V row. */
typedef struct {
    const TGKvCacheDesc* caches; /* device table, or NULL: every item uses cache0 */
    TGKvCacheDesc cache0;
    const float* q;              /* [items][n_heads][head_dim] fp32 */
    float*       out;            /* same shape */
    const float* k_new;          /* NULL, or [items][kv_dim] fp32: row n_pos[i]-1 of item i's */
    const float* v_new;          /*   cache is written first (decode append fused in) */
    float*       part_o;         /* [n_chunks][GT][head_dim]  scratch */
    float*       part_ml;        /* [n_chunks][GT][2]         scratch */
    uint32_t*    counters;       /* [items][n_sub*n_kv_heads], zero, self-resetting */
    uint32_t*    tile_ctr;       /* tensor-core decode only: NULL (each CTA streams its
                                  * chunk), or per-segment tile queues laid out as
                                  * counters (zero, reset by the merging CTA): the
                                  * segment's CTAs take 128-position tiles from it */
    int32_t*     err;            /* device error word (0 = fine) */
    uint32_t cache_stride;       /* cache index = item * cache_stride */
    uint32_t n_items;
    uint32_t n_heads;
    uint32_t n_kv_heads;
    uint32_t n_sub;              /* head subsets per KV head = G / GT */
    uint32_t chunk;              /* positions per chunk, multiple of TGKV_TILE */
    float    qscale;             /* softmax scale * log2(e) */
    uint32_t item_base;          /* first item of this launch (q/out/counter offset) */
    /* Output gather over NVLink (KV heads split over ranks).  When
     * gather_world > 0 every finished output element is also stored at
     * gather_out[r][gather_base + its index in out] for each rank r (peer
     * memory), and the CTA that finished a segment then adds 1 to each rank's
     * *gather_flag[r] (system scope, after a system fence). */
    float*    gather_out[TGKV_MAX_RANKS];
    uint32_t* gather_flag[TGKV_MAX_RANKS];
    uint64_t  gather_base;
    uint32_t  gather_world;
    /* Failure injection for tests: nonzero makes the producer issue no loads,
     * so every wait of the launch runs out and reports through err. */
    uint32_t  stall_loads;
    /* Two-level merge for segments of more than two_level_min chunks (0:
     * never): chunks merge in groups of 16 (the last of a group to finish
     * merges it into partial slot l1_base + first + group, counting on
     * counters[gctr_base + first + group]), then the last group to finish
     * merges the group partials. */
    uint32_t  two_level_min;
    uint32_t  l1_base;
    uint32_t  gctr_base;
    /* Used when cache0.tmap is 0 (the no-allocation entry): the cache's tensor
     * map travels in the parameter block itself. */
    CUtensorMap tmap0;
    uint32_t n_pos[TGKV_MAX_ITEMS];
    uint32_t chunk_prefix[TGKV_MAX_ITEMS + 1];
} TGKvAttnParams;

/* Append of one fp32 row per item into cache (item * cache_stride) at
 * position pos[i] (batched decode), or of n_rows consecutive rows into one
 * cache starting at pos[0] (cache_stride = 0, rows_per_item = n_rows). */
typedef struct {
    const TGKvCacheDesc* caches; /* device table, or NULL: every item uses cache0 */
    TGKvCacheDesc cache0;
    const float* k;              /* [rows][kv_dim] fp32 */
    const float* v;
    uint32_t cache_stride;
    uint32_t n_items;
    uint32_t rows_per_item;
    uint32_t kv_dim;
    uint32_t pos[TGKV_MAX_ITEMS];
} TGKvAppendParams;

/* RoPE + KV write with shaders/rope.comp semantics (f32 tables). */
typedef struct {
    const float* qkv;            /* [n_tokens][q_dim + 2*kv_dim] */
    const float* cs;             /* [max_seq][head_dim/2] */
    const float* sn;
    void*        kvc;            /* cache buffer */
    float*       qout;           /* [n_tokens][q_dim] */
    uint32_t n_tokens, n_heads, n_kv_heads, head_dim, start_pos, max_seq;
    int      dtype;
} TGKvRopeParams;

/* Tensor-core causal attention of n_q consecutive query rows over one bf16
 * cache with head_dim 128 (tgkv_prefill.cu).  Query row t sits at position
 * pos0 + t.  Grid (ceil(n_q / (128/G)), n_kv_heads, n_split) in clusters of
 * (1, 1, n_split): the n_split CTAs of a row block share its KV tiles and
 * merge through distributed shared memory.  G = n_heads/n_kv_heads in
 * {1, 2, 4, 8}; n_split in [1, 8]. */
typedef struct {
    /* q as a 3-D map (128 head dims, n_heads, n_q), fp32, 128B swizzle, box
     * (32, G, 128/G): one box = 32 head dims of a CTA's 128 rows */
    CUtensorMap  qmap;
    uint64_t     tmap_sw;        /* device address: tensor map with 128B swizzle, box (64,128,1) */
    const float* q;              /* [n_q][n_heads][128] fp32, 16-byte aligned */
    float*       out;            /* same shape */
    int32_t*     err;
    uint32_t n_q, n_heads, n_kv_heads;
    uint32_t pos0;
    float    qscale;             /* softmax scale * log2(e) */
    uint32_t n_split;
    /* The turn's append fused in: NULL, or the n_q new rows [n_q][kv_dim]
     * fp32 of K and V, stored (bf16, round to nearest even) at positions
     * pos0 .. pos0 + n_q - 1 of kvc before they are read.  Each CTA stores
     * the new rows of its own KV head and tile range; CTAs of different row
     * blocks store the same bytes for the rows they share. */
    const float* k_new;
    const float* v_new;
    uint16_t*    kvc;            /* the cache buffer [2][max_seq][kv_dim], bf16 */
    uint32_t     max_seq;
} TGKvPrefillParams;

/* Causal attention of n_q consecutive query rows over one fp32 cache on the
 * CUDA cores (tgkv_prefill_f32.cu): row r at position pos0 + r attends
 * positions [0, pos0 + r] of kv ([2][max_seq][n_kv_heads * head_dim]).  q and
 * out: [n_q][n_heads][head_dim], 16-byte aligned.  head_dim 32/64/128, group
 * n_heads / n_kv_heads 1, 2, 3, 4 or 8.  Row blocks of 64 / group rows; a
 * block's K/V tiles are dealt to splits of tps tiles (tgkv_prefill_f32_plan);
 * with more than one split, part holds n_kv_heads * n_blocks * n_split
 * partials of 64 vectors x (head_dim + 4) floats and ctr one zeroed counter
 * per (KV head, block), returned to zero by the kernel. */
typedef struct {
    const float* q;
    float*       out;
    const float* kv;
    float*       part;
    uint32_t*    ctr;
    uint32_t n_q, n_heads, n_kv_heads, head_dim, max_seq, pos0;
    float    qscale;             /* softmax scale * log2(e) */
    uint32_t n_blocks, tps, n_split;
} TGKvPrefillF32Params;
void tgkv_prefill_f32_plan(uint32_t n_q, uint32_t pos0, uint32_t group, uint32_t n_kv_heads,
                           uint32_t sm_count, uint32_t* n_blocks, uint32_t* tps,
                           uint32_t* n_split);

/* Launchers (tgkv_kernels.cu, tgkv_prefill.cu, tgkv_prefill_f32.cu).  Return 0
 * on success, else a cudaError_t. */
int tgkv_launch_prefill_f32(const TGKvPrefillF32Params* p, void* stream);
int tgkv_prefill_f32_supported(uint32_t head_dim, uint32_t group);
int tgkv_launch_prefill(const TGKvPrefillParams* p, void* stream);
/* Clusters of n_split prefill CTAs resident at once on the current device. */
uint32_t tgkv_prefill_max_clusters(uint32_t n_split);
int tgkv_launch_attention(const TGKvAttnParams* p, int dtype, uint32_t head_dim,
                          uint32_t g_tile, uint32_t grid, void* stream);
/* The tensor-core decode kernel (tgkv_decode_tc.cuh): bf16 caches of
 * head_dim 128 with a swizzled tensor map, g_tile 1, 2 or 4, chunks planned
 * with tiles of 128 positions and one CTA per SM. */
int tgkv_launch_attention_tc(const TGKvAttnParams* p, uint32_t g_tile, uint32_t grid,
                             void* stream);
int tgkv_launch_append(const TGKvAppendParams* p, int dtype, void* stream);
/* One thread waits (acquire, system scope; bounded, error word on expiry)
 * until *flag has reached target (wrap-safe). */
int tgkv_launch_gather_wait(const uint32_t* flag, uint32_t target, int32_t* err, void* stream);
int tgkv_launch_rope_append(const TGKvRopeParams* p, void* stream);
/* dst (device) = a | b | c: device-mapped pointers of page-locked host
 * memory, byte counts multiples of 16, all 16-byte aligned.  A programmatic
 * dependent that overlaps the previous kernel and completes after it. */
int tgkv_launch_stage_host(const void* a, uint64_t na, const void* b, uint64_t nb,
                           const void* c, uint64_t nc, void* dst, void* stream);
/* Chunk length the planner uses for a launch of total_positions (bridge). */
uint32_t tgkv_pick_chunk(const uint32_t* n_pos, uint32_t n_items, uint32_t mult, uint32_t sm_count);
/* The same with `slots` resident CTAs per wave and chunks a multiple of tile. */
uint32_t tgkv_pick_chunk_tiled(const uint32_t* n_pos, uint32_t n_items, uint32_t mult,
                               uint32_t slots, uint32_t tile);
/* Heads per CTA the attention kernel supports for this head_dim (<= G). */
uint32_t tgkv_attention_g_tile(uint32_t head_dim, uint32_t group);
/* 1 if (dtype, head_dim) has an attention kernel. */
int tgkv_attention_supported(int dtype, uint32_t head_dim);

#ifdef __cplusplus
}
#endif
#endif
