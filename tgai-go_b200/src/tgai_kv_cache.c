/* tgai_kv_cache.c -- TGAI GO's KV-cache API on a B200.
 *
 * Host C.  Follows the reference implementation's rules (src/tgai_kv_cache.c):
 * argument checks and the 64 GB request cap at create (:28-44), memory from
 * the selected backend (:33, :55, :74), len-only reset (:78-83), the capacity
 * rule of append (:95-98) and the clamped advance (:112-116).  Device work
 * goes through tgai_gpu_dispatch.c / tgai_cuda_bridge.c; nothing here falls
 * back to the CPU.
 */
#include "tgai_kv_cache.h"
#include "tgai_backend.h"
#include "tgai_cuda_bridge.h"
#include "tgai_gpu_dispatch.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

struct TGKvCache {
    uint32_t max_seq, n_kv_heads, head_dim, kv_dim;
    int      dtype;
    uint32_t esize;
    size_t   bytes;               /* 2 * max_seq * kv_dim * esize */
    void*    dev;                 /* device address of the buffer */
    float*   host;                /* always NULL (not mappable) */
    uint32_t len;
    TGBackend* be;                /* backend that owns dev */
    void*    scratch;             /* split-sequence partials */
    uint64_t scratch_bytes;
    uint32_t* counters;
    uint64_t counter_slots;
    float*   staging;             /* device staging of host rows (bf16 append) */
    size_t   staging_bytes;
    void*    tmap;                /* TMA tensor map of dev (NULL: no attention kernel) */
    void*    tmap_sw;             /* swizzled map for the tensor-core suffix kernel, or NULL */
    uint32_t* npos;               /* host item table for attention */
    uint32_t npos_cap;
    float    mscale;              /* YaRN temperature on the 1/sqrt(head_dim) scale */
};

static _Thread_local char t_err[256] = "kv: no error";

static void set_err(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}

const char* tg_kv_last_error(void) { return t_err; }

/* Lets the allocation-free attention entry point in tgkv_kernels.cu report
 * through tg_kv_last_error(); not exported. */
__attribute__((visibility("hidden"))) void tgkv_set_last_error(const char* msg) {
    set_err("%s", msg ? msg : "unknown");
}

TGKvCache* tg_kv_create_ex(uint32_t max_seq, uint32_t n_kv_heads, uint32_t head_dim, int dtype) {
    if (max_seq == 0 || n_kv_heads == 0 || head_dim == 0) {
        set_err("invalid argument (0)");
        return NULL;
    }
    if (dtype != TG_KV_F32 && dtype != TG_KV_BF16) {
        set_err("invalid dtype %d", dtype);
        return NULL;
    }
    TGBackend* b = tg_be_current();
    if (!b || !b->alloc) {
        set_err("no backend selected (call tg_be_select first)");
        return NULL;
    }
    const uint32_t es = dtype == TG_KV_BF16 ? 2u : 4u;
    const uint64_t kv_dim = (uint64_t)n_kv_heads * head_dim;
    const uint64_t bytes64 = 2ull * max_seq * kv_dim * es;
    if (bytes64 > (64ull << 30) || kv_dim > 0xffffffffull) {
        set_err("request too large");
        return NULL;
    }
    TGKvCache* c = (TGKvCache*)calloc(1, sizeof(TGKvCache));
    if (!c) { set_err("calloc failed"); return NULL; }
    c->max_seq = max_seq;
    c->n_kv_heads = n_kv_heads;
    c->head_dim = head_dim;
    c->kv_dim = (uint32_t)kv_dim;
    c->dtype = dtype;
    c->esize = es;
    c->bytes = (size_t)bytes64;
    c->be = b;
    c->mscale = 1.0f;
    c->dev = b->alloc(c->bytes);              /* zero-filled by the cuda backend */
    if (!c->dev) {
        set_err("device allocation failed: %s", b->last_error ? b->last_error() : "?");
        free(c);
        return NULL;
    }
    c->host = (float*)(b->map ? b->map(c->dev) : NULL);
    if (tg_cuda_kv_attn_supported(dtype, head_dim)) {
        c->tmap = tg_cuda_kv_tmap_create(dtype, (uint64_t)(uintptr_t)c->dev, max_seq, n_kv_heads,
                                         head_dim);
        if (!c->tmap) {
            set_err("tensor map: %s", tg_cuda_kv_last_error());
            b->free(c->dev);
            free(c);
            return NULL;
        }
    }
    if (dtype == TG_KV_BF16 && head_dim == 128) {
        c->tmap_sw = tg_cuda_kv_tmap_sw_create((uint64_t)(uintptr_t)c->dev, max_seq, n_kv_heads);
        if (!c->tmap_sw) {
            set_err("tensor map: %s", tg_cuda_kv_last_error());
            if (c->tmap) tg_cuda_kv_free(c->tmap);
    if (c->tmap_sw) tg_cuda_kv_free(c->tmap_sw);
            b->free(c->dev);
            free(c);
            return NULL;
        }
    }
    tg_gpu_kv_register(c->dev, dtype, max_seq, n_kv_heads, head_dim, c->tmap);
    return c;
}

TGKvCache* tg_kv_create(uint32_t max_seq, uint32_t n_kv_heads, uint32_t head_dim) {
    return tg_kv_create_ex(max_seq, n_kv_heads, head_dim, TG_KV_F32);
}

void tg_kv_destroy(TGKvCache* c) {
    if (!c) return;
    TGBackend* b = c->be;
    if (c->dev) tg_gpu_kv_unregister(c->dev);
    if (b && b->free) {
        if (c->dev) b->free(c->dev);
        if (c->scratch) b->free(c->scratch);
        if (c->counters) b->free(c->counters);
        if (c->staging) b->free(c->staging);
    }
    if (c->tmap) tg_cuda_kv_free(c->tmap);
    free(c->npos);
    free(c);
}

void tg_kv_reset(TGKvCache* c) {
    if (!c) return;
    c->len = 0;                 /* rows stay; attention reads only [0, len) */
}

uint32_t tg_kv_len(const TGKvCache* c) { return c ? c->len : 0; }
uint32_t tg_kv_capacity(const TGKvCache* c) { return c ? c->max_seq : 0; }
void* tg_kv_device_handle(TGKvCache* c) { return c ? c->dev : NULL; }
float* tg_kv_host_ptr(TGKvCache* c) { return c ? c->host : NULL; }
int tg_kv_dtype(const TGKvCache* c) { return c ? c->dtype : -1; }
uint32_t tg_kv_n_kv_heads(const TGKvCache* c) { return c ? c->n_kv_heads : 0; }
uint32_t tg_kv_head_dim(const TGKvCache* c) { return c ? c->head_dim : 0; }
uint64_t tg_kv_bytes(const TGKvCache* c) { return c ? (uint64_t)c->bytes : 0; }

void tg_kv_set_attn_mscale(TGKvCache* c, float mscale) {
    if (c) c->mscale = mscale;
}

/* (1/sqrt(head_dim)) * mscale, as src/tgai_engine.c:3947 forms it */
static float score_scale(const TGKvCache* c) {
    return (1.0f / sqrtf((float)c->head_dim)) * c->mscale;
}

void tg_kv_advance(TGKvCache* c, uint32_t n_tokens) {
    if (!c) return;
    uint64_t l = (uint64_t)c->len + n_tokens;
    c->len = l > c->max_seq ? c->max_seq : (uint32_t)l;
}

int tg_kv_truncate(TGKvCache* c, uint32_t n) {
    if (!c) { set_err("null cache"); return 0; }
    if (n > c->len) { set_err("truncate to %u beyond length %u", n, c->len); return 0; }
    c->len = n;
    return 1;
}

static int ensure_dev(TGKvCache* c, void** p, uint64_t* have, uint64_t need) {
    if (need <= *have) return 1;
    if (*p) c->be->free(*p);
    const uint64_t want = need + need / 2;
    *p = c->be->alloc((size_t)want);
    if (!*p) {
        *have = 0;
        set_err("device allocation failed: %s",
                c->be->last_error ? c->be->last_error() : "?");
        return 0;
    }
    *have = want;
    return 1;
}

int tg_kv_append(TGKvCache* c, const float* k_src, const float* v_src, uint32_t n_tokens) {
    if (!c || !k_src || !v_src) { set_err("null argument"); return 0; }
    if (n_tokens == 0) return 1;
    if ((uint64_t)c->len + n_tokens > c->max_seq) { set_err("capacity exceeded"); return 0; }
    const size_t row = (size_t)c->kv_dim * 4;
    if (c->host) {                                   /* mappable backends (not cuda) */
        memcpy(c->host + (size_t)c->len * c->kv_dim, k_src, row * n_tokens);
        memcpy(c->host + (size_t)c->max_seq * c->kv_dim + (size_t)c->len * c->kv_dim, v_src,
               row * n_tokens);
        c->len += n_tokens;
        return 1;
    }
    /* Stage the fp32 rows in HBM, then the append kernel writes them in the
     * cache's storage type; blocks so the caller's buffers are free again. */
    uint64_t have = c->staging_bytes;
    if (!ensure_dev(c, (void**)&c->staging, &have, 2ull * row * n_tokens)) return 0;
    c->staging_bytes = (size_t)have;
    float* ks = c->staging;
    float* vs = (float*)((char*)c->staging + row * n_tokens);
    if (!tg_cuda_kv_h2d(ks, k_src, row * n_tokens, NULL) ||
        !tg_cuda_kv_h2d(vs, v_src, row * n_tokens, NULL)) {
        set_err("%s", tg_cuda_kv_last_error());
        return 0;
    }
    if (!tg_gpu_kv_append_dev(c->dtype, c->dev, c->max_seq, c->kv_dim, c->len, ks, vs, n_tokens,
                              NULL) ||
        !tg_cuda_kv_sync(NULL)) {
        set_err("%s", tg_gpu_kv_error());
        return 0;
    }
    c->len += n_tokens;
    return 1;
}

int tg_kv_append_dev(TGKvCache* c, const float* k_dev, const float* v_dev, uint32_t n_tokens,
                     void* stream) {
    if (!c || !k_dev || !v_dev) { set_err("null argument"); return 0; }
    if (n_tokens == 0) return 1;
    if ((uint64_t)c->len + n_tokens > c->max_seq) { set_err("capacity exceeded"); return 0; }
    if (!tg_gpu_kv_append_dev(c->dtype, c->dev, c->max_seq, c->kv_dim, c->len, k_dev, v_dev,
                              n_tokens, stream)) {
        set_err("%s", tg_gpu_kv_error());
        return 0;
    }
    c->len += n_tokens;
    return 1;
}

int tg_kv_download(const TGKvCache* c, void* dst) {
    if (!c || !dst) { set_err("null argument"); return 0; }
    if (!tg_cuda_kv_d2h(dst, c->dev, c->bytes, NULL)) {
        set_err("%s", tg_cuda_kv_last_error());
        return 0;
    }
    return 1;
}

/* Make sure the split-sequence scratch of a call fits (grows with slack). */
static int ensure_attn_scratch(TGBackend* be, const TGCudaAttnCall* call, void** scratch,
                               uint64_t* scratch_bytes, uint32_t** counters, uint64_t* slots) {
    const uint64_t need = tg_cuda_kv_attn_scratch_bytes(call);
    const uint64_t nslots = tg_cuda_kv_attn_counters(call);
    if (need == 0 || nslots == 0) { set_err("%s", tg_cuda_kv_last_error()); return 0; }
    if (need > *scratch_bytes) {
        if (*scratch) be->free(*scratch);
        const uint64_t want = need + need / 2;
        *scratch = be->alloc((size_t)want);
        *scratch_bytes = *scratch ? want : 0;
        if (!*scratch) { set_err("scratch allocation failed"); return 0; }
    }
    if (nslots > *slots) {
        /* counters must start at zero; the kernel returns them to zero */
        if (*counters) be->free(*counters);
        *counters = (uint32_t*)be->alloc((size_t)nslots * 4);
        *slots = *counters ? nslots : 0;
        if (!*counters) { set_err("counter allocation failed"); return 0; }
    }
    return 1;
}

int tg_kv_attention(TGKvCache* c, const float* q_dev, float* out_dev, uint32_t n_heads,
                    uint32_t n_q, void* stream) {
    if (!c || !q_dev || !out_dev) { set_err("null argument"); return 0; }
    if (n_q == 0 || n_q > c->len) {
        set_err("n_q %u must be in [1, len=%u]", n_q, c->len);
        return 0;
    }
    if (n_heads == 0 || n_heads % c->n_kv_heads) {
        set_err("n_heads %u is not a multiple of n_kv_heads %u", n_heads, c->n_kv_heads);
        return 0;
    }
    if (n_q > c->npos_cap) {
        uint32_t* np = (uint32_t*)realloc(c->npos, (size_t)n_q * sizeof(uint32_t));
        if (!np) { set_err("realloc failed"); return 0; }
        c->npos = np;
        c->npos_cap = n_q;
    }
    for (uint32_t t = 0; t < n_q; t++) c->npos[t] = c->len - n_q + t + 1;
    TGCudaAttnCall call;
    memset(&call, 0, sizeof(call));
    call.dtype = c->dtype;
    call.n_heads = n_heads;
    call.n_kv_heads = c->n_kv_heads;
    call.head_dim = c->head_dim;
    call.cache.base = (uint64_t)(uintptr_t)c->dev;
    call.cache.max_seq = c->max_seq;
    call.cache.tmap = (uint64_t)(uintptr_t)c->tmap;
    call.cache.tmap_sw = (uint64_t)(uintptr_t)c->tmap_sw;
    call.n_pos = c->npos;
    call.n_items = n_q;
    if (!ensure_attn_scratch(c->be, &call, &c->scratch, &c->scratch_bytes, &c->counters,
                             &c->counter_slots))
        return 0;
    if (!c->tmap) {
        set_err("attention: no kernel for dtype %d head_dim %u", c->dtype, c->head_dim);
        return 0;
    }
    if (!tg_gpu_kv_attention(c->dtype, c->dev, c->max_seq, c->tmap, c->tmap_sw, n_heads,
                             c->n_kv_heads,
                             c->head_dim,
                             q_dev, out_dev, c->npos, n_q, score_scale(c),
                             c->scratch, c->counters, stream)) {
        set_err("%s", tg_gpu_kv_error());
        return 0;
    }
    return 1;
}

int tg_kv_append_attention(TGKvCache* c, const float* k_dev, const float* v_dev,
                           const float* q_dev, float* out_dev, uint32_t n_heads, uint32_t n,
                           void* stream) {
    if (!c || !k_dev || !v_dev || !q_dev || !out_dev) { set_err("null argument"); return 0; }
    if (n == 0) { set_err("n must be at least 1"); return 0; }
    if ((uint64_t)c->len + n > c->max_seq) { set_err("capacity exceeded"); return 0; }
    if (n_heads == 0 || n_heads % c->n_kv_heads) {
        set_err("n_heads %u is not a multiple of n_kv_heads %u", n_heads, c->n_kv_heads);
        return 0;
    }
    if (n > c->npos_cap) {
        uint32_t* np = (uint32_t*)realloc(c->npos, (size_t)n * sizeof(uint32_t));
        if (!np) { set_err("realloc failed"); return 0; }
        c->npos = np;
        c->npos_cap = n;
    }
    for (uint32_t t = 0; t < n; t++) c->npos[t] = c->len + t + 1;
    TGCudaAttnCall call;
    memset(&call, 0, sizeof(call));
    call.dtype = c->dtype;
    call.n_heads = n_heads;
    call.n_kv_heads = c->n_kv_heads;
    call.head_dim = c->head_dim;
    call.cache.base = (uint64_t)(uintptr_t)c->dev;
    call.cache.max_seq = c->max_seq;
    call.cache.tmap = (uint64_t)(uintptr_t)c->tmap;
    call.cache.tmap_sw = (uint64_t)(uintptr_t)c->tmap_sw;
    call.q = q_dev;
    call.out = out_dev;
    call.k_new = k_dev;
    call.v_new = v_dev;
    call.n_pos = c->npos;
    call.n_items = n;
    call.scale = score_scale(c);
    /* TGKV_FUSE_SUFFIX=1: one launch, the suffix kernel storing the rows
     * itself before it reads them.  Off by default: on configs[2]'s turns it
     * measured 0.506 ms per turn against 0.448 with the append kernel first
     * (each row block's clusters store the rows they read, so the stores are
     * repeated per row block and sit on every cluster's critical path). */
    const char* fz = getenv("TGKV_FUSE_SUFFIX");
    if (fz && fz[0] == '1' && tg_be_current() == &tg_backend_cuda &&
        tg_cuda_kv_attn_fuses_suffix(&call)) {
        /* one launch: the suffix kernel stores the rows, then attends them */
        if (!ensure_attn_scratch(c->be, &call, &c->scratch, &c->scratch_bytes, &c->counters,
                                 &c->counter_slots))
            return 0;
        call.scratch = c->scratch;
        call.counters = c->counters;
        if (!tg_cuda_kv_attention(&call, stream)) {
            set_err("%s", tg_cuda_kv_last_error());
            return 0;
        }
        c->len += n;
        return 1;
    }
    /* the append launch, then the attention */
    return tg_kv_append_dev(c, k_dev, v_dev, n, stream) &&
           tg_kv_attention(c, q_dev, out_dev, n_heads, n, stream);
}

/* ---- batched decode ----------------------------------------------------- */
struct TGKvBatch {
    uint32_t n, n_heads, n_kv_heads, head_dim, kv_dim;
    int dtype;
    TGBackend* be;
    TGKvCache** caches;
    TGCudaCacheDesc* table_dev;
    uint32_t* npos;                   /* host: attended positions per cache */
    void* scratch;
    uint64_t scratch_bytes;
    uint32_t* counters;
    uint64_t counter_slots;
    /* host-buffer variant: two device staging slots, used in turn, so that a
     * call's uploads (on the plan's copy stream) overlap the previous call's
     * kernel; in_ready orders a slot's kernel after its uploads, slot_free a
     * slot's next uploads after its last reader */
    float* io[2];
    uint64_t io_bytes[2];
    void* copy_stream;
    void* in_ready[2];
    void* slot_free[2];
    int slot_used[2];
    uint32_t slot;
    uint32_t last_launches;
    /* small page-locked inputs: two device slots the staging kernel fills in
     * turn, and the device pointers of the last host buffers seen */
    float* small_io[2];
    uint64_t small_bytes;
    uint32_t small_slot;
};

TGKvBatch* tg_kv_batch_create(TGKvCache* const* caches, uint32_t n, uint32_t n_heads) {
    if (!caches || n == 0 || n > 1024) { set_err("batch: need 1..1024 caches"); return NULL; }
    const TGKvCache* c0 = caches[0];
    if (!c0) { set_err("batch: null cache"); return NULL; }
    for (uint32_t i = 1; i < n; i++) {
        const TGKvCache* c = caches[i];
        if (!c || c->n_kv_heads != c0->n_kv_heads || c->head_dim != c0->head_dim ||
            c->dtype != c0->dtype) {
            set_err("batch: cache %u differs in geometry or dtype", i);
            return NULL;
        }
    }
    if (n_heads == 0 || n_heads % c0->n_kv_heads) {
        set_err("batch: n_heads %u is not a multiple of n_kv_heads %u", n_heads, c0->n_kv_heads);
        return NULL;
    }
    for (uint32_t i = 0; i < n; i++)
        if (!caches[i]->tmap) {
            set_err("batch: no attention kernel for dtype %d head_dim %u", c0->dtype,
                    c0->head_dim);
            return NULL;
        }
    TGKvBatch* b = (TGKvBatch*)calloc(1, sizeof(TGKvBatch));
    if (!b) { set_err("calloc failed"); return NULL; }
    b->n = n;
    b->n_heads = n_heads;
    b->n_kv_heads = c0->n_kv_heads;
    b->head_dim = c0->head_dim;
    b->kv_dim = c0->kv_dim;
    b->dtype = c0->dtype;
    b->be = c0->be;
    b->caches = (TGKvCache**)malloc(n * sizeof(TGKvCache*));
    b->npos = (uint32_t*)malloc(n * sizeof(uint32_t));
    TGCudaCacheDesc* table = (TGCudaCacheDesc*)calloc(n, sizeof(TGCudaCacheDesc));
    if (!b->caches || !b->npos || !table) {
        free(table);
        tg_kv_batch_destroy(b);
        set_err("malloc failed");
        return NULL;
    }
    for (uint32_t i = 0; i < n; i++) {
        b->caches[i] = caches[i];
        table[i].base = (uint64_t)(uintptr_t)caches[i]->dev;
        table[i].max_seq = caches[i]->max_seq;
        table[i].tmap = (uint64_t)(uintptr_t)caches[i]->tmap;
        table[i].tmap_sw = (uint64_t)(uintptr_t)caches[i]->tmap_sw;
    }
    b->table_dev = (TGCudaCacheDesc*)b->be->alloc(n * sizeof(TGCudaCacheDesc));
    if (!b->table_dev || !tg_cuda_kv_h2d(b->table_dev, table, n * sizeof(TGCudaCacheDesc), NULL)) {
        free(table);
        tg_kv_batch_destroy(b);
        set_err("batch: descriptor table upload failed");
        return NULL;
    }
    free(table);
    return b;
}

void tg_kv_batch_destroy(TGKvBatch* b) {
    if (!b) return;
    if (b->be && b->be->free) {
        if (b->table_dev) b->be->free(b->table_dev);
        if (b->scratch) b->be->free(b->scratch);
        if (b->counters) b->be->free(b->counters);
        for (int i = 0; i < 2; i++)
            if (b->io[i]) b->be->free(b->io[i]);
    }
    for (int i = 0; i < 2; i++) {
        tg_cuda_kv_event_destroy(b->in_ready[i]);
        tg_cuda_kv_event_destroy(b->slot_free[i]);
    }
    tg_cuda_kv_stream_destroy(b->copy_stream);
    if (b->be && b->be->free)
        for (int i = 0; i < 2; i++)
            if (b->small_io[i]) b->be->free(b->small_io[i]);
    free(b->caches);
    free(b->npos);
    free(b);
}

uint32_t tg_kv_batch_last_launches(const TGKvBatch* b) { return b ? b->last_launches : 0; }

/* ---- output gather over NVLink ------------------------------------------ */

#define TGKV_GATHER_MAX 8

/* Two halves of [world][elems] gathered outputs and one arrival counter per
 * half, used by alternate calls.  A call's outputs stay in their half until
 * the call after next: before any rank's call n+2 stores into a peer's half,
 * that rank has waited for every rank's call n+1 arrivals, and a rank's call
 * n+1 kernel runs only after the work it queued on its stream before that call
 * -- the consumers of call n's outputs -- has finished.  The counters are
 * separate for the same reason: no arrival of call n+2 can reach a counter
 * before its owner has finished waiting for call n. */
struct TGKvGather {
    uint32_t world, rank;
    uint64_t elems;                   /* outputs of one rank */
    uint64_t half_bytes;              /* one half: [world][elems] fp32, 256-byte multiple */
    uint64_t flag_off;                /* byte offset of the two arrival counters (128 B apart) */
    unsigned char* mem;               /* this rank's allocation */
    unsigned char* peer[TGKV_GATHER_MAX];   /* every rank's allocation (own at [rank]) */
    int imported;
    uint64_t calls;                   /* gathered calls so far; call n uses half n & 1 */
    uint32_t last_half;               /* half of the last call */
    uint32_t target[2];               /* arrivals expected per half after the last call */
};

TGKvGather* tg_kv_gather_create(uint32_t world, uint32_t rank, uint64_t elems) {
    if (world == 0 || world > TGKV_GATHER_MAX || rank >= world || elems == 0) {
        set_err("gather: bad shape (world %u, rank %u, %llu elements)", world, rank,
                (unsigned long long)elems);
        return NULL;
    }
    TGKvGather* g = (TGKvGather*)calloc(1, sizeof(TGKvGather));
    if (!g) { set_err("out of host memory"); return NULL; }
    g->world = world;
    g->rank = rank;
    g->elems = elems;
    g->half_bytes = ((uint64_t)world * elems * 4 + 255) / 256 * 256;
    g->flag_off = 2 * g->half_bytes;
    g->mem = (unsigned char*)tg_cuda_kv_malloc((size_t)(g->flag_off + 256));   /* zeroed */
    if (!g->mem) {
        set_err("gather: %s", tg_cuda_kv_last_error());
        free(g);
        return NULL;
    }
    g->peer[rank] = g->mem;
    g->imported = world == 1;
    return g;
}

void tg_kv_gather_destroy(TGKvGather* g) {
    if (!g) return;
    for (uint32_t r = 0; r < g->world; r++)
        if (r != g->rank && g->peer[r]) tg_cuda_kv_ipc_close(g->peer[r]);
    tg_cuda_kv_free(g->mem);
    free(g);
}

int tg_kv_gather_export(const TGKvGather* g, void* handle64) {
    if (!g || !handle64) { set_err("null argument"); return 0; }
    if (!tg_cuda_kv_ipc_handle(g->mem, handle64)) { set_err("%s", tg_cuda_kv_last_error()); return 0; }
    return 1;
}

int tg_kv_gather_import(TGKvGather* g, const void* handles) {
    if (!g || !handles) { set_err("null argument"); return 0; }
    for (uint32_t r = 0; r < g->world; r++) {
        if (r == g->rank || g->peer[r]) continue;
        g->peer[r] = (unsigned char*)tg_cuda_kv_ipc_open((const unsigned char*)handles + 64u * r);
        if (!g->peer[r]) {
            set_err("gather: rank %u: %s", r, tg_cuda_kv_last_error());
            return 0;
        }
    }
    g->imported = 1;
    return 1;
}

float* tg_kv_gather_buffer(const TGKvGather* g) {
    return g ? (float*)(g->mem + (uint64_t)g->last_half * g->half_bytes) : NULL;
}

/* One decode step of the plan; with g, the outputs also go to every rank's
 * gathered buffer and the stream then waits for all ranks' outputs. */
static int batch_decode(TGKvBatch* b, const float* q, const float* k_new, const float* v_new,
                        float* out, TGKvGather* g, void* stream) {
    if (!b || !q || !k_new || !v_new || !out) { set_err("null argument"); return 0; }
    if (g && !g->imported) { set_err("gather: peers not imported"); return 0; }
    if (g && (uint64_t)b->n * b->n_heads * b->head_dim != g->elems) {
        set_err("gather: plan outputs %llu elements, gather slices hold %llu",
                (unsigned long long)b->n * b->n_heads * b->head_dim, (unsigned long long)g->elems);
        return 0;
    }
    b->last_launches = 0;
    for (uint32_t i = 0; i < b->n; i++) {
        const TGKvCache* c = b->caches[i];
        if (c->len >= c->max_seq) { set_err("batch: cache %u is full", i); return 0; }
        b->npos[i] = c->len + 1;
    }
    TGCudaAttnCall call;
    memset(&call, 0, sizeof(call));
    call.dtype = b->dtype;
    call.n_heads = b->n_heads;
    call.n_kv_heads = b->n_kv_heads;
    call.head_dim = b->head_dim;
    call.table_dev = b->table_dev;
    call.q = q;
    call.out = out;
    call.n_pos = b->npos;
    call.n_items = b->n;
    call.scale = score_scale(b->caches[0]);
    if (!ensure_attn_scratch(b->be, &call, &b->scratch, &b->scratch_bytes, &b->counters,
                             &b->counter_slots))
        return 0;
    call.scratch = b->scratch;
    call.counters = b->counters;
    call.k_new = k_new;               /* the append runs inside the attention launch */
    call.v_new = v_new;
    const uint32_t half = g ? (uint32_t)(g->calls & 1u) : 0;
    if (g) {
        call.gather_world = g->world;
        call.gather_base = (uint64_t)g->rank * g->elems;
        for (uint32_t r = 0; r < g->world; r++) {
            call.gather_out[r] = (float*)(g->peer[r] + (uint64_t)half * g->half_bytes);
            call.gather_flag[r] = (uint32_t*)(g->peer[r] + g->flag_off + 128u * half);
        }
    }
    if (tg_be_current() != &tg_backend_cuda) {
        set_err("KV-cache path needs the cuda backend; no fallback");
        return 0;
    }
    if (!tg_cuda_kv_attention(&call, stream)) {
        set_err("%s", tg_cuda_kv_last_error());
        return 0;
    }
    b->last_launches += tg_cuda_kv_attn_last_launches();
    for (uint32_t i = 0; i < b->n; i++) b->caches[i]->len++;
    if (g) {
        /* every rank finishes the same number of segments and signals each
         * rank once per segment */
        g->target[half] += g->world * (uint32_t)tg_cuda_kv_attn_segments(&call);
        g->calls++;
        g->last_half = half;
        if (!tg_cuda_kv_gather_wait((const uint32_t*)(g->mem + g->flag_off + 128u * half),
                                    g->target[half], stream)) {
            set_err("%s", tg_cuda_kv_last_error());
            return 0;
        }
        b->last_launches++;
    }
    return 1;
}

int tg_kv_batch_decode(TGKvBatch* b, const float* q, const float* k_new, const float* v_new,
                       float* out, void* stream) {
    return batch_decode(b, q, k_new, v_new, out, NULL, stream);
}

int tg_kv_batch_decode_gather(TGKvBatch* b, const float* q, const float* k_new,
                              const float* v_new, float* out, TGKvGather* g, void* stream) {
    if (!g) { set_err("null gather"); return 0; }
    return batch_decode(b, q, k_new, v_new, out, g, stream);
}

/* The step from host buffers: upload q/k/v into one of the plan's two
 * staging slots on the plan's copy stream (overlapping the previous call's
 * kernel when the host buffers are pinned), run the step on `stream` once
 * they are in, and bring the outputs back: a page-locked out_host receives
 * them straight from the kernel (no copy; the stores overlap the streaming),
 * else they are copied back on `stream` -- with g, the whole gathered buffer
 * is copied.  Synchronising `stream` covers the results either way. */
/* Page-locked inputs of at most this many bytes per call are staged by one
 * small kernel on the launch stream instead of three copies on the plan's
 * copy stream ordered by events: for a few KB those CUDA calls cost more host
 * time than the decode kernel takes. */
#define TGKV_SMALL_UPLOAD (256u << 10)

static int batch_decode_host(TGKvBatch* b, const float* q_host, const float* k_host,
                             const float* v_host, float* out_host, TGKvGather* g, void* stream) {
    if (!b || !q_host || !k_host || !v_host || !out_host) { set_err("null argument"); return 0; }
    const uint64_t qb = (uint64_t)b->n * b->n_heads * b->head_dim * 4;
    const uint64_t kb = (uint64_t)b->n * b->kv_dim * 4;
    const uint64_t need = 2 * qb + 2 * kb + 64;
    if (qb + 2 * kb <= TGKV_SMALL_UPLOAD && !(qb % 16) && !(kb % 16)) {
        void* dq = tg_cuda_kv_host_device_ptr(q_host);
        void* dk = tg_cuda_kv_host_device_ptr(k_host);
        void* dv = tg_cuda_kv_host_device_ptr(v_host);
        if (dq && dk && dv && !(((uintptr_t)dq | (uintptr_t)dk | (uintptr_t)dv) & 15)) {
            if (b->small_bytes < need) {
                for (int i = 0; i < 2; i++) {
                    if (b->small_io[i]) b->be->free(b->small_io[i]);   /* waits for readers */
                    b->small_io[i] = (float*)b->be->alloc((size_t)need);
                }
                b->small_bytes = b->small_io[0] && b->small_io[1] ? need : 0;
                if (!b->small_bytes) { set_err("batch: staging allocation failed"); return 0; }
            }
            float* q = b->small_io[b->small_slot];
            float* k = (float*)((char*)q + qb);
            float* v = (float*)((char*)k + kb);
            float* o = (float*)((char*)v + kb);
            b->small_slot ^= 1u;
            if (!tg_cuda_kv_stage_host(q, dq, qb, dk, kb, dv, kb, stream)) {
                set_err("%s", tg_cuda_kv_last_error());
                return 0;
            }
            /* the kernel stores a page-locked out_host's rows itself; with a
             * gather, the whole gathered buffer comes back after the wait */
            float* direct = g ? NULL : (float*)tg_cuda_kv_host_device_ptr(out_host);
            if (!batch_decode(b, q, k, v, direct ? direct : o, g, stream)) return 0;
            b->last_launches++;
            const void* src = g ? (const void*)tg_kv_gather_buffer(g) : (const void*)o;
            const uint64_t ob = g ? (uint64_t)g->world * g->elems * 4 : qb;
            if (!direct && !tg_cuda_kv_d2h_async(out_host, src, ob, stream)) {
                set_err("%s", tg_cuda_kv_last_error());
                return 0;
            }
            return 1;
        }
    }
    if (!b->copy_stream) {
        b->copy_stream = tg_cuda_kv_stream_create();
        for (int i = 0; i < 2; i++) {
            b->in_ready[i] = tg_cuda_kv_event_create();
            b->slot_free[i] = tg_cuda_kv_event_create();
        }
        if (!b->copy_stream || !b->in_ready[0] || !b->in_ready[1] || !b->slot_free[0] ||
            !b->slot_free[1]) {
            set_err("batch: %s", tg_cuda_kv_last_error());
            return 0;
        }
    }
    const uint32_t s = b->slot;
    if (need > b->io_bytes[s]) {
        if (b->io[s]) b->be->free(b->io[s]);          /* cudaFree waits for its readers */
        b->io[s] = (float*)b->be->alloc((size_t)need);
        b->io_bytes[s] = b->io[s] ? need : 0;
        if (!b->io[s]) { set_err("batch: staging allocation failed"); return 0; }
    }
    float* q = b->io[s];
    float* o = (float*)((char*)q + qb);
    float* k = (float*)((char*)o + qb);
    float* v = (float*)((char*)k + kb);
    void* cp = b->copy_stream;
    int ok = (!b->slot_used[s] || tg_cuda_kv_stream_wait(cp, b->slot_free[s])) &&
             tg_cuda_kv_h2d(q, q_host, qb, cp) && tg_cuda_kv_h2d(k, k_host, kb, cp) &&
             tg_cuda_kv_h2d(v, v_host, kb, cp) && tg_cuda_kv_event_record(b->in_ready[s], cp) &&
             tg_cuda_kv_stream_wait(stream, b->in_ready[s]);
    if (!ok) { set_err("%s", tg_cuda_kv_last_error()); return 0; }
    float* direct = g ? NULL : (float*)tg_cuda_kv_host_device_ptr(out_host);
    if (!batch_decode(b, q, k, v, direct ? direct : o, g, stream)) return 0;
    const void* src = g ? (const void*)tg_kv_gather_buffer(g) : (const void*)o;
    const uint64_t ob = g ? (uint64_t)g->world * g->elems * 4 : qb;
    if ((!direct && !tg_cuda_kv_d2h_async(out_host, src, ob, stream)) ||
        !tg_cuda_kv_event_record(b->slot_free[s], stream)) {
        set_err("%s", tg_cuda_kv_last_error());
        return 0;
    }
    b->slot_used[s] = 1;
    b->slot ^= 1u;
    return 1;
}

int tg_kv_batch_decode_host(TGKvBatch* b, const float* q_host, const float* k_host,
                            const float* v_host, float* out_host, void* stream) {
    return batch_decode_host(b, q_host, k_host, v_host, out_host, NULL, stream);
}

int tg_kv_batch_decode_gather_host(TGKvBatch* b, const float* q_host, const float* k_host,
                                   const float* v_host, float* out_host, TGKvGather* g,
                                   void* stream) {
    if (!g) { set_err("null gather"); return 0; }
    return batch_decode_host(b, q_host, k_host, v_host, out_host, g, stream);
}
