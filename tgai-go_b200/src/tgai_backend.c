/* tgai_backend.c -- the TGBackend table for CUDA and backend selection.
 *
 * Fills the slot the reference leaves empty (src/tgai_backend.c:301-305) with
 * a CUDA implementation of the KV-cache path's entries: memory, single-query
 * attention and RoPE + KV write.  Selection keeps the reference's API and
 * TG_BACKEND variable (src/tgai_backend.c:336-364) but only "cuda" can be
 * selected; "cpu" and "vulkan" are known names that are not compiled in.
 */
#include "tgai_backend.h"
#include "tgai_cuda_bridge.h"
#include "tgai_gpu_dispatch.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static char g_cuda_err[256] = "cuda backend: not initialized";

static int cu_init(void) {
    if (!tg_cuda_kv_init()) {
        snprintf(g_cuda_err, sizeof(g_cuda_err), "%s", tg_cuda_kv_last_error());
        return 0;
    }
    snprintf(g_cuda_err, sizeof(g_cuda_err), "cuda backend: ready");
    return 1;
}
static void cu_shutdown(void) { /* device memory is owned by the caches */ }
static int cu_ready(void) { return tg_cuda_kv_ready(); }
static const char* cu_last_error(void) { return g_cuda_err; }

static int cu_info(TGBackendInfo* out) {
    if (!out || !tg_cuda_kv_ready()) return 0;
    memset(out, 0, sizeof(*out));
    out->name = "cuda";
    out->device_name = tg_cuda_kv_device_name();
    out->caps = tg_backend_cuda.caps;
    out->mem_bytes = tg_cuda_kv_device_mem();
    out->is_gpu = 1;
    out->is_uma = 0;
    return 1;
}

static void* cu_alloc(size_t bytes) {
    void* p = tg_cuda_kv_malloc(bytes);
    if (!p) snprintf(g_cuda_err, sizeof(g_cuda_err), "%s", tg_cuda_kv_last_error());
    return p;
}
static void cu_free(void* p) { tg_cuda_kv_free(p); }
static void* cu_map(void* p) { (void)p; return NULL; }   /* discrete HBM: not mappable */

static int cu_upload(void* dst, const void* src, size_t bytes) {
    if (!dst || !src) return 0;
    return tg_cuda_kv_h2d(dst, src, bytes, NULL);
}
static int cu_download(void* dst, const void* src, size_t bytes) {
    if (!dst || !src) return 0;
    return tg_cuda_kv_d2h(dst, src, bytes, NULL);
}

/* Split-sequence scratch shared by the table's blocking attention calls. */
static pthread_mutex_t g_attn_mu = PTHREAD_MUTEX_INITIALIZER;
static void* g_scratch = NULL;
static uint64_t g_scratch_bytes = 0;
static uint32_t* g_counters = NULL;
static uint64_t g_counter_slots = 0;
static void* g_tmap = NULL;            /* tensor map for caller-owned cache buffers */

static int cu_attention(void* q, void* kvc, void* out, uint32_t nh, uint32_t nkvh, uint32_t hd,
                        uint32_t n_kv, uint32_t pos, uint32_t max_seq) {
    if (!q || !kvc || !out || nkvh == 0 || hd == 0) return 0;
    uint32_t n = n_kv < pos + 1 ? n_kv : pos + 1;       /* j < n_kv and j <= pos */
    if (n > max_seq) n = max_seq;
    if (n == 0) {                                        /* no position: output 0 */
        return tg_cuda_kv_memset(out, 0, (size_t)nh * hd * 4, NULL);
    }
    int dtype = tg_gpu_kv_lookup_dtype(kvc);
    if (dtype < 0) dtype = 0;
    pthread_mutex_lock(&g_attn_mu);
    const void* tmap = tg_gpu_kv_lookup_tmap(kvc, max_seq, nkvh, hd);
    if (!tmap) {                     /* a buffer this library did not create */
        if (!g_tmap) g_tmap = tg_cuda_kv_malloc(128);
        if (!g_tmap || !tg_cuda_kv_tmap_write(dtype, (uint64_t)(uintptr_t)kvc, max_seq, nkvh, hd,
                                              g_tmap)) {
            snprintf(g_cuda_err, sizeof(g_cuda_err), "%s", tg_cuda_kv_last_error());
            pthread_mutex_unlock(&g_attn_mu);
            return 0;
        }
        tmap = g_tmap;
    }
    TGCudaAttnCall c;
    memset(&c, 0, sizeof(c));
    c.dtype = dtype;
    c.n_heads = nh;
    c.n_kv_heads = nkvh;
    c.head_dim = hd;
    c.cache.base = (uint64_t)(uintptr_t)kvc;
    c.cache.max_seq = max_seq;
    c.cache.tmap = (uint64_t)(uintptr_t)tmap;
    c.q = (const float*)q;
    c.out = (float*)out;
    c.n_pos = &n;
    c.n_items = 1;
    c.scale = 1.0f / sqrtf((float)hd);
    const uint64_t need = tg_cuda_kv_attn_scratch_bytes(&c);
    const uint64_t slots = tg_cuda_kv_attn_counters(&c);
    int ok = 1;
    if (need > g_scratch_bytes) {
        tg_cuda_kv_free(g_scratch);
        g_scratch = tg_cuda_kv_malloc(need);
        g_scratch_bytes = g_scratch ? need : 0;
        ok = g_scratch != NULL;
    }
    if (ok && slots > g_counter_slots) {
        tg_cuda_kv_free(g_counters);
        g_counters = (uint32_t*)tg_cuda_kv_malloc(slots * 4);
        g_counter_slots = g_counters ? slots : 0;
        ok = g_counters != NULL;
    }
    if (ok)
        ok = tg_gpu_kv_attention(dtype, kvc, max_seq, tmap, NULL, nh, nkvh, hd, c.q, c.out, &n, 1,
                                 c.scale,
                                 g_scratch, g_counters, NULL) &&
             tg_cuda_kv_sync(NULL);
    if (!ok) snprintf(g_cuda_err, sizeof(g_cuda_err), "%s", tg_gpu_kv_error());
    pthread_mutex_unlock(&g_attn_mu);
    return ok;
}

static int cu_rope(void* qkv, void* cs, void* sn, void* kvc, void* qout, uint32_t n_tokens,
                   uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, uint32_t start_pos,
                   uint32_t max_seq) {
    int dtype = tg_gpu_kv_lookup_dtype(kvc);
    if (dtype < 0) dtype = 0;
    int ok = tg_cuda_kv_rope_append(dtype, (const float*)qkv, (const float*)cs, (const float*)sn,
                                    kvc, (float*)qout, n_tokens, n_heads, n_kv_heads, head_dim,
                                    start_pos, max_seq, NULL) &&
             tg_cuda_kv_sync(NULL);
    if (!ok) snprintf(g_cuda_err, sizeof(g_cuda_err), "%s", tg_cuda_kv_last_error());
    return ok;
}

TGBackend tg_backend_cuda = {
    "cuda",
    TG_BE_CAP_F32 | TG_BE_CAP_BF16 | TG_BE_CAP_ROPE | TG_BE_CAP_ATTN | TG_BE_CAP_KV,
    cu_init, cu_shutdown, cu_ready, cu_info, cu_last_error,
    cu_alloc, cu_free, cu_upload, cu_download, cu_map,
    NULL, NULL, NULL,                 /* rmsnorm, silu_mul, softmax: not on this path */
    cu_rope, NULL, cu_attention, NULL,
    NULL,
};

/* Known names without an implementation in this library. */
TGBackend tg_backend_cpu = {"cpu", 0, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL,
                            NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL};
TGBackend tg_backend_vulkan = {"vulkan", 0, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL,
                               NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL, NULL};

static TGBackend* g_cur = NULL;
static const char* g_names[] = {"cuda", "vulkan", "cpu", NULL};

const char* const* tg_be_list(void) { return g_names; }
TGBackend* tg_be_current(void) { return g_cur; }

int tg_be_probe(void) {
    return (tg_backend_cuda.init ? 1 : 0) + (tg_backend_vulkan.init ? 1 : 0) +
           (tg_backend_cpu.init ? 1 : 0);
}

static TGBackend* by_name(const char* nm) {
    if (!nm) return NULL;
    if (strcmp(nm, "cuda") == 0) return &tg_backend_cuda;
    if (strcmp(nm, "vulkan") == 0) return &tg_backend_vulkan;
    if (strcmp(nm, "cpu") == 0) return &tg_backend_cpu;
    return NULL;
}

int tg_be_select(const char* name) {
    if (g_cur) tg_be_shutdown();
    if (!name || !name[0] || strcmp(name, "auto") == 0) {
        const char* env = getenv("TG_BACKEND");
        name = (env && env[0] && strcmp(env, "auto") != 0) ? env : "cuda";
    }
    TGBackend* b = by_name(name);
    if (!b) {
        fprintf(stderr, "[backend] unknown: %s\n", name);
        return 0;
    }
    if (!b->init) {
        fprintf(stderr, "[backend] %s not compiled in (this library is CUDA only)\n", name);
        return 0;
    }
    if (!b->init()) {
        fprintf(stderr, "[backend] %s init failed: %s\n", name, b->last_error ? b->last_error() : "?");
        return 0;
    }
    g_cur = b;
    return 1;
}

int tg_be_current_info(TGBackendInfo* out) {
    if (!g_cur || !g_cur->info) return 0;
    return g_cur->info(out);
}

void tg_be_shutdown(void) {
    if (g_cur && g_cur->shutdown) g_cur->shutdown();
    g_cur = NULL;
}
