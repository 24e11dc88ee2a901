/* tgai_gpu_dispatch.c -- KV-cache path router (CUDA only, no fallback).
 *
 * Portable C; the reference router is Win32-only (<windows.h>, _stricmp,
 * src/tgai_gpu_dispatch.c:89-90) and routes matmul to Vulkan.  Here it routes
 * the KV-cache path's device work to tgai_cuda_bridge.c and keeps the
 * reference's tg_gpu_backend_* status surface.
 */
#include "tgai_gpu_dispatch.h"
#include "tgai_backend.h"
#include "tgai_cuda_bridge.h"

#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <strings.h>

static _Thread_local char t_err[256] = "dispatch: no error";
static char g_reason[256] = "not initialized";
static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static uint64_t g_calls = 0, g_ok = 0;

static void set_err(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}

const char* tg_gpu_kv_error(void) { return t_err; }

/* TG_BACKEND as the reference reads it (src/tgai_gpu_dispatch.c:467-492,
 * case-insensitive): unset, "auto" or "cuda" bring the CUDA path up; "cpu"
 * and "vulkan" are refused with a reason (this build has neither, and the
 * KV-cache path never falls back); any other value is refused as unknown.
 * A backend the caller already selected with tg_be_select is kept. */
int tg_gpu_backend_init(void) {
    TGBackend* b = tg_be_current();
    if (!b) {
        const char* env = getenv("TG_BACKEND");
        if (env && env[0] && strcasecmp(env, "auto") != 0 && strcasecmp(env, "cuda") != 0) {
            if (strcasecmp(env, "cpu") == 0 || strcasecmp(env, "vulkan") == 0)
                snprintf(g_reason, sizeof(g_reason),
                         "TG_BACKEND=%s refused: this build routes the KV-cache path to CUDA "
                         "only (no %s path, no fallback)", env, env);
            else
                snprintf(g_reason, sizeof(g_reason),
                         "TG_BACKEND=%s not recognised (auto or cuda; cpu and vulkan are "
                         "refused)", env);
            return 0;
        }
        if (!tg_be_select("cuda")) {
            snprintf(g_reason, sizeof(g_reason), "cuda: %s", tg_cuda_kv_last_error());
            return 0;
        }
        b = tg_be_current();
    }
    if (b != &tg_backend_cuda) {
        snprintf(g_reason, sizeof(g_reason), "backend %s is not cuda", b ? b->name : "(none)");
        return 0;
    }
    snprintf(g_reason, sizeof(g_reason), "cuda: KV-cache path on %s", tg_cuda_kv_device_name());
    return 1;
}

int tg_gpu_backend_ready(void) { return tg_be_current() == &tg_backend_cuda && tg_cuda_kv_ready(); }
const char* tg_gpu_backend_name(void) { return tg_gpu_backend_ready() ? "cuda" : "none"; }
const char* tg_gpu_backend_reason(void) { return g_reason; }
const char* tg_gpu_backend_device(void) { return tg_gpu_backend_ready() ? tg_cuda_kv_device_name() : ""; }
void tg_gpu_backend_shutdown(void) {
    tg_be_shutdown();
    snprintf(g_reason, sizeof(g_reason), "shut down");
}

void tg_gpu_kv_stats(uint64_t* calls, uint64_t* ok, uint64_t* fallbacks) {
    pthread_mutex_lock(&g_mu);
    if (calls) *calls = g_calls;
    if (ok) *ok = g_ok;
    if (fallbacks) *fallbacks = 0;
    pthread_mutex_unlock(&g_mu);
}

/* ---- cache registry (small open list; caches are few and long-lived) ---- */
typedef struct {
    const void* base;
    int dtype;
    uint32_t max_seq, n_kv_heads, head_dim;
    const void* tmap;
} RegEntry;
static RegEntry* g_reg = NULL;
static size_t g_reg_n = 0, g_reg_cap = 0;

void tg_gpu_kv_register(const void* base, int dtype, uint32_t max_seq, uint32_t n_kv_heads,
                        uint32_t head_dim, const void* tmap) {
    pthread_mutex_lock(&g_mu);
    if (g_reg_n == g_reg_cap) {
        size_t nc = g_reg_cap ? g_reg_cap * 2 : 64;
        RegEntry* r = (RegEntry*)realloc(g_reg, nc * sizeof(RegEntry));
        if (!r) { pthread_mutex_unlock(&g_mu); return; }
        g_reg = r;
        g_reg_cap = nc;
    }
    g_reg[g_reg_n].base = base;
    g_reg[g_reg_n].dtype = dtype;
    g_reg[g_reg_n].max_seq = max_seq;
    g_reg[g_reg_n].n_kv_heads = n_kv_heads;
    g_reg[g_reg_n].head_dim = head_dim;
    g_reg[g_reg_n].tmap = tmap;
    g_reg_n++;
    pthread_mutex_unlock(&g_mu);
}

void tg_gpu_kv_unregister(const void* base) {
    pthread_mutex_lock(&g_mu);
    for (size_t i = 0; i < g_reg_n; i++)
        if (g_reg[i].base == base) { g_reg[i] = g_reg[--g_reg_n]; break; }
    pthread_mutex_unlock(&g_mu);
}

int tg_gpu_kv_lookup_dtype(const void* base) {
    int d = -1;
    pthread_mutex_lock(&g_mu);
    for (size_t i = 0; i < g_reg_n; i++)
        if (g_reg[i].base == base) { d = g_reg[i].dtype; break; }
    pthread_mutex_unlock(&g_mu);
    return d;
}

const void* tg_gpu_kv_lookup_tmap(const void* base, uint32_t max_seq, uint32_t n_kv_heads,
                                  uint32_t head_dim) {
    const void* t = NULL;
    pthread_mutex_lock(&g_mu);
    for (size_t i = 0; i < g_reg_n; i++)
        if (g_reg[i].base == base && g_reg[i].max_seq == max_seq &&
            g_reg[i].n_kv_heads == n_kv_heads && g_reg[i].head_dim == head_dim) {
            t = g_reg[i].tmap;
            break;
        }
    pthread_mutex_unlock(&g_mu);
    return t;
}

/* ---- routing ------------------------------------------------------------ */
static int route_begin(void) {
    pthread_mutex_lock(&g_mu);
    g_calls++;
    pthread_mutex_unlock(&g_mu);
    if (tg_be_current() != &tg_backend_cuda) {
        set_err("KV-cache path needs the cuda backend (tg_be_select(\"cuda\")); no fallback");
        return 0;
    }
    if (!tg_cuda_kv_ready() && !tg_cuda_kv_init()) {
        set_err("%s", tg_cuda_kv_last_error());
        return 0;
    }
    return 1;
}

static int route_end(int ok) {
    if (!ok) { set_err("%s", tg_cuda_kv_last_error()); return 0; }
    pthread_mutex_lock(&g_mu);
    g_ok++;
    pthread_mutex_unlock(&g_mu);
    return 1;
}

int tg_gpu_kv_append_dev(int dtype, void* base, uint32_t max_seq, uint32_t kv_dim,
                         uint32_t row0, const float* k, const float* v, uint32_t n,
                         void* stream) {
    if (!route_begin()) return 0;
    TGCudaCacheDesc d = {(uint64_t)(uintptr_t)base, max_seq, 0, 0, 0};
    return route_end(tg_cuda_kv_append(dtype, d, kv_dim, row0, k, v, n, stream));
}

int tg_gpu_kv_attention(int dtype, void* base, uint32_t max_seq, const void* tmap,
                        const void* tmap_sw, uint32_t n_heads,
                        uint32_t n_kv_heads, uint32_t head_dim, const float* q, float* out,
                        const uint32_t* n_pos, uint32_t n_items, float scale,
                        void* scratch, uint32_t* counters, void* stream) {
    if (!route_begin()) return 0;
    TGCudaAttnCall c;
    memset(&c, 0, sizeof(c));
    c.dtype = dtype;
    c.n_heads = n_heads;
    c.n_kv_heads = n_kv_heads;
    c.head_dim = head_dim;
    c.cache.base = (uint64_t)(uintptr_t)base;
    c.cache.max_seq = max_seq;
    c.cache.tmap = (uint64_t)(uintptr_t)tmap;
    c.cache.tmap_sw = (uint64_t)(uintptr_t)tmap_sw;
    c.q = q;
    c.out = out;
    c.n_pos = n_pos;
    c.n_items = n_items;
    c.scale = scale;
    c.scratch = scratch;
    c.counters = counters;
    return route_end(tg_cuda_kv_attention(&c, stream));
}
