/* tgai_engine_bridge.c -- the engine's CUDA seam (cuda/tgai_cuda_bridge.h:31-60)
 * over the whole-model forward of tgai_forward.c.
 *
 * Contract of the reference bridge (cuda/tgai_cuda_bridge.c): init runs once
 * per process (again only after shutdown), only when TGAI_USE_GPU is set to
 * a non-zero value, and returns 0 with a reason when the GPU path does not
 * take the model; forward returns 0 without counting when the bridge is not
 * ready or the model is not the one it took, and counts a fallback when the
 * GPU forward itself fails.  The reference reads the model through the
 * engine's exported accessors; so does this file, resolving tg_config,
 * find_weight, get_cached_weight and tg_preload_all in the engine object that
 * called tg_engine_cuda_init (else anywhere in the process;
 * src/tgai_engine.h:60-117), so that the library links without the engine.
 */
#define _GNU_SOURCE
#include "tgai_engine_bridge.h"

#include <dlfcn.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* The .TG file header as tg_config returns it: the 128-byte packed layout of
 * src/tgai_format.h:156-188 (fields this bridge reads). */
#pragma pack(push, 1)
typedef struct {
    uint32_t magic, version, weight_dtype;
    uint32_t n_layers, d_model, n_heads, d_ff, vocab_size, max_seq_len;
    uint32_t n_experts, n_activated, rope_theta;
    uint32_t pad_token_id, bos_token_id, eos_token_id, unk_token_id;
    uint64_t tokenizer_off, tokenizer_len, weight_table_off, weight_table_count;
    uint64_t weight_data_off, weight_data_len;
    uint32_t arch_type, num_kv_heads, modality_flags, extension_off;
} EngineHeader;

/* One weight-table entry: src/tgai_format.h:190-200 (52 bytes). */
typedef struct {
    uint64_t name_hash, offset, length;
    uint32_t dtype, ndim;
    uint32_t shape[4];
    uint32_t scale_or_pad;
} EngineWeightEntry;
#pragma pack(pop)

_Static_assert(sizeof(EngineHeader) == 128, "TG header is 128 bytes");
_Static_assert(sizeof(EngineWeightEntry) == 52, "TG weight entry is 52 bytes");

typedef const EngineHeader* (*config_fn)(const TGModel*);
typedef const EngineWeightEntry* (*find_fn)(TGModel*, const char*);
typedef float* (*get_fn)(TGModel*, const EngineWeightEntry*);
typedef int (*preload_fn)(TGModel*);

/* Slot introspection of tgai_forward.c (internal). */
int tgkv_fwd_slot_index(TGFwdModel* m, const void* key);
long long tgkv_fwd_rejects(const TGFwdModel* m);
uint32_t tgkv_fwd_max_slots(const TGFwdModel* m);

static pthread_mutex_t g_lock = PTHREAD_MUTEX_INITIALIZER;
static TGFwdModel* g_fwd;
static TGModel* g_model;
static int g_ready, g_inited;
static long long g_calls, g_fallbacks;
static char g_reason[256] = "not initialized";
static config_fn p_config;
static find_fn p_find;
static get_fn p_get;

typedef struct {
    TGModel* m;
} EngineCtx;

/* TGFwdWeightFn over the engine's accessors; rows = shape[0], columns = the
 * product of the rest (the engine stores Linear weights as [out, in]). */
static const float* engine_weight(void* ctx, const char* name, uint32_t shape[2]) {
    TGModel* m = ((EngineCtx*)ctx)->m;
    const EngineWeightEntry* e = p_find(m, name);
    if (!e || e->ndim < 1 || e->ndim > 4) return NULL;
    uint64_t cols = 1;
    for (uint32_t i = 1; i < e->ndim; i++) cols *= e->shape[i];
    if (cols > 0xffffffffu) return NULL;
    shape[0] = e->shape[0];
    shape[1] = (uint32_t)cols;
    return p_get(m, e);
}

static int env_on(void) {
    const char* e = getenv("TGAI_USE_GPU");
    return e && e[0] && e[0] != '0';
}

int tg_engine_cuda_init(TGModel* m) {
    pthread_mutex_lock(&g_lock);
    if (g_inited) {
        const int r = g_ready;
        pthread_mutex_unlock(&g_lock);
        return r;
    }
    g_inited = 1;
    int ok = 0;
    if (!m) {
        snprintf(g_reason, sizeof(g_reason), "model handle is NULL");
    } else if (!env_on()) {
        snprintf(g_reason, sizeof(g_reason),
                 "TGAI_USE_GPU not enabled (set to 1 to enable GPU forward)");
    } else {
        /* the accessors of the engine that called us (tg_load), else any in the process */
        void* eng = NULL;
        Dl_info di;
        if (dladdr(__builtin_return_address(0), &di) && di.dli_fname)
            eng = dlopen(di.dli_fname, RTLD_LAZY | RTLD_NOLOAD);
        if (eng && !dlsym(eng, "tg_config")) {
            dlclose(eng);
            eng = NULL;
        }
        void* const held = eng;            /* the engine stays loaded: it called us */
        if (!eng) eng = RTLD_DEFAULT;
        p_config = (config_fn)dlsym(eng, "tg_config");
        p_find = (find_fn)dlsym(eng, "find_weight");
        p_get = (get_fn)dlsym(eng, "get_cached_weight");
        preload_fn preload = (preload_fn)dlsym(eng, "tg_preload_all");
        if (held) dlclose(held);
        const EngineHeader* h = p_config && p_find && p_get ? p_config(m) : NULL;
        if (!p_config || !p_find || !p_get) {
            snprintf(g_reason, sizeof(g_reason),
                     "engine accessors tg_config/find_weight/get_cached_weight not found in the process");
        } else if (!h || h->magic != 0x49414754u) {
            snprintf(g_reason, sizeof(g_reason), "failed to read model header (bad magic)");
        } else if (p_find(m, "blocks.0.attn.q_norm.weight")) {
            snprintf(g_reason, sizeof(g_reason), "QK-Norm models stay on the CPU path");
        } else if (p_find(m, "blocks.0.attn_res_proj.proj.weight")) {
            snprintf(g_reason, sizeof(g_reason), "block AttnRes models stay on the CPU path");
        } else {
            if (preload) preload(m);
            TGFwdConfig c;
            memset(&c, 0, sizeof(c));
            c.n_layers = h->n_layers;
            c.d_model = h->d_model;
            c.n_heads = h->n_heads;
            c.n_kv_heads = h->num_kv_heads ? h->num_kv_heads : h->n_heads;
            /* head_dim from q_proj's rows, as the engine infers it
             * (src/tgai_engine.c:1893-1905) */
            const EngineWeightEntry* q = p_find(m, "blocks.0.attn.q_proj.weight");
            c.head_dim = (q && h->n_heads && q->shape[0] % h->n_heads == 0)
                             ? q->shape[0] / h->n_heads : h->d_model / (h->n_heads ? h->n_heads : 1);
            c.d_ff = h->d_ff;
            c.vocab_size = h->vocab_size;
            c.max_seq_len = h->max_seq_len;
            c.n_experts = h->n_experts;
            c.n_activated = h->n_activated;
            c.rope_theta = (float)h->rope_theta;
            c.unk_id = (int32_t)h->unk_token_id;
            EngineCtx ctx = {m};
            g_fwd = tg_fwd_create(&c, engine_weight, &ctx);
            if (!g_fwd) {
                snprintf(g_reason, sizeof(g_reason), "GPU forward not available: %s",
                         tg_fwd_last_error());
            } else {
                g_model = m;
                g_ready = ok = 1;
                snprintf(g_reason, sizeof(g_reason),
                         "TAKEN OVER (GPU forward; model resident in HBM, %llu weight bytes)",
                         (unsigned long long)tg_fwd_weight_bytes(g_fwd));
            }
        }
    }
    pthread_mutex_unlock(&g_lock);
    return ok;
}

int tg_engine_cuda_forward(TGModel* m, const int32_t* input_ids, int seq_len, TGKVCache* cache,
                           int cache_pos, const float** out_logits) {
    if (out_logits) *out_logits = NULL;
    if (!g_ready || !g_fwd || m != g_model) return 0;
    if (seq_len <= 0 || !input_ids || cache_pos < 0) return 0;
    const float* lg = tg_fwd_forward(g_fwd, cache, input_ids, (uint32_t)seq_len,
                                     (uint32_t)cache_pos);
    if (!lg) {
        __atomic_add_fetch(&g_fallbacks, 1, __ATOMIC_RELAXED);
        return 0;
    }
    __atomic_add_fetch(&g_calls, 1, __ATOMIC_RELAXED);
    if (out_logits) *out_logits = lg;
    return 1;
}

void tg_engine_cuda_reset_slot(TGKVCache* cache) {
    if (g_ready && g_fwd) tg_fwd_reset_slot(g_fwd, cache);
}

void tg_engine_cuda_free_slot(TGKVCache* cache) {
    if (g_ready && g_fwd) tg_fwd_free_slot(g_fwd, cache);
}

void tg_engine_cuda_reset(void) {
    pthread_mutex_lock(&g_lock);
    if (g_ready && g_fwd) tg_fwd_reset_all(g_fwd);
    pthread_mutex_unlock(&g_lock);
}

void tg_engine_cuda_shutdown(void) {
    pthread_mutex_lock(&g_lock);
    tg_fwd_destroy(g_fwd);
    g_fwd = NULL;
    g_model = NULL;
    g_ready = g_inited = 0;
    snprintf(g_reason, sizeof(g_reason), "shut down");
    pthread_mutex_unlock(&g_lock);
}

int tg_engine_cuda_ready(void) { return g_ready; }
const char* tg_engine_cuda_reason(void) { return g_reason; }
long long tg_engine_cuda_calls(void) { return __atomic_load_n(&g_calls, __ATOMIC_RELAXED); }
long long tg_engine_cuda_fallbacks(void) { return __atomic_load_n(&g_fallbacks, __ATOMIC_RELAXED); }

/* Slot introspection of the reference bridge (cuda/tgai_cuda_bridge.c):
 * -1 when the GPU forward has not taken over. */
int tg_gpu_kv_slot_of(void* cache) {
    return g_ready && g_fwd ? tgkv_fwd_slot_index(g_fwd, cache) : -1;
}
int tg_gpu_kv_slot_seq(void* cache) {
    return g_ready && g_fwd ? tg_fwd_slot_last_pos(g_fwd, cache) : -1;
}
int tg_gpu_kv_slot_live(void) { return g_ready && g_fwd ? (int)tg_fwd_slot_count(g_fwd) : -1; }
int tg_gpu_kv_slot_max(void) { return g_ready && g_fwd ? (int)tgkv_fwd_max_slots(g_fwd) : -1; }
long long tg_gpu_kv_slot_rejects(void) { return g_ready && g_fwd ? tgkv_fwd_rejects(g_fwd) : -1; }
long long tg_gpu_cuda_calls(void) { return tg_engine_cuda_calls(); }
long long tg_gpu_cuda_fallbacks(void) { return tg_engine_cuda_fallbacks(); }
