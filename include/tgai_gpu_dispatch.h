/* tgai_gpu_dispatch.h -- routes TGAI GO's KV-cache path to the CUDA kernels.
 *
 * The reference router (src/tgai_gpu_dispatch.c) reads TG_BACKEND
 * (tgai_gpu_dispatch.c:467-492), reports status through tg_gpu_backend_*
 * (tgai_gpu_dispatch.c:773-819) and falls back to the CPU when the GPU path is
 * unavailable.  This router keeps the status names, routes only the KV-cache
 * path, accepts TG_BACKEND = auto | cuda, and never falls back: a call that
 * cannot run on the GPU fails with a reason.
 */
#ifndef TGAI_GPU_DISPATCH_H
#define TGAI_GPU_DISPATCH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status (tgai_gpu_dispatch.c:773-819 names). */
int         tg_gpu_backend_init(void);      /* selects "cuda" if no backend is selected */
int         tg_gpu_backend_ready(void);
const char* tg_gpu_backend_name(void);      /* "cuda" or "none" */
const char* tg_gpu_backend_reason(void);
const char* tg_gpu_backend_device(void);
void        tg_gpu_backend_shutdown(void);

/* Counters of routed KV-path calls; `fallbacks` is always 0 (kept so callers
 * written against the reference's tg_gpu_stats-style counters can assert it). */
void tg_gpu_kv_stats(uint64_t* calls, uint64_t* ok, uint64_t* fallbacks);

/* Registry of live caches by device address, so that TGBackend.attention
 * given only `kvc` knows the storage type (a bf16 cache reads as bf16). */
void tg_gpu_kv_register(const void* base, int dtype, uint32_t max_seq, uint32_t n_kv_heads,
                        uint32_t head_dim, const void* tmap);
void tg_gpu_kv_unregister(const void* base);
int  tg_gpu_kv_lookup_dtype(const void* base);   /* -1 if not a registered cache */
/* Tensor map of a registered cache with exactly this geometry, else NULL. */
const void* tg_gpu_kv_lookup_tmap(const void* base, uint32_t max_seq, uint32_t n_kv_heads,
                                  uint32_t head_dim);

/* Routed operations (1 = done, 0 = failed; reason in tg_kv_last_error()). */
int tg_gpu_kv_append_dev(int dtype, void* base, uint32_t max_seq, uint32_t kv_dim,
                         uint32_t row0, const float* k, const float* v, uint32_t n,
                         void* stream);
/* tmap: the cache's tensor map; tmap_sw: its 128B-swizzled map (bf16
 * head_dim-128 caches, for the tensor-core suffix kernel) or NULL. */
int tg_gpu_kv_attention(int dtype, void* base, uint32_t max_seq, const void* tmap,
                        const void* tmap_sw, uint32_t n_heads,
                        uint32_t n_kv_heads, uint32_t head_dim, const float* q, float* out,
                        const uint32_t* n_pos, uint32_t n_items, float scale,
                        void* scratch, uint32_t* counters, void* stream);
const char* tg_gpu_kv_error(void);               /* reason of the last failure */

#ifdef __cplusplus
}
#endif
#endif
