/* tgai_backend.h -- TGAI GO's compute-backend function table, CUDA only.
 *
 * Keeps the reference's struct TGBackend field order and signatures
 * (src/tgai_backend.h:55-94) and its selection API (src/tgai_backend.h:99-118)
 * so code written against the reference table compiles and links unchanged.
 * Only "cuda" is implemented: "cpu" and "vulkan" exist as names (their tables
 * have no init), and selecting them fails with "not compiled in" -- there is
 * no CPU or Vulkan fallback in this library.
 *
 * For "cuda": device handles are raw device addresses; alloc zero-fills;
 * map returns NULL (discrete HBM); upload/download/attention/rope block until
 * done.  rmsnorm, silu_mul, softmax, mm_bf16 and moe_router are NULL (outside
 * the KV-cache path).
 */
#ifndef TGAI_BACKEND_H
#define TGAI_BACKEND_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Capability bits (src/tgai_backend.h:31-40). */
#define TG_BE_CAP_F32   (1u << 0)
#define TG_BE_CAP_BF16  (1u << 1)
#define TG_BE_CAP_Q4    (1u << 2)
#define TG_BE_CAP_MM    (1u << 3)
#define TG_BE_CAP_NORM  (1u << 4)
#define TG_BE_CAP_ROPE  (1u << 5)
#define TG_BE_CAP_ATTN  (1u << 6)
#define TG_BE_CAP_MOE   (1u << 7)
#define TG_BE_CAP_KV    (1u << 8)
#define TG_BE_CAP_TRAIN (1u << 9)

/* src/tgai_backend.h:43-50 */
typedef struct {
    const char* name;
    const char* device_name;
    uint32_t    caps;
    uint64_t    mem_bytes;
    int         is_gpu;
    int         is_uma;
} TGBackendInfo;

typedef struct TGBackend TGBackend;

/* src/tgai_backend.h:55-94 -- field order is part of the ABI. */
struct TGBackend {
    const char* name;
    uint32_t    caps;

    int  (*init)(void);
    void (*shutdown)(void);
    int  (*ready)(void);
    int  (*info)(TGBackendInfo* out);
    const char* (*last_error)(void);

    void* (*alloc)(size_t bytes);
    void  (*free)(void* p);
    int   (*upload)(void* dst, const void* src, size_t bytes);
    int   (*download)(void* dst, const void* src, size_t bytes);
    void* (*map)(void* p);

    int (*rmsnorm)(void* x, void* w, void* y, uint32_t n_rows, uint32_t d, float eps);
    int (*silu_mul)(void* g, void* u, void* o, uint32_t n);
    int (*softmax)(void* x, void* y, uint32_t n_rows, uint32_t n_cols);
    /* RoPE + KV write, shaders/rope.comp semantics: qkv fp32
     * [n_tokens][q_dim + 2*kv_dim], cs/sn fp32 [max_seq][head_dim/2]; writes
     * rotated Q to qout [n_tokens][q_dim] and rotated K plus V into the cache
     * buffer kvc at positions start_pos + t. */
    int (*rope)(void* qkv, void* cs, void* sn, void* kvc, void* qout,
                uint32_t n_tokens, uint32_t n_heads, uint32_t n_kv_heads,
                uint32_t head_dim, uint32_t start_pos, uint32_t max_seq);
    int (*mm_bf16)(void* w, void* x, void* ypart,
                   uint32_t n_out, uint32_t n_in, uint32_t seq, uint32_t split);
    /* Single-query attention (tgai_vk_kernels.h:81-85 shape): q, out fp32
     * [n_heads][head_dim]; kvc a cache buffer [2][max_seq][kv_dim]; positions
     * j < n_kv with j <= pos; scale 1/sqrt(head_dim).  kvc from
     * tg_kv_device_handle() of a bf16 cache is read as bf16, any other
     * address as fp32. */
    int (*attention)(void* q, void* kvc, void* out,
                     uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                     uint32_t n_kv, uint32_t pos, uint32_t max_seq);
    int (*moe_router)(void* x, void* router_w, void* qbias, void* topids, void* topprob,
                      uint32_t n_experts, uint32_t d_model, uint32_t top_k, int use_qb);

    void* priv;
};

/* src/tgai_backend.h:99-118 */
int tg_be_probe(void);
int tg_be_select(const char* name);          /* NULL/"auto" -> TG_BACKEND or "cuda" */
TGBackend* tg_be_current(void);
int tg_be_current_info(TGBackendInfo* out);
void tg_be_shutdown(void);
const char* const* tg_be_list(void);

extern TGBackend tg_backend_cpu;              /* name only: not compiled in */
extern TGBackend tg_backend_vulkan;           /* name only: not compiled in */
extern TGBackend tg_backend_cuda;             /* the implementation */

#ifdef __cplusplus
}
#endif
#endif /* TGAI_BACKEND_H */
