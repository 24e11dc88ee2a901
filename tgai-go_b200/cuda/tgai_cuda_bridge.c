/* tgai_cuda_bridge.c -- thin C layer from TGAI GO host code to CUDA for the
 * KV-cache path.  Plain C (C11); talks to the CUDA runtime and to the kernel
 * launchers of tgkv_kernels.cu, nothing else.
 *
 * Host-side planning of split-sequence attention lives here: the per-item
 * position counts, the chunk length and the chunk prefix table are computed
 * on the host and handed to the kernel by value (tgkv_launch.h), so a launch
 * needs no copy of its own.
 */
#include "tgai_cuda_bridge.h"
#include "tgkv_launch.h"

#include <cuda.h>                 /* CUtensorMap types; the encoder comes from the runtime */
#include <cuda_runtime_api.h>
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static _Thread_local char t_err[256] = "cuda bridge: no error";
static _Thread_local uint32_t t_last_launches = 0;
static _Thread_local int t_last_kernel = 0;
static _Thread_local uint32_t t_last_split = 0;

static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;
static int g_ready = 0;
static int g_sm_count = 0;
static uint64_t g_mem = 0;
static char g_name[256] = "";
static int32_t* g_err_word = NULL;      /* device error word for bounded waits */
static int g_fail_allocs = 0;           /* testing hook */

static void set_err(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}

static int cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return 1;
    set_err("%s: %s", what, cudaGetErrorString(e));
    return 0;
}

const char* tg_cuda_kv_last_error(void) { return t_err; }

int tg_cuda_kv_init(void) {
    pthread_mutex_lock(&g_mu);
    if (g_ready) { pthread_mutex_unlock(&g_mu); return 1; }
    const char* fa = getenv("TGKV_FAIL_ALLOC");
    if (fa && fa[0]) g_fail_allocs = atoi(fa);
    int n = 0, dev = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n <= 0) {
        set_err("no CUDA device: %s", e == cudaSuccess ? "count is 0" : cudaGetErrorString(e));
        pthread_mutex_unlock(&g_mu);
        return 0;
    }
    struct cudaDeviceProp prop;
    if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice") ||
        !cuda_ok(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties")) {
        pthread_mutex_unlock(&g_mu);
        return 0;
    }
    if (prop.major < 10) {
        set_err("device %s is sm_%d%d; this build targets sm_100a", prop.name, prop.major,
                prop.minor);
        pthread_mutex_unlock(&g_mu);
        return 0;
    }
    snprintf(g_name, sizeof(g_name), "%s", prop.name);
    g_sm_count = prop.multiProcessorCount;
    g_mem = (uint64_t)prop.totalGlobalMem;
    if (!cuda_ok(cudaMalloc((void**)&g_err_word, 256), "cudaMalloc(error word)") ||
        !cuda_ok(cudaMemset(g_err_word, 0, 256), "cudaMemset(error word)")) {
        pthread_mutex_unlock(&g_mu);
        return 0;
    }
    g_ready = 1;
    pthread_mutex_unlock(&g_mu);
    return 1;
}

/* ---- TMA tensor maps -------------------------------------------------------
 * cuTensorMapEncodeTiled is reached through cudaGetDriverEntryPoint, so the
 * library needs no link against libcuda. */
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn g_encode = NULL;

static int resolve_encode(void) {
    if (g_encode) return 1;
    enum cudaDriverEntryPointQueryResult q;
    void* fn = NULL;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess || !fn) {
        set_err("cuTensorMapEncodeTiled unavailable");
        return 0;
    }
    g_encode = (EncodeTiledFn)fn;
    return 1;
}

static int encode_tmap_box(int dtype, uint64_t base, uint32_t max_seq, uint32_t n_kv_heads,
                           uint32_t head_dim, uint32_t box_x, uint32_t box_y, int swizzle128,
                           CUtensorMap* out) {
    if (!resolve_encode()) return 0;
    const uint64_t es = dtype == 1 ? 2 : 4;
    const uint64_t kv_dim = (uint64_t)n_kv_heads * head_dim;
    if ((base & 15u) || (kv_dim * es) % 16 || (head_dim * es) % 16 || head_dim > 256) {
        set_err("tensor map: cache layout not TMA-compatible (head_dim %u)", head_dim);
        return 0;
    }
    cuuint64_t dims[3] = {kv_dim, max_seq, 2};
    cuuint64_t strides[2] = {kv_dim * es, (uint64_t)max_seq * kv_dim * es};
    cuuint32_t box[3] = {box_x, box_y, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(out, dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                          3, (void*)(uintptr_t)base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_err("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return 0;
    }
    return 1;
}

static int encode_tmap(int dtype, uint64_t base, uint32_t max_seq, uint32_t n_kv_heads,
                       uint32_t head_dim, CUtensorMap* out) {
    return encode_tmap_box(dtype, base, max_seq, n_kv_heads, head_dim, head_dim, TGKV_TILE, 0,
                           out);
}

/* The suffix kernel's map over q [n_q][n_heads][128] fp32: dims (128,
 * n_heads, n_q), 128B swizzle, box (32, g, 128/g) -- 32 head dims of the 128
 * (token, head) rows one CTA owns; rows past n_q read as zero. */
static int encode_qmap(const float* q, uint32_t n_heads, uint32_t n_q, uint32_t g, CUtensorMap* out) {
    if (!resolve_encode()) return 0;
    cuuint64_t dims[3] = {128, n_heads, n_q};
    cuuint64_t strides[2] = {128 * 4, (uint64_t)n_heads * 128 * 4};
    cuuint32_t box[3] = {32, g, 128 / g};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void*)q, dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_err("cuTensorMapEncodeTiled (q) failed (%d)", (int)r);
        return 0;
    }
    return 1;
}

void* tg_cuda_kv_tmap_sw_create(uint64_t base, uint32_t max_seq, uint32_t n_kv_heads) {
    if (!g_ready && !tg_cuda_kv_init()) return NULL;
    CUtensorMap m;
    if (!encode_tmap_box(1, base, max_seq, n_kv_heads, 128, 64, 128, 1, &m)) return NULL;
    void* d = tg_cuda_kv_malloc(sizeof(CUtensorMap));
    if (!d) return NULL;
    if (!cuda_ok(cudaMemcpy(d, &m, sizeof(m), cudaMemcpyHostToDevice), "tensor map h2d")) {
        tg_cuda_kv_free(d);
        return NULL;
    }
    return d;
}

int tg_cuda_kv_tmap_write(int dtype, uint64_t base, uint32_t max_seq, uint32_t n_kv_heads,
                          uint32_t head_dim, void* tmap_dev) {
    if (!g_ready && !tg_cuda_kv_init()) return 0;
    if (!tmap_dev || ((uintptr_t)tmap_dev & 63u)) { set_err("tensor map: bad destination"); return 0; }
    CUtensorMap m;
    if (!encode_tmap(dtype, base, max_seq, n_kv_heads, head_dim, &m)) return 0;
    return cuda_ok(cudaMemcpy(tmap_dev, &m, sizeof(m), cudaMemcpyHostToDevice), "tensor map h2d");
}

void* tg_cuda_kv_tmap_create(int dtype, uint64_t base, uint32_t max_seq, uint32_t n_kv_heads,
                             uint32_t head_dim) {
    void* d = tg_cuda_kv_malloc(sizeof(CUtensorMap));
    if (!d) return NULL;
    if (!tg_cuda_kv_tmap_write(dtype, base, max_seq, n_kv_heads, head_dim, d)) {
        tg_cuda_kv_free(d);
        return NULL;
    }
    return d;
}

int tg_cuda_kv_set_device(int device) {
    if (!cuda_ok(cudaSetDevice(device), "cudaSetDevice")) return 0;
    pthread_mutex_lock(&g_mu);
    const int was_ready = g_ready;
    pthread_mutex_unlock(&g_mu);
    if (was_ready) {                 /* re-read properties for the new device */
        tg_cuda_kv_shutdown();
        return tg_cuda_kv_init();
    }
    return 1;
}

void tg_cuda_kv_shutdown(void) {
    pthread_mutex_lock(&g_mu);
    if (g_err_word) cudaFree(g_err_word);
    g_err_word = NULL;
    g_ready = 0;
    pthread_mutex_unlock(&g_mu);
}

int tg_cuda_kv_ready(void) { return g_ready; }
const char* tg_cuda_kv_device_name(void) { return g_name; }
uint64_t tg_cuda_kv_device_mem(void) { return g_mem; }
int tg_cuda_kv_sm_count(void) { return g_sm_count; }

void tg_cuda_kv_inject_alloc_failures(int n) {
    pthread_mutex_lock(&g_mu);
    g_fail_allocs = n;
    pthread_mutex_unlock(&g_mu);
}

void* tg_cuda_kv_malloc(size_t bytes) {
    if (!g_ready && !tg_cuda_kv_init()) return NULL;
    pthread_mutex_lock(&g_mu);
    if (g_fail_allocs > 0) {
        g_fail_allocs--;
        pthread_mutex_unlock(&g_mu);
        set_err("cudaMalloc(%zu): injected failure (TGKV_FAIL_ALLOC)", bytes);
        return NULL;
    }
    pthread_mutex_unlock(&g_mu);
    void* p = NULL;
    if (!cuda_ok(cudaMalloc(&p, bytes ? bytes : 1), "cudaMalloc")) return NULL;
    /* the zero fill completes before the pointer is returned: work queued on
     * non-blocking streams is not ordered after the legacy stream's memset */
    if (!cuda_ok(cudaMemset(p, 0, bytes), "cudaMemset") ||
        !cuda_ok(cudaStreamSynchronize(0), "cudaMemset sync")) {
        cudaFree(p);
        return NULL;
    }
    return p;
}

void tg_cuda_kv_free(void* p) {
    if (p) cudaFree(p);
}

void* tg_cuda_kv_stream_create(void) {
    if (!g_ready && !tg_cuda_kv_init()) return NULL;
    cudaStream_t s = NULL;
    if (!cuda_ok(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) return NULL;
    return (void*)s;
}

void tg_cuda_kv_stream_destroy(void* stream) {
    if (stream) cudaStreamDestroy((cudaStream_t)stream);
}

void* tg_cuda_kv_event_create(void) {
    if (!g_ready && !tg_cuda_kv_init()) return NULL;
    cudaEvent_t e = NULL;
    if (!cuda_ok(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate")) return NULL;
    return (void*)e;
}

void tg_cuda_kv_event_destroy(void* event) {
    if (event) cudaEventDestroy((cudaEvent_t)event);
}

int tg_cuda_kv_event_record(void* event, void* stream) {
    if (!event) { set_err("event record: null event"); return 0; }
    return cuda_ok(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream), "cudaEventRecord");
}

int tg_cuda_kv_stream_wait(void* stream, void* event) {
    if (!event) { set_err("stream wait: null event"); return 0; }
    return cuda_ok(cudaStreamWaitEvent((cudaStream_t)stream, (cudaEvent_t)event, 0),
                   "cudaStreamWaitEvent");
}

void* tg_cuda_kv_host_device_ptr(const void* host) {
    if (!host || (!g_ready && !tg_cuda_kv_init())) return NULL;
    struct cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, host) != cudaSuccess) {
        cudaGetLastError();
        return NULL;
    }
    return a.type == cudaMemoryTypeHost ? a.devicePointer : NULL;
}

static int launch_rc(int rc, const char* what);

int tg_cuda_kv_ipc_handle(const void* dev, void* handle64) {
    if (!g_ready && !tg_cuda_kv_init()) return 0;
    if (!dev || !handle64) { set_err("ipc: null argument"); return 0; }
    cudaIpcMemHandle_t h;
    if (!cuda_ok(cudaIpcGetMemHandle(&h, (void*)dev), "cudaIpcGetMemHandle")) return 0;
    memcpy(handle64, &h, sizeof(h) < 64 ? sizeof(h) : 64);
    return 1;
}

void* tg_cuda_kv_ipc_open(const void* handle64) {
    if (!g_ready && !tg_cuda_kv_init()) return NULL;
    if (!handle64) { set_err("ipc: null handle"); return NULL; }
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    void* p = NULL;
    if (!cuda_ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
        return NULL;
    return p;
}

void tg_cuda_kv_ipc_close(void* dev) {
    if (dev) cudaIpcCloseMemHandle(dev);
}

int tg_cuda_kv_gather_wait(const uint32_t* flag, uint32_t target, void* stream) {
    if (!g_ready && !tg_cuda_kv_init()) return 0;
    if (!flag) { set_err("gather wait: null flag"); return 0; }
    return launch_rc(tgkv_launch_gather_wait(flag, target, g_err_word, stream), "gather wait");
}

int tg_cuda_kv_h2d(void* dst, const void* src, size_t bytes, void* stream) {
    if (!bytes) return 1;
    if (!stream) return cuda_ok(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice), "h2d");
    return cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream),
                   "h2d async");
}

int tg_cuda_kv_h2d_async(void* dst, const void* src, size_t bytes, void* stream) {
    if (!bytes) return 1;
    return cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream),
                   "h2d async");
}

int tg_cuda_kv_d2h_async(void* dst, const void* src, size_t bytes, void* stream) {
    if (!bytes) return 1;
    return cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream),
                   "d2h async");
}

int tg_cuda_kv_stage_host(void* dst, const void* a, size_t na, const void* b, size_t nb,
                          const void* c, size_t nc, void* stream) {
    if ((na | nb | nc) % 16 || (((uintptr_t)dst | (uintptr_t)a | (uintptr_t)b | (uintptr_t)c) & 15)) {
        set_err("stage: sizes and addresses must be multiples of 16 bytes");
        return 0;
    }
    return launch_rc(tgkv_launch_stage_host(a, na, b, nb, c, nc, dst, stream), "host staging");
}

int tg_cuda_kv_d2h(void* dst, const void* src, size_t bytes, void* stream) {
    if (!bytes) return 1;
    if (!stream) return cuda_ok(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost), "d2h");
    return cuda_ok(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream),
                   "d2h async");
}

int tg_cuda_kv_memset(void* dst, int value, size_t bytes, void* stream) {
    if (!bytes) return 1;
    if (!stream) return cuda_ok(cudaMemset(dst, value, bytes), "memset");
    return cuda_ok(cudaMemsetAsync(dst, value, bytes, (cudaStream_t)stream), "memset async");
}

int tg_cuda_kv_sync(void* stream) {
    if (!stream) return cuda_ok(cudaDeviceSynchronize(), "device sync");
    return cuda_ok(cudaStreamSynchronize((cudaStream_t)stream), "stream sync");
}

__attribute__((visibility("hidden"))) int32_t* tgkv_bridge_err_word(void) { return g_err_word; }

int tg_cuda_kv_device_error(void) {
    if (!g_ready) return 0;
    int32_t v = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    if (cudaMemcpy(&v, g_err_word, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (v) cudaMemset(g_err_word, 0, 4);
    return v;
}

/* ---- append ------------------------------------------------------------- */
static int launch_rc(int rc, const char* what) {
    if (rc == 0) return 1;
    set_err("%s: %s", what, cudaGetErrorString((cudaError_t)rc));
    return 0;
}

int tg_cuda_kv_append(int dtype, TGCudaCacheDesc cache, uint32_t kv_dim, uint32_t row0,
                      const float* k, const float* v, uint32_t n_rows, void* stream) {
    if (!g_ready && !tg_cuda_kv_init()) return 0;
    if (n_rows == 0) return 1;
    if (!k || !v || !cache.base) { set_err("append: NULL pointer"); return 0; }
    if ((uint64_t)row0 + n_rows > cache.max_seq) { set_err("append: capacity exceeded"); return 0; }
    if (kv_dim % 8) { set_err("append: kv_dim %u is not a multiple of 8", kv_dim); return 0; }
    if (((uintptr_t)k | (uintptr_t)v) & 15u) {
        set_err("append: source rows must be 16-byte aligned");
        return 0;
    }
    static _Thread_local TGKvAppendParams p;   /* ~4 KB: keep off the stack */
    memset(&p, 0, offsetof(TGKvAppendParams, pos));
    p.caches = NULL;
    p.cache0.base = cache.base;
    p.cache0.max_seq = cache.max_seq;
    p.k = k;
    p.v = v;
    p.cache_stride = 0;
    p.n_items = 1;
    p.rows_per_item = n_rows;
    p.kv_dim = kv_dim;
    p.pos[0] = row0;
    return launch_rc(tgkv_launch_append(&p, dtype, stream), "append kernel");
}

int tg_cuda_kv_append_batch(int dtype, const TGCudaCacheDesc* table_dev, uint32_t kv_dim,
                            const uint32_t* pos, uint32_t n_items,
                            const float* k, const float* v, void* stream) {
    if (!g_ready && !tg_cuda_kv_init()) return 0;
    if (n_items == 0) return 1;
    if (!table_dev || !pos || !k || !v) { set_err("append_batch: NULL pointer"); return 0; }
    if (kv_dim % 8) { set_err("append_batch: kv_dim %u is not a multiple of 8", kv_dim); return 0; }
    static _Thread_local TGKvAppendParams p;
    for (uint32_t b0 = 0; b0 < n_items; b0 += TGKV_MAX_ITEMS) {
        const uint32_t n = (n_items - b0) < TGKV_MAX_ITEMS ? (n_items - b0) : TGKV_MAX_ITEMS;
        memset(&p, 0, offsetof(TGKvAppendParams, pos));
        p.caches = (const TGKvCacheDesc*)(table_dev + b0);
        p.k = k + (uint64_t)b0 * kv_dim;
        p.v = v + (uint64_t)b0 * kv_dim;
        p.cache_stride = 1;
        p.n_items = n;
        p.rows_per_item = 1;
        p.kv_dim = kv_dim;
        memcpy(p.pos, pos + b0, n * sizeof(uint32_t));
        if (!launch_rc(tgkv_launch_append(&p, dtype, stream), "append_batch kernel")) return 0;
    }
    return 1;
}

/* ---- attention planning ------------------------------------------------- */
int tg_cuda_kv_attn_supported(int dtype, uint32_t head_dim) {
    return tgkv_attention_supported(dtype, head_dim);
}

typedef struct {
    uint32_t gt, n_sub, chunk;
    uint64_t max_chunks;      /* most chunks in any launch of the call */
    int tc;                   /* the tensor-core decode kernel runs it */
} AttnPlan;


/* Chunk length (one CTA per chunk of one item's positions for one KV head
 * and head subset).  CTAs run in waves (two per SM on the CUDA-core kernel,
 * one on the tensor-core one), and every wave costs a fixed start-up, tail
 * and merge time besides its streaming, measured on B200 at about the time
 * of 768 positions per CTA (cfg5: 103 / 124 / 139 us per layer at 1 / 2 / 3
 * waves against 83 us of pure streaming).  So the planner takes, over 1 to 16
 * waves, the smallest chunk whose CTAs fill exactly that many waves, and of
 * those the one minimising waves x (chunk + 768); never below 128 positions,
 * a multiple of the kernel's tile.  (Rounding the chunk up from total / slots
 * can spill a few CTAs into one more wave: one 131072-position sequence with
 * 8 KV heads made 152 CTAs for 148 slots.)  TGKV_CHUNK overrides (tests use it
 * to force split boundaries); TGKV_WAVES fixes the wave count. */
enum { kWaveOverheadPositions = 768 };

static uint64_t count_chunks(const uint32_t* n_pos, uint32_t n_items, uint32_t chunk, uint32_t mult) {
    uint64_t n = 0;
    for (uint32_t i = 0; i < n_items; i++) n += (n_pos[i] + chunk - 1) / chunk;   /* 32-bit */
    return n * mult;
}

static uint32_t round_up(uint64_t x, uint32_t tile) { return (uint32_t)((x + tile - 1) / tile * tile); }

__attribute__((visibility("hidden"))) uint32_t tgkv_pick_chunk(const uint32_t* n_pos, uint32_t n_items,
                                                             uint32_t mult, uint32_t sm_count) {
    return tgkv_pick_chunk_tiled(n_pos, n_items, mult, (sm_count ? sm_count : 148) * 2, TGKV_TILE);
}

__attribute__((visibility("hidden"))) uint32_t tgkv_pick_chunk_tiled(const uint32_t* n_pos,
                                                                   uint32_t n_items, uint32_t mult,
                                                                   uint32_t slots_in,
                                                                   uint32_t tile) {
    const char* e = getenv("TGKV_CHUNK");
    if (e && e[0] && atol(e) >= 1) return round_up((uint64_t)atol(e), tile);
    const uint64_t slots = slots_in ? slots_in : 296;
    uint32_t longest = 1;
    for (uint32_t i = 0; i < n_items; i++)
        if (n_pos[i] > longest) longest = n_pos[i];
    const uint32_t cmax = round_up(longest < 128 ? 128 : longest, tile);
    const char* w = getenv("TGKV_WAVES");
    const uint64_t forced = (w && w[0] && atol(w) >= 1) ? (uint64_t)atol(w) : 0;
    uint64_t best_cost = ~0ull, best = cmax;
    for (uint64_t waves = forced ? forced : 1; waves <= (forced ? forced : 16); waves++) {
        /* the smallest chunk (a multiple of tile, >= 128) whose CTAs fit in
         * `waves` full waves: the CTA count only falls as the chunk grows */
        const uint64_t cap = slots * waves;
        if (count_chunks(n_pos, n_items, cmax, mult) > cap) continue;
        uint32_t lo = 128 / tile, hi = cmax / tile;      /* in tiles; hi always fits */
        if (lo == 0) lo = 1;
        while (lo < hi) {
            const uint32_t mid = lo + (hi - lo) / 2;
            if (count_chunks(n_pos, n_items, mid * tile, mult) <= cap) hi = mid;
            else lo = mid + 1;
        }
        const uint64_t c = (uint64_t)lo * tile;
        const uint64_t n = count_chunks(n_pos, n_items, (uint32_t)c, mult);
        const uint64_t cost = (n + slots - 1) / slots * (c + kWaveOverheadPositions);
        if (cost < best_cost) {
            best_cost = cost;
            best = c;
        }
    }
    return (uint32_t)best;
}

/* Decode calls over bf16 head_dim-128 caches with a swizzled tensor map (a
 * batch's caches all have one when they are bf16 / 128) run on the
 * tensor-core decode kernel when the launch streams at least 131072
 * (position, KV head, head subset) rows -- about one wave of 16-tile CTAs.
 * That kernel keeps one CTA per SM and pays more per CTA (TMEM, the q terms,
 * the pipeline fill) but streams HBM at full speed; small launches are
 * latency-bound and stay on the CUDA-core kernel.  Measured on B200: 64
 * ragged sequences (cfg4) 0.99-1.02 of HBM against 0.86; one 131072-position
 * sequence 0.888 against 0.866; one 4096-position sequence (16384 rows)
 * 1739 against 2072 tok/s.  TGKV_DECODE_TC=1 takes every eligible call to
 * the tensor-core kernel, TGKV_DECODE_TC=0 none. */
static int use_decode_tc(const TGCudaAttnCall* c, uint32_t gt) {
    const char* e = getenv("TGKV_DECODE_TC");
    const int mode = (e && e[0] == '0') ? 0 : (e && e[0] == '1') ? 1 : -1;
    if (mode == 0 || c->dtype != 1 || c->head_dim != 128 || gt > 4 ||
        !(c->table_dev != NULL || c->cache.tmap_sw != 0))
        return 0;
    if (mode == 1) return 1;
    uint64_t rows = 0;
    for (uint32_t i = 0; i < c->n_items; i++) rows += c->n_pos[i];
    rows *= (uint64_t)c->n_heads / gt;                 /* KV heads x head subsets */
    /* one KV head of a 131072-position context (a GPU's share of configs[4]
     * split over 8): 1337 tok/s here against 1234 on the CUDA-core kernel;
     * one 4096-position sequence of 4 KV heads (16384 rows) stays there */
    return rows >= 131072;
}

static int plan_attention(const TGCudaAttnCall* c, AttnPlan* pl) {
    if (!c || c->n_kv_heads == 0 || c->n_heads == 0 || c->n_heads % c->n_kv_heads) {
        set_err("attention: n_heads must be a positive multiple of n_kv_heads");
        return 0;
    }
    if (!tgkv_attention_supported(c->dtype, c->head_dim)) {
        set_err("attention: no kernel for dtype %d head_dim %u", c->dtype, c->head_dim);
        return 0;
    }
    const uint32_t group = c->n_heads / c->n_kv_heads;
    pl->gt = tgkv_attention_g_tile(c->head_dim, group);
    pl->n_sub = group / pl->gt;
    for (uint32_t i = 0; i < c->n_items; i++)
        if (c->n_pos[i] == 0) { set_err("attention: item %u attends no position", i); return 0; }
    pl->tc = use_decode_tc(c, pl->gt);
    pl->chunk = pl->tc ? tgkv_pick_chunk_tiled(c->n_pos, c->n_items, c->n_kv_heads * pl->n_sub,
                                               (uint32_t)(g_sm_count ? g_sm_count : 148), 128)
                       : tgkv_pick_chunk(c->n_pos, c->n_items, c->n_kv_heads * pl->n_sub,
                                         (uint32_t)g_sm_count);
    pl->max_chunks = 0;
    for (uint32_t b0 = 0; b0 < c->n_items; b0 += TGKV_MAX_ITEMS) {
        const uint32_t n = (c->n_items - b0) < TGKV_MAX_ITEMS ? (c->n_items - b0) : TGKV_MAX_ITEMS;
        uint64_t chunks = 0;
        for (uint32_t i = 0; i < n; i++)
            chunks += (uint64_t)((c->n_pos[b0 + i] + pl->chunk - 1) / pl->chunk) * c->n_kv_heads *
                      pl->n_sub;
        if (chunks > 0x7fffffffu) { set_err("attention: too many chunks in one launch"); return 0; }
        if (chunks > pl->max_chunks) pl->max_chunks = chunks;
    }
    return 1;
}

/* Two-level merge of long segments (in groups of 16 chunks, then the
 * groups) above merge2_min() chunks; TGKV_MERGE2=0 merges every segment in
 * one CTA. */
static int merge2_on(void) {
    const char* e = getenv("TGKV_MERGE2");
    return !(e && e[0] == '0');
}
static uint32_t merge2_min(void) {
    const char* e = getenv("TGKV_MERGE2_MIN");
    return e && atoi(e) > 0 ? (uint32_t)atoi(e) : 96u;
}

/* Partial slots of a launch: one per chunk, and with the two-level merge as
 * many again for the group partials. */
static uint64_t part_slots(const AttnPlan* pl) {
    return pl->max_chunks * (merge2_on() ? 2u : 1u);
}

static uint64_t part_o_bytes(const AttnPlan* pl, uint32_t head_dim) {
    return (part_slots(pl) * pl->gt * head_dim * 4 + 255) / 256 * 256;
}

/* Blocks of query rows over one bf16 head_dim-128 cache go to the tensor-core
 * kernel (tgkv_prefill.cu) when there are at least 128 (row, head) pairs:
 * consecutive positions, group size 1/2/4/8, no fused append, q and out
 * 16-byte aligned.  TGKV_PREFILL=0
 * keeps them on the split-sequence kernel. */
static int use_prefill(const TGCudaAttnCall* c) {
    const char* e = getenv("TGKV_PREFILL");
    if (e && e[0] == '0') return 0;
    if (!c || !c->n_kv_heads || !c->n_heads || c->n_heads % c->n_kv_heads || !c->n_pos ||
        !c->n_items || c->n_pos[0] == 0)
        return 0;
    if (c->dtype != 1 || c->head_dim != 128 || c->table_dev || !c->cache.tmap_sw) return 0;
    /* new rows (the fused append): item i's row lands at position n_pos[i] - 1,
     * consecutive like the items; 16-byte rows for the kernel's loads */
    if (c->k_new && (!c->v_new || !c->cache.base ||
                     (((uintptr_t)c->k_new | (uintptr_t)c->v_new) & 15u)))
        return 0;
    const uint32_t g = c->n_heads / c->n_kv_heads;
    if (!(g == 1 || g == 2 || g == 4 || g == 8)) return 0;
    if ((uint64_t)c->n_items * g < 128) return 0;
    if (((uintptr_t)c->q | (uintptr_t)c->out) & 15u) return 0;   /* float4 rows */
    for (uint32_t i = 1; i < c->n_items; i++)
        if (c->n_pos[i] != c->n_pos[0] + i) return 0;
    return 1;
}

/* KV split of the suffix kernel: the most CTAs per row block (<= 8) that
 * keep the launch to one wave of clusters, no more than the first row block
 * has tiles.  TGKV_PF_SPLIT=n forces n (clamped to the same limits). */
static uint32_t prefill_split(const TGCudaAttnCall* c, uint32_t pos0) {
    const uint32_t g = c->n_heads / c->n_kv_heads;
    const uint32_t toks = 128 / g;
    const uint32_t blocks = (c->n_items + toks - 1) / toks * c->n_kv_heads;
    const uint32_t first = c->n_items < toks ? c->n_items : toks;
    const uint32_t tiles0 = (pos0 + first - 1) / 128 + 1;
    const char* e = getenv("TGKV_PF_SPLIT");
    uint32_t cap = e && atoi(e) > 0 ? (uint32_t)atoi(e) : 8;
    if (cap > 8) cap = 8;
    if (cap > tiles0) cap = tiles0;
    for (uint32_t ns = cap; ns > 1; ns--) {
        if (e && atoi(e) > 0) return ns;
        if ((uint64_t)blocks * ns <= (uint64_t)g_sm_count && blocks <= tgkv_prefill_max_clusters(ns)) return ns;
    }
    return 1;
}

int tg_cuda_kv_attn_fuses_suffix(const TGCudaAttnCall* c) { return use_prefill(c); }

/* Blocks of query rows over one fp32 cache (the forward's prefill: its caches
 * are fp32 like the engine's) go to the CUDA-core block kernel
 * (tgkv_prefill_f32.cu) when there are at least 32 (row, head) pairs:
 * consecutive positions, head_dim 32/64/128, group 1/2/3/4/8, no fused
 * append, no gather, q and out 16-byte aligned.  The split-sequence kernel
 * would run one query row per item: a 512-token prefill of the V2.7-shaped
 * model took 150 us a layer there.  TGKV_PREFILL=0 keeps them on it. */
static int use_prefill_f32(const TGCudaAttnCall* c) {
    const char* e = getenv("TGKV_PREFILL");
    if (e && e[0] == '0') return 0;
    if (!c || !c->n_kv_heads || !c->n_heads || c->n_heads % c->n_kv_heads || !c->n_pos ||
        !c->n_items || c->n_pos[0] == 0)
        return 0;
    if (c->dtype != 0 || c->table_dev || !c->cache.base || c->k_new || c->v_new ||
        c->gather_world)
        return 0;
    const uint32_t g = c->n_heads / c->n_kv_heads;
    if (!tgkv_prefill_f32_supported(c->head_dim, g)) return 0;
    if ((uint64_t)c->n_items * g < 32) return 0;
    if (((uintptr_t)c->q | (uintptr_t)c->out) & 15u) return 0;
    if ((uint64_t)c->n_pos[0] - 1 + c->n_items > c->cache.max_seq) return 0;
    for (uint32_t i = 1; i < c->n_items; i++)
        if (c->n_pos[i] != c->n_pos[0] + i) return 0;
    return 1;
}

/* The fp32 block kernel's plan: row blocks, tiles per split, splits of the
 * longest block; its partials (floats) and counters. */
typedef struct {
    uint32_t n_blocks, tps, n_split;
    uint64_t part_floats, ctrs;
} Block32Plan;
static Block32Plan plan_block32(const TGCudaAttnCall* c) {
    Block32Plan b;
    tgkv_prefill_f32_plan(c->n_items, c->n_pos[0] - 1, c->n_heads / c->n_kv_heads,
                          c->n_kv_heads, (uint32_t)(g_sm_count ? g_sm_count : 148), &b.n_blocks,
                          &b.tps, &b.n_split);
    b.ctrs = (uint64_t)c->n_kv_heads * b.n_blocks;
    b.part_floats = b.n_split > 1 ? b.ctrs * b.n_split * 64u * (c->head_dim + 4u) : 0;
    return b;
}

/* Calls that go to the tensor-core suffix kernel need no split scratch: one
 * token byte and one counter keep the caller's sizing logic uniform; the fp32
 * block kernel needs its split partials and a counter per row block. */
uint64_t tg_cuda_kv_attn_scratch_bytes(const TGCudaAttnCall* c) {
    if (use_prefill(c)) return 256;
    if (use_prefill_f32(c)) {
        const Block32Plan b = plan_block32(c);
        return b.part_floats ? b.part_floats * 4 : 256;
    }
    AttnPlan pl;
    if (!plan_attention(c, &pl)) return 0;
    return part_o_bytes(&pl, c->head_dim) + part_slots(&pl) * pl.gt * 2 * 4;
}

/* One arrival counter per segment; the tensor-core decode kernel also keeps
 * one tile queue per segment after them; the two-level merge one counter
 * per chunk group after those. */
uint64_t tg_cuda_kv_attn_counters(const TGCudaAttnCall* c) {
    if (use_prefill(c)) return 1;
    if (use_prefill_f32(c)) return plan_block32(c).ctrs;
    AttnPlan pl;
    if (!plan_attention(c, &pl)) return 0;
    return (uint64_t)c->n_items * c->n_kv_heads * pl.n_sub * (pl.tc ? 2u : 1u) +
           (merge2_on() ? pl.max_chunks : 0);
}

/* Segments of the call: (item, KV head, head subset) triples, each finished
 * (and, with a gather, signalled) once. */
uint64_t tg_cuda_kv_attn_segments(const TGCudaAttnCall* c) {
    if (use_prefill(c) || use_prefill_f32(c)) return 0;
    AttnPlan pl;
    if (!plan_attention(c, &pl)) return 0;
    return (uint64_t)c->n_items * c->n_kv_heads * pl.n_sub;
}

/* Tile stealing inside a segment (tensor-core decode), opt-in with
 * TGKV_STEAL=1: the segment's CTAs take 128-position tiles from a shared
 * queue instead of streaming fixed chunks.  Measured on B200 it did not pay
 * overall: cfg4 0.961 against 0.977 of HBM with fixed chunks on the same
 * box, one 131072-position sequence in one wave 0.894 against 0.888. */
static int steal_on(void) {
    const char* e = getenv("TGKV_STEAL");
    return e && e[0] == '1';
}

uint32_t tg_cuda_kv_attn_last_launches(void) { return t_last_launches; }
int tg_cuda_kv_attn_last_kernel(void) { return t_last_kernel; }
uint32_t tg_cuda_kv_attn_last_split(void) { return t_last_split; }

int tg_cuda_kv_attention(const TGCudaAttnCall* c, void* stream) {
    t_last_launches = 0;
    t_last_kernel = 0;
    t_last_split = 0;
    if (!g_ready && !tg_cuda_kv_init()) return 0;
    /* the tensor-core suffix and the fp32 block routes need none of the
     * split planning */
    const int prefill = use_prefill(c);
    const int block32 = !prefill && use_prefill_f32(c);
    AttnPlan pl;
    if (!prefill && !block32 && !plan_attention(c, &pl)) return 0;
    if (c->n_items == 0) return 1;
    if (!c->q || !c->out || (!c->table_dev && (!c->cache.base || !c->cache.tmap))) {
        set_err("attention: NULL pointer");
        return 0;
    }
    if (((uintptr_t)c->q | (uintptr_t)c->out) & 7u) {
        set_err("attention: q/out must be 8-byte aligned");
        return 0;
    }
    if (!c->k_new != !c->v_new) {
        set_err("attention: k_new and v_new go together");
        return 0;
    }
    if (c->gather_world > TGKV_MAX_RANKS) {
        set_err("attention: gather over %u ranks, at most %d", c->gather_world, TGKV_MAX_RANKS);
        return 0;
    }
    for (uint32_t r = 0; r < c->gather_world; r++)
        if (!c->gather_out[r] || !c->gather_flag[r]) {
            set_err("attention: gather rank %u has no buffer or flag", r);
            return 0;
        }
    if (c->gather_world && prefill) {
        set_err("attention: the output gather is for decode calls (one query row per item)");
        return 0;
    }
    if (prefill) {
        TGKvPrefillParams pp;
        memset(&pp, 0, sizeof(pp));
        pp.k_new = c->k_new;
        pp.v_new = c->v_new;
        pp.kvc = (uint16_t*)(uintptr_t)c->cache.base;
        pp.max_seq = c->cache.max_seq;
        pp.tmap_sw = c->cache.tmap_sw;
        pp.q = c->q;
        pp.out = c->out;
        pp.err = g_err_word;
        pp.n_q = c->n_items;
        pp.n_heads = c->n_heads;
        pp.n_kv_heads = c->n_kv_heads;
        pp.pos0 = c->n_pos[0] - 1;
        pp.qscale = c->scale * 1.4426950408889634f;
        pp.n_split = prefill_split(c, pp.pos0);
        if (!encode_qmap(c->q, c->n_heads, c->n_items, c->n_heads / c->n_kv_heads, &pp.qmap))
            return 0;
        t_last_split = pp.n_split;
        if (!launch_rc(tgkv_launch_prefill(&pp, stream), "prefill kernel")) return 0;
        t_last_launches = 1;
        t_last_kernel = 2;
        return 1;
    }
    if (block32) {
        const Block32Plan bp = plan_block32(c);
        if (bp.n_split > 1 && (!c->scratch || !c->counters)) {
            set_err("attention: fp32 block scratch not provided");
            return 0;
        }
        TGKvPrefillF32Params pp;
        memset(&pp, 0, sizeof(pp));
        pp.part = (float*)c->scratch;
        pp.ctr = c->counters;
        pp.n_blocks = bp.n_blocks;
        pp.tps = bp.tps;
        pp.n_split = bp.n_split;
        pp.q = c->q;
        pp.out = c->out;
        pp.kv = (const float*)(uintptr_t)c->cache.base;
        pp.n_q = c->n_items;
        pp.n_heads = c->n_heads;
        pp.n_kv_heads = c->n_kv_heads;
        pp.head_dim = c->head_dim;
        pp.max_seq = c->cache.max_seq;
        pp.pos0 = c->n_pos[0] - 1;
        pp.qscale = c->scale * 1.4426950408889634f;
        if (!launch_rc(tgkv_launch_prefill_f32(&pp, stream), "fp32 block kernel")) return 0;
        t_last_launches = 1;
        t_last_kernel = 4;
        t_last_split = bp.n_split;
        return 1;
    }
    if (!c->scratch || !c->counters) {
        set_err("attention: split-sequence scratch not provided");
        return 0;
    }
    static _Thread_local TGKvAttnParams p;     /* ~8 KB: keep off the stack */
    const uint64_t po = part_o_bytes(&pl, c->head_dim);
    for (uint32_t b0 = 0; b0 < c->n_items; b0 += TGKV_MAX_ITEMS) {
        const uint32_t n = (c->n_items - b0) < TGKV_MAX_ITEMS ? (c->n_items - b0) : TGKV_MAX_ITEMS;
        memset(&p, 0, offsetof(TGKvAttnParams, n_pos));
        p.caches = (const TGKvCacheDesc*)(c->table_dev ? c->table_dev + b0 : NULL);
        p.cache0.base = c->cache.base;
        p.cache0.max_seq = c->cache.max_seq;
        p.cache0.tmap = c->cache.tmap;
        p.cache0.tmap_sw = c->cache.tmap_sw;
        p.q = c->q;
        p.out = c->out;
        p.k_new = c->k_new ? c->k_new + (uint64_t)b0 * c->n_kv_heads * c->head_dim : NULL;
        p.v_new = c->v_new ? c->v_new + (uint64_t)b0 * c->n_kv_heads * c->head_dim : NULL;
        p.part_o = (float*)c->scratch;
        p.part_ml = (float*)((char*)c->scratch + po);
        p.counters = c->counters;
        if (merge2_on()) {
            p.two_level_min = merge2_min();
            p.l1_base = (uint32_t)pl.max_chunks;
            p.gctr_base = (uint32_t)((uint64_t)c->n_items * c->n_kv_heads * pl.n_sub *
                                     (pl.tc ? 2u : 1u));
        }
        p.tile_ctr = (pl.tc && steal_on())
                         ? c->counters + (uint64_t)c->n_items * c->n_kv_heads * pl.n_sub
                         : NULL;
        p.err = g_err_word;
        p.cache_stride = c->table_dev ? 1u : 0u;
        p.n_items = n;
        p.n_heads = c->n_heads;
        p.n_kv_heads = c->n_kv_heads;
        p.n_sub = pl.n_sub;
        p.chunk = pl.chunk;
        p.qscale = c->scale * 1.4426950408889634f;
        p.item_base = b0;
        p.gather_world = c->gather_world;
        p.gather_base = c->gather_base;
        for (uint32_t r = 0; r < c->gather_world; r++) {
            p.gather_out[r] = c->gather_out[r];
            p.gather_flag[r] = c->gather_flag[r];
        }
        uint32_t acc = 0;
        for (uint32_t i = 0; i < n; i++) {
            const uint32_t np = c->n_pos[b0 + i];
            p.n_pos[i] = np;
            p.chunk_prefix[i] = acc;
            acc += ((np + pl.chunk - 1) / pl.chunk) * c->n_kv_heads * pl.n_sub;
        }
        p.chunk_prefix[n] = acc;
        if (pl.tc) {
            if (!launch_rc(tgkv_launch_attention_tc(&p, pl.gt, acc, stream),
                           "tensor-core decode kernel"))
                return 0;
        } else if (!launch_rc(tgkv_launch_attention(&p, c->dtype, c->head_dim, pl.gt, acc, stream),
                              "attention kernel")) {
            return 0;
        }
        t_last_launches++;
        t_last_kernel = pl.tc ? 3 : 1;
    }
    return 1;
}

/* ---- RoPE + append ------------------------------------------------------ */
int tg_cuda_kv_rope_append(int dtype, const float* qkv, const float* cs, const float* sn,
                           void* kvc, float* qout, uint32_t n_tokens, uint32_t n_heads,
                           uint32_t n_kv_heads, uint32_t head_dim, uint32_t start_pos,
                           uint32_t max_seq, void* stream) {
    if (!g_ready && !tg_cuda_kv_init()) return 0;
    if (n_tokens == 0) return 1;
    if (!qkv || !cs || !sn || !kvc || !qout) { set_err("rope: NULL pointer"); return 0; }
    if (head_dim == 0 || (head_dim & 1) || n_kv_heads == 0 || n_kv_heads > n_heads) {
        set_err("rope: bad head geometry");
        return 0;
    }
    if ((uint64_t)start_pos + n_tokens > max_seq) { set_err("rope: capacity exceeded"); return 0; }
    TGKvRopeParams p;
    p.qkv = qkv;
    p.cs = cs;
    p.sn = sn;
    p.kvc = kvc;
    p.qout = qout;
    p.n_tokens = n_tokens;
    p.n_heads = n_heads;
    p.n_kv_heads = n_kv_heads;
    p.head_dim = head_dim;
    p.start_pos = start_pos;
    p.max_seq = max_seq;
    p.dtype = dtype;
    return launch_rc(tgkv_launch_rope_append(&p, stream), "rope kernel");
}
