// tgkv_prefill_f32.cu -- causal attention of n_q consecutive query rows over
// one fp32 cache, on the CUDA cores: the whole-model forward's prefill, whose
// caches are fp32 like the engine's (src/tgai_engine.c:3943-4011 computes the
// same scores, softmax and weighted sum one query row at a time).
//
// One CTA of 256 threads takes up to 32 query vectors -- R = 32 / G
// consecutive rows times the G query heads of one KV head -- and walks the
// K/V tiles of 32 positions up to its last row's position, two tiles in
// flight (cp.async into shared memory, rows past that position zero-filled:
// stale rows of a truncated turn never enter).  Per tile:
//   S   thread (v, j) scores query vector v = t / 8 against positions
//       j, j + 8, j + 16, j + 24 of the tile (q pre-scaled by scale * log2 e);
//   softmax: online, in the log2 domain, over the 8 threads of a vector;
//   PV  the same thread accumulates dimensions 4 (t % 8) + 32 k of O.
// Row r attends positions [0, pos0 + r].  The per-row (one query row a CTA)
// split-sequence kernel re-read every K/V row once per query row and ran
// thousands of one-tile CTAs; here a K/V tile serves 32 query vectors.
#include <cuda_runtime.h>
#include <stdint.h>

#include "tgkv_launch.h"

namespace tgkvp32 {

constexpr int kThreads = 256;
constexpr int kT = 32;     // positions per K/V tile
constexpr int kQV = 32;    // query vectors per CTA at most

template <int HD>
struct Cfg {
    static constexpr int RS = HD + 4;          // row stride in floats: rows 16 bytes apart in banks
    static constexpr int TILE = kT * RS;       // floats of one K or V tile
    static constexpr int OFF_K = kQV * RS;     // after Q: stage s at OFF_K + 2 s TILE (K, then V)
    static constexpr int FLOATS = OFF_K + 4 * TILE;
    static constexpr int BYTES = FLOATS * 4;
    static constexpr int NV = HD / 32;         // float4 of O per thread
};

__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// K and V rows [p0, p0 + kT) of KV head kvh into stage st; rows past last
// (inclusive) are zeros.
template <int HD>
__device__ __forceinline__ void load_tile(float* st, const TGKvPrefillF32Params& p, uint32_t kvh,
                                          uint32_t p0, uint32_t last) {
    using C = Cfg<HD>;
    constexpr int kChunks = kT * (HD / 4);     // 16-byte pieces of one tile
    const uint64_t kv_dim = (uint64_t)p.n_kv_heads * HD;
    const float* kb = p.kv + (uint64_t)kvh * HD;
    const float* vb = p.kv + (uint64_t)p.max_seq * kv_dim + (uint64_t)kvh * HD;
    for (int c = threadIdx.x; c < 2 * kChunks; c += kThreads) {
        const int m = c / kChunks, e = c % kChunks;         // m: K or V
        const int r = e / (HD / 4), q4 = e % (HD / 4);
        const uint32_t pos = p0 + (uint32_t)r;
        const bool valid = pos <= last;
        const float* src = (m ? vb : kb) + (uint64_t)(valid ? pos : 0) * kv_dim + q4 * 4;
        cp_async16(st + m * C::TILE + r * C::RS + q4 * 4, src, valid);
    }
}

template <int HD, int G>
__global__ void __launch_bounds__(kThreads, 2) prefill_f32_kernel(const TGKvPrefillF32Params p) {
    using C = Cfg<HD>;
    extern __shared__ __align__(16) float sm[];
    constexpr int R = kQV / G;                 // query rows per CTA
    const int t = threadIdx.x, lane = t & 31;
    const int v = t >> 3, jl = t & 7;          // query vector, lane within its 8
    const uint32_t kvh = blockIdx.y, r0 = blockIdx.x * R;
    const uint32_t rows = p.n_q - r0 < (uint32_t)R ? p.n_q - r0 : (uint32_t)R;
    const bool on = v < (int)(rows * G);
    const uint32_t row = r0 + (uint32_t)(v / G), head = kvh * G + (uint32_t)(v % G);
    const uint32_t lim = p.pos0 + row;                    // this vector's last position
    const uint32_t last = p.pos0 + r0 + rows - 1;         // the CTA's last position
    const uint32_t n_tiles = last / kT + 1;

    // the K/V of tile 0 in flight while q is staged (scaled; zeros for idle vectors)
    load_tile<HD>(sm + C::OFF_K, p, kvh, 0, last);
    cp_commit();
    for (int e = t; e < kQV * (HD / 4); e += kThreads) {
        const int qv = e / (HD / 4), q4 = e % (HD / 4);
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qv < (int)(rows * G)) {
            const uint32_t rr = r0 + (uint32_t)(qv / G), hh = kvh * G + (uint32_t)(qv % G);
            x = *reinterpret_cast<const float4*>(p.q + ((uint64_t)rr * p.n_heads + hh) * HD + q4 * 4);
            x.x *= p.qscale;
            x.y *= p.qscale;
            x.z *= p.qscale;
            x.w *= p.qscale;
        }
        *reinterpret_cast<float4*>(sm + qv * C::RS + q4 * 4) = x;
    }

    float m = -INFINITY, l = 0.f;
    float4 o[C::NV];
#pragma unroll
    for (int k = 0; k < C::NV; ++k) o[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* qrow = sm + v * C::RS;

    for (uint32_t ti = 0; ti < n_tiles; ++ti) {
        float* st = sm + C::OFF_K + (int)(ti & 1) * 2 * C::TILE;
        if (ti + 1 < n_tiles) {
            // the other stage was last read in tile ti - 1, before the barrier
            // that closed it
            load_tile<HD>(sm + C::OFF_K + (int)((ti + 1) & 1) * 2 * C::TILE, p, kvh,
                          (ti + 1) * kT, last);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        const float* kt = st;
        const float* vt = st + C::TILE;
        const uint32_t p0 = ti * kT;

        // ---- S: positions jl + 8 u of the tile
        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
        for (int d = 0; d < HD; d += 4) {
            const float4 q4 = *reinterpret_cast<const float4*>(qrow + d);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float4 k4 = *reinterpret_cast<const float4*>(kt + (jl + 8 * u) * C::RS + d);
                s[u] = fmaf(q4.x, k4.x, s[u]);
                s[u] = fmaf(q4.y, k4.y, s[u]);
                s[u] = fmaf(q4.z, k4.z, s[u]);
                s[u] = fmaf(q4.w, k4.w, s[u]);
            }
        }
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (!on || p0 + (uint32_t)(jl + 8 * u) > lim) s[u] = -INFINITY;
            mx = fmaxf(mx, s[u]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        const float m_new = fmaxf(m, mx);
        // a vector with no position yet in this tile (only the idle ones:
        // every row attends position 0) keeps m = -inf and adds nothing
        const float corr = m == -INFINITY ? 0.f : exp2f(m - m_new);
        float pr[4], ps = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            pr[u] = s[u] == -INFINITY ? 0.f : exp2f(s[u] - m_new);
            ps += pr[u];
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        m = m_new;
        l = l * corr + ps;
#pragma unroll
        for (int k = 0; k < C::NV; ++k) {
            o[k].x *= corr;
            o[k].y *= corr;
            o[k].z *= corr;
            o[k].w *= corr;
        }

        // ---- PV: position jj + 8 u's weight from lane jj of this vector's 8
        const int base = lane & ~7;
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll 4
        for (int jj = 0; jj < 8; ++jj) {
            const float w = __shfl_sync(0xffffffffu, pr[u], base | jj);
            const int j = jj + 8 * u;
#pragma unroll
            for (int k = 0; k < C::NV; ++k) {
                const float4 v4 = *reinterpret_cast<const float4*>(vt + j * C::RS + jl * 4 + 32 * k);
                o[k].x = fmaf(w, v4.x, o[k].x);
                o[k].y = fmaf(w, v4.y, o[k].y);
                o[k].z = fmaf(w, v4.z, o[k].z);
                o[k].w = fmaf(w, v4.w, o[k].w);
            }
        }
        __syncthreads();                       // the stage is read; tile ti + 2 may refill it
    }

    if (on) {
        const float inv = 1.0f / l;
        float* dst = p.out + ((uint64_t)row * p.n_heads + head) * HD;
#pragma unroll
        for (int k = 0; k < C::NV; ++k)
            *reinterpret_cast<float4*>(dst + jl * 4 + 32 * k) =
                make_float4(o[k].x * inv, o[k].y * inv, o[k].z * inv, o[k].w * inv);
    }
}

template <int HD, int G>
int launch(const TGKvPrefillF32Params* p, cudaStream_t st) {
    using C = Cfg<HD>;
    // the shared-memory opt-in, once per device (threads that race here
    // set the same value)
    static volatile bool attr[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    if (!attr[dev]) {
        e = cudaFuncSetAttribute(prefill_f32_kernel<HD, G>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, C::BYTES);
        if (e != cudaSuccess) return (int)e;
        attr[dev] = true;
    }
    constexpr int R = kQV / G;
    const dim3 grid((p->n_q + R - 1) / R, p->n_kv_heads);
    prefill_f32_kernel<HD, G><<<grid, kThreads, C::BYTES, st>>>(*p);
    return (int)cudaGetLastError();
}

}  // namespace tgkvp32

extern "C" int tgkv_prefill_f32_supported(uint32_t head_dim, uint32_t group) {
    return (head_dim == 32 || head_dim == 64 || head_dim == 128) &&
           (group == 1 || group == 2 || group == 3 || group == 4 || group == 8);
}

extern "C" int tgkv_launch_prefill_f32(const TGKvPrefillF32Params* p, void* stream) {
    if (!p || !p->n_q || !p->n_kv_heads || p->n_heads % p->n_kv_heads) return (int)cudaErrorInvalidValue;
    const uint32_t g = p->n_heads / p->n_kv_heads;
    cudaStream_t st = (cudaStream_t)stream;
#define TGKV_P32_CASE(HD, G) \
    if (p->head_dim == HD && g == G) return tgkvp32::launch<HD, G>(p, st);
    TGKV_P32_CASE(128, 1) TGKV_P32_CASE(128, 2) TGKV_P32_CASE(128, 3) TGKV_P32_CASE(128, 4)
    TGKV_P32_CASE(128, 8)
    TGKV_P32_CASE(64, 1) TGKV_P32_CASE(64, 2) TGKV_P32_CASE(64, 3) TGKV_P32_CASE(64, 4)
    TGKV_P32_CASE(64, 8)
    TGKV_P32_CASE(32, 1) TGKV_P32_CASE(32, 2) TGKV_P32_CASE(32, 3) TGKV_P32_CASE(32, 4)
    TGKV_P32_CASE(32, 8)
#undef TGKV_P32_CASE
    return (int)cudaErrorInvalidValue;
}
