// tgkv_prefill_f32.cu -- causal attention of n_q consecutive query rows over
// one fp32 cache, on the CUDA cores: the whole-model forward's prefill, whose
// caches are fp32 like the engine's (src/tgai_engine.c:3943-4011 computes the
// same scores, softmax and weighted sum one query row at a time).
//
// A row block is R = 64 / G consecutive rows times the G query heads of one
// KV head: up to 64 query vectors, staged once in shared memory pre-scaled by
// scale * log2 e.  Its K/V tiles of 32 positions (up to the block's last
// row's position) are dealt to CTAs of at most `tps` tiles each, so that the
// long blocks of the causal triangle do not leave most SMs idle; a block of
// one split writes its rows, a block of several writes one partial per split
// (running maximum, sum, unnormalised output) and the split that finishes
// last merges them.  Inside a CTA (256 threads) two tiles are in flight
// (cp.async, rows past the block's last position zero-filled: stale rows of a
// truncated turn never enter), and thread (p, j) takes query vectors p and
// p + 32 against positions j + 8 u of the tile (S), keeps their online
// softmax in the log2 domain with the 8 threads of the pair, and accumulates
// their dimensions 4 j + 32 k of O (PV): every shared-memory load of a K or V
// row serves two query vectors.  Row r attends positions [0, pos0 + r].
#include <cuda_runtime.h>
#include <stdint.h>

#include "tgkv_launch.h"

namespace tgkvp32 {

constexpr int kThreads = 256;
constexpr int kT = 32;     // positions per K/V tile
constexpr int kQV = 64;    // query vectors per row block at most

template <int HD>
struct Cfg {
    static constexpr int RS = HD + 4;          // row stride in floats: rows 16 bytes apart in banks
    static constexpr int TILE = kT * RS;       // floats of one K or V tile
    static constexpr int OFF_K = kQV * RS;     // after Q: stage s at OFF_K + 2 s TILE (K, then V)
    static constexpr int FLOATS = OFF_K + 4 * TILE;
    static constexpr int BYTES = FLOATS * 4;
    static constexpr int NV = HD / 32;         // float4 of O per thread and vector
    static constexpr int PS = HD + 4;          // floats of a partial: m, l, 2 pad, O
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

// grid (n_blocks, n_split, n_kv_heads): row block x, split y of its tiles
template <int HD, int G>
__global__ void __launch_bounds__(kThreads, 2) prefill_f32_kernel(const TGKvPrefillF32Params p) {
    using C = Cfg<HD>;
    extern __shared__ __align__(16) float sm[];
    __shared__ int s_last;
    constexpr int R = kQV / G;                 // query rows of a row block
    const int t = threadIdx.x, lane = t & 31;
    const int vp = t >> 3, jl = t & 7;         // vectors vp and vp + 32, lane within the 8
    const uint32_t b = blockIdx.x, split = blockIdx.y, kvh = blockIdx.z;
    const uint32_t r0 = b * R;
    const uint32_t rows = p.n_q - r0 < (uint32_t)R ? p.n_q - r0 : (uint32_t)R;
    const uint32_t nvec = rows * G;
    const uint32_t last = p.pos0 + r0 + rows - 1;         // the block's last position
    const uint32_t n_tiles = last / kT + 1;
    const uint32_t n_splits = (n_tiles + p.tps - 1) / p.tps;
    const uint32_t t0 = split * p.tps;
    if (t0 >= n_tiles) return;                 // a short block has fewer splits
    const uint32_t t1 = t0 + p.tps < n_tiles ? t0 + p.tps : n_tiles;

    bool on[2];
    uint32_t lim[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t v = (uint32_t)(vp + 32 * h);
        on[h] = v < nvec;
        lim[h] = p.pos0 + r0 + v / G;          // this vector's last position
    }

    // the K/V of the first tile in flight while q is staged (scaled; zeros
    // for idle vectors)
    load_tile<HD>(sm + C::OFF_K, p, kvh, t0 * kT, last);
    cp_commit();
    for (int e = t; e < kQV * (HD / 4); e += kThreads) {
        const int qv = e / (HD / 4), q4 = e % (HD / 4);
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if ((uint32_t)qv < nvec) {
            const uint32_t rr = r0 + (uint32_t)(qv / G), hh = kvh * G + (uint32_t)(qv % G);
            x = *reinterpret_cast<const float4*>(p.q + ((uint64_t)rr * p.n_heads + hh) * HD + q4 * 4);
            x.x *= p.qscale;
            x.y *= p.qscale;
            x.z *= p.qscale;
            x.w *= p.qscale;
        }
        *reinterpret_cast<float4*>(sm + qv * C::RS + q4 * 4) = x;
    }

    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float4 o[2][C::NV];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int k = 0; k < C::NV; ++k) o[h][k] = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* q0 = sm + vp * C::RS;
    const float* q1 = sm + (vp + 32) * C::RS;
    const int base = lane & ~7;

    for (uint32_t ti = t0; ti < t1; ++ti) {
        const uint32_t i = ti - t0;
        float* st = sm + C::OFF_K + (int)(i & 1) * 2 * C::TILE;
        if (ti + 1 < t1) {
            // the other stage was last read in the previous tile, before the
            // barrier that closed it
            load_tile<HD>(sm + C::OFF_K + (int)((i + 1) & 1) * 2 * C::TILE, p, kvh,
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

        // ---- S: vectors vp and vp + 32 against positions jl + 8 u of the tile
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            const float4 a = *reinterpret_cast<const float4*>(q0 + d);
            const float4 c = *reinterpret_cast<const float4*>(q1 + d);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float4 k4 = *reinterpret_cast<const float4*>(kt + (jl + 8 * u) * C::RS + d);
                s[0][u] = fmaf(a.x, k4.x, s[0][u]);
                s[0][u] = fmaf(a.y, k4.y, s[0][u]);
                s[0][u] = fmaf(a.z, k4.z, s[0][u]);
                s[0][u] = fmaf(a.w, k4.w, s[0][u]);
                s[1][u] = fmaf(c.x, k4.x, s[1][u]);
                s[1][u] = fmaf(c.y, k4.y, s[1][u]);
                s[1][u] = fmaf(c.z, k4.z, s[1][u]);
                s[1][u] = fmaf(c.w, k4.w, s[1][u]);
            }
        }
        // ---- online softmax of each vector over its 8 threads
        float pr[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float mx = -INFINITY;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (!on[h] || p0 + (uint32_t)(jl + 8 * u) > lim[h]) s[h][u] = -INFINITY;
                mx = fmaxf(mx, s[h][u]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            const float m_new = fmaxf(m[h], mx);
            // a vector with no position yet (an idle one, or a later split's
            // rows past this tile) keeps m = -inf and adds nothing
            const float corr = m[h] == -INFINITY ? 0.f : exp2f(m[h] - m_new);
            float ps = 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                pr[h][u] = s[h][u] == -INFINITY ? 0.f : exp2f(s[h][u] - m_new);
                ps += pr[h][u];
            }
            ps += __shfl_xor_sync(0xffffffffu, ps, 1);
            ps += __shfl_xor_sync(0xffffffffu, ps, 2);
            ps += __shfl_xor_sync(0xffffffffu, ps, 4);
            m[h] = m_new;
            l[h] = l[h] * corr + ps;
#pragma unroll
            for (int k = 0; k < C::NV; ++k) {
                o[h][k].x *= corr;
                o[h][k].y *= corr;
                o[h][k].z *= corr;
                o[h][k].w *= corr;
            }
        }

        // ---- PV: position jj + 8 u's weights from lane jj of the pair's 8
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll 4
        for (int jj = 0; jj < 8; ++jj) {
            const float w0 = __shfl_sync(0xffffffffu, pr[0][u], base | jj);
            const float w1 = __shfl_sync(0xffffffffu, pr[1][u], base | jj);
            const float* vr = vt + (jj + 8 * u) * C::RS + jl * 4;
#pragma unroll
            for (int k = 0; k < C::NV; ++k) {
                const float4 v4 = *reinterpret_cast<const float4*>(vr + 32 * k);
                o[0][k].x = fmaf(w0, v4.x, o[0][k].x);
                o[0][k].y = fmaf(w0, v4.y, o[0][k].y);
                o[0][k].z = fmaf(w0, v4.z, o[0][k].z);
                o[0][k].w = fmaf(w0, v4.w, o[0][k].w);
                o[1][k].x = fmaf(w1, v4.x, o[1][k].x);
                o[1][k].y = fmaf(w1, v4.y, o[1][k].y);
                o[1][k].z = fmaf(w1, v4.z, o[1][k].z);
                o[1][k].w = fmaf(w1, v4.w, o[1][k].w);
            }
        }
        __syncthreads();                       // the stage is read; the tile after next may refill it
    }

    if (n_splits == 1) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (!on[h]) continue;
            const uint32_t v = (uint32_t)(vp + 32 * h);
            const uint32_t row = r0 + v / G, head = kvh * G + v % G;
            const float inv = 1.0f / l[h];
            float* dst = p.out + ((uint64_t)row * p.n_heads + head) * HD;
#pragma unroll
            for (int k = 0; k < C::NV; ++k)
                *reinterpret_cast<float4*>(dst + jl * 4 + 32 * k) =
                    make_float4(o[h][k].x * inv, o[h][k].y * inv, o[h][k].z * inv, o[h][k].w * inv);
        }
        return;
    }

    // ---- several splits: this split's partial, then the last to finish merges
    const uint64_t blk = (uint64_t)kvh * p.n_blocks + b;
    const uint64_t pstride = (uint64_t)kQV * C::PS;         // floats of one split's partials
    float* part = p.part + (blk * p.n_split + split) * pstride;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float* dst = part + (uint64_t)(vp + 32 * h) * C::PS;
        if (jl == 0) {
            dst[0] = m[h];
            dst[1] = l[h];
        }
#pragma unroll
        for (int k = 0; k < C::NV; ++k)
            *reinterpret_cast<float4*>(dst + 4 + jl * 4 + 32 * k) = o[h][k];
    }
    __syncthreads();
    if (t == 0) {
        __threadfence();                       // this CTA's partial, then the count
        s_last = atomicAdd(p.ctr + blk, 1u) == n_splits - 1;
        if (s_last) __threadfence();           // every split's partial before the merge
    }
    __syncthreads();
    if (!s_last) return;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (!on[h]) continue;
        const uint32_t v = (uint32_t)(vp + 32 * h);
        const float* src = p.part + blk * p.n_split * pstride + (uint64_t)v * C::PS;
        float M = -INFINITY;
        for (uint32_t s2 = 0; s2 < n_splits; ++s2) M = fmaxf(M, __ldcg(src + s2 * pstride));
        float L = 0.f;
        float4 O[C::NV];
#pragma unroll
        for (int k = 0; k < C::NV; ++k) O[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t s2 = 0; s2 < n_splits; ++s2) {
            const float* ps = src + s2 * pstride;
            const float ms = __ldcg(ps);
            const float f = ms == -INFINITY ? 0.f : exp2f(ms - M);
            L = fmaf(f, __ldcg(ps + 1), L);
#pragma unroll
            for (int k = 0; k < C::NV; ++k) {
                const float4 x = __ldcg(reinterpret_cast<const float4*>(ps + 4 + jl * 4 + 32 * k));
                O[k].x = fmaf(f, x.x, O[k].x);
                O[k].y = fmaf(f, x.y, O[k].y);
                O[k].z = fmaf(f, x.z, O[k].z);
                O[k].w = fmaf(f, x.w, O[k].w);
            }
        }
        const uint32_t row = r0 + v / G, head = kvh * G + v % G;
        const float inv = 1.0f / L;
        float* dst = p.out + ((uint64_t)row * p.n_heads + head) * HD;
#pragma unroll
        for (int k = 0; k < C::NV; ++k)
            *reinterpret_cast<float4*>(dst + jl * 4 + 32 * k) =
                make_float4(O[k].x * inv, O[k].y * inv, O[k].z * inv, O[k].w * inv);
    }
    if (t == 0) p.ctr[blk] = 0u;               // counted again only by a later launch
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
    const dim3 grid(p->n_blocks, p->n_split, p->n_kv_heads);
    prefill_f32_kernel<HD, G><<<grid, kThreads, C::BYTES, st>>>(*p);
    return (int)cudaGetLastError();
}

}  // namespace tgkvp32

extern "C" int tgkv_prefill_f32_supported(uint32_t head_dim, uint32_t group) {
    return (head_dim == 32 || head_dim == 64 || head_dim == 128) &&
           (group == 1 || group == 2 || group == 3 || group == 4 || group == 8);
}

extern "C" void tgkv_prefill_f32_plan(uint32_t n_q, uint32_t pos0, uint32_t group,
                                      uint32_t n_kv_heads, uint32_t sm_count, uint32_t* n_blocks,
                                      uint32_t* tps, uint32_t* n_split) {
    const uint32_t R = tgkvp32::kQV / group;
    const uint32_t nb = (n_q + R - 1) / R;
    // tiles of every block; the last block's are the most
    uint64_t total = 0;
    uint32_t longest = 1;
    for (uint32_t b = 0; b < nb; ++b) {
        const uint32_t rows = n_q - b * R < R ? n_q - b * R : R;
        const uint32_t nt = (pos0 + b * R + rows - 1) / tgkvp32::kT + 1;
        total += nt;
        if (nt > longest) longest = nt;
    }
    total *= n_kv_heads;
    // splits of about total / (4 sm_count) tiles: two CTAs on each SM and a
    // second round of them; at least 2 tiles (one lands while the other is
    // used) unless the longest block has fewer
    const uint64_t want = (uint64_t)(sm_count ? sm_count : 148) * 4;
    uint32_t t = (uint32_t)((total + want - 1) / want);
    if (t < 2) t = 2;
    if (t > longest) t = longest;
    *n_blocks = nb;
    *tps = t;
    *n_split = (longest + t - 1) / t;
}

extern "C" int tgkv_launch_prefill_f32(const TGKvPrefillF32Params* p, void* stream) {
    if (!p || !p->n_q || !p->n_kv_heads || p->n_heads % p->n_kv_heads || !p->tps ||
        !p->n_split || !p->n_blocks || (p->n_split > 1 && (!p->part || !p->ctr)))
        return (int)cudaErrorInvalidValue;
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
