// tgkv_forward.cu -- the kernels of the whole-model forward around the KV path
// (sm_100a): token embedding, RMSNorm, bias, SwiGLU, the MoE router and the
// expert FFN grouped by expert, and the MoE combine.  The projections and the
// LM head are plain GEMMs (cuBLAS, from tgai_forward.c); RoPE + KV append and
// attention are the KV path's own kernels (tgkv_kernels.cu, tgkv_prefill.cu).
//
// Every kernel here is HBM- or latency-bound elementwise / row work: rows are
// read with coalesced float4 loads, reductions are warp shuffles, and nothing
// is shaped into a GEMM.  The arithmetic follows the engine's CPU forward
// (src/tgai_engine.c) term for term where the order is observable: RMSNorm's
// 1/sqrt(ss/d + eps) then x * s * w (:2729-2784), the dense FFN's clamp to
// +-88 (:4118-4123), the router's strict-greater top-k with -1e30 start and
// its max-shifted softmax (:4166-4192), and the k-ordered fused
// multiply-add of the expert outputs (:4304).
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "tgkv_forward.h"

namespace tgkvf {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    return fmaf(a.w, b.w, acc);
}

__device__ __forceinline__ float silu_mul(float a, float b) { return (a / (1.0f + expf(-a))) * b; }

// Programmatic dependent launch: the decode kernels are launched so that they
// may start while their predecessor on the stream finishes.  Before
// pdl_wait() they touch only weights (constant during a forward), which they
// prefetch into L2; pdl_wait() returns once the predecessor has completed and
// its writes are visible (at once for a launch without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// One warp prefetches a weight row of n floats into L2, one 128-byte line per lane step.
__device__ __forceinline__ void prefetch_row(const float* w, uint32_t n) {
    for (uint32_t i = (threadIdx.x & 31) * 32; i < n; i += 32 * 32)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(w + i));
}
// Share `part` of `parts` of [pf, pf + n floats) prefetched into L2 by this
// CTA's threads: the weights of a LATER launch on the stream.  A decode
// step's kernels are short and latency-bound, with HBM bandwidth to spare;
// pulling the next kernel's weights into L2 meanwhile leaves that kernel
// L2 latency instead of HBM latency.  Every line prefetched lies inside
// [pf, pf + n).
__device__ __forceinline__ void prefetch_share(const float* pf, uint64_t n, uint32_t part,
                                               uint32_t parts) {
    if (!pf || n == 0) return;
    const uint64_t lines = (n + 31) / 32;
    const uint64_t per = (lines + parts - 1) / parts;
    const uint64_t l0 = (uint64_t)part * per;
    const uint64_t l1 = l0 + per < lines ? l0 + per : lines;
    for (uint64_t l = l0 + threadIdx.x; l < l1; l += blockDim.x)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(pf + l * 32));
}
__device__ __forceinline__ uint32_t cta_rank() { return blockIdx.x + gridDim.x * blockIdx.y; }
__device__ __forceinline__ uint32_t cta_count() { return gridDim.x * gridDim.y; }

__global__ void __launch_bounds__(256) embed_kernel(float* x, const float* emb, const int32_t* ids,
                                                   uint32_t d, uint32_t rows, int32_t unk) {
    const uint32_t t = blockIdx.x;
    int32_t id = ids[t];
    if (id < 0 || (uint32_t)id >= rows) id = unk;
    const float* src = emb + (uint64_t)id * d;
    float* dst = x + (uint64_t)t * d;
    for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) dst[i] = src[i];
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(float* out, const float* x, const float* w,
                                                      uint32_t d, uint64_t out_stride,
                                                      uint64_t x_stride, float eps) {
    __shared__ float red[8];
    const float* xr = x + (uint64_t)blockIdx.x * x_stride;
    float* orow = out + (uint64_t)blockIdx.x * out_stride;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < d; i += 256) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float s = 1.0f / sqrtf(tot / (float)d + eps);
    for (uint32_t i = threadIdx.x; i < d; i += 256) orow[i] = xr[i] * s * w[i];
}

__global__ void __launch_bounds__(256) bias_kernel(float* y, const float* b, uint64_t n,
                                                   uint32_t cols) {
    const uint64_t i = (uint64_t)blockIdx.x * 256 + threadIdx.x;
    if (i < n) y[i] += b[i % cols];
}

__global__ void __launch_bounds__(256) silu_mul_kernel(float* h, const float* ab, uint64_t n,
                                                       uint32_t dff, int clamp) {
    const uint64_t i = (uint64_t)blockIdx.x * 256 + threadIdx.x;
    if (i >= n) return;
    const uint64_t r = i / dff, j = i % dff;
    float a = ab[r * 2 * dff + j];
    const float b = ab[r * 2 * dff + dff + j];
    if (clamp) a = fminf(fmaxf(a, -88.0f), 88.0f);
    h[i] = silu_mul(a, b);
}

// One thread per token: at most 16 experts and top-8.
__global__ void __launch_bounds__(128) route_kernel(const float* logits, const float* bias,
                                                    int32_t* top_ids, float* top_w,
                                                    uint32_t* counts, uint32_t* lists,
                                                    uint32_t seq, uint32_t ne, uint32_t na) {
    const uint32_t t = blockIdx.x * 128 + threadIdx.x;
    if (t >= seq) return;
    float lg[16];
    for (uint32_t e = 0; e < ne; ++e) {
        lg[e] = logits[(uint64_t)t * ne + e];
        if (bias) lg[e] += bias[e];
    }
    int ids[8];
    float vals[8];
    for (uint32_t k = 0; k < na; ++k) {
        int best = -1;
        float best_v = -1e30f;
        for (uint32_t e = 0; e < ne; ++e) {
            bool used = false;
            for (uint32_t kk = 0; kk < k; ++kk) used |= ids[kk] == (int)e;
            if (used) continue;
            if (lg[e] > best_v) { best_v = lg[e]; best = (int)e; }
        }
        ids[k] = best;
        vals[k] = best_v;
    }
    float mx = vals[0];
    for (uint32_t k = 1; k < na; ++k) if (vals[k] > mx) mx = vals[k];
    float ss = 0.f;
    for (uint32_t k = 0; k < na; ++k) { vals[k] = expf(vals[k] - mx); ss += vals[k]; }
    for (uint32_t k = 0; k < na; ++k) {
        vals[k] /= ss;
        top_ids[(uint64_t)t * na + k] = ids[k];
        top_w[(uint64_t)t * na + k] = vals[k];
        if (ids[k] >= 0) {
            const uint32_t slot = atomicAdd(&counts[ids[k]], 1u);
            lists[(uint64_t)ids[k] * seq * na + slot] = t * na + k;
        }
    }
}

// Rows of one expert's weight against the inputs of the pairs routed to it:
// one warp per weight row, float4 loads, kPairs pairs per pass so that each
// weight row is read once per kPairs pairs (expert weights stay L2-resident
// across the passes of a prefill).
constexpr int kRowsPerCta = 8;
constexpr int kPairs = 4;

template <bool kW12>
__global__ void __launch_bounds__(256) expert_kernel(const float* __restrict__ w,
                                                     const float* __restrict__ in,
                                                     float* __restrict__ out,
                                                     const uint32_t* __restrict__ counts,
                                                     const uint32_t* __restrict__ lists,
                                                     uint32_t list_stride, uint32_t n_rows,
                                                     uint32_t k_dim, uint32_t na,
                                                     uint64_t expert_stride) {
    const uint32_t e = blockIdx.y;
    const uint32_t n = counts[e];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t row = blockIdx.x * kRowsPerCta + warp;
    if (n == 0 || row >= n_rows) return;
    const float* wa = w + (uint64_t)e * expert_stride + (uint64_t)row * k_dim;
    const float* wb = wa + (uint64_t)n_rows * k_dim;          // W2 row (phase 1 only)
    const uint32_t* lst = lists + (uint64_t)e * list_stride;
    for (uint32_t p0 = 0; p0 < n; p0 += kPairs) {
        const float* src[kPairs];
#pragma unroll
        for (int u = 0; u < kPairs; ++u) {
            const uint32_t p = lst[min(p0 + u, n - 1)];
            src[u] = in + (uint64_t)(kW12 ? p / na : p) * k_dim;
        }
        float acc_a[kPairs], acc_b[kPairs];
#pragma unroll
        for (int u = 0; u < kPairs; ++u) acc_a[u] = acc_b[u] = 0.f;
#pragma unroll 4
        for (uint32_t i = lane * 4; i < k_dim; i += 128) {
            const float4 a4 = __ldg(reinterpret_cast<const float4*>(wa + i));
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (kW12) b4 = __ldg(reinterpret_cast<const float4*>(wb + i));
#pragma unroll
            for (int u = 0; u < kPairs; ++u) {
                const float4 x4 = *reinterpret_cast<const float4*>(src[u] + i);
                acc_a[u] = dot4(a4, x4, acc_a[u]);
                if (kW12) acc_b[u] = dot4(b4, x4, acc_b[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < kPairs; ++u) {
            acc_a[u] = warp_sum(acc_a[u]);
            if (kW12) acc_b[u] = warp_sum(acc_b[u]);
        }
        if (lane == 0) {
#pragma unroll
            for (int u = 0; u < kPairs; ++u) {
                if (p0 + u >= n) break;
                const uint32_t p = lst[p0 + u];
                out[(uint64_t)p * n_rows + row] = kW12 ? silu_mul(acc_a[u], acc_b[u]) : acc_a[u];
            }
        }
    }
}

__global__ void __launch_bounds__(256) combine_kernel(float* x, const float* y,
                                                      const int32_t* top_ids,
                                                      const float* top_w, uint32_t d,
                                                      uint32_t ne, uint32_t na) {
    const uint32_t t = blockIdx.x;
    for (uint32_t i = threadIdx.x; i < d; i += 256) {
        float ot = 0.f;
        for (uint32_t k = 0; k < na; ++k) {
            const int e = top_ids[(uint64_t)t * na + k];
            if (e < 0 || (uint32_t)e >= ne) continue;
            ot = fmaf(top_w[(uint64_t)t * na + k], y[((uint64_t)t * na + k) * d + i], ot);
        }
        x[(uint64_t)t * d + i] += ot;
    }
}

// ---------------------------------------------------------------- decode
// Kernels for steps of at most kDecRows tokens (decode).  Each CTA stages the
// token rows (RMS-normalised when a norm weight is given) in shared memory
// and every warp streams whole weight rows with 16-byte loads, so a weight
// byte is read once per step and the norm, bias, residual and SwiGLU ride in
// the same launch.  Several warps per SM keep many loads in flight: the step
// is bound by how fast the weights stream from HBM.
constexpr int kDecRows = 4;

// Shared-memory layout of a decode CTA: the per-warp partial sums of squares
// [32][kDecRows], the norm weight g [K], then the staged rows sx [R][K].
__host__ __device__ constexpr uint32_t dec_red_floats() { return 32 * kDecRows; }

// Rows [0, R) of x (row stride ldx, K columns) staged in shared memory and
// returned as sx [R][K]; with g, each row becomes x * (1/sqrt(mean(x^2) +
// eps)) * g.  One pass brings x and g in (all loads of a thread in flight
// together) and sums each thread's squares in registers; the block then
// reduces the sums (warp shuffles, one barrier) and every thread rescales the
// elements it staged.  Ends with __syncthreads.
__device__ __forceinline__ float* stage_rows(float* dsm, const float* x, uint64_t ldx, uint32_t R,
                                             uint32_t K, const float* g, float eps) {
    float* red = dsm;
    float* sg = dsm + dec_red_floats();
    float* sx = sg + K;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float ss[kDecRows];
#pragma unroll
    for (int r = 0; r < kDecRows; ++r) ss[r] = 0.f;
    for (uint32_t i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
        if (g) *reinterpret_cast<float4*>(sg + i) = *reinterpret_cast<const float4*>(g + i);
#pragma unroll
        for (int r = 0; r < kDecRows; ++r) {
            if ((uint32_t)r >= R) break;
            const float4 v = *reinterpret_cast<const float4*>(x + r * ldx + i);
            *reinterpret_cast<float4*>(sx + r * K + i) = v;
            ss[r] = fmaf(v.x, v.x, ss[r]);
            ss[r] = fmaf(v.y, v.y, ss[r]);
            ss[r] = fmaf(v.z, v.z, ss[r]);
            ss[r] = fmaf(v.w, v.w, ss[r]);
        }
    }
    if (g) {
#pragma unroll
        for (int r = 0; r < kDecRows; ++r) {
            const float t = warp_sum(ss[r]);
            if (lane == 0) red[warp * kDecRows + r] = t;
        }
    }
    __syncthreads();
    if (!g) return sx;
    float sc[kDecRows];
#pragma unroll
    for (int r = 0; r < kDecRows; ++r) {
        float t = 0.f;
        for (uint32_t w = 0; w < (blockDim.x >> 5); ++w) t += red[w * kDecRows + r];
        sc[r] = 1.0f / sqrtf(t / (float)K + eps);
    }
    for (uint32_t i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
        const float4 g4 = *reinterpret_cast<const float4*>(sg + i);
#pragma unroll
        for (int r = 0; r < kDecRows; ++r) {
            if ((uint32_t)r >= R) break;
            float4 v = *reinterpret_cast<const float4*>(sx + r * K + i);
            v.x = v.x * sc[r] * g4.x;
            v.y = v.y * sc[r] * g4.y;
            v.z = v.z * sc[r] * g4.z;
            v.w = v.w * sc[r] * g4.w;
            *reinterpret_cast<float4*>(sx + r * K + i) = v;
        }
    }
    __syncthreads();
    return sx;
}

// acc[n][r] = W_n . x_n[r] for NW weight rows of one warp (x_n holds R rows
// of K floats; all lanes hold the sums on return).  A lane owns columns
// lane*4 + 128*m; the 16-byte loads of kU consecutive m of every row are
// issued (the last batch predicated) before any product is formed, so a row
// costs ceil(K / (128 kU)) memory round trips.  Large kU suits launches with
// few rows per SM; small kU keeps registers low so that many CTAs stay
// resident.  Each lane sums its columns in increasing m and the warp then
// reduces by shuffles, whatever kU is.
template <int NW, int kU>
__device__ __forceinline__ void row_dots_n(const float* const (&w)[NW],
                                           const float* const (&x)[NW], uint32_t R, uint32_t K,
                                           float (&acc)[NW][kDecRows]) {
    const uint32_t lane = threadIdx.x & 31;
#pragma unroll
    for (int n = 0; n < NW; ++n)
#pragma unroll
        for (int r = 0; r < kDecRows; ++r) acc[n][r] = 0.f;
    for (uint32_t i0 = lane * 4; i0 < K; i0 += kU * 128) {
        float4 a4[NW][kU];
#pragma unroll
        for (int u = 0; u < kU; ++u)
#pragma unroll
            for (int n = 0; n < NW; ++n)
                a4[n][u] = i0 + u * 128 < K
                               ? __ldg(reinterpret_cast<const float4*>(w[n] + i0 + u * 128))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            if (i0 + u * 128 >= K) break;
#pragma unroll
            for (int n = 0; n < NW; ++n)
#pragma unroll
                for (int r = 0; r < kDecRows; ++r)
                    if ((uint32_t)r < R)
                        acc[n][r] = dot4(a4[n][u],
                                         *reinterpret_cast<const float4*>(x[n] + r * K + i0 + u * 128),
                                         acc[n][r]);
        }
    }
#pragma unroll
    for (int n = 0; n < NW; ++n)
#pragma unroll
        for (int r = 0; r < kDecRows; ++r)
            if ((uint32_t)r < R) acc[n][r] = warp_sum(acc[n][r]);    // R is warp-uniform
}

// Lane r < R picks row r's sum.
__device__ __forceinline__ float pick_row(const float (&a)[kDecRows]) {
    const uint32_t lane = threadIdx.x & 31;
    float v = a[0];
#pragma unroll
    for (int r = 1; r < kDecRows; ++r)
        if ((uint32_t)r == lane) v = a[r];
    return v;
}

enum { kStore = 0, kAdd = 1, kSwiglu = 2 };

template <int MODE, int KU = 8>
__global__ void __launch_bounds__(256) dec_gemv_kernel(const float* __restrict__ w, const float* x,
                                                       uint64_t ldx, const float* g,
                                                       const float* bias, float* out,
                                                       uint64_t ldo, uint32_t R, uint32_t N,
                                                       uint32_t K, int clamp, const float* pf,
                                                       uint64_t pf_n) {
    extern __shared__ __align__(16) float dsm[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the warp's first row only: a launch whose rows exceed the L2 (the LM
    // head) would otherwise evict its own prefetched lines before use
    if (const uint32_t n = blockIdx.x * 8 + warp; n < N) {
        prefetch_row(w + (uint64_t)n * K, K);
        if (MODE == kSwiglu) prefetch_row(w + (uint64_t)(N + n) * K, K);
    }
    prefetch_share(pf, pf_n, cta_rank(), cta_count());
    pdl_wait();
    pdl_trigger();
    const float* sx = stage_rows(dsm, x, ldx, R, K, g, 1e-6f);
    for (uint32_t n = blockIdx.x * 8 + warp; n < N; n += gridDim.x * 8) {
        float v, vb = 0.f;
        if (MODE == kSwiglu) {
            float ab[2][kDecRows];
            row_dots_n<2, 4>({w + (uint64_t)n * K, w + (uint64_t)(N + n) * K}, {sx, sx}, R, K, ab);
            v = pick_row(ab[0]);
            vb = pick_row(ab[1]);
        } else {
            float a[1][kDecRows];
            row_dots_n<1, KU>({w + (uint64_t)n * K}, {sx}, R, K, a);
            v = pick_row(a[0]);
        }
        if (lane < R) {                      // lane r writes row r's output
            float* o = out + lane * ldo + n;
            if (MODE == kStore) {
                *o = bias ? v + bias[n] : v;
            } else if (MODE == kAdd) {
                *o += v;
            } else {
                if (clamp) v = fminf(fmaxf(v, -88.0f), 88.0f);
                *o = silu_mul(v, vb);
            }
        }
    }
}

// Q/K/V projection of a decode step with its norm, bias, RoPE and the KV
// append fused: one warp per pair of adjacent output rows (2m, 2m+1), which
// RoPE rotates together.  Query rows go to q_out [R][q_dim]; key and value
// rows of token r go to position pos0 + r of the fp32 cache [2][max_seq]
// [kv_dim].  The rotation is the KV path's (tgkv_kernels.cu rope_append), so
// the bits equal a separate RoPE launch's.
__global__ void __launch_bounds__(384, 1) dec_qkv_rope_kernel(const float* __restrict__ w,
                                                           const float* x, const float* g,
                                                           const float* bias, const float* cs,
                                                           const float* sn, float* q_out,
                                                           float* kvc, uint32_t R, uint32_t d,
                                                           uint32_t q_dim, uint32_t kv_dim,
                                                           uint32_t hd, uint32_t pos0,
                                                           uint32_t max_seq, const float* pf,
                                                           uint64_t pf_n, const uint32_t* pos_rows,
                                                           float* k_out, float* v_out) {
    extern __shared__ __align__(16) float dsm[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t npair = (q_dim + 2 * kv_dim) / 2;
    const uint32_t nw = blockDim.x >> 5;
    for (uint32_t m = blockIdx.x * nw + warp; m < npair; m += gridDim.x * nw)
        prefetch_row(w + (uint64_t)(2 * m) * d, 2 * d);
    prefetch_share(pf, pf_n, cta_rank(), cta_count());
    pdl_wait();
    pdl_trigger();
    const float* sx = stage_rows(dsm, x, d, R, d, g, 1e-6f);
    for (uint32_t m = blockIdx.x * nw + warp; m < npair; m += gridDim.x * nw) {
        const uint32_t n0 = 2 * m;
        // the epilogue's bias and rotation factors, loaded ahead of the weight rows
        const bool rot = n0 < q_dim + kv_dim;
        const uint32_t half = hd >> 1, col = n0 < q_dim ? n0 : n0 - q_dim;
        float b0 = 0.f, b1 = 0.f, c = 0.f, sn_ = 0.f;
        // row r's position: consecutive from pos0 (one sequence), or its own
        // (rows of different sequences)
        const uint64_t pos = lane < R ? (pos_rows ? pos_rows[lane] : pos0 + lane) : 0;
        if (lane < R) {
            if (bias) { b0 = bias[n0]; b1 = bias[n0 + 1]; }
            if (rot) {
                c = cs[pos * half + (col % hd) / 2];
                sn_ = sn[pos * half + (col % hd) / 2];
            }
        }
        float ab[2][kDecRows];
        row_dots_n<2, 12>({w + (uint64_t)n0 * d, w + (uint64_t)(n0 + 1) * d}, {sx, sx}, R, d, ab);
        float v0 = pick_row(ab[0]), v1 = pick_row(ab[1]);
        if (lane < R) {
            if (bias) { v0 += b0; v1 += b1; }
            if (rot) {
                const float r0 = __fmaf_rn(v0, c, -__fmul_rn(v1, sn_));
                const float r1 = __fmaf_rn(v0, sn_, __fmul_rn(v1, c));
                float* dst = n0 < q_dim ? q_out + (uint64_t)lane * q_dim + col
                             : kvc      ? kvc + pos * kv_dim + col
                                        : k_out + (uint64_t)lane * kv_dim + col;
                dst[0] = r0;
                dst[1] = r1;
            } else {
                const uint32_t vc = n0 - q_dim - kv_dim;
                float* dst = kvc ? kvc + ((uint64_t)max_seq + pos) * kv_dim + vc
                                 : v_out + (uint64_t)lane * kv_dim + vc;
                dst[0] = v0;
                dst[1] = v1;
            }
        }
    }
}

// Expert W3, the k-ordered weighted sum and the residual of a decode step:
// x[r][i] += sum_k top_w[r][k] * (W3[e_k][i] . h[r * na + k]).  One warp per
// row i; the dot products of two k at a time share one load batch (24 weight
// loads per lane in flight).
__global__ void __launch_bounds__(384, 1) dec_w3_combine_kernel(const float* __restrict__ w3,
                                                             const float* __restrict__ h,
                                                             const int32_t* top_ids,
                                                             const float* top_w, float* x,
                                                             uint32_t R, uint32_t d, uint32_t dff,
                                                             uint32_t ne, uint32_t na,
                                                             const float* pf, uint64_t pf_n) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t i = blockIdx.x * (blockDim.x >> 5) + warp;
    prefetch_share(pf, pf_n, cta_rank(), cta_count());
    pdl_wait();
    pdl_trigger();
    if (i >= d) return;
    for (uint32_t r = 0; r < R; ++r) {
        float ot = 0.f;
        for (uint32_t k = 0; k < na; k += 2) {
            const int e0 = top_ids[r * na + k];
            const int e1 = k + 1 < na ? top_ids[r * na + k + 1] : -1;
            const bool v0 = e0 >= 0 && (uint32_t)e0 < ne, v1 = e1 >= 0 && (uint32_t)e1 < ne;
            const float* h0 = h + (uint64_t)(r * na + k) * dff;
            const float* w0 = w3 + ((uint64_t)(v0 ? e0 : 0) * d + i) * dff;
            float a0, a1 = 0.f;
            if (v1) {
                float a[2][kDecRows];
                row_dots_n<2, 12>({w0, w3 + ((uint64_t)e1 * d + i) * dff}, {h0, h0 + dff}, 1, dff, a);
                a0 = a[0][0];
                a1 = a[1][0];
            } else {
                float a[1][kDecRows];
                row_dots_n<1, 12>({w0}, {h0}, 1, dff, a);
                a0 = a[0][0];
            }
            if (v0) ot = fmaf(top_w[r * na + k], a0, ot);
            if (v1) ot = fmaf(top_w[r * na + k + 1], a1, ot);
        }
        if (lane == 0) x[(uint64_t)r * d + i] += ot;
    }
}

// MoE front and expert W1/W2 + SiLU of a decode step in one launch: grid row
// p = (token r, choice k).  Every CTA normalises token r's row, computes its
// router logits (+ bias) and the engine's top-k and softmax -- the same
// arithmetic in every CTA, so all agree -- then streams W1/W2 rows of its
// expert e_k: h[p][j] = silu(W1[e][j] . ln) * (W2[e][j] . ln), one warp per j.
// The CTAs of column 0 publish top_ids / top_w for the W3 launch.
__global__ void __launch_bounds__(256, 2) dec_moe_w12_kernel(const float* x, const float* g,
                                                          const float* __restrict__ router,
                                                          const float* bias,
                                                          const float* __restrict__ w12,
                                                          int32_t* top_ids, float* top_w, float* h,
                                                          uint32_t d, uint32_t dff, uint32_t ne,
                                                          uint32_t na, const float* w3_pf) {
    extern __shared__ __align__(16) float dsm[];
    __shared__ float slog[16];
    __shared__ int s_ids[8];
    const uint32_t p = blockIdx.y, r = p / na, kk = p % na;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t e = warp; e < ne; e += 8) prefetch_row(router + (uint64_t)e * d, d);
    pdl_wait();
    pdl_trigger();
    const float* sx = stage_rows(dsm, x + (uint64_t)r * d, d, 1, d, g, 1e-6f);
    for (uint32_t e = warp; e < ne; e += 8) {
        float a[1][kDecRows];
        row_dots_n<1, 12>({router + (uint64_t)e * d}, {sx}, 1, d, a);
        if (lane == 0) slog[e] = bias ? a[0][0] + bias[e] : a[0][0];
    }
    __syncthreads();
    if (warp == 0) {
        // The engine's top-k: for k = 0..na-1 the first expert (lowest index)
        // of the largest logit above -1e30 not chosen yet, else -1 with
        // -1e30; lane k keeps choice k.  Argmax over the warp by shuffles on
        // the order (larger value, then lower index; no candidate last).
        const float v = lane < ne ? slog[lane] : 0.f;
        bool used = false;
        float my_v = -1e30f;
        int my_id = -1;
        for (uint32_t k = 0; k < na; ++k) {
            const bool cand = lane < ne && !used && v > -1e30f;
            float bv = cand ? v : -1e30f;
            int bi = cand ? (int)lane : -1;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (bi >= 0 && (uint32_t)bi == lane) used = true;
            if (lane == k) {
                my_v = bi >= 0 ? bv : -1e30f;
                my_id = bi;
            }
        }
        // softmax over the chosen logits: max (lanes >= na hold -1e30, below
        // or equal to every choice), then the exponentials summed in k order
        float mx = my_v;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float ek = lane < na ? expf(my_v - mx) : 0.f;
        float ss = 0.f;
        for (uint32_t k = 0; k < na; ++k) ss += __shfl_sync(0xffffffffu, ek, k);
        if (lane < na) {
            s_ids[lane] = my_id;
            if (blockIdx.x == 0 && kk == 0) {
                top_ids[r * na + lane] = my_id;
                top_w[r * na + lane] = ek / ss;
            }
        }
    }
    __syncthreads();
    const int e = s_ids[kk];
    if (e < 0 || (uint32_t)e >= ne) return;
    // the W3 launch reads expert e's [d][dff] rows: this column of CTAs pulls them into L2
    if (w3_pf) prefetch_share(w3_pf + (uint64_t)e * d * dff, (uint64_t)d * dff, blockIdx.x, gridDim.x);
    const float* we = w12 + (uint64_t)e * 2 * dff * d;
    for (uint32_t j = blockIdx.x * 8 + warp; j < dff; j += gridDim.x * 8) {
        const float* wa = we + (uint64_t)j * d;
        float ab[2][kDecRows];
        row_dots_n<2, 12>({wa, wa + (uint64_t)dff * d}, {sx, sx}, 1, d, ab);
        if (lane == 0) h[(uint64_t)p * dff + j] = silu_mul(ab[0][0], ab[1][0]);
    }
}

inline uint32_t blocks_for(uint64_t n, uint32_t per) { return (uint32_t)((n + per - 1) / per); }

}  // namespace tgkvf

using namespace tgkvf;

extern "C" int tgkv_fwd_embed(float* x, const float* emb, const int32_t* ids, uint32_t seq,
                              uint32_t d, uint32_t rows, int32_t unk, void* stream) {
    embed_kernel<<<seq, 256, 0, (cudaStream_t)stream>>>(x, emb, ids, d, rows, unk);
    return (int)cudaGetLastError();
}

extern "C" int tgkv_fwd_rmsnorm(float* out, const float* x, const float* w, uint32_t n_rows,
                                uint32_t d, uint64_t out_stride, uint64_t x_stride, float eps,
                                void* stream) {
    rmsnorm_kernel<<<n_rows, 256, 0, (cudaStream_t)stream>>>(out, x, w, d, out_stride, x_stride,
                                                             eps);
    return (int)cudaGetLastError();
}

extern "C" int tgkv_fwd_bias(float* y, const float* b, uint32_t rows, uint32_t cols,
                             void* stream) {
    const uint64_t n = (uint64_t)rows * cols;
    bias_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(y, b, n, cols);
    return (int)cudaGetLastError();
}

extern "C" int tgkv_fwd_silu_mul(float* h, const float* ab, uint32_t rows, uint32_t dff,
                                 int clamp, void* stream) {
    const uint64_t n = (uint64_t)rows * dff;
    silu_mul_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t)stream>>>(h, ab, n, dff, clamp);
    return (int)cudaGetLastError();
}

extern "C" int tgkv_fwd_route(const float* logits, const float* bias, int32_t* top_ids,
                              float* top_w, uint32_t* counts, uint32_t* lists, uint32_t seq,
                              uint32_t ne, uint32_t na, void* stream) {
    if (ne == 0 || ne > 16 || na == 0 || na > 8 || na > ne) return (int)cudaErrorInvalidValue;
    route_kernel<<<blocks_for(seq, 128), 128, 0, (cudaStream_t)stream>>>(
        logits, bias, top_ids, top_w, counts, lists, seq, ne, na);
    return (int)cudaGetLastError();
}

extern "C" int tgkv_fwd_expert_w12(const float* w12, const float* x, float* h,
                                   const uint32_t* counts, const uint32_t* lists, uint32_t seq,
                                   uint32_t ne, uint32_t na, uint32_t d, uint32_t dff,
                                   void* stream) {
    if (d % 4 || dff % 4) return (int)cudaErrorInvalidValue;
    const dim3 grid(blocks_for(dff, kRowsPerCta), ne);
    expert_kernel<true><<<grid, 256, 0, (cudaStream_t)stream>>>(
        w12, x, h, counts, lists, seq * na, dff, d, na, (uint64_t)2 * dff * d);
    return (int)cudaGetLastError();
}

extern "C" int tgkv_fwd_expert_w3(const float* w3, const float* h, float* y,
                                  const uint32_t* counts, const uint32_t* lists, uint32_t seq,
                                  uint32_t ne, uint32_t na, uint32_t d, uint32_t dff,
                                  void* stream) {
    if (d % 4 || dff % 4) return (int)cudaErrorInvalidValue;
    const dim3 grid(blocks_for(d, kRowsPerCta), ne);
    expert_kernel<false><<<grid, 256, 0, (cudaStream_t)stream>>>(
        w3, h, y, counts, lists, seq * na, d, dff, na, (uint64_t)d * dff);
    return (int)cudaGetLastError();
}

extern "C" int tgkv_fwd_moe_combine(float* x, const float* y, const int32_t* top_ids,
                                    const float* top_w, uint32_t seq, uint32_t d, uint32_t ne,
                                    uint32_t na, void* stream) {
    combine_kernel<<<seq, 256, 0, (cudaStream_t)stream>>>(x, y, top_ids, top_w, d, ne, na);
    return (int)cudaGetLastError();
}


// ---- decode launchers
static size_t dec_smem(uint32_t R, uint32_t K) {
    return ((size_t)dec_red_floats() + K + (size_t)R * K) * 4;
}

// SMs of the current device (grids of the streaming launches are sized to
// what stays resident, so that no CTA waits for a second wave).
static uint32_t sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return 148;
    return (uint32_t)n;
}

static bool pdl_on() {
    static const bool on = [] {
        const char* e = getenv("TGKV_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Launch as a programmatic dependent of the previous work on the stream.
template <typename... KArgs, typename... Args>
static int launch_pdl_n(void (*k)(KArgs...), dim3 grid, uint32_t threads, size_t smem,
                        void* stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_on() ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}
template <typename... KArgs, typename... Args>
static int launch_pdl(void (*k)(KArgs...), dim3 grid, size_t smem, void* stream, Args... args) {
    return launch_pdl_n(k, grid, 256, smem, stream, args...);
}

// Warps per CTA (at most 12) for a launch of `units` equal warp tasks with
// one CTA per SM: the fewest warps whose CTAs fit on the SMs, so that no SM
// streams more than ceil(units / SMs) tasks.
static uint32_t warps_for(uint32_t units, uint32_t sms) {
    for (uint32_t w = 8; w < 12; ++w)
        if ((units + w - 1) / w <= sms) return w;
    return 12;
}

template <typename F>
static int set_smem(F* f, size_t bytes) {
    if (bytes <= 48 * 1024) return 0;
    return (int)cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

extern "C" uint32_t tgkv_fwd_decode_rows(void) { return kDecRows; }

extern "C" int tgkv_fwd_dec_gemv(int mode, const float* w, const float* x, uint64_t ldx,
                                 const float* g, const float* bias, float* out, uint64_t ldo,
                                 uint32_t R, uint32_t N, uint32_t K, int clamp, const float* pf,
                                 uint64_t pf_n, void* stream) {
    if (R == 0 || R > kDecRows || K % 4 || ldx % 4) return (int)cudaErrorInvalidValue;
    const size_t sm = dec_smem(R, K);
    if (sm > 200 * 1024) return (int)cudaErrorInvalidValue;
    // CTAs loop over rows: at most 4 per SM (64 registers a thread) so that the
    // LM head's 32000 rows stage the normalised input once per CTA
    const uint32_t nb = blocks_for(N, 8), cap = 4 * sm_count();
    const dim3 grid(nb < cap ? nb : cap);
    int e;
    switch (mode) {
    case kStore:
        if ((e = set_smem(dec_gemv_kernel<kStore>, sm))) return e;
        return launch_pdl(dec_gemv_kernel<kStore>, grid, sm, stream, w, x, ldx, g, bias, out, ldo,
                          R, N, K, clamp, pf, pf_n);
    case kAdd:
        if ((e = set_smem(dec_gemv_kernel<kAdd>, sm))) return e;
        return launch_pdl(dec_gemv_kernel<kAdd>, grid, sm, stream, w, x, ldx, g, bias, out, ldo,
                          R, N, K, clamp, pf, pf_n);
    case kSwiglu:
        if ((e = set_smem(dec_gemv_kernel<kSwiglu>, sm))) return e;
        return launch_pdl(dec_gemv_kernel<kSwiglu>, grid, sm, stream, w, x, ldx, g, bias, out,
                          ldo, R, N, K, clamp, pf, pf_n);
    default:
        return (int)cudaErrorInvalidValue;
    }
}

extern "C" int tgkv_fwd_dec_qkv_rope(const float* w, const float* x, const float* g,
                                     const float* bias, const float* cs, const float* sn,
                                     float* q_out, float* kvc, uint32_t R, uint32_t d,
                                     uint32_t q_dim, uint32_t kv_dim, uint32_t hd, uint32_t pos0,
                                     uint32_t max_seq, const float* pf, uint64_t pf_n,
                                     void* stream) {
    if (R == 0 || R > kDecRows || d % 4 || hd % 2 || q_dim % hd || kv_dim % hd ||
        (uint64_t)pos0 + R > max_seq)
        return (int)cudaErrorInvalidValue;
    const size_t sm = dec_smem(R, d);
    if (sm > 200 * 1024) return (int)cudaErrorInvalidValue;
    int e;
    if ((e = set_smem(dec_qkv_rope_kernel, sm))) return e;
    // one warp per pair of rows, one CTA per SM
    const uint32_t npair = (q_dim + 2 * kv_dim) / 2, nw = warps_for(npair, sm_count());
    return launch_pdl_n(dec_qkv_rope_kernel, dim3(blocks_for(npair, nw)), nw * 32, sm, stream, w,
                        x, g, bias, cs, sn, q_out, kvc, R, d, q_dim, kv_dim, hd, pos0, max_seq,
                        pf, pf_n, (const uint32_t*)nullptr, (float*)nullptr, (float*)nullptr);
}

extern "C" int tgkv_fwd_dec_qkv_rows(const float* w, const float* x, const float* g,
                                     const float* bias, const float* cs, const float* sn,
                                     float* q_out, float* k_out, float* v_out, uint32_t R,
                                     uint32_t d, uint32_t q_dim, uint32_t kv_dim, uint32_t hd,
                                     const uint32_t* pos_rows, uint32_t max_seq, const float* pf,
                                     uint64_t pf_n, void* stream) {
    if (R == 0 || R > kDecRows || d % 4 || hd % 2 || q_dim % hd || kv_dim % hd || !pos_rows ||
        !k_out || !v_out)
        return (int)cudaErrorInvalidValue;
    const size_t sm = dec_smem(R, d);
    if (sm > 200 * 1024) return (int)cudaErrorInvalidValue;
    int e;
    if ((e = set_smem(dec_qkv_rope_kernel, sm))) return e;
    const uint32_t npair = (q_dim + 2 * kv_dim) / 2, nw = warps_for(npair, sm_count());
    return launch_pdl_n(dec_qkv_rope_kernel, dim3(blocks_for(npair, nw)), nw * 32, sm, stream, w,
                        x, g, bias, cs, sn, q_out, (float*)nullptr, R, d, q_dim, kv_dim, hd, 0u,
                        max_seq, pf, pf_n, pos_rows, k_out, v_out);
}

extern "C" int tgkv_fwd_dec_w3_combine(const float* w3, const float* h, const int32_t* top_ids,
                                       const float* top_w, float* x, uint32_t R, uint32_t d,
                                       uint32_t dff, uint32_t ne, uint32_t na, const float* pf,
                                       uint64_t pf_n, void* stream) {
    if (R == 0 || R > kDecRows || dff % 4) return (int)cudaErrorInvalidValue;
    // one warp per output row, one CTA per SM
    const uint32_t nw = warps_for(d, sm_count());
    return launch_pdl_n(dec_w3_combine_kernel, dim3(blocks_for(d, nw)), nw * 32, 0, stream, w3, h,
                        top_ids, top_w, x, R, d, dff, ne, na, pf, pf_n);
}

extern "C" int tgkv_fwd_dec_moe_w12(const float* x, const float* g, const float* router,
                                    const float* bias, const float* w12, int32_t* top_ids,
                                    float* top_w, float* h, uint32_t R, uint32_t d, uint32_t dff,
                                    uint32_t ne, uint32_t na, const float* w3_pf, void* stream) {
    if (R == 0 || R > kDecRows || d % 4 || ne == 0 || ne > 16 || na == 0 || na > 8 || na > ne)
        return (int)cudaErrorInvalidValue;
    const size_t sm = dec_smem(1, d);
    int e;
    if ((e = set_smem(dec_moe_w12_kernel, sm))) return e;
    // two CTAs per SM over all (token, choice) columns; warps loop over rows
    const uint32_t cols = R * na, per = 2 * sm_count() / cols;
    const uint32_t gx = blocks_for(dff, 8) < per ? blocks_for(dff, 8) : (per ? per : 1);
    return launch_pdl(dec_moe_w12_kernel, dim3(gx, cols), sm, stream, x, g,
                      router, bias, w12, top_ids, top_w, h, d, dff, ne, na, w3_pf);
}

extern "C" void* tgkv_fwd_host_alloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMallocHost(&p, bytes) != cudaSuccess) return nullptr;
    return p;
}

extern "C" void tgkv_fwd_host_free(void* p) {
    if (p) cudaFreeHost(p);
}
