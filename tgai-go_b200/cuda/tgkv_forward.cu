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
        for (uint32_t i = lane * 4; i < k_dim; i += 128) {
            const float4 a4 = *reinterpret_cast<const float4*>(wa + i);
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (kW12) b4 = *reinterpret_cast<const float4*>(wb + i);
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

extern "C" void* tgkv_fwd_host_alloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMallocHost(&p, bytes) != cudaSuccess) return nullptr;
    return p;
}

extern "C" void tgkv_fwd_host_free(void* p) {
    if (p) cudaFreeHost(p);
}
