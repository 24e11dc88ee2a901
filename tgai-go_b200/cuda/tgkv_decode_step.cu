// tgkv_decode_step.cu -- one decode token through every layer of the model in
// ONE cooperative launch (sm_100a): one CTA per SM, the phases of a layer
// separated by grid barriers instead of kernel boundaries.
//
// The per-launch decode path (tgkv_forward.cu) runs five dependent launches
// per layer; each pays a fixed chain of launch, wait, input staging and
// epilogue (2.5-3 us), which is most of a layer's time on a 3B MoE.  Here a
// layer is five phases of one resident grid:
//   P1  RMSNorm(x) . Wqkv in row pairs, bias, RoPE, K/V row appended at pos;
//   P2  split attention over the cache: warp tasks of (query head, position
//       range), online softmax, partials; the task that finishes a head last
//       merges its partials;
//   P3  the merged heads into shared memory, then the out projection +
//       residual;
//   P4  RMSNorm(x), router + top-k (every CTA, same arithmetic as the
//       engine's), routed experts' W1/W2 rows + SiLU (or the dense FFN's);
//   P5  routed experts' W3 rows, k-ordered sum + residual (or dense W3).
// Before each barrier a warp loads the first column block of its first rows
// of the next phase into registers where they are known (all but the routed
// experts' W1/W2), so those loads stream while the grid waits.
// Every barrier is bounded: a CTA that waits more than ~1 s sets the error
// word and the grid leaves at the next barrier, so a broken run returns a
// status instead of hanging the GPU.  Data written inside the launch (x, q,
// the K/V rows, partials, h) is read with ld.global.cg (L2, not the SM's L1,
// which other SMs' stores do not update); weights with the read-only path.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "tgkv_forward.h"

namespace tgkvs {

constexpr int kThreads = 384;        // 12 warps, one CTA per SM
constexpr int kWarps = kThreads / 32;
constexpr int kSub = 8;              // positions per attention load batch
constexpr int kErrBarrier = 6;       // error word: a grid barrier timed out
constexpr long long kSpinCycles = 2000000000ll;   // ~1 s at 2 GHz

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
__device__ __forceinline__ float4 ldcg4(const float* p) {
    return __ldcg(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ float silu_mul(float a, float b) { return (a / (1.0f + expf(-a))) * b; }

// Grid barrier over a counter that only grows within the launch: barrier b
// completes when the counter reaches (b + 1) * gridDim.x.  Thread 0 of each
// CTA arrives with a release reduction (the CTA's writes, ordered before it by
// __syncthreads, become visible with it) and spins on acquire loads; the
// result (1 = go on) is read by all threads of the CTA from shared memory, so
// the CTA leaves together.
__device__ __forceinline__ int grid_sync(uint32_t* bar, uint32_t& target, int* err, int* s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        target += gridDim.x;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        const long long t0 = clock64();
        int ok = 1;
        for (uint32_t it = 0;; ++it) {
            uint32_t v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
            if (v >= target) break;
            if ((it & 63) == 63) {
                if (*(volatile int*)err) { ok = 0; break; }
                if (clock64() - t0 > kSpinCycles) {
                    atomicExch(err, kErrBarrier);
                    ok = 0;
                    break;
                }
            }
        }
        if (ok && *(volatile int*)err) ok = 0;
        *s_ok = ok;
    }
    __syncthreads();
    return *(volatile int*)s_ok;
}

// dst[0, K) = src * (1/sqrt(mean(src^2) + eps)) * g  (g NULL: plain copy);
// src written inside the launch.  Ends with __syncthreads.
__device__ __forceinline__ void stage(float* dst, const float* src, const float* g, uint32_t K,
                                      float* red) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x * 4; i < K; i += kThreads * 4) {
        const float4 v = ldcg4(src + i);
        *reinterpret_cast<float4*>(dst + i) = v;
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
    if (!g) {
        __syncthreads();
        return;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += red[w];
    const float sc = 1.0f / sqrtf(t / (float)K + 1e-6f);
    for (uint32_t i = threadIdx.x * 4; i < K; i += kThreads * 4) {
        float4 v = *reinterpret_cast<const float4*>(dst + i);
        const float4 g4 = __ldg(reinterpret_cast<const float4*>(g + i));
        v.x = v.x * sc * g4.x;
        v.y = v.y * sc * g4.y;
        v.z = v.z * sc * g4.z;
        v.w = v.w * sc * g4.w;
        *reinterpret_cast<float4*>(dst + i) = v;
    }
    __syncthreads();
}

// A weight load: read-only path, not kept in L1, and marked first to leave
// L2 (every weight is read once per token, 3.4 GB on the V2.7-shaped model,
// while the K/V rows, activations and partials should stay there).
__device__ __forceinline__ float4 ld_weight(const float* p, uint64_t policy) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(policy));
    return v;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// The column block [i0, i0 + kU * 128) of NW rows into registers: lane l
// loads float4 l, l + 32, ... of it (zeros past K).
template <int NW, int kU>
__device__ __forceinline__ void load_block(float4 (&a4)[NW][kU], const float* const (&w)[NW],
                                           uint32_t K, uint32_t i0) {
    const uint64_t pol = evict_first_policy();
#pragma unroll
    for (int u = 0; u < kU; ++u)
#pragma unroll
        for (int n = 0; n < NW; ++n)
            a4[n][u] = i0 + u * 128 < K ? ld_weight(w[n] + i0 + u * 128, pol)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
}

// acc[n] = W_n . x_n over K columns (x_n in shared memory), NW rows of one
// warp, with the rows' first column block already in a4 (load_block at
// lane * 4, issued earlier -- before a grid barrier, so that it streams
// while the grid waits); each later block's loads are all issued before its
// products.  All lanes hold the sums.
template <int NW, int kU>
__device__ __forceinline__ void dots_from(float4 (&a4)[NW][kU], const float* const (&w)[NW],
                                          const float* const (&x)[NW], uint32_t K,
                                          float (&acc)[NW]) {
    const uint32_t lane = threadIdx.x & 31;
#pragma unroll
    for (int n = 0; n < NW; ++n) acc[n] = 0.f;
    for (uint32_t i0 = lane * 4; i0 < K;) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            if (i0 + u * 128 >= K) break;
#pragma unroll
            for (int n = 0; n < NW; ++n)
                acc[n] = dot4(a4[n][u], *reinterpret_cast<const float4*>(x[n] + i0 + u * 128), acc[n]);
        }
        i0 += kU * 128;
        if (i0 < K) load_block<NW, kU>(a4, w, K, i0);
    }
#pragma unroll
    for (int n = 0; n < NW; ++n) acc[n] = warp_sum(acc[n]);
}

}  // namespace tgkvs

using namespace tgkvs;

// P2 for query head h's position range [p_begin, p_end) against the K/V rows
// of its KV head kvh in the fp32 cache, lane l owning dimensions [4l, 4l + 4)
// (lanes past head_dim / 4 idle); kSub positions' rows in flight at a time.
// Online softmax in the natural exponent; the partial goes to part as
// [m, l, 0, 0, o[head_dim]] (running max, sum, unnormalised output; stride
// head_dim + 4 keeps o 16-byte aligned), slot h * kTgStepMaxTasks + task.
__device__ __forceinline__ void attn_task(const TGFwdStepParams& p, const float* kvc, uint32_t h,
                                          uint32_t kvh, uint32_t task, uint32_t p_begin,
                                          uint32_t p_end) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t hd = p.head_dim, kv_dim = p.n_kv_heads * hd;
    const bool on = lane * 4 < hd;
    const float4 qv = on ? ldcg4(p.q + (uint64_t)h * hd + lane * 4) : make_float4(0.f, 0.f, 0.f, 0.f);
    float m = -INFINITY, l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* K = kvc + (uint64_t)kvh * hd + lane * 4;
    const float* V = kvc + (uint64_t)p.max_seq * kv_dim + (uint64_t)kvh * hd + lane * 4;
    for (uint32_t p0 = p_begin; p0 < p_end; p0 += kSub) {
        float4 kr[kSub], vr[kSub];
#pragma unroll
        for (int u = 0; u < kSub; ++u) {
            const bool in = on && p0 + u < p_end;
            kr[u] = in ? ldcg4(K + (uint64_t)(p0 + u) * kv_dim) : make_float4(0.f, 0.f, 0.f, 0.f);
            vr[u] = in ? ldcg4(V + (uint64_t)(p0 + u) * kv_dim) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float sc[kSub];
        float mx = m;
#pragma unroll
        for (int u = 0; u < kSub; ++u) {
            sc[u] = warp_sum(dot4(qv, kr[u], 0.f)) * p.scale;
            if (p0 + u >= p_end) sc[u] = -INFINITY;
            mx = fmaxf(mx, sc[u]);
        }
        const float corr = m == -INFINITY ? 0.f : expf(m - mx);
        float4 acc = make_float4(o.x * corr, o.y * corr, o.z * corr, o.w * corr);
        float ls = l * corr;
#pragma unroll
        for (int u = 0; u < kSub; ++u) {
            const float e = sc[u] == -INFINITY ? 0.f : expf(sc[u] - mx);
            ls += e;
            acc.x = fmaf(e, vr[u].x, acc.x);
            acc.y = fmaf(e, vr[u].y, acc.y);
            acc.z = fmaf(e, vr[u].z, acc.z);
            acc.w = fmaf(e, vr[u].w, acc.w);
        }
        m = mx;
        l = ls;
        o = acc;
    }
    float* dst = p.part + ((uint64_t)h * kTgStepMaxTasks + task) * (hd + 4);
    if (lane == 0) {
        dst[0] = m;
        dst[1] = l;
    }
    if (on) *reinterpret_cast<float4*>(dst + 4 + lane * 4) = o;
}

// Head h's attention output from its n_tasks partials, by the one warp that
// finished the head's last task, into attn (global, [q_dim]): the maximum M
// of the partials' maxima, L = sum exp(m_i - M) l_i (lane i % 32 holding
// partial i's m and l), O = sum exp(m_i - M) o_i / L with lane l owning
// dimensions [4l, 4l + 4), sixteen partials' rows in flight at a time.
__device__ __forceinline__ void attn_merge(const TGFwdStepParams& p, uint32_t h, uint32_t n_tasks) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t hd = p.head_dim, stride = hd + 4;
    const bool on = lane * 4 < hd;
    const float* base = p.part + (uint64_t)h * kTgStepMaxTasks * stride;
    constexpr int kPer = kTgStepMaxTasks / 32;
    float w[kPer], li[kPer];
    float M = -INFINITY;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        const uint32_t i = lane + 32 * u;
        w[u] = i < n_tasks ? __ldcg(base + (uint64_t)i * stride) : -INFINITY;
        li[u] = i < n_tasks ? __ldcg(base + (uint64_t)i * stride + 1) : 0.f;
        M = fmaxf(M, w[u]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.f;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
        w[u] = w[u] == -INFINITY ? 0.f : expf(w[u] - M);     // the weight of partial i
        L = fmaf(w[u], li[u], L);
    }
    L = warp_sum(L);
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
    for (uint32_t i0 = 0; i0 < n_tasks; i0 += 16) {
        float4 oc[16];
#pragma unroll
        for (int u = 0; u < 16; ++u)
            oc[u] = on && i0 + u < n_tasks ? ldcg4(base + (uint64_t)(i0 + u) * stride + 4 + lane * 4)
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            const uint32_t i = i0 + u;
            float f = 0.f;
#pragma unroll
            for (int v = 0; v < kPer; ++v) {
                const float fv = __shfl_sync(0xffffffffu, w[v], i & 31);
                if (i >> 5 == (uint32_t)v) f = fv;
            }
            if (i >= n_tasks) f = 0.f;
            O.x = fmaf(f, oc[u].x, O.x);
            O.y = fmaf(f, oc[u].y, O.y);
            O.z = fmaf(f, oc[u].z, O.z);
            O.w = fmaf(f, oc[u].w, O.w);
        }
    }
    if (on) {
        const float inv = 1.0f / L;
        *reinterpret_cast<float4*>(p.attn + (uint64_t)h * hd + lane * 4) =
            make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
    }
}

// The engine's top-k of warp 0 over slog[0, ne): for k = 0..na-1 the first
// expert (lowest index) of the largest logit above -1e30 not chosen yet, else
// -1 with -1e30 (src/tgai_engine.c:4166-4192), then the softmax over the
// chosen logits with the exponentials summed in k order.
__device__ __forceinline__ void top_k_warp(const float* slog, uint32_t ne, uint32_t na,
                                           int* s_ids, float* s_w) {
    const uint32_t lane = threadIdx.x & 31;
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
    float mx = my_v;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float ek = lane < na ? expf(my_v - mx) : 0.f;
    float ss = 0.f;
    for (uint32_t k = 0; k < na; ++k) ss += __shfl_sync(0xffffffffu, ek, k);
    if (lane < na) {
        s_ids[lane] = my_id;
        s_w[lane] = ek / ss;
    }
}

template <int G>
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const TGFwdStepParams p) {
    extern __shared__ __align__(16) float smem[];
    __shared__ float red[kWarps];
    __shared__ float slog[16];
    __shared__ int s_ids[8];
    __shared__ float s_w[8];
    __shared__ int s_ok;
    const uint32_t d = p.d, hd = p.head_dim, nkv = p.n_kv_heads;
    const uint32_t q_dim = nkv * G * hd, kv_dim = nkv * hd, dff = p.dff, ne = p.ne, na = p.na;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // warp tasks go round the CTAs first (task t to CTA t % grid), so that
    // a phase with fewer tasks than warps still keeps every SM loading
    const uint32_t gw = blockIdx.x + gridDim.x * warp, tw = gridDim.x * kWarps;
    float* sx = smem;                     // [max(d, q_dim)]
    float* sh = smem + p.sx_floats;       // [na or 1][dff]
    uint32_t* bar = p.state;
    int* err = reinterpret_cast<int*>(p.state + 1);
    uint32_t* head_ctr = p.state + 2;     // finished attention tasks per query head
    uint32_t target = 0;
    // attention split: at most kTgStepMaxTasks position ranges per KV head,
    // each a multiple of kSub positions, about 16 positions where L allows
    const uint32_t L = p.pos + 1;
    uint32_t n_tasks = (L + 15) / 16;
    if (n_tasks > kTgStepMaxTasks) n_tasks = kTgStepMaxTasks;
    const uint32_t ch = ((L + n_tasks - 1) / n_tasks + kSub - 1) / kSub * kSub;
    n_tasks = (L + ch - 1) / ch;
    const uint32_t half = hd >> 1;
    const uint32_t npair = (q_dim + 2 * kv_dim) / 2;
    // The first column block of the warp's first rows of the next phase,
    // loaded before the grid barrier that precedes it (pf_for: which phase
    // it is for; 0: none): Q/K/V pair, out-projection row, router row, W3
    // rows of the first two experts (or the dense W3 row).
    enum { kPfNone = 0, kPfQkv, kPfWo, kPfRouter, kPfW3 };
    // Every task loads its rows through pf too, and every prefetch point
    // writes it (zeros where the warp has no such row), so that it is the
    // one block of row registers of the kernel and dead during the attention.
    float4 pf[2][12];
    float4 (&pf1)[1][12] = reinterpret_cast<float4 (&)[1][12]>(pf);
    int pf_for;
    const uint32_t lane4 = lane * 4;
    {
        const float* r0 = p.layers[0].wqkv + (uint64_t)(2 * (gw < npair ? gw : 0)) * d;
        load_block<2, 12>(pf, {r0, r0 + d}, gw < npair ? d : 0, lane4);
        pf_for = gw < npair ? kPfQkv : kPfNone;
    }

    for (uint32_t l = 0; l < p.n_layers; ++l) {
        const TGFwdStepLayer W = p.layers[l];
        float* kvc = p.kvc[l];
        // ---- P1: norm, Q/K/V row pairs, bias, RoPE at pos, K/V append
        stage(sx, p.x, W.ln1, d, red);
        for (uint32_t mp = gw; mp < npair; mp += tw) {
            const uint32_t n0 = 2 * mp;
            const float* r0 = W.wqkv + (uint64_t)n0 * d;
            float a[2];
            if (!(mp == gw && pf_for == kPfQkv)) load_block<2, 12>(pf, {r0, r0 + d}, d, lane4);
            dots_from<2, 12>(pf, {r0, r0 + d}, {sx, sx}, d, a);
            if (lane == 0) {
                float v0 = a[0], v1 = a[1];
                if (W.bqkv) {
                    v0 += W.bqkv[n0];
                    v1 += W.bqkv[n0 + 1];
                }
                if (n0 < q_dim + kv_dim) {
                    const uint32_t col = n0 < q_dim ? n0 : n0 - q_dim;
                    const uint64_t ti = (uint64_t)p.pos * half + (col % hd) / 2;
                    const float c = p.cs[ti], s = p.sn[ti];
                    const float r0 = __fmaf_rn(v0, c, -__fmul_rn(v1, s));
                    const float r1 = __fmaf_rn(v0, s, __fmul_rn(v1, c));
                    float* dst = n0 < q_dim ? p.q + col : kvc + (uint64_t)p.pos * kv_dim + col;
                    dst[0] = r0;
                    dst[1] = r1;
                } else {
                    float* dst = kvc + ((uint64_t)p.max_seq + p.pos) * kv_dim + (n0 - q_dim - kv_dim);
                    dst[0] = v0;
                    dst[1] = v1;
                }
            }
        }
        if (!grid_sync(bar, target, err, &s_ok)) return;
        // ---- P2: split attention, partials per (query head, position
        // range), one task per CTA before any CTA takes a second; the task
        // that finishes a head last merges it into attn
        for (uint32_t t = gw; t < nkv * G * n_tasks; t += tw) {
            const uint32_t h = t / n_tasks, task = t % n_tasks;
            const uint32_t pb = task * ch, pe = pb + ch < L ? pb + ch : L;
            attn_task(p, kvc, h, h / G, task, pb, pe);
            __syncwarp();
            uint32_t prev = 0;
            if (lane == 0) {
                __threadfence();                     // this task's partial, then the count
                prev = atomicAdd(head_ctr + h, 1u);
            }
            prev = __shfl_sync(0xffffffffu, prev, 0);
            if (prev == n_tasks - 1) {
                __threadfence();                     // every task's partial before the merge
                attn_merge(p, h, n_tasks);
                if (lane == 0) head_ctr[h] = 0;      // counted again only a layer later
            }
        }
        load_block<1, 12>(pf1, {W.wo + (uint64_t)(gw < d ? gw : 0) * q_dim}, gw < d ? q_dim : 0,
                          lane4);
        pf_for = gw < d ? kPfWo : kPfNone;
        if (!grid_sync(bar, target, err, &s_ok)) return;
        // ---- P3: the merged heads into sx, then out projection + residual
        stage(sx, p.attn, nullptr, q_dim, red);
        for (uint32_t n = gw; n < d; n += tw) {
            const float* r = W.wo + (uint64_t)n * q_dim;
            float a[1];
            if (!(n == gw && pf_for == kPfWo)) load_block<1, 12>(pf1, {r}, q_dim, lane4);
            dots_from<1, 12>(pf1, {r}, {sx}, q_dim, a);
            if (lane == 0) p.x[n] = __ldcg(p.x + n) + a[0];
        }
        {
            const bool r = ne && warp < ne;
            load_block<1, 12>(pf1, {W.router + (uint64_t)(r ? warp : 0) * d}, r ? d : 0, lane4);
            pf_for = r ? kPfRouter : kPfNone;
        }
        if (!grid_sync(bar, target, err, &s_ok)) return;
        // ---- P4: norm, router + top-k (every CTA), expert W1/W2 rows + SiLU
        stage(sx, p.x, W.ln2, d, red);
        if (ne) {
            for (uint32_t e = warp; e < ne; e += kWarps) {
                const float* r = W.router + (uint64_t)e * d;
                float a[1];
                if (!(e == warp && pf_for == kPfRouter)) load_block<1, 12>(pf1, {r}, d, lane4);
                dots_from<1, 12>(pf1, {r}, {sx}, d, a);
                if (lane == 0) slog[e] = W.qb ? a[0] + W.qb[e] : a[0];
            }
            __syncthreads();
            if (warp == 0) top_k_warp(slog, ne, na, s_ids, s_w);
            __syncthreads();
            for (uint32_t t = gw; t < na * dff; t += tw) {
                const uint32_t k = t / dff, j = t % dff;
                const int e = s_ids[k];
                float hv = 0.f;
                if (e >= 0 && (uint32_t)e < ne) {
                    const float* wa = W.w12 + ((uint64_t)e * 2 * dff + j) * d;
                    float a[2];
                    load_block<2, 12>(pf, {wa, wa + (uint64_t)dff * d}, d, lane4);
                    dots_from<2, 12>(pf, {wa, wa + (uint64_t)dff * d}, {sx, sx}, d, a);
                    hv = silu_mul(a[0], a[1]);
                }
                if (lane == 0) p.h[(uint64_t)k * dff + j] = hv;
            }
        } else {
            for (uint32_t j = gw; j < dff; j += tw) {
                const float* r0 = W.w12 + (uint64_t)j * d;
                const float* r1 = W.w12 + (uint64_t)(dff + j) * d;
                float a[2];
                load_block<2, 12>(pf, {r0, r1}, d, lane4);
                dots_from<2, 12>(pf, {r0, r1}, {sx, sx}, d, a);
                if (lane == 0) p.h[j] = silu_mul(fminf(fmaxf(a[0], -88.0f), 88.0f), a[1]);
            }
        }
        {
            // dense: the W3 row of output gw; experts: the rows of output gw
            // of the first two experts when both are routed
            const bool two = ne && na > 1 && s_ids[0] >= 0 && (uint32_t)s_ids[0] < ne &&
                             s_ids[1] >= 0 && (uint32_t)s_ids[1] < ne;
            const bool on = gw < d && (!ne || two);
            const uint32_t i = on ? gw : 0;
            const float* r0 = ne ? W.w3 + ((uint64_t)(two ? s_ids[0] : 0) * d + i) * dff
                                 : W.w3 + (uint64_t)i * dff;
            const float* r1 = ne ? W.w3 + ((uint64_t)(two ? s_ids[1] : 0) * d + i) * dff : r0;
            load_block<2, 12>(pf, {r0, ne ? r1 : r0}, on ? dff : 0, lane4);
            pf_for = on ? kPfW3 : kPfNone;
        }
        if (!grid_sync(bar, target, err, &s_ok)) return;
        // ---- P5: W3 rows, k-ordered weighted sum (or dense W3) + residual
        stage(sh, p.h, nullptr, (ne ? na : 1) * dff, red);
        for (uint32_t i = gw; i < d; i += tw) {
            float ot = 0.f;
            if (ne) {
                for (uint32_t k = 0; k < na; k += 2) {
                    const int e0 = s_ids[k];
                    const int e1 = k + 1 < na ? s_ids[k + 1] : -1;
                    const bool v0 = e0 >= 0 && (uint32_t)e0 < ne, v1 = e1 >= 0 && (uint32_t)e1 < ne;
                    const float* w0 = W.w3 + ((uint64_t)(v0 ? e0 : 0) * d + i) * dff;
                    float a0 = 0.f, a1 = 0.f;
                    if (v1) {
                        const float* w1 = W.w3 + ((uint64_t)e1 * d + i) * dff;
                        float a[2];
                        if (!(k == 0 && i == gw && pf_for == kPfW3))
                            load_block<2, 12>(pf, {w0, w1}, dff, lane4);
                        dots_from<2, 12>(pf, {w0, w1},
                                         {sh + (uint64_t)k * dff, sh + (uint64_t)(k + 1) * dff}, dff, a);
                        a0 = a[0];
                        a1 = a[1];
                    } else if (v0) {
                        float a[1];
                        load_block<1, 12>(pf1, {w0}, dff, lane4);
                        dots_from<1, 12>(pf1, {w0}, {sh + (uint64_t)k * dff}, dff, a);
                        a0 = a[0];
                    }
                    if (v0) ot = fmaf(s_w[k], a0, ot);
                    if (v1) ot = fmaf(s_w[k + 1], a1, ot);
                }
            } else {
                const float* r = W.w3 + (uint64_t)i * dff;
                float a[1];
                if (!(i == gw && pf_for == kPfW3)) load_block<1, 12>(pf1, {r}, dff, lane4);
                dots_from<1, 12>(pf1, {r}, {sh}, dff, a);
                ot = a[0];
            }
            if (lane == 0) p.x[i] = __ldcg(p.x + i) + ot;
        }
        {
            const bool on = l + 1 < p.n_layers && gw < npair;
            const float* r0 = p.layers[on ? l + 1 : l].wqkv + (uint64_t)(2 * (on ? gw : 0)) * d;
            load_block<2, 12>(pf, {r0, r0 + d}, on ? d : 0, lane4);
            pf_for = on ? kPfQkv : kPfNone;
        }
        if (!grid_sync(bar, target, err, &s_ok)) return;
    }
}

namespace {

// A step launch holds every SM for its whole duration, and two of them
// resident at once could each wait at a barrier for CTAs the other one keeps
// out.  Launches from different streams (forward slots) are therefore chained
// on each device through one event: each waits for the previous one's end.
constexpr int kMaxDevices = 64;
std::mutex g_step_mu;
cudaEvent_t g_step_done[kMaxDevices];

template <int G>
int launch_step(const TGFwdStepParams& p, size_t smem, uint32_t grid, cudaStream_t st) {
    void* args[] = {const_cast<TGFwdStepParams*>(&p)};
    int dev = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_step_mu);
    cudaEvent_t& done = g_step_done[dev];
    if (!done && (e = cudaEventCreateWithFlags(&done, cudaEventDisableTiming)) != cudaSuccess) {
        done = nullptr;
        return (int)e;
    }
    if ((e = cudaStreamWaitEvent(st, done, 0)) != cudaSuccess) return (int)e;
    e = cudaLaunchCooperativeKernel((const void*)decode_step_kernel<G>, dim3(grid),
                                    dim3(kThreads), args, smem, st);
    if (e == cudaErrorCooperativeLaunchTooLarge) {
        (void)cudaGetLastError();
        return -1;                             // refused before anything ran
    }
    if (e != cudaSuccess) return (int)e;
    return (int)cudaEventRecord(done, st);
}

template <int G>
int step_grid(size_t smem, uint32_t* grid) {
    int dev = 0, sms = 0, per = 0, coop = 0;
    cudaError_t e;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return (int)e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return (int)e;
    if ((e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev)) != cudaSuccess)
        return (int)e;
    if (!coop) return -1;
    if (smem > 48 * 1024 &&
        (e = cudaFuncSetAttribute(decode_step_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem)) != cudaSuccess)
        return (int)e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, decode_step_kernel<G>, kThreads,
                                                           smem)) != cudaSuccess)
        return (int)e;
    if (per < 1) return -1;
    *grid = (uint32_t)sms;                 // one CTA per SM
    return 0;
}

}  // namespace

extern "C" int tgkv_fwd_step_supported(uint32_t d, uint32_t n_heads, uint32_t n_kv_heads,
                                       uint32_t head_dim, uint32_t dff, uint32_t ne, uint32_t na) {
    if (!n_kv_heads || n_heads % n_kv_heads) return 0;
    const uint32_t g = n_heads / n_kv_heads;
    if (g != 1 && g != 2 && g != 3 && g != 4 && g != 8) return 0;
    if (head_dim != 32 && head_dim != 64 && head_dim != 128) return 0;
    if (d % 4 || dff % 4 || ne > 16 || na > 8 || (ne && (na == 0 || na > ne))) return 0;
    if (n_heads > kTgStepStateWords - 2) return 0;
    return tgkv_fwd_step_smem(d, n_heads * head_dim, dff, ne, na) <= 160 * 1024;
}

extern "C" size_t tgkv_fwd_step_smem(uint32_t d, uint32_t q_dim, uint32_t dff, uint32_t ne,
                                     uint32_t na) {
    const size_t sx = d > q_dim ? d : q_dim;
    return (sx + (size_t)(ne ? na : 1) * dff) * 4;
}

extern "C" size_t tgkv_fwd_step_part_floats(uint32_t n_heads, uint32_t n_kv_heads,
                                            uint32_t head_dim) {
    (void)n_kv_heads;
    return (size_t)n_heads * kTgStepMaxTasks * (head_dim + 4);
}

extern "C" int tgkv_fwd_decode_step(const TGFwdStepParams* p, void* stream) {
    if (!p || !p->n_kv_heads || p->n_heads % p->n_kv_heads || p->pos >= p->max_seq)
        return (int)cudaErrorInvalidValue;
    const uint32_t g = p->n_heads / p->n_kv_heads;
    const size_t smem = tgkv_fwd_step_smem(p->d, p->n_heads * p->head_dim, p->dff, p->ne, p->na);
    if (p->sx_floats != (smem / 4 - (size_t)(p->ne ? p->na : 1) * p->dff))
        return (int)cudaErrorInvalidValue;
    cudaStream_t st = (cudaStream_t)stream;
    uint32_t grid = 0;
    int e;
    switch (g) {
#define TGKV_STEP_CASE(GV)                                       \
    case GV:                                                     \
        if ((e = step_grid<GV>(smem, &grid))) return e;          \
        return launch_step<GV>(*p, smem, grid, st);
        TGKV_STEP_CASE(1)
        TGKV_STEP_CASE(2)
        TGKV_STEP_CASE(3)
        TGKV_STEP_CASE(4)
        TGKV_STEP_CASE(8)
#undef TGKV_STEP_CASE
    default:
        return (int)cudaErrorInvalidValue;
    }
}
