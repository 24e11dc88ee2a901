// tgkv_prefill.cu -- tensor-core (tcgen05) causal attention of a block of query
// rows over a bf16 KV cache with head_dim 128: the suffix attention of an LCP
// re-append (a turn's 64-512 new tokens attending the whole cache), the one
// place on the KV-cache path that is a dense contraction.
//
// Semantics are those of the decode kernel (src/tgai_engine.c:3943-4011):
// q head h reads KV head h*nkv/nh, scores scaled by 1/sqrt(head_dim) (times
// the YaRN temperature if set), query row t at position pos0 + t sees
// positions [0, pos0 + t].
//
// One CTA owns 128 "rows" -- 128/G tokens x the G query heads of one KV head --
// and walks the cache in tiles of 128 positions:
//   warp 4       TMA: K and V tiles, 2 x 64-column boxes each, 128-byte
//                swizzled, into a 2-stage ring;
//   warp 5       allocates 512 TMEM columns; one lane issues the MMAs:
//                S = Q K^T into TMEM (q split into bf16 hi + lo parts so the
//                scores keep ~16 mantissa bits), then O += P V with P read
//                from TMEM (also hi + lo) and V as an MN-major operand;
//   warps 0-3    one query row per thread (= one TMEM lane): read S, mask,
//                online softmax in the log2 domain with lazy rescale, write P
//                into TMEM; at the end read O and write the output row.
// TMEM columns: S [0,128) fp32, O [128,256) fp32, P_hi [256,320) and
// P_lo [320,384) bf16 pairs.  Every mbarrier wait is bounded.

#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include "tgkv_launch.h"
#include "tgkv_ptx.cuh"

namespace tgkv {
namespace prefill {

constexpr int kRows = 128;          // query rows per CTA (TMEM lanes)
constexpr int kPos = 128;           // positions per KV tile
constexpr int kHD = 128;            // head dim
constexpr int kThreads = 192;       // warps 0-3 softmax, 4 TMA, 5 MMA
constexpr int kBlockBytes = 16384;  // 128 rows x 64 bf16, one swizzled box

// shared memory (offsets from a 1024-aligned base)
constexpr uint32_t OFF_QHI = 0;                 // 2 blocks (head dims 0-63, 64-127)
constexpr uint32_t OFF_QLO = 2 * kBlockBytes;
constexpr uint32_t OFF_STAGE = 4 * kBlockBytes; // per stage: K0 K1 V0 V1
constexpr uint32_t STAGE_BYTES = 4 * kBlockBytes;
constexpr int kStages = 2;
constexpr uint32_t OFF_BAR = OFF_STAGE + kStages * STAGE_BYTES;
constexpr uint32_t SMEM_USED = OFF_BAR + 256;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;   // slack to align the base

// barriers (uint64 each) at OFF_BAR
constexpr int B_KV_FULL = 0;    // [2]
constexpr int B_KV_EMPTY = 2;   // [2]
constexpr int B_S_FULL = 4;
constexpr int B_P_FULL = 5;
constexpr int B_PV_DONE = 6;
constexpr int B_Q_READY = 7;
constexpr int B_MMA_DONE = 8;
constexpr uint32_t OFF_TSLOT = OFF_BAR + 16 * 8;
constexpr uint32_t OFF_ABORT = OFF_TSLOT + 8;

constexpr uint32_t TM_S = 0, TM_O = 128, TM_PHI = 256, TM_PLO = 320, TM_COLS = 512;

constexpr int kErrTimeout = 3;

// Byte offset of element (row, d) of a 128 x 128 bf16 tile stored as two
// K-major 128-byte-swizzled blocks (head dims 0-63 | 64-127): rows of 128
// bytes, 16-byte chunk c of row r at chunk c ^ (r % 8) -- the layout TMA
// writes with CU_TENSOR_MAP_SWIZZLE_128B and UMMA reads with layout type 2.
__device__ __forceinline__ uint32_t swz_offset(int row, int d) {
    const int blk = d >> 6, dd = d & 63, chunk = dd >> 3, e = dd & 7;
    return (uint32_t)(blk * kBlockBytes + row * 128 + ((chunk ^ (row & 7)) << 4) + e * 2);
}

__device__ __forceinline__ void set_abort(const TGKvPrefillParams& p, volatile int* flag) {
    atomicExch(p.err, kErrTimeout);
    *flag = 1;
}

__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ TGKvPrefillParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(base);
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + OFF_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(base + OFF_TSLOT);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(base + OFF_ABORT);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = p.n_heads / p.n_kv_heads;
    const uint32_t toks = kRows / G;
    const uint32_t kvh = blockIdx.y;
    const uint32_t t0 = blockIdx.x * toks;
    const uint32_t t_end = min(t0 + toks, p.n_q);
    const uint32_t pmax = p.pos0 + t_end - 1;
    const int ntiles = (int)((pmax + kPos) / kPos);

    if (tid == 0) {
        mbar_init(&bar[B_KV_FULL + 0], 1);
        mbar_init(&bar[B_KV_FULL + 1], 1);
        mbar_init(&bar[B_KV_EMPTY + 0], 1);
        mbar_init(&bar[B_KV_EMPTY + 1], 1);
        mbar_init(&bar[B_S_FULL], 1);
        mbar_init(&bar[B_P_FULL], 128);
        mbar_init(&bar[B_PV_DONE], 1);
        mbar_init(&bar[B_Q_READY], 128);
        mbar_init(&bar[B_MMA_DONE], 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 5) {
        tmem_alloc(tslot, TM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 4) {
        // ---------------- TMA producer
        if (lane == 0) {
            const int x = (int)(kvh * kHD);
            for (int j = 0; j < ntiles; ++j) {
                const int s = j & 1;
                if (j >= 2 && !mbar_wait(&bar[B_KV_EMPTY + s], ((j >> 1) - 1) & 1)) {
                    set_abort(p, abort_flag);
                    break;
                }
                unsigned char* st = base + OFF_STAGE + s * STAGE_BYTES;
                uint64_t* full = &bar[B_KV_FULL + s];
                mbar_arrive_expect_tx(full, STAGE_BYTES);
                const int y = j * kPos;
                tma_load_3d(st + 0 * kBlockBytes, p.tmap_sw, x, y, 0, full);
                tma_load_3d(st + 1 * kBlockBytes, p.tmap_sw, x + 64, y, 0, full);
                tma_load_3d(st + 2 * kBlockBytes, p.tmap_sw, x, y, 1, full);
                tma_load_3d(st + 3 * kBlockBytes, p.tmap_sw, x + 64, y, 1, full);
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer
        if (lane == 0) {
            const uint32_t id_qk = umma_idesc_bf16(kRows, kPos, 0, 0);
            const uint32_t id_pv = umma_idesc_bf16(kRows, kHD, 0, 1);
            bool ok = mbar_wait(&bar[B_Q_READY], 0);
            if (!ok) set_abort(p, abort_flag);
            tc_fence_after();
            for (int j = 0; ok && j < ntiles; ++j) {
                const int s = j & 1;
                if (!mbar_wait(&bar[B_KV_FULL + s], (j >> 1) & 1)) {
                    set_abort(p, abort_flag);
                    break;
                }
                tc_fence_after();
                const uint32_t st = sbase + OFF_STAGE + s * STAGE_BYTES;
                // S = (Q_hi + Q_lo) K^T over 128 head dims in 8 steps of 16
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t qb = sbase + (h ? OFF_QLO : OFF_QHI);
#pragma unroll
                    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            const uint64_t ad = umma_desc_sw128(qb + kb * kBlockBytes + ks * 32, 16, 1024);
                            const uint64_t bd = umma_desc_sw128(st + kb * kBlockBytes + ks * 32, 16, 1024);
                            umma_ss(tmem + TM_S, ad, bd, id_qk, (h | kb | ks) != 0);
                        }
                }
                umma_commit(&bar[B_S_FULL]);
                if (!mbar_wait(&bar[B_P_FULL], j & 1)) {
                    set_abort(p, abort_flag);
                    break;
                }
                tc_fence_after();
                // O += (P_hi + P_lo) V over 128 positions in 8 steps of 16;
                // V is MN-major: 64-dim blocks 16 KB apart, 8-row groups 1 KB apart
                const uint32_t vb = st + 2 * kBlockBytes;
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t bd = umma_desc_sw128(vb + kk * 16 * 128, kBlockBytes, 1024);
                        umma_ts(tmem + TM_O, tmem + (h ? TM_PLO : TM_PHI) + kk * 8, bd, id_pv,
                                (j | h | kk) != 0);
                    }
                umma_commit(&bar[B_KV_EMPTY + s]);
            }
            umma_commit(&bar[B_PV_DONE]);
            umma_commit(&bar[B_MMA_DONE]);
            if (!mbar_wait(&bar[B_MMA_DONE], 0)) set_abort(p, abort_flag);
        }
    } else {
        // ---------------- softmax / epilogue: thread = query row = TMEM lane
        const int r = tid;
        const uint32_t tk = t0 + (uint32_t)r / G;
        const uint32_t hq = kvh * G + (uint32_t)r % G;
        const bool valid = tk < p.n_q;
        const uint32_t prow = p.pos0 + tk;
        const float* qrow = p.q + ((uint64_t)tk * p.n_heads + hq) * kHD;
        // q * scale * log2(e) split into bf16 hi + lo, swizzled into smem
#pragma unroll 4
        for (int c = 0; c < 16; ++c) {
            float x[8];
            if (valid) {
                const float4 a = *reinterpret_cast<const float4*>(qrow + c * 8);
                const float4 b = *reinterpret_cast<const float4*>(qrow + c * 8 + 4);
                x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
                x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = 0.f;
            }
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float a0 = x[2 * e] * p.qscale, a1 = x[2 * e + 1] * p.qscale;
                hi[e] = pack_bf16x2(a0, a1);
                lo[e] = pack_bf16x2(a0 - bf16_bits_to_f32((uint16_t)(hi[e] & 0xffffu)),
                                    a1 - bf16_bits_to_f32((uint16_t)(hi[e] >> 16)));
            }
            const uint32_t off = swz_offset(r, c * 8);
            *reinterpret_cast<uint4*>(base + OFF_QHI + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(base + OFF_QLO + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&bar[B_Q_READY]);

        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < ntiles; ++j) {
            // warp-uniform outcome: the TMEM loads below are warp-collective
            if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_S_FULL], j & 1))) {
                if (lane == 0) set_abort(p, abort_flag);
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t pbase = (uint32_t)j * kPos;
            // pass 1: masked row maximum
            float tm = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_off + TM_S + c * 32, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const uint32_t pos = pbase + c * 32 + i;
                    if (valid && pos <= prow) tm = fmaxf(tm, __uint_as_float(v[i]));
                }
            }
            // lazy rescale: the running maximum moves only when exceeded by > 2^8
            float alpha = 1.f;
            const bool grow = tm > m + 8.f;
            if (grow) {
                alpha = (m == -INFINITY) ? 0.f : exp2f(m - tm);
                m = tm;
                l *= alpha;
            }
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t v[32];
                    tmem_ld32(tmem + lane_off + TM_O + c * 32, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                    tmem_st32(tmem + lane_off + TM_O + c * 32, v);
                }
            }
            // pass 2: P = exp2(s - m) as bf16 hi + lo pairs
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
                uint32_t va[32], vb[32], ph[32], pl[32];
                tmem_ld32(tmem + lane_off + TM_S + c2 * 64, va);
                tmem_ld32(tmem + lane_off + TM_S + c2 * 64 + 32, vb);
                tmem_wait_ld();
#pragma unroll
                for (int cc = 0; cc < 32; ++cc) {
                    const int i0 = 2 * cc;
                    const uint32_t pos0 = pbase + c2 * 64 + i0;
                    const float s0 = __uint_as_float(i0 < 32 ? va[i0] : vb[i0 - 32]);
                    const float s1 = __uint_as_float(i0 + 1 < 32 ? va[i0 + 1] : vb[i0 + 1 - 32]);
                    const float p0 = (valid && pos0 <= prow) ? exp2f(s0 - m) : 0.f;
                    const float p1 = (valid && pos0 + 1 <= prow) ? exp2f(s1 - m) : 0.f;
                    l += p0 + p1;
                    ph[cc] = pack_bf16x2(p0, p1);
                    pl[cc] = pack_bf16x2(p0 - bf16_bits_to_f32((uint16_t)(ph[cc] & 0xffffu)),
                                         p1 - bf16_bits_to_f32((uint16_t)(ph[cc] >> 16)));
                }
                tmem_st32(tmem + lane_off + TM_PHI + c2 * 32, ph);
                tmem_st32(tmem + lane_off + TM_PLO + c2 * 32, pl);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bar[B_P_FULL]);
        }
        // epilogue: O / l
        if (ok && !__all_sync(0xffffffffu, mbar_wait(&bar[B_PV_DONE], 0)) && lane == 0)
            set_abort(p, abort_flag);
        tc_fence_after();
        const float inv = (l > 0.f) ? 1.f / l : 0.f;
        float* orow = p.out + ((uint64_t)tk * p.n_heads + hq) * kHD;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_off + TM_O + c * 32, v);
            tmem_wait_ld();
            if (valid) {
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    *reinterpret_cast<float4*>(orow + c * 32 + i) =
                        make_float4(__uint_as_float(v[i]) * inv, __uint_as_float(v[i + 1]) * inv,
                                    __uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, TM_COLS);
    }
}

}  // namespace prefill
}  // namespace tgkv

extern "C" int tgkv_launch_prefill(const TGKvPrefillParams* p, void* stream) {
    using namespace tgkv::prefill;
    const uint32_t G = p->n_heads / p->n_kv_heads;
    if (p->n_q == 0) return 0;
    if (!(G == 1 || G == 2 || G == 4 || G == 8) || p->n_heads % p->n_kv_heads)
        return (int)cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(prefill_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return (int)e;
        configured = true;
    }
    const uint32_t toks = kRows / G;
    dim3 grid((p->n_q + toks - 1) / toks, p->n_kv_heads);
    prefill_kernel<<<grid, kThreads, SMEM_BYTES, (cudaStream_t)stream>>>(*p);
    return (int)cudaGetLastError();
}
