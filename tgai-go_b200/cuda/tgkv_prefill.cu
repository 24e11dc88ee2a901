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
// Work split.  A row block is 128 "rows" -- 128/G tokens x the G query heads
// of one KV head -- and its KV tiles of 128 positions are divided among the
// n_split CTAs of one thread-block cluster, so that a turn's few row blocks
// still fill the GPU.  Each CTA keeps an unnormalised partial (O, running max
// m, sum l) per row; after a cluster barrier every CTA merges a slice of the
// rows from all partials over distributed shared memory and writes them out.
//
// Inside a CTA:
//   warp 4       TMA: K and V tiles (2 x 64-column boxes each, 128-byte
//                swizzled) into separate 2-stage rings;
//   warp 5       allocates 512 TMEM columns; one lane issues the MMAs:
//                S = Q K^T into one of two S buffers (q split into bf16 hi +
//                lo parts so the scores keep ~16 mantissa bits), and
//                O += P V with P read from TMEM (hi + lo) and V as an
//                MN-major operand.  S for tile j+2 is issued as soon as the
//                PV of tile j has released its buffer, so the tensor core
//                works on the next tile while the softmax runs on this one;
//   warps 0-3    one query row per thread (= one TMEM lane): read S, mask the
//                causal diagonal, online softmax in the log2 domain with lazy
//                rescale, write P (bf16 hi, lo) over S in place; at the end
//                read O and publish the partial.
// TMEM columns: S/P buffer 0 [0,128), S/P buffer 1 [128,256), O [256,384).
// Every mbarrier wait is bounded; a timeout sets the error word and the CTA
// still reaches both cluster barriers.

#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include "tgkv_launch.h"
#include "tgkv_ptx.cuh"

namespace tgkv {
namespace prefill {

constexpr int kRows = 128;                   // query rows per CTA (TMEM lanes)
constexpr int kPos = 128;                    // positions per KV tile
constexpr int kHD = 128;                     // head dim
constexpr int kThreads = 192;                // warps 0-3 softmax, 4 TMA, 5 MMA
constexpr uint32_t kBlockBytes = 16384;      // 128 rows x 64 bf16: one swizzled box
constexpr uint32_t kTileBytes = 2 * kBlockBytes;
constexpr uint32_t kMaxSplit = 8;

// shared memory, offsets from a 1024-aligned base
constexpr uint32_t OFF_QHI = 0;
constexpr uint32_t OFF_QLO = kTileBytes;
constexpr uint32_t OFF_K = 2 * kTileBytes;   // [2] K tiles
constexpr uint32_t OFF_V = 4 * kTileBytes;   // [2] V tiles
constexpr uint32_t OFF_BAR = 6 * kTileBytes;
constexpr uint32_t OFF_TSLOT = OFF_BAR + 32 * 8;
constexpr uint32_t OFF_ML = OFF_BAR + 512;   // m[128], l[128] of this CTA's partial
constexpr uint32_t SMEM_USED = OFF_ML + 2 * kRows * 4;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;   // slack to align the base
// Once the last MMA is done the Q region holds this CTA's partial O: fp32
// [128 rows][32 float4 groups], group g of row r stored at g ^ (r % 32).
constexpr uint32_t OFF_OPART = 0;
static_assert(kRows * kHD * 4 <= 2 * kTileBytes, "partial O must fit the Q region");

// barriers (uint64 each) at OFF_BAR
constexpr int B_KFULL = 0;     // [2]
constexpr int B_KEMPTY = 2;    // [2]
constexpr int B_VFULL = 4;     // [2]
constexpr int B_VEMPTY = 6;    // [2]
constexpr int B_SFULL = 8;     // [2] S of the tile in buffer s is in TMEM
constexpr int B_PFULL = 10;    // [2] P of buffer s written (128 arrivals)
constexpr int B_PVDONE = 12;   // one phase per tile: its PV is complete
constexpr int B_QREADY = 13;
constexpr int B_OREADY = 14;   // every MMA of the CTA is complete

constexpr uint32_t TM_SP = 0, TM_O = 256, TM_COLS = 512;

constexpr int kErrTimeout = 3;

// Byte offset of element (row, d) of a 128 x 128 bf16 tile stored as two
// K-major 128-byte-swizzled blocks (head dims 0-63 | 64-127): rows of 128
// bytes, 16-byte chunk c of row r at chunk c ^ (r % 8) -- the layout TMA
// writes with CU_TENSOR_MAP_SWIZZLE_128B and UMMA reads with layout type 2.
__device__ __forceinline__ uint32_t swz_offset(int row, int d) {
    const int blk = d >> 6, dd = d & 63, chunk = dd >> 3, e = dd & 7;
    return (uint32_t)(blk * (int)kBlockBytes + row * 128 + ((chunk ^ (row & 7)) << 4) + e * 2);
}

__device__ __forceinline__ uint32_t opart_offset(uint32_t row, uint32_t grp) {
    return OFF_OPART + row * 512u + ((grp ^ (row & 31u)) << 4);
}

__device__ __forceinline__ float bf16_lo_f(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi_f(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

__device__ __forceinline__ void fail(const TGKvPrefillParams& p) { atomicExch(p.err, kErrTimeout); }

// The MMAs of S(j) = (Q_hi + Q_lo) K_j^T into S buffer j % 2, after K_j has
// landed; commits release the K stage and signal the softmax.
__device__ __forceinline__ bool issue_s(uint64_t* bar, uint32_t sbase, uint32_t tmem, int j) {
    const int s = j & 1;
    if (!mbar_wait(&bar[B_KFULL + s], (uint32_t)(j >> 1) & 1u)) return false;
    tc_fence_after();
    constexpr uint32_t id_qk = umma_idesc_bf16(kRows, kPos, 0, 0);
    const uint32_t kb = sbase + OFF_K + (uint32_t)s * kTileBytes;
    const uint32_t d = tmem + TM_SP + (uint32_t)s * 128u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t qb = sbase + (h ? OFF_QLO : OFF_QHI);
#pragma unroll
        for (int blk = 0; blk < 2; ++blk)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint32_t o = (uint32_t)blk * kBlockBytes + (uint32_t)ks * 32u;
                umma_ss(d, umma_desc_sw128(qb + o, 16, 1024), umma_desc_sw128(kb + o, 16, 1024),
                        id_qk, (h | blk | ks) != 0);
            }
    }
    umma_commit(&bar[B_KEMPTY + s]);
    umma_commit(&bar[B_SFULL + s]);
    return true;
}

__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ TGKvPrefillParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(base);
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + OFF_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(base + OFF_TSLOT);
    float* sm_m = reinterpret_cast<float*>(base + OFF_ML);
    float* sm_l = sm_m + kRows;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t G = p.n_heads / p.n_kv_heads;
    const uint32_t lg = (uint32_t)(__ffs((int)G) - 1);       // G is a power of two
    const uint32_t kvh = blockIdx.y;
    const uint32_t t0 = blockIdx.x * ((uint32_t)kRows >> lg);
    const uint32_t t_end = min(t0 + ((uint32_t)kRows >> lg), p.n_q);
    const uint32_t prow_min = p.pos0 + t0;                  // first row's last position
    const uint32_t pmax = p.pos0 + t_end - 1;               // last row's last position
    const int ntx = (int)(pmax / kPos) + 1;                 // KV tiles of this row block
    const uint32_t ns = p.n_split;
    const uint32_t z = cluster_ctarank();                   // = blockIdx.z
    const int j0 = (int)(z * (uint32_t)ntx / ns);
    const int nt = (int)((z + 1) * (uint32_t)ntx / ns) - j0;   // this CTA's tiles

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar[B_KFULL + i], 1);
            mbar_init(&bar[B_KEMPTY + i], 1);
            mbar_init(&bar[B_VFULL + i], 1);
            mbar_init(&bar[B_VEMPTY + i], 1);
            mbar_init(&bar[B_SFULL + i], 1);
            mbar_init(&bar[B_PFULL + i], kRows);
        }
        mbar_init(&bar[B_PVDONE], 1);
        mbar_init(&bar[B_QREADY], kRows);
        mbar_init(&bar[B_OREADY], 1);
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
        if (lane == 0 && nt > 0) {
            prefetch_tmap(p.tmap_sw);
            const int x = (int)(kvh * kHD);
            int nk = 0, nv = 0;                 // tiles whose K / V copies are issued
            for (int j = 0; j < nt; ++j) {
                const int s = j & 1;
                const int y = (j0 + j) * kPos;
                const uint32_t ph = (uint32_t)((j >> 1) - 1) & 1u;
                if (j >= 2 && !mbar_wait(&bar[B_KEMPTY + s], ph)) { fail(p); break; }
                unsigned char* kd = base + OFF_K + s * kTileBytes;
                mbar_arrive_expect_tx(&bar[B_KFULL + s], kTileBytes);
                tma_load_3d(kd, p.tmap_sw, x, y, 0, &bar[B_KFULL + s]);
                tma_load_3d(kd + kBlockBytes, p.tmap_sw, x + 64, y, 0, &bar[B_KFULL + s]);
                nk = j + 1;
                if (j >= 2 && !mbar_wait(&bar[B_VEMPTY + s], ph)) { fail(p); break; }
                unsigned char* vd = base + OFF_V + s * kTileBytes;
                mbar_arrive_expect_tx(&bar[B_VFULL + s], kTileBytes);
                tma_load_3d(vd, p.tmap_sw, x, y, 1, &bar[B_VFULL + s]);
                tma_load_3d(vd + kBlockBytes, p.tmap_sw, x + 64, y, 1, &bar[B_VFULL + s]);
                nv = j + 1;
            }
            // every copy this thread issued has landed before the CTA may exit
            // (immediate in a normal run: the MMA warp consumed them all)
            for (int j = nk > 2 ? nk - 2 : 0; j < nk; ++j)
                if (!mbar_wait(&bar[B_KFULL + (j & 1)], (uint32_t)(j >> 1) & 1u)) fail(p);
            for (int j = nv > 2 ? nv - 2 : 0; j < nv; ++j)
                if (!mbar_wait(&bar[B_VFULL + (j & 1)], (uint32_t)(j >> 1) & 1u)) fail(p);
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer
        if (lane == 0 && nt > 0) {
            constexpr uint32_t id_pv = umma_idesc_bf16(kRows, kHD, 0, 1);
            bool ok = mbar_wait(&bar[B_QREADY], 0);
            tc_fence_after();
            if (ok) ok = issue_s(bar, sbase, tmem, 0);
            if (ok && nt > 1) ok = issue_s(bar, sbase, tmem, 1);
            for (int j = 0; ok && j < nt; ++j) {
                const int s = j & 1;
                const uint32_t ph = (uint32_t)(j >> 1) & 1u;
                if (!mbar_wait(&bar[B_PFULL + s], ph) || !mbar_wait(&bar[B_VFULL + s], ph)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // O += (P_hi + P_lo) V over 128 positions in 8 steps of 16.  P of
                // positions 64h + [0,64) sits at columns 64h + [0,32) (hi) and
                // 64h + [32,64) (lo) of the buffer.  V is MN-major: 64-dim
                // blocks 16 KB apart, 8-row groups 1 KB apart.
                const uint32_t vb = sbase + OFF_V + (uint32_t)s * kTileBytes;
                const uint32_t pc = tmem + TM_SP + (uint32_t)s * 128u;
#pragma unroll
                for (int part = 0; part < 2; ++part)
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t a = pc + (uint32_t)(kk >> 2) * 64u + (uint32_t)part * 32u +
                                           (uint32_t)(kk & 3) * 8u;
                        umma_ts(tmem + TM_O, a, umma_desc_sw128(vb + kk * 16 * 128, kBlockBytes, 1024),
                                id_pv, (j | part | kk) != 0);
                    }
                umma_commit(&bar[B_VEMPTY + s]);
                umma_commit(&bar[B_PVDONE]);
                if (j + 2 < nt) {
                    // S(j+2) goes into this buffer once PV(j) has read P out of it
                    if (!mbar_wait(&bar[B_PVDONE], (uint32_t)j & 1u)) { ok = false; break; }
                    tc_fence_after();
                    ok = issue_s(bar, sbase, tmem, j + 2);
                }
            }
            if (!ok) fail(p);
            umma_commit(&bar[B_OREADY]);
            if (!mbar_wait(&bar[B_OREADY], 0)) fail(p);
        }
    } else {
        // ---------------- softmax / epilogue: thread = query row = TMEM lane
        const int r = tid;
        const uint32_t tk = t0 + ((uint32_t)r >> lg);
        const uint32_t prow = min(p.pos0 + tk, pmax);
        // q block * scale * log2(e) -> bf16 hi + lo, swizzled into smem.  The
        // 128 threads walk the block's 4096 float4s coalesced: float4 f is
        // row f / 32, head dims 4 (f % 32) .. +3.
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            float4 x[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t f = (uint32_t)(b * 16 + i) * 128u + (uint32_t)r;
                const uint32_t row = f >> 5, c4 = f & 31u;
                const uint32_t ttk = t0 + (row >> lg);
                const uint32_t thq = (kvh << lg) + (row & (G - 1));
                x[i] = ttk < p.n_q ? *reinterpret_cast<const float4*>(
                                         p.q + ((uint64_t)ttk * p.n_heads + thq) * kHD + c4 * 4)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t f = (uint32_t)(b * 16 + i) * 128u + (uint32_t)r;
                const uint32_t row = f >> 5, c4 = f & 31u;
                const float a0 = x[i].x * p.qscale, a1 = x[i].y * p.qscale;
                const float a2 = x[i].z * p.qscale, a3 = x[i].w * p.qscale;
                const uint32_t h01 = cvt_bf16x2(a0, a1), h23 = cvt_bf16x2(a2, a3);
                const uint32_t l01 = cvt_bf16x2(a0 - bf16_lo_f(h01), a1 - bf16_hi_f(h01));
                const uint32_t l23 = cvt_bf16x2(a2 - bf16_lo_f(h23), a3 - bf16_hi_f(h23));
                const uint32_t off = swz_offset((int)row, (int)(c4 * 4));
                *reinterpret_cast<uint2*>(base + OFF_QHI + off) = make_uint2(h01, h23);
                *reinterpret_cast<uint2*>(base + OFF_QLO + off) = make_uint2(l01, l23);
            }
        }
        fence_proxy_async_smem();
        mbar_arrive(&bar[B_QREADY]);

        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            const int s = j & 1;
            const int jt = j0 + j;
            const uint32_t pbase = (uint32_t)jt * kPos;
            const uint32_t sp = tmem + lane_off + TM_SP + (uint32_t)s * 128u;
            const uint32_t ph = (uint32_t)(j >> 1) & 1u;
            // warp-uniform outcome: the TMEM loads below are warp-collective
            if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_SFULL + s], ph))) { ok = false; break; }
            tc_fence_after();
            if (jt == ntx - 1) {
                // Rows past the block's last position hold whatever the cache
                // kept there (truncated turns); P is 0 for them, but 0 * inf
                // would still poison O, so zero those V rows before PV reads them.
                if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_VFULL + s], ph))) { ok = false; break; }
                if (pbase + (uint32_t)r > pmax) {
                    unsigned char* vrow = base + OFF_V + s * kTileBytes + r * 128;
#pragma unroll
                    for (int b = 0; b < 2; ++b)
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            *reinterpret_cast<uint4*>(vrow + b * kBlockBytes + c * 16) =
                                make_uint4(0u, 0u, 0u, 0u);
                }
                fence_proxy_async_smem();
            }
            // positions past some row's own one only occur from prow_min on
            const bool diag = pbase + (kPos - 1) > prow_min;

            // pass 1: row maximum
            float tm = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t v[32];
                tmem_ld32(sp + c * 32, v);
                tmem_wait_ld(v);
                if (diag) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (pbase + (uint32_t)(c * 32 + i) <= prow) tm = fmaxf(tm, __uint_as_float(v[i]));
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) tm = fmaxf(tm, __uint_as_float(v[i]));
                }
            }
            // lazy rescale: the running maximum moves only when exceeded by > 2^8
            float alpha = 1.f;
            const bool grow = tm > m + 8.f;
            if (grow) {
                alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - tm);
                m = tm;
                l *= alpha;
            }
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
                // O holds tiles < j: wait for PV(j-1), then scale it
                if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_PVDONE], (uint32_t)(j - 1) & 1u))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t v[32];
                    tmem_ld32(tmem + lane_off + TM_O + c * 32, v);
                    tmem_wait_ld(v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                    tmem_st32(tmem + lane_off + TM_O + c * 32, v);
                }
            }
            // pass 2: P = 2^(s - m) as bf16 hi + lo over S, 64 positions at a time
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint32_t va[32], vb[32], phi[32], plo[32];
                tmem_ld32(sp + hh * 64, va);
                tmem_ld32(sp + hh * 64 + 32, vb);
                tmem_wait_ld(va, vb);
#pragma unroll
                for (int cc = 0; cc < 32; ++cc) {
                    const int i0 = 2 * cc;
                    const float s0 = __uint_as_float(i0 < 32 ? va[i0] : vb[i0 - 32]);
                    const float s1 = __uint_as_float(i0 + 1 < 32 ? va[i0 + 1] : vb[i0 + 1 - 32]);
                    float p0 = ex2_approx(s0 - m), p1 = ex2_approx(s1 - m);
                    if (diag) {
                        const uint32_t pos = pbase + (uint32_t)(hh * 64 + i0);
                        p0 = pos <= prow ? p0 : 0.f;
                        p1 = pos + 1 <= prow ? p1 : 0.f;
                    }
                    l += p0 + p1;
                    const uint32_t h = cvt_bf16x2(p0, p1);
                    phi[cc] = h;
                    plo[cc] = cvt_bf16x2(p0 - bf16_lo_f(h), p1 - bf16_hi_f(h));
                }
                tmem_st32(sp + hh * 64, phi);
                tmem_st32(sp + hh * 64 + 32, plo);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bar[B_PFULL + s]);
        }
        // partial of this CTA: O (after every MMA is done) -> the Q region
        if (ok && nt > 0 && !__all_sync(0xffffffffu, mbar_wait(&bar[B_OREADY], 0))) ok = false;
        tc_fence_after();
        if (!ok && lane == 0) fail(p);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            if (nt > 0) {
                tmem_ld32(tmem + lane_off + TM_O + c * 32, v);
                tmem_wait_ld(v);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0u;
            }
#pragma unroll
            for (int g = 0; g < 8; ++g)
                *reinterpret_cast<uint4*>(base + opart_offset((uint32_t)r, (uint32_t)(c * 8 + g))) =
                    make_uint4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
        }
        sm_m[r] = m;
        sm_l[r] = l;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, TM_COLS);
    }
    __syncwarp();
    cluster_sync();

    // ---------------- merge: this CTA finishes rows [z*128/ns, (z+1)*128/ns)
    // from the partials of every CTA of the cluster; one item = one row's
    // float4 group, a warp covers a row (512 contiguous bytes out).
    {
        const uint32_t rb0 = z * (uint32_t)kRows / ns, rb1 = (z + 1) * (uint32_t)kRows / ns;
        const uint32_t items = (rb1 - rb0) * 32u;
        for (uint32_t it = (uint32_t)tid; it < items; it += kThreads) {
            const uint32_t row = rb0 + (it >> 5), grp = it & 31u;
            const uint32_t ttk = t0 + (row >> lg);
            if (ttk >= p.n_q) continue;
            const uint32_t thq = (kvh << lg) + (row & (G - 1));
            float mz[kMaxSplit], lz[kMaxSplit];
            float M = -INFINITY;
#pragma unroll
            for (uint32_t zz = 0; zz < kMaxSplit; ++zz)
                if (zz < ns) {
                    mz[zz] = dsmem_ld_f32(dsmem_map(sbase + OFF_ML + row * 4u, zz));
                    lz[zz] = dsmem_ld_f32(dsmem_map(sbase + OFF_ML + (kRows + row) * 4u, zz));
                    M = fmaxf(M, mz[zz]);
                }
            float L = 0.f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (uint32_t zz = 0; zz < kMaxSplit; ++zz)
                if (zz < ns && mz[zz] != -INFINITY) {
                    const float w = ex2_approx(mz[zz] - M);
                    L += w * lz[zz];
                    const float4 o = dsmem_ld_f4(dsmem_map(sbase + opart_offset(row, grp), zz));
                    acc.x += w * o.x;
                    acc.y += w * o.y;
                    acc.z += w * o.z;
                    acc.w += w * o.w;
                }
            const float inv = L > 0.f ? 1.f / L : 0.f;
            *reinterpret_cast<float4*>(p.out + ((uint64_t)ttk * p.n_heads + thq) * kHD + grp * 4) =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
    }
    __syncwarp();
    cluster_sync();      // peers read this CTA's shared memory until here
}

}  // namespace prefill
}  // namespace tgkv

extern "C" int tgkv_launch_prefill(const TGKvPrefillParams* p, void* stream) {
    using namespace tgkv::prefill;
    const uint32_t G = p->n_heads / p->n_kv_heads;
    if (p->n_q == 0) return 0;
    if (!(G == 1 || G == 2 || G == 4 || G == 8) || p->n_heads % p->n_kv_heads ||
        p->n_split == 0 || p->n_split > kMaxSplit)
        return (int)cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    static bool configured[64];
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 SMEM_BYTES);
        if (e != cudaSuccess) return (int)e;
        configured[dev] = true;
    }
    const uint32_t toks = kRows / G;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((p->n_q + toks - 1) / toks, p->n_kv_heads, p->n_split);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = p->n_split;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, prefill_kernel, *p);
    return (int)e;
}

// Clusters of n_split prefill CTAs that fit on the current device at once
// (0 if the query fails); the planner sizes the split with it.
extern "C" uint32_t tgkv_prefill_max_clusters(uint32_t n_split) {
    using namespace tgkv::prefill;
    if (n_split == 0 || n_split > kMaxSplit) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    static uint32_t cache[64][kMaxSplit + 1];
    if (cache[dev][n_split]) return cache[dev][n_split];
    if (cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BYTES) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, n_split);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = n_split;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, prefill_kernel, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return 0;
    }
    cache[dev][n_split] = (uint32_t)n;
    return (uint32_t)n;
}
