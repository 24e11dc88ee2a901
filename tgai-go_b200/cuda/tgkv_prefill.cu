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
// m, sum l) per row.  At the end each CTA finishes a slice of the rows: every
// CTA copies its partial rows into the staging area of the CTA that finishes
// them (shared-to-peer-shared bulk copies inside the cluster), and that CTA
// merges them from its own shared memory and writes the output rows.
//
// Inside a CTA (320 threads):
//   warps 0-7    softmax: row r = TMEM lane r is shared by warps r/32 and
//                r/32 + 4, which take positions [0,64) and [64,128) of each
//                tile; they exchange the tile's row maximum through shared
//                memory.  First they write q * scale * log2(e) into TMEM as
//                bf16 hi + lo parts (so the scores keep ~16 mantissa bits);
//                per tile: read S, mask the causal diagonal, online softmax
//                in the log2 domain with lazy rescale, write P (bf16 hi, lo)
//                over S in place; at the end read O and publish the partial;
//   warp 8       TMA: the q block (4 swizzled boxes of 32 head dims, rows past
//                n_q zero-filled) into the staging area, then K and V tiles
//                (2 x 64-column boxes each, 128-byte swizzled) into separate
//                2-stage rings;
//   warp 9       allocates the 512 TMEM columns; one lane issues the MMAs,
//                both with the A operand in TMEM: S = (Q_hi + Q_lo) K^T into
//                one of two S buffers, O += (P_hi + P_lo) V with V as an
//                MN-major operand.  S for tile j+2 is issued as soon as the
//                PV of tile j has released its buffer, so the tensor core
//                works on the next tile while the softmax runs on this one.
// TMEM columns: S/P buffers [0,128) and [128,256), O [256,384), Q [384,512).
// Every mbarrier wait is bounded; a timeout sets the error word and the CTA
// still reaches both cluster barriers.

#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include "tgkv_launch.h"
#include "tgkv_ptx.cuh"

namespace tgkv {
namespace prefill {

constexpr int kRows = 128;                   // query rows per CTA (TMEM lanes)
constexpr int kPos = 128;                    // positions per KV tile
constexpr int kHD = 128;                     // head dim
constexpr int kSoftmaxWarps = 8;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kTmaWarp = 8, kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr uint32_t kBlockBytes = 16384;      // 128 rows x 64 bf16: one swizzled box
constexpr uint32_t kTileBytes = 2 * kBlockBytes;
constexpr uint32_t kMaxSplit = 8;

// shared memory, offsets from a 1024-aligned base
constexpr uint32_t OFF_K = 0;                   // [2] K tiles
constexpr uint32_t OFF_V = 2 * kTileBytes;      // [2] V tiles
// A partial row travels as a 528-byte slot: O (fp32, float4 group g at byte
// 16g) and a 16-byte tail (m, l of column half 0, l of half 1, 0).  The
// 33-chunk stride spreads a warp's 32 consecutive slots over all banks, and
// a warp reading one slot's 32 groups is conflict-free as well.
constexpr uint32_t kSlotBytes = 528;
// Staging area: first the block's q, fp32, as TMA writes it (4 boxes of 32
// head dims x 128 rows, 128-byte rows, 128B swizzle); once every CTA of the
// cluster has moved its q into TMEM, the partial
// rows that the cluster's CTAs copy to this CTA: slot = source rank * (rows
// this CTA finishes) + row.
constexpr uint32_t kStgRows = 136;              // >= n_split * ceil(128 / n_split), n_split <= 8
constexpr uint32_t OFF_STG = 4 * kTileBytes;
constexpr uint32_t STG_BYTES = kStgRows * kSlotBytes;
constexpr uint32_t OFF_BAR = OFF_STG + STG_BYTES;
constexpr uint32_t OFF_TSLOT = OFF_BAR + 32 * 8;
constexpr uint32_t OFF_TMX = OFF_BAR + 512;     // tile maxima [2 parities][2 halves][128]
constexpr uint32_t SMEM_USED = OFF_TMX + 4 * kRows * 4;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;      // slack to align the base
// Once every MMA is done the K and V rings hold this CTA's outgoing partial
// rows (row r at r * kSlotBytes, laid out for its destination slot) and the
// merge weights.
constexpr uint32_t OFF_OUT = OFF_K;
constexpr uint32_t OFF_WTS = OFF_K + kRows * kSlotBytes;
static_assert(STG_BYTES >= kRows * kHD * 4, "q staging must fit");
static_assert(OFF_WTS + kRows * (kMaxSplit + 1) * 4 <= OFF_STG, "outgoing rows and weights fit the rings");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");

// barriers (uint64 each) at OFF_BAR
constexpr int B_KFULL = 0;     // [2]
constexpr int B_KEMPTY = 2;    // [2]
constexpr int B_VFULL = 4;     // [2]
constexpr int B_VEMPTY = 6;    // [2]
constexpr int B_SFULL = 8;     // [2] S of the tile in buffer s is in TMEM
constexpr int B_PFULL = 10;    // [2] P of buffer s written (256 arrivals)
constexpr int B_PVDONE = 12;   // one phase per tile: its PV is complete
constexpr int B_QREADY = 13;   // Q is in TMEM (256 arrivals)
constexpr int B_OREADY = 14;   // every MMA of the CTA is complete
constexpr int B_PUSH = 15;     // the partial rows of every cluster CTA have landed here
constexpr int B_QLOAD = 16;    // the q block has landed in the staging area

constexpr uint32_t TM_SP = 0, TM_O = 256, TM_Q = 384, TM_COLS = 512;

constexpr int kErrTimeout = 3;

// Byte offset of float4 group grp (head dims 4grp .. +3) inside a slot.
__device__ __forceinline__ uint32_t slot_group(uint32_t grp) { return grp << 4; }
// First row that CTA z of the cluster finishes in the merge.
__device__ __forceinline__ uint32_t row_begin(uint32_t z, uint32_t ns) { return z * (uint32_t)kRows / ns; }

__device__ __forceinline__ float bf16_lo_f(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi_f(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

__device__ __forceinline__ void fail(const TGKvPrefillParams& p) { atomicExch(p.err, kErrTimeout); }

// Named barrier of the two softmax warps that share a TMEM lane quarter.
__device__ __forceinline__ void pair_sync(int quarter) {
    asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
}
// Named barrier of the eight softmax warps.
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 5, 256;" ::: "memory"); }

// The MMAs of S(j) = (Q_hi + Q_lo) K_j^T into S buffer j % 2, after K_j has
// landed: A = Q from TMEM (head dims 16ks .. +15 at column 8ks of each
// part), B = the K tile, K-major, 128-byte swizzled.  The commits release
// the K stage and signal the softmax.
__device__ __forceinline__ bool issue_s(uint64_t* bar, uint32_t sbase, uint32_t tmem, int j) {
    const int s = j & 1;
    if (!mbar_wait(&bar[B_KFULL + s], (uint32_t)(j >> 1) & 1u)) return false;
    tc_fence_after();
    constexpr uint32_t id_qk = umma_idesc_bf16(kRows, kPos, 0, 0);
    const uint64_t kd = umma_desc_sw128(sbase + OFF_K + (uint32_t)s * kTileBytes, 16, 1024);
    const uint32_t d = tmem + TM_SP + (uint32_t)s * 128u;
    // step i: part h = i / 8 (Q hi, Q lo), head dims 16 ks .. +15, ks = i % 8;
    // the descriptor's start address field counts 16-byte units.  Unrolled:
    // the tensor core should never wait on the issuing thread.
#pragma unroll
    for (uint32_t i = 0; i < 16; ++i) {
        const uint32_t h = i >> 3, ks = i & 7u;
        const uint32_t bo = (ks >> 2) * kBlockBytes + (ks & 3u) * 32u;
        umma_ts(d, tmem + TM_Q + h * 64u + ks * 8u, kd + (bo >> 4), id_qk, i != 0);
    }
    umma_commit(&bar[B_KEMPTY + s]);
    umma_commit(&bar[B_SFULL + s]);
    return true;
}

// Row maximum over 32 scores (MASK: only the first lim + 1 count), as a tree.
template <bool MASK>
__device__ __forceinline__ float max32(const uint32_t (&v)[32], float tm, int lim) {
    float a[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float x0 = __uint_as_float(v[2 * i]), x1 = __uint_as_float(v[2 * i + 1]);
        if (MASK) {
            x0 = 2 * i <= lim ? x0 : -INFINITY;
            x1 = 2 * i + 1 <= lim ? x1 : -INFINITY;
        }
        a[i] = fmaxf(x0, x1);
    }
#pragma unroll
    for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
        for (int i = 0; i < w; ++i) a[i] = fmaxf(a[i], a[i + w]);
    return fmaxf(tm, a[0]);
}

// P = 2^(s - m) of 32 positions as bf16 pairs: hi words -> ph, the rounding
// residuals (lo) -> pl; the fp32 values accumulate into l2.  MASK: positions
// past lim (chunk-relative) get P = 0.
template <bool MASK>
__device__ __forceinline__ void p32(const uint32_t (&v)[32], float m, int lim, float2& l2,
                                    uint32_t (&ph)[16], uint32_t (&pl)[16]) {
    const float2 nm = make_float2(-m, -m);
    const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        const float2 d = __fadd2_rn(make_float2(__uint_as_float(v[2 * c]), __uint_as_float(v[2 * c + 1])), nm);
        float p0 = ex2_approx(d.x), p1 = ex2_approx(d.y);
        if (MASK) {
            p0 = 2 * c <= lim ? p0 : 0.f;
            p1 = 2 * c + 1 <= lim ? p1 : 0.f;
        }
        const float2 pp = make_float2(p0, p1);
        l2 = __fadd2_rn(l2, pp);
        const uint32_t h = cvt_bf16x2(p0, p1);
        ph[c] = h;
        const float2 res = __ffma2_rn(make_float2(bf16_lo_f(h), bf16_hi_f(h)), neg1, pp);
        pl[c] = cvt_bf16x2(res.x, res.y);
    }
}

// The P of chunk c (32 positions) replaces its S: hi words at columns
// 32c + [0,16), lo words at 32c + [16,32) of the buffer.
__device__ __forceinline__ void p_chunk(const uint32_t (&v)[32], bool mask, float m, int lim,
                                        float2& l2, uint32_t col) {
    uint32_t ph[16], pl[16];
    if (mask) p32<true>(v, m, lim, l2, ph, pl);
    else p32<false>(v, m, lim, l2, ph, pl);
    tmem_st16(col, ph);
    tmem_st16(col + 16, pl);
}

__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ TGKvPrefillParams p) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(base);
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + OFF_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(base + OFF_TSLOT);
    float* sm_tmx = reinterpret_cast<float*>(base + OFF_TMX);

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

    // softmax thread: row r (TMEM lane), column half hf of every tile
    const int r = (warp & 3) * 32 + lane, hf = warp >> 2;
    const uint32_t tk = t0 + ((uint32_t)r >> lg);
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar[B_KFULL + i], 1);
            mbar_init(&bar[B_KEMPTY + i], 1);
            mbar_init(&bar[B_VFULL + i], 1);
            mbar_init(&bar[B_VEMPTY + i], 1);
            mbar_init(&bar[B_SFULL + i], 1);
            mbar_init(&bar[B_PFULL + i], kSoftmaxThreads);
        }
        mbar_init(&bar[B_PVDONE], 1);
        mbar_init(&bar[B_QREADY], kSoftmaxThreads);
        mbar_init(&bar[B_OREADY], 1);
        mbar_init(&bar[B_PUSH], 1);
        mbar_init(&bar[B_QLOAD], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // the partial rows this CTA finishes, from the cluster's other CTAs
        mbar_arrive_expect_tx(&bar[B_PUSH],
                              (ns - 1) * (row_begin(z + 1, ns) - row_begin(z, ns)) * kSlotBytes);
        prefetch_tmap(p.tmap_sw);
        prefetch_tmap(reinterpret_cast<uint64_t>(&p.qmap));
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tslot, TM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    // Launched as a programmatic dependent: everything above overlaps the
    // previous kernel on the stream; nothing below reads global memory
    // before that kernel has completed.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (p.k_new) {
        // The fused append: the row block's new K/V rows -- KV head kvh,
        // positions [pos0, pmax] -- go into the cache (bf16, the append
        // kernel's rounding), shared out over the cluster's CTAs, every
        // thread's loads in flight before its stores.  A cluster barrier then
        // orders them before any CTA's TMA loads.  Other row blocks store the
        // same bytes for the rows they share.
        const uint32_t kv_dim = p.n_kv_heads * kHD;
        const uint64_t vofs = (uint64_t)p.max_seq * kv_dim;
        const uint32_t total = (pmax + 1 - p.pos0) * 32;      // 16-byte chunks of K and V rows
        const uint32_t per = (total + ns - 1) / ns;
        const uint32_t c0 = z * per, c1 = min(total, c0 + per);
        constexpr int kU = 4;
#pragma unroll 1
        for (uint32_t i0 = c0 + tid; i0 < c1; i0 += kThreads * kU) {
            float4 a[kU], b[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const uint32_t i = i0 + u * kThreads;
                if (i < c1) {
                    const uint32_t row = p.pos0 + (i >> 5), part = i & 31, e = (part & 15) * 8;
                    const float* src = (part < 16 ? p.k_new : p.v_new) +
                                       (uint64_t)(row - p.pos0) * kv_dim + kvh * kHD + e;
                    a[u] = *reinterpret_cast<const float4*>(src);
                    b[u] = *reinterpret_cast<const float4*>(src + 4);
                }
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const uint32_t i = i0 + u * kThreads;
                if (i < c1) {
                    const uint32_t row = p.pos0 + (i >> 5), part = i & 31, e = (part & 15) * 8;
                    uint4 w;
                    w.x = pack_bf16x2(a[u].x, a[u].y);
                    w.y = pack_bf16x2(a[u].z, a[u].w);
                    w.z = pack_bf16x2(b[u].x, b[u].y);
                    w.w = pack_bf16x2(b[u].z, b[u].w);
                    *reinterpret_cast<uint4*>(p.kvc + (part < 16 ? 0 : vofs) +
                                              (uint64_t)row * kv_dim + kvh * kHD + e) = w;
                }
            }
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");
        __syncwarp();                 // the .aligned cluster barrier wants whole warps
        cluster_sync();
        asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    // Cluster barrier, first phase: a CTA arrives once its staging area is
    // free (q moved into TMEM) and waits before copying partials to peers.
    if (warp >= kSoftmaxWarps) cluster_arrive();

    if (warp == kTmaWarp) {
        // ---------------- TMA producer: the q block, then the K/V tiles
        if (lane == 0) {
            mbar_arrive_expect_tx(&bar[B_QLOAD], kRows * kHD * 4);
#pragma unroll 1
            for (int b = 0; b < 4; ++b)
                tma_load_3d(base + OFF_STG + b * kBlockBytes, reinterpret_cast<uint64_t>(&p.qmap),
                            32 * b, (int)(kvh << lg), (int)t0, &bar[B_QLOAD]);
        }
        if (lane == 0 && nt > 0) {
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
        __syncwarp();
        cluster_wait();
    } else if (warp == kMmaWarp) {
        // ---------------- MMA issuer
        if (lane == 0 && nt > 0) {
            constexpr uint32_t id_pv = umma_idesc_bf16(kRows, kHD, 0, 1);
            bool ok = mbar_wait(&bar[B_QREADY], 0);
            tc_fence_after();
#pragma unroll 1
            for (int j = 0; ok && j < nt && j < 2; ++j) ok = issue_s(bar, sbase, tmem, j);
            for (int j = 0; ok && j < nt; ++j) {
                const int s = j & 1;
                const uint32_t ph = (uint32_t)(j >> 1) & 1u;
                if (!mbar_wait(&bar[B_PFULL + s], ph) || !mbar_wait(&bar[B_VFULL + s], ph)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // O += (P_hi + P_lo) V over 128 positions in 8 steps of 16.  P of
                // positions 32c + [0,32) sits at columns 32c + [0,16) (hi) and
                // 32c + [16,32) (lo) of the buffer.  V is MN-major: 64-dim
                // blocks 16 KB apart, 8-row groups 1 KB apart.
                const uint64_t vd =
                    umma_desc_sw128(sbase + OFF_V + (uint32_t)s * kTileBytes, kBlockBytes, 1024);
                const uint32_t pc = tmem + TM_SP + (uint32_t)s * 128u;
                // step i: part = i / 8 (P hi, P lo), positions 16 kk .. +15, kk = i % 8
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) {
                    const uint32_t part = i >> 3, kk = i & 7u;
                    const uint32_t a = pc + (kk >> 1) * 32u + part * 16u + (kk & 1u) * 8u;
                    umma_ts(tmem + TM_O, a, vd + ((kk * 16u * 128u) >> 4), id_pv, (j | (int)i) != 0);
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
        __syncwarp();
        cluster_wait();
    } else {
        // ---------------- softmax / epilogue
        const uint32_t prow = min(p.pos0 + tk, pmax);
        const int quarter = warp & 3;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        // q * scale * log2(e) -> bf16 hi + lo words (word w = head dims 2w,
        // 2w+1), this thread's half of row r: hi words at Q columns 32hf +
        // [0,32), lo words at 64 + 32hf + [0,32).  In the staging area head
        // dims 32b .. 32b+31 of row r sit in box b, 16-byte chunk c at c ^ (r % 8).
        {
            if (!__all_sync(0xffffffffu, mbar_wait(&bar[B_QLOAD], 0)) && lane == 0) fail(p);
            const float2 sc = make_float2(p.qscale, p.qscale);
            const unsigned char* qrow = base + OFF_STG + (uint32_t)r * 128u;
#pragma unroll 1
            for (uint32_t k = 0; k < 8; ++k) {
                // head dims 64hf + 8k .. +7: box 2hf + k/4, chunks 2(k%4), 2(k%4)+1
                const unsigned char* bx = qrow + (2u * hf + (k >> 2)) * kBlockBytes;
                const uint32_t c0 = 2u * (k & 3u);
                const float4 x0 = *reinterpret_cast<const float4*>(bx + ((c0 ^ ((uint32_t)r & 7u)) << 4));
                const float4 x1 =
                    *reinterpret_cast<const float4*>(bx + (((c0 + 1u) ^ ((uint32_t)r & 7u)) << 4));
                const float2 a0 = __fmul2_rn(make_float2(x0.x, x0.y), sc);
                const float2 a1 = __fmul2_rn(make_float2(x0.z, x0.w), sc);
                const float2 a2 = __fmul2_rn(make_float2(x1.x, x1.y), sc);
                const float2 a3 = __fmul2_rn(make_float2(x1.z, x1.w), sc);
                const uint32_t h0 = cvt_bf16x2(a0.x, a0.y), h1 = cvt_bf16x2(a1.x, a1.y);
                const uint32_t h2 = cvt_bf16x2(a2.x, a2.y), h3 = cvt_bf16x2(a3.x, a3.y);
                tmem_st4(tmem + lane_off + TM_Q + (uint32_t)hf * 32u + 4u * k, h0, h1, h2, h3);
                tmem_st4(tmem + lane_off + TM_Q + 64u + (uint32_t)hf * 32u + 4u * k,
                         cvt_bf16x2(a0.x - bf16_lo_f(h0), a0.y - bf16_hi_f(h0)),
                         cvt_bf16x2(a1.x - bf16_lo_f(h1), a1.y - bf16_hi_f(h1)),
                         cvt_bf16x2(a2.x - bf16_lo_f(h2), a2.y - bf16_hi_f(h2)),
                         cvt_bf16x2(a3.x - bf16_lo_f(h3), a3.y - bf16_hi_f(h3)));
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bar[B_QREADY]);
            cluster_arrive();         // this CTA's staging area is free
        }

        // Both warps of a pair meet at a (non-timed) named barrier every tile,
        // so neither leaves the loop early: after a failed wait a warp skips
        // its waits and TMEM work but keeps the barrier count.
        float m = -INFINITY;
        float2 l2 = make_float2(0.f, 0.f);
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            const int s = j & 1;
            const int jt = j0 + j;
            const uint32_t pbase = (uint32_t)jt * kPos;
            const uint32_t sp = tmem + lane_off + TM_SP + (uint32_t)s * 128u + (uint32_t)hf * 64u;
            const uint32_t ph = (uint32_t)(j >> 1) & 1u;
            // warp-uniform outcomes: the TMEM loads below are warp-collective
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar[B_SFULL + s], ph));
            if (ok) tc_fence_after();
            if (ok && jt == ntx - 1 && hf == 0) {
                // Rows past the block's last position hold whatever the cache
                // kept there (truncated turns); P is 0 for them, but 0 * inf
                // would still poison O, so zero those V rows before PV reads them.
                ok = __all_sync(0xffffffffu, mbar_wait(&bar[B_VFULL + s], ph));
                if (ok && pbase + (uint32_t)r > pmax) {
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
            // last visible position relative to this warp's 64 columns
            const int lim = (int)prow - (int)pbase - hf * 64;

            // pass 1: maximum over this half, then over the row
            float tm = -INFINITY;
            if (ok) {
                uint32_t va[32], vb[32];
                tmem_ld32(sp, va);
                tmem_ld32(sp + 32, vb);
                tmem_wait_ld(va, vb);
                if (diag) tm = max32<true>(vb, max32<true>(va, -INFINITY, lim), lim - 32);
                else tm = max32<false>(vb, max32<false>(va, -INFINITY, 0), 0);
            }
            float* tmx = sm_tmx + (j & 1) * 2 * kRows;
            tmx[hf * kRows + r] = tm;
            pair_sync(quarter);
            tm = fmaxf(tm, tmx[(hf ^ 1) * kRows + r]);
            if (ok) {
                // lazy rescale: the running maximum moves only when exceeded by > 2^8
                float alpha = 1.f;
                const bool grow = tm > m + 8.f;
                if (grow) {
                    alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - tm);
                    m = tm;
                    l2.x *= alpha;
                    l2.y *= alpha;
                }
                if (j > 0 && __any_sync(0xffffffffu, grow)) {
                    // O holds tiles < j: wait for PV(j-1), then scale this half
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(&bar[B_PVDONE], (uint32_t)(j - 1) & 1u));
                    if (ok) {
                        tc_fence_after();
#pragma unroll
                        for (int c = 0; c < 2; ++c) {
                            uint32_t v[32];
                            const uint32_t oc = tmem + lane_off + TM_O + (uint32_t)hf * 64u + c * 32;
                            tmem_ld32(oc, v);
                            tmem_wait_ld(v);
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
                            tmem_st32(oc, v);
                        }
                    }
                }
            }
            if (ok) {
                // pass 2: P over S, 32 positions at a time, the second chunk's
                // scores loading while the first is converted
                uint32_t va[32], vb[32];
                tmem_ld32(sp, va);
                tmem_wait_ld(va);
                tmem_ld32(sp + 32, vb);
                p_chunk(va, diag, m, lim, l2, sp);
                tmem_wait_ld(vb);
                p_chunk(vb, diag, m, lim - 32, l2, sp + 32);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bar[B_PFULL + s]);
        }
        // partial of this CTA (after every MMA is done): this thread's half
        // of O row r, with m and l, goes into its slot here when this CTA
        // finishes row r, else into outgoing row r; one bulk copy per peer
        // then moves that peer's rows in one piece.
        if (ok && nt > 0 && !__all_sync(0xffffffffu, mbar_wait(&bar[B_OREADY], 0))) ok = false;
        tc_fence_after();
        if (!ok && lane == 0) fail(p);
        if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        uint32_t zo = 0;
        while (zo + 1 < ns && row_begin(zo + 1, ns) <= (uint32_t)r) ++zo;
        const uint32_t rbo = row_begin(zo, ns);
        const uint32_t slot = z * (row_begin(zo + 1, ns) - rbo) + ((uint32_t)r - rbo);
        unsigned char* orow = zo == z ? base + OFF_STG + slot * kSlotBytes
                                      : base + OFF_OUT + (uint32_t)r * kSlotBytes;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            uint32_t v[32];
            if (nt > 0) {
                tmem_ld32(tmem + lane_off + TM_O + (uint32_t)hf * 64u + c * 32, v);
                tmem_wait_ld(v);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0u;
            }
#pragma unroll
            for (int g = 0; g < 8; ++g)
                *reinterpret_cast<uint4*>(orow + slot_group((uint32_t)(hf * 16 + c * 8 + g))) =
                    make_uint4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
        }
        float* tail = reinterpret_cast<float*>(orow + 512);
        if (hf == 0) {
            tail[0] = m;
            tail[3] = 0.f;
        }
        tail[1 + hf] = l2.x + l2.y;
        fence_proxy_async_smem();     // the rows are read by the bulk copies
        softmax_sync();
        __syncwarp();
        cluster_wait();               // every CTA's staging area is free
        if (tid == 0) {
            for (uint32_t d = 0; d < ns; ++d) {
                if (d == z) continue;
                const uint32_t rbd = row_begin(d, ns), nrd = row_begin(d + 1, ns) - rbd;
                bulk_copy_to_peer(dsmem_map(sbase + OFF_STG + z * nrd * kSlotBytes, d),
                                  sbase + OFF_OUT + rbd * kSlotBytes, nrd * kSlotBytes,
                                  dsmem_map(sbase + OFF_BAR + B_PUSH * 8, d));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, TM_COLS);
    }
    // Second phase: a CTA arrives once every partial row it finishes has
    // landed, and waits (at the very end) until all have, so that no CTA
    // exits while a copy still reads its shared memory.
    if (!mbar_wait(&bar[B_PUSH], 0) && tid == 0) fail(p);
    __syncwarp();
    cluster_arrive();

    // ---------------- merge: this CTA finishes rows [rb0, rb0 + nr) from the
    // slots in its own staging area.  First one thread per row turns the
    // (m, l) of all partials into weights; then one item = one row's float4
    // group, a warp covering a row (512 contiguous bytes out).
    const uint32_t rb0 = row_begin(z, ns), nr = row_begin(z + 1, ns) - rb0;
    float* wts = reinterpret_cast<float*>(base + OFF_WTS);   // [row - rb0][kMaxSplit + 1]
    if ((uint32_t)tid < nr) {
        const uint32_t rl = (uint32_t)tid;
        const unsigned char* tails = base + OFF_STG + rl * kSlotBytes + 512;   // slot (0, rl)
        float M = -INFINITY;
#pragma unroll 1
        for (uint32_t zz = 0; zz < ns; ++zz)
            M = fmaxf(M, *reinterpret_cast<const float*>(tails + zz * nr * kSlotBytes));
        float L = 0.f;
        float* w = wts + rl * (kMaxSplit + 1);
#pragma unroll 1
        for (uint32_t zz = 0; zz < ns; ++zz) {
            const float4 t = *reinterpret_cast<const float4*>(tails + zz * nr * kSlotBytes);
            const float wz = t.x == -INFINITY ? 0.f : ex2_approx(t.x - M);
            L += wz * (t.y + t.z);
            w[zz] = wz;
        }
        w[kMaxSplit] = L > 0.f ? 1.f / L : 0.f;
    }
    __syncthreads();
    {
        const uint32_t items = nr * 32u;
#pragma unroll 4
        for (uint32_t it = (uint32_t)tid; it < items; it += kThreads) {
            const uint32_t rl = it >> 5, grp = it & 31u;
            const uint32_t row = rb0 + rl;
            const uint32_t ttk = t0 + (row >> lg);
            const uint32_t thq = (kvh << lg) + (row & (G - 1));
            const float* w = wts + rl * (kMaxSplit + 1);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
            for (uint32_t zz = 0; zz < ns; ++zz) {
                const float wz = w[zz];
                const uint32_t sl = zz * nr + rl;
                const float4 o = *reinterpret_cast<const float4*>(
                    base + OFF_STG + sl * kSlotBytes + slot_group(grp));
                acc.x += wz * o.x;
                acc.y += wz * o.y;
                acc.z += wz * o.z;
                acc.w += wz * o.w;
            }
            const float inv = w[kMaxSplit];
            if (ttk < p.n_q)
                *reinterpret_cast<float4*>(p.out + ((uint64_t)ttk * p.n_heads + thq) * kHD + grp * 4) =
                    make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
    }
    __syncwarp();
    cluster_wait();
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
    // Programmatic dependent launch (TGKV_PDL=0 turns it off): the kernel
    // waits (griddepcontrol.wait) before its first global access.
    static const bool pdl = [] {
        const char* v = getenv("TGKV_PDL");
        return !(v && v[0] == '0');
    }();
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = p->n_split;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 2 : 1;
    e = cudaLaunchKernelEx(&cfg, prefill_kernel, *p);
    return (int)e;
}

// Clusters of n_split prefill CTAs that fit on the current device at once
// (0 if the query fails); the planner sizes the split with it.  The first
// call on a device asks for every split size, so that no later call pays
// for the occupancy query.
extern "C" uint32_t tgkv_prefill_max_clusters(uint32_t n_split) {
    using namespace tgkv::prefill;
    if (n_split == 0 || n_split > kMaxSplit) return 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    static uint32_t cache[64][kMaxSplit + 1];
    static bool filled[64];
    if (!filled[dev]) {
        if (cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 SMEM_BYTES) != cudaSuccess)
            return 0;
        for (uint32_t ns = 1; ns <= kMaxSplit; ++ns) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(1, 1, ns);
            cfg.blockDim = dim3(kThreads, 1, 1);
            cfg.dynamicSmemBytes = SMEM_BYTES;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = 1;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = ns;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, prefill_kernel, &cfg) != cudaSuccess || n < 0) {
                cudaGetLastError();
                n = 0;
            }
            cache[dev][ns] = (uint32_t)n;
        }
        filled[dev] = true;
    }
    return cache[dev][n_split];
}
