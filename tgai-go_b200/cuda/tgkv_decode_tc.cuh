// tgkv_decode_tc.cuh -- decode attention over a bf16, head_dim-128 cache on the
// tensor cores (tcgen05), included by tgkv_kernels.cu after attention_kernel,
// whose parameter block, chunk plan, fused append, partial layout and merge
// it shares.
//
// Why: the CUDA-core kernel spends about 52 warp-instructions per 512-byte
// K+V row (bf16 unpacking, QK and PV FMAs, reductions), which at full HBM
// bandwidth is more than half of the B200's issue rate; its bandwidth then
// follows the SM clock.  Here the contractions run on the tensor core and a
// row costs about two warp-instructions of softmax.
//
// Per CTA: one chunk of positions of one (query row, KV head, head subset),
// tiles of 128 positions, GT <= 4 query heads.  The three bf16 terms of q and
// of P are stacked along the MMA's N (row t * GT + h holds term t of head h;
// 3 GT <= 12 rows, zero-padded to N = 16), so one 8-step MMA chain per
// product computes all terms side by side and the softmax adds them:
//   S^T = K_tile . Qs^T       M = 128 positions, N = 16, K = 128 head dims
//   O^T += V_tile^T . Ps^T    M = 128 head dims, N = 16, K = 128 positions
// K and V tiles arrive by TMA in the 128-byte-swizzled boxes of the cache's
// second tensor map (64 dims x 128 positions); K is the K-major A operand of
// the first MMA, V the MN-major A operand of the second.  q and P enter as
// three bf16 terms (hi + mid + lo: all 24 mantissa bits of the fp32 value),
// so the products are those of the fp32 values and only the order of the
// fp32 accumulation differs from the CUDA-core kernel.
// Warps 0-3 (TMEM lane quarters 0-3): per tile, one position per thread --
// read its GT scores from TMEM, mask, share the tile maxima, online softmax
// in the log2 domain with the CUDA-core kernel's lazy rescale (the running
// maximum moves only when exceeded by 2^8; O^T is then rescaled in TMEM),
// write P^T into shared memory.  Warp 4: the fused append, then TMA.  Warp 5:
// TMEM and the MMAs (one lane).  Every mbarrier wait is bounded.
namespace tgkv {
namespace tc {

constexpr int kPos = 128;                       // positions per tile (MMA M of S^T)
constexpr int kN = 16;                          // MMA N: query heads, zero-padded
constexpr int kStages = 3;
constexpr int kThreads = 192;                   // warps 0-3 softmax, 4 TMA, 5 MMA
constexpr int kTmaWarp = 4, kMmaWarp = 5;
constexpr uint32_t kBlk = 16384;                // one box: 128 positions x 64 dims bf16
constexpr uint32_t kStage = 4 * kBlk;           // K (2 boxes) then V (2 boxes)
constexpr uint32_t kRowBlk = kN * 128;          // 16 rows x 64 bf16 (128 B): 2 KB
constexpr uint32_t kPart = 2 * kRowBlk;         // 16 rows x 128 bf16: one N = 16 operand
constexpr int kTerms = 3;                       // bf16 terms of q and of P
// shared memory, offsets from a 1024-aligned base
constexpr uint32_t OFF_RING = 0;
constexpr uint32_t OFF_Q = kStages * kStage;            // the stacked Q terms
constexpr uint32_t OFF_P = OFF_Q + kPart;               // [2 buffers] stacked P terms
constexpr uint32_t OFF_BAR = OFF_P + 2 * kPart;
constexpr uint32_t OFF_TSLOT = OFF_BAR + 32 * 8;
constexpr uint32_t OFF_RED = OFF_TSLOT + 16;            // [4 warps][16] tile maxima / sums
constexpr uint32_t OFF_CRED = OFF_RED + 4 * kN * 4;     // [4][GT][2] for the merge
constexpr uint32_t OFF_FLAG = OFF_CRED + 4 * 4 * 2 * 4;
constexpr uint32_t OFF_TPOS = OFF_FLAG + 16;            // [3] first position of each stage's tile
constexpr uint32_t SMEM_USED = OFF_TPOS + 16;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;       // slack to align the base
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
// the merge reuses the idle ring: (m, l) pairs, then 128 float4 sums
constexpr uint32_t OFF_ACC = OFF_Q - 128 * 16;

// barriers
constexpr int B_FULL = 0;      // [3] K and V of the stage landed
constexpr int B_EMPTY = 3;     // [3] the stage's PV is complete
constexpr int B_SFULL = 6;     // [2] S^T of the buffer is in TMEM
constexpr int B_SFREE = 8;     // [2] the softmax has read the S^T buffer (128 arrivals)
constexpr int B_PFULL = 10;    // [2] P buffer written, O^T rescaled (128 arrivals)
constexpr int B_PEMPTY = 12;   // [2] the PV that read the P buffer is complete (its
                               //     commit also marks O^T up to date)
constexpr int B_QREADY = 14;   // Q in shared memory (128 arrivals)

// TMEM columns: S^T buffers [0,16), [16,32); O^T [32,48)
constexpr uint32_t TM_S = 0, TM_O = 32, TM_COLS = 64;

constexpr int kErrTcTimeout = 5;
constexpr uint32_t kEnd = 0xffffffffu;          // a stage's tile position: no more tiles

// Byte offset of element (row r, column c) of a 16-row, 128-column bf16
// operand stored as two 64-column blocks in the canonical 128-byte swizzle
// (16-byte chunk k of row r at chunk k ^ (r & 7)).
__device__ __forceinline__ uint32_t sw_off(uint32_t r, uint32_t c) {
    const uint32_t b = c >> 6, cc = c & 63u;
    const uint32_t chunk = (cc >> 3) ^ (r & 7u);
    return b * kRowBlk + r * 128u + chunk * 16u + (cc & 7u) * 2u;
}

__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
}

// 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld16(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])::"memory");
}

// Named barrier of the four softmax warps (the merge's consumer_bar id).
__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// The same barrier, returning whether every softmax thread passed `v`: the
// softmax warps leave their tile loop only together, so that every thread
// meets every named barrier even after a bounded wait gave up.
__device__ __forceinline__ bool softmax_bar_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.and.pred po, 1, 128, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}
// Softmax warps and the MMA warp, before TMEM is freed.
__device__ __forceinline__ void dealloc_bar() { asm volatile("bar.sync 3, 160;" ::: "memory"); }

}  // namespace tc

template <int GT>
__global__ void __launch_bounds__(tc::kThreads, 1)
attention_tc_kernel(const __grid_constant__ TGKvAttnParams p) {
    using namespace tc;
    constexpr int HD = 128;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(base);
    uint64_t* bar = reinterpret_cast<uint64_t*>(base + OFF_BAR);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(base + OFF_TSLOT);
    float* red = reinterpret_cast<float*>(base + OFF_RED);
    int* flag = reinterpret_cast<int*>(base + OFF_FLAG);      // [0] abort, [1] last
    volatile uint32_t* tpos = reinterpret_cast<volatile uint32_t*>(base + OFF_TPOS);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t u = blockIdx.x;
    const Chunk ck = decode_chunk(p, u);
    const uint32_t n_item = p.n_pos[ck.item];
    const uint64_t cidx = (uint64_t)(p.item_base + ck.item) * (p.n_sub * p.n_kv_heads) + ck.seg;
    // Tile stealing (tile_ctr set, opt-in): the segment's CTAs take tiles of
    // [0, n_item) from its queue, so a CTA on a slower SM takes fewer;
    // otherwise each CTA streams the tiles of its own chunk.  Either way the
    // producer ends the stream with a stage marked kEnd and the other warps
    // stop there.
    const bool steal = p.tile_ctr != nullptr;
    const uint32_t lim = steal ? n_item : ck.pos1;          // positions past lim are masked

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bar[B_FULL + s], 1);
            mbar_init(&bar[B_EMPTY + s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bar[B_SFULL + b], 1);
            mbar_init(&bar[B_SFREE + b], 128);
            mbar_init(&bar[B_PFULL + b], 128);
            mbar_init(&bar[B_PEMPTY + b], 1);
        }
        mbar_init(&bar[B_QREADY], 128);
        flag[0] = 0;
        flag[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tslot, TM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    // A one-cache launch's tensor map was written when the cache was made:
    // its descriptor is fetched while the previous kernel finishes.
    if (!p.caches && warp == kTmaWarp && lane == 0 && p.cache0.tmap_sw) prefetch_tmap(p.cache0.tmap_sw);
    // Programmatic dependent launch: nothing above reads global memory
    // written by the previous kernels.
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == kTmaWarp) {
        const TGKvCacheDesc cd = p.caches ? p.caches[ck.item * p.cache_stride] : p.cache0;
        if (p.k_new && (steal || ck.pos1 == n_item)) {
            // fused append, as in attention_kernel: this KV head's slice of the
            // new row, then visible to this CTA's TMA reads below (with
            // stealing any CTA of the segment may load the last tile, so each
            // writes the same bytes first)
            const uint64_t kv_dim = (uint64_t)p.n_kv_heads * HD;
            const uint64_t src = (uint64_t)(p.item_base + ck.item) * kv_dim + ck.kvh * HD;
            const uint64_t dst = (uint64_t)(n_item - 1) * kv_dim + ck.kvh * HD;   // the new row
            const uint64_t vofs = (uint64_t)cd.max_seq * kv_dim;
            uint16_t* c = reinterpret_cast<uint16_t*>(cd.base);
            for (int e = lane; e < HD; e += 32) {
                c[dst + e] = f32_to_bf16_rne(p.k_new[src + e]);
                c[vofs + dst + e] = f32_to_bf16_rne(p.v_new[src + e]);
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
            __syncwarp();
        }
        if (lane == 0) {
            prefetch_tmap(cd.tmap_sw);
            const int x = (int)(ck.kvh * HD);
            const uint32_t seg_tiles = (n_item + kPos - 1) / kPos;
            for (int t = 0;; ++t) {
                uint32_t yy;
                bool done;
                if (steal) {
                    const uint32_t g = atomicAdd(p.tile_ctr + cidx, 1u);
                    done = g >= seg_tiles;
                    yy = g * kPos;
                } else {
                    yy = ck.pos0 + (uint32_t)t * kPos;
                    done = yy >= ck.pos1;
                }
                const int s = t % kStages;
                if (t >= kStages && !mbar_wait(&bar[B_EMPTY + s], (uint32_t)((t / kStages) - 1) & 1u)) {
                    atomicExch(p.err, kErrTcTimeout);
                    flag[0] = 1;
                    break;
                }
                tpos[s] = done ? kEnd : yy;
                if (done) {                     // the end marker: the phase completes without data
                    mbar_arrive(&bar[B_FULL + s]);
                    break;
                }
                const int y = (int)yy;
                unsigned char* st = base + OFF_RING + s * kStage;
                mbar_arrive_expect_tx(&bar[B_FULL + s], kStage);
                tma_load_3d(st, cd.tmap_sw, x, y, 0, &bar[B_FULL + s]);
                tma_load_3d(st + kBlk, cd.tmap_sw, x + 64, y, 0, &bar[B_FULL + s]);
                tma_load_3d(st + 2 * kBlk, cd.tmap_sw, x, y, 1, &bar[B_FULL + s]);
                tma_load_3d(st + 3 * kBlk, cd.tmap_sw, x + 64, y, 1, &bar[B_FULL + s]);
            }
        }
        return;
    }

    if (warp == kMmaWarp) {
        bool ok = true;
        if (lane == 0) {
            constexpr uint32_t id_s = umma_idesc_bf16(kPos, kN, 0, 0);
            constexpr uint32_t id_pv = umma_idesc_bf16(HD, kN, 1, 0);
            ok = mbar_wait(&bar[B_QREADY], 0);
            int nt = -1;                        // tiles of this CTA, once the end marker is seen
            // S^T(j) into buffer j % 2: A = the K tile (K-major), B = the stacked Q.
            // Returns false on a timeout; at the end marker sets nt = j instead.
            auto issue_s = [&](int j) -> bool {
                const int s = j % kStages, b = j & 1;
                if (!mbar_wait(&bar[B_FULL + s], (uint32_t)(j / kStages) & 1u)) return false;
                if (tpos[s] == kEnd) {
                    nt = j;
                    return true;
                }
                if (j >= 2 && !mbar_wait(&bar[B_SFREE + b], (uint32_t)((j >> 1) - 1) & 1u))
                    return false;
                tc_fence_after();
                const uint64_t ad = umma_desc_sw128(sbase + OFF_RING + s * kStage, 16, 1024);
#pragma unroll
                for (uint32_t ks = 0; ks < 8; ++ks) {
                    const uint32_t ao = (ks >> 2) * kBlk + (ks & 3u) * 32u;
                    const uint32_t bo = (ks >> 2) * kRowBlk + (ks & 3u) * 32u;
                    const uint64_t bd = umma_desc_sw128(sbase + OFF_Q + bo, 16, 1024);
                    umma_ss(tmem + TM_S + (uint32_t)b * kN, ad + (ao >> 4), bd, id_s, ks != 0);
                }
                umma_commit(&bar[B_SFULL + b]);
                return true;
            };
            if (ok) ok = issue_s(0);
            if (ok && nt < 0) ok = issue_s(1);
            for (int j = 0; ok && (nt < 0 || j < nt); ++j) {
                const int s = j % kStages, b = j & 1;
                if (!mbar_wait(&bar[B_PFULL + b], (uint32_t)(j >> 1) & 1u)) { ok = false; break; }
                tc_fence_after();
                // O^T += V^T Ps^T: A = the V tile, MN-major (64-dim blocks 16 KB
                // apart, 8-position groups 1 KB apart), 16 positions per step;
                // B = the stacked P rows of buffer b (K-major)
                const uint64_t vd =
                    umma_desc_sw128(sbase + OFF_RING + s * kStage + 2 * kBlk, kBlk, 1024);
#pragma unroll
                for (uint32_t kk = 0; kk < 8; ++kk) {
                    const uint32_t po = OFF_P + (uint32_t)b * kPart + (kk >> 2) * kRowBlk +
                                        (kk & 3u) * 32u;
                    umma_ss(tmem + TM_O, vd + ((kk * 16u * 128u) >> 4),
                            umma_desc_sw128(sbase + po, 16, 1024), id_pv, (j | (int)kk) != 0);
                }
                umma_commit(&bar[B_EMPTY + s]);
                umma_commit(&bar[B_PEMPTY + b]);
                if (nt < 0) ok = issue_s(j + 2);
            }
            if (!ok) {
                atomicExch(p.err, kErrTcTimeout);
                flag[0] = 1;
            }
        }
        __syncwarp();
        dealloc_bar();
        if (lane == 0) tc_fence_after();
        __syncwarp();
        tmem_dealloc(tmem, TM_COLS);
        return;
    }

    // ---------------- softmax warps 0-3: TMEM lane quarter = warp
    const uint32_t group = p.n_heads / p.n_kv_heads;
    const uint32_t head0 = ck.kvh * group + ck.sub * GT;
    const uint64_t row = (uint64_t)(p.item_base + ck.item) * p.n_heads * HD;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    // rows >= 3 GT of the Q and P operands stay zero; row t * GT + h of Q:
    // term t of q * scale (log2 domain) for head h
    for (uint32_t o = (uint32_t)tid * 16; o < 3 * kPart; o += 128 * 16)
        st_shared_zero16(sbase + OFF_Q + o);
    softmax_bar();
    for (uint32_t e = (uint32_t)tid; e < (uint32_t)GT * (HD / 2); e += 128) {
        const uint32_t h = e / (HD / 2), d = (e % (HD / 2)) * 2;
        const float2 x = *reinterpret_cast<const float2*>(p.q + row + (uint64_t)(head0 + h) * HD + d);
        float r0 = x.x * p.qscale, r1 = x.y * p.qscale;
#pragma unroll
        for (int t = 0; t < kTerms; ++t) {
            const uint32_t w = cvt_bf16x2(r0, r1);
            st_shared_u32(sbase + OFF_Q + sw_off((uint32_t)t * GT + h, d), w);
            r0 -= __uint_as_float(w << 16);
            r1 -= __uint_as_float(w & 0xffff0000u);
        }
    }
    fence_proxy_async_smem();
    mbar_arrive(&bar[B_QREADY]);

    float m_run[GT], l_part[GT];
#pragma unroll
    for (int h = 0; h < GT; ++h) { m_run[h] = -INFINITY; l_part[h] = 0.f; }
    bool ok = true;
    const uint32_t pp = (uint32_t)(warp * 32 + lane);              // position within a tile
    // P buffer j % 2 is free again, and O^T holds everything up to PV(j),
    // once PV(j)'s commit has landed (phase j / 2 of PEMPTY[j % 2]; the
    // buffer's earlier PV has been waited for by then, so the parity is
    // unambiguous)
    auto pv_done = [&](int j) -> bool {
        return mbar_wait(&bar[B_PEMPTY + (j & 1)], (uint32_t)(j >> 1) & 1u);
    };
    int nt = 0;                                          // tiles this CTA attended
    for (int j = 0;; ++j) {
        const int b = j & 1, s = j % kStages;
        uint32_t sv[16];
        // the stage's tile position, or the end marker, once its FULL phase is
        // complete; every thread reads the same word, and the barrier makes
        // the exit (end or timeout) common to the four warps
        bool mine = mbar_wait(&bar[B_FULL + s], (uint32_t)(j / kStages) & 1u);
        uint32_t tp = kEnd;
        if (mine) tp = tpos[s];
        if (!softmax_bar_all(ok && mine)) { ok = false; break; }
        if (tp == kEnd) break;
        nt = j + 1;
        // tcgen05.ld / st are warp-collective: every guard around them is made
        // warp-uniform
        mine = __all_sync(0xffffffffu, mbar_wait(&bar[B_SFULL + b], (uint32_t)(j >> 1) & 1u));
        const uint32_t pos = tp + pp;
        const bool valid = pos < lim;
        float sc[GT], tmx[GT];
        if (mine) {
            tc_fence_after();
            tmem_ld16(tmem + lane_off + TM_S + (uint32_t)b * kN, sv);
            tmem_wait_ld16(sv);
            tc_fence_before();
            mbar_arrive(&bar[B_SFREE + b]);
        }
#pragma unroll
        for (int h = 0; h < GT; ++h) {
            const float st = (__uint_as_float(sv[h]) + __uint_as_float(sv[GT + h])) +
                             __uint_as_float(sv[2 * GT + h]);
            sc[h] = (mine && valid) ? st : -INFINITY;
            float t = sc[h];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
            tmx[h] = t;
        }
        if (lane == 0)
#pragma unroll
            for (int h = 0; h < GT; ++h) red[warp * kN + h] = tmx[h];
        ok = softmax_bar_all(ok && mine);
        if (!ok) break;
#pragma unroll
        for (int h = 0; h < GT; ++h)
            tmx[h] = fmaxf(fmaxf(red[h], red[kN + h]), fmaxf(red[2 * kN + h], red[3 * kN + h]));
        softmax_bar();                                  // red is rewritten next tile
        // PV(j - 2) has released P buffer j % 2
        if (j >= 2) mine = __all_sync(0xffffffffu, pv_done(j - 2));
        // lazy rescale, as in attention_kernel: the running maximum moves only
        // when a score exceeds it by more than 2^8
        bool need = false;
#pragma unroll
        for (int h = 0; h < GT; ++h) need |= tmx[h] > m_run[h] + 8.f;
        if (need) {
            float alpha[GT];
#pragma unroll
            for (int h = 0; h < GT; ++h) {
                const float m_new = fmaxf(m_run[h], tmx[h]);
                alpha[h] = (m_new == -INFINITY) ? 1.f : exp2f(m_run[h] - m_new);
                m_run[h] = m_new;
                l_part[h] *= alpha[h];
            }
            if (j > 0 && mine) mine = __all_sync(0xffffffffu, pv_done(j - 1));
            if (j > 0 && mine) {
                // O^T holds PV(0 .. j-1): scale its columns
                tc_fence_after();
                uint32_t ov[16];
                tmem_ld16(tmem + lane_off + TM_O, ov);
                tmem_wait_ld16(ov);
#pragma unroll
                for (int h = 0; h < GT; ++h)
#pragma unroll
                    for (int t = 0; t < kTerms; ++t)
                        ov[t * GT + h] = __float_as_uint(__uint_as_float(ov[t * GT + h]) * alpha[h]);
                tmem_st16(tmem + lane_off + TM_O, ov);
                tmem_wait_st();
            }
        }
        if (!mine) { ok = false; continue; }           // leaves at the next tile's barrier
        const uint32_t pb = sbase + OFF_P + (uint32_t)b * kPart;
#pragma unroll
        for (int h = 0; h < GT; ++h) {
            const float pv = valid ? ex2_approx(sc[h] - m_run[h]) : 0.f;
            l_part[h] += pv;
            float r = pv;
#pragma unroll
            for (int t = 0; t < kTerms; ++t) {
                const uint32_t w = cvt_bf16x2(r, 0.f) & 0xffffu;
                st_shared_u16(pb + sw_off((uint32_t)(t * GT + h), pp), (uint16_t)w);
                r -= __uint_as_float(w << 16);
            }
        }
        if (pos >= n_item) {
            // rows past the item's length may hold anything (a truncated turn):
            // P = 0 there, but 0 x Inf/NaN is NaN, so clear this V row (its
            // stage has landed: FULL was waited for above)
            const uint32_t vr = sbase + OFF_RING + s * kStage + 2 * kBlk + pp * 128u;
#pragma unroll
            for (uint32_t c = 0; c < 128; c += 16) {
                st_shared_zero16(vr + c);
                st_shared_zero16(vr + kBlk + c);
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bar[B_PFULL + b]);
    }
    if (!ok) {
        atomicExch(p.err, kErrTcTimeout);
        flag[0] = 1;
    }
    // the streaming is over: the next kernel on the stream may start launching
    if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // ---- l over the CTA, O^T out of TMEM (lane = head dim)
    float ov_f[GT];
    if (ok && nt > 0 && !__all_sync(0xffffffffu, pv_done(nt - 1))) {   // every MMA is done
        ok = false;
        atomicExch(p.err, kErrTcTimeout);
        flag[0] = 1;
    }
    tc_fence_after();
#pragma unroll
    for (int h = 0; h < GT; ++h) ov_f[h] = 0.f;          // a CTA left without tiles
    if (nt > 0) {
        uint32_t ov[16];
        tmem_ld16(tmem + lane_off + TM_O, ov);
        tmem_wait_ld16(ov);
#pragma unroll
        for (int h = 0; h < GT; ++h)
            ov_f[h] = (__uint_as_float(ov[h]) + __uint_as_float(ov[GT + h])) +
                      __uint_as_float(ov[2 * GT + h]);
    }
    tc_fence_before();
    dealloc_bar();
#pragma unroll
    for (int h = 0; h < GT; ++h) {
        float t = l_part[h];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        l_part[h] = t;
    }
    if (lane == 0)
#pragma unroll
        for (int h = 0; h < GT; ++h) red[warp * kN + h] = l_part[h];
    softmax_bar();
    float L[GT];
#pragma unroll
    for (int h = 0; h < GT; ++h) L[h] = (red[h] + red[kN + h]) + (red[2 * kN + h] + red[3 * kN + h]);

    const uint32_t d = (uint32_t)tid;                    // head dim of this thread
    const bool whole = ck.nch == 1;
#pragma unroll
    for (int h = 0; h < GT; ++h) {
        if (whole) {
            const float o = (L[h] > 0.f) ? ov_f[h] / L[h] : 0.f;
            p.out[row + (uint64_t)(head0 + h) * HD + d] = o;
            if (p.gather_world) gather_store(p, row + (uint64_t)(head0 + h) * HD + d, o);
        } else {
            p.part_o[((uint64_t)u * GT + h) * HD + d] = ov_f[h];
            if (d == 0) {
                p.part_ml[((uint64_t)u * GT + h) * 2 + 0] = m_run[h];
                p.part_ml[((uint64_t)u * GT + h) * 2 + 1] = L[h];
            }
        }
    }
    if (whole) {
        if (steal && tid == 0) p.tile_ctr[cidx] = 0u;      // this CTA was the segment
        if (p.gather_world) gather_signal(p, tid);
        return;
    }
    // ---- the chunk that completes the segment merges it
    constexpr int kCap = (int)(OFF_ACC / (GT * 8));
    if (merge_segment<GT, HD, kCap>(p, ck, u, cidx, row, head0,
                                    reinterpret_cast<float2*>(base + OFF_RING),
                                    reinterpret_cast<float4*>(base + OFF_ACC),
                                    reinterpret_cast<float*>(base + OFF_CRED), flag, tid, lane,
                                    warp) &&
        steal && tid == 0)
        // every CTA of the segment has arrived, so every producer is past its
        // last take from the queue
        p.tile_ctr[cidx] = 0u;
}

}  // namespace tgkv
