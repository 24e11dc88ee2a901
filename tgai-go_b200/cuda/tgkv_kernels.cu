// tgkv_kernels.cu -- sm_100a kernels for TGAI GO's KV-cache path.
//
//   * attention: split-sequence (flash-decoding) GQA attention over caches in
//     the [2][max_seq][kv_dim] layout of src/tgai_kv_cache.h:15-21.  Each
//     (query row, KV head) segment is cut into fixed-size chunks, one CTA per
//     chunk (about eight waves).  A producer warp moves 32-row
//     boxes of K and V of one KV head into a shared-memory ring with tiled TMA
//     (cp.async.bulk.tensor, mbarrier completion); four consumer warps compute
//     the scores of all GT query heads of the group from the same staged rows
//     (K/V read once per KV head), keep an online softmax in the log2 domain
//     with warp-shuffle reductions, and accumulate P*V with packed fp32 FMAs.
//     The chunks of one segment merge in the last CTA to finish one.
//     Semantics follow src/tgai_engine.c:3943-4011: kvh = h*nkv/nh, scores
//     scaled by 1/sqrt(head_dim), causal, softmax, P*V.
//   * append: fp32 rows -> cache rows (fp32 copy or bf16 round-to-nearest-
//     even), 16-byte vector loads and stores.
//   * rope_append: shaders/rope.comp semantics (rotate Q and K, write K and V
//     into the cache).
//
// Every wait on an mbarrier is bounded by %globaltimer; on expiry the kernel
// records an error code in p.err and returns instead of spinning.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <math.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <mutex>
#include "tgkv_launch.h"
#include "tgkv_ptx.cuh"

namespace tgkv {

constexpr int kTile = TGKV_TILE;     // positions per stage
constexpr int kConsumerWarps = 4;    // 8 positions of a stage per warp
constexpr int kThreads = (kConsumerWarps + 1) * 32;


// Error codes written to p.err.
constexpr int kErrFullTimeout = 1;
constexpr int kErrEmptyTimeout = 2;
constexpr int kErrGatherTimeout = 4;

// Kernels launch as programmatic dependents unless TGKV_PDL=0.
bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("TGKV_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

}  // namespace tgkv

namespace tgkv {

// ------------------------------------------------------------ attention
// Compile-time geometry of one (dtype, head_dim, heads-per-CTA) variant.
template <int DT, int HD, int GT>
struct AttnCfg {
    static constexpr int ES = DT ? 2 : 4;              // bytes per element
    static constexpr int RB = HD * ES;                 // bytes per K/V row of one head
    static constexpr int LB = RB / 8;                  // bytes of a row per lane (8 lanes/row)
    static constexpr int VW = LB >= 16 ? 16 : LB;      // vector width in bytes
    static constexpr int NVEC = LB / VW;               // vectors per lane per row
    static constexpr int EPV = VW / ES;                // elements per vector
    static constexpr int NP = (HD / 8) / 2;            // float2 per lane per row
    static constexpr int STAGE = 2 * kTile * RB;       // K tile + V tile
    static constexpr int NSTAGE = (98304 / STAGE) > 8 ? 8 : (98304 / STAGE);
    static constexpr int HSTEP = 4 / GT;               // lane stride between heads
    static_assert(RB % 64 == 0, "row must be a multiple of 64 bytes");
    static_assert(GT == 1 || GT == 2 || GT == 4, "GT");
    static_assert(NSTAGE >= 2, "stages");
    // shared memory carve-up (bytes)
    static constexpr int OFF_BAR = NSTAGE * STAGE;
    static constexpr int OFF_P = OFF_BAR + 2 * NSTAGE * 8;
    static constexpr int OFF_ALPHA = OFF_P + kConsumerWarps * 32 * 4;
    static constexpr int OFF_CO = OFF_ALPHA + kConsumerWarps * 4 * 4;
    static constexpr int OFF_CML = OFF_CO + kConsumerWarps * GT * HD * 4;
    static constexpr int OFF_RED = OFF_CML + kConsumerWarps * GT * 2 * 4;   // [4][GT][2]
    static constexpr int OFF_FLAG = OFF_RED + kConsumerWarps * GT * 2 * 4;
    static constexpr int SMEM = OFF_FLAG + 16;
    // the combine reuses the idle ring: (m, l) pairs, then 128 float4 sums
    static constexpr int OFF_ACC = OFF_BAR - 128 * 16;
    static constexpr int ML_CAP = OFF_ACC / (GT * 8);                  // partials
};

// Unpack one lane vector (VW bytes at p) into EPV/2 float2.
template <int DT, int VW>
__device__ __forceinline__ void load_vec(const unsigned char* p, float2* o) {
    if constexpr (DT == 0) {
        static_assert(VW == 16, "f32 rows use 16-byte vectors");
        const float4 x = *reinterpret_cast<const float4*>(p);
        o[0] = make_float2(x.x, x.y);
        o[1] = make_float2(x.z, x.w);
    } else if constexpr (VW == 16) {
        const uint4 w = *reinterpret_cast<const uint4*>(p);
        o[0] = bf16pair_to_f2(w.x);
        o[1] = bf16pair_to_f2(w.y);
        o[2] = bf16pair_to_f2(w.z);
        o[3] = bf16pair_to_f2(w.w);
    } else {
        const uint2 w = *reinterpret_cast<const uint2*>(p);
        o[0] = bf16pair_to_f2(w.x);
        o[1] = bf16pair_to_f2(w.y);
    }
}

// A lane's slice of one row: vector v covers bytes v*8*VW + j*VW.
template <int DT, int HD, int GT>
__device__ __forceinline__ void load_row(const unsigned char* row, int j, float2* o) {
    using C = AttnCfg<DT, HD, GT>;
#pragma unroll
    for (int v = 0; v < C::NVEC; ++v)
        load_vec<DT, C::VW>(row + v * 8 * C::VW + j * C::VW, o + v * (C::EPV / 2));
}

// Element index of float2 slot i of lane j (first of the pair).
template <int DT, int HD, int GT>
__device__ __forceinline__ int elem_of(int j, int i) {
    using C = AttnCfg<DT, HD, GT>;
    const int v = i / (C::EPV / 2), w = i % (C::EPV / 2);
    return (v * 8 * C::VW + j * C::VW) / C::ES + 2 * w;
}

// Reduce N per-lane values over the 8 lanes of a group (xor 4, 2, 1) so that
// each lane ends with one complete sum: lane bit 2 picks the upper half of
// the values first, then bit 1, then bit 0 (while values remain to split).
template <int N>
__device__ __forceinline__ float group_transpose_reduce(float (&v)[N], int lane) {
    int n = N;
#pragma unroll
    for (int mask = 4; mask >= 1; mask >>= 1) {
        if (n >= 2) {
            const int half = n / 2;
            const bool upper = (lane & mask) != 0;
#pragma unroll
            for (int i = 0; i < N / 2; ++i) {
                if (i < half) {
                    const float send = upper ? v[i] : v[i + half];
                    const float keep = upper ? v[i + half] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
                }
            }
            n = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], mask);
        }
    }
    return v[0];
}

__device__ __forceinline__ void consumer_bar() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

// A chunk of a segment (see TGKvAttnParams), decoded from its number.
struct Chunk {
    uint32_t item, seg, kvh, sub;
    uint32_t pos0, pos1;         // positions [pos0, pos1) of the segment
    uint32_t nch;                // chunks of this segment
    uint32_t first;              // number of the segment's first chunk
};

__device__ __forceinline__ Chunk decode_chunk(const TGKvAttnParams& p, uint32_t u) {
    uint32_t lo = 0, hi = p.n_items;            // largest i with chunk_prefix[i] <= u
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (p.chunk_prefix[mid] <= u) lo = mid; else hi = mid;
    }
    Chunk c;
    c.item = lo;
    const uint32_t np = p.n_pos[lo];
    c.nch = (np + p.chunk - 1) / p.chunk;
    const uint32_t rem = u - p.chunk_prefix[lo];
    c.seg = rem / c.nch;
    const uint32_t ci = rem % c.nch;
    c.first = u - ci;
    c.kvh = c.seg % p.n_kv_heads;
    c.sub = c.seg / p.n_kv_heads;
    c.pos0 = ci * p.chunk;
    c.pos1 = min(c.pos0 + p.chunk, np);
    return c;
}

// Output gather over NVLink: one finished element to every rank's buffer.
__device__ __forceinline__ void gather_store(const TGKvAttnParams& p, uint64_t idx, float v) {
    for (uint32_t r = 0; r < p.gather_world; ++r) p.gather_out[r][p.gather_base + idx] = v;
}
// Four consecutive finished elements (idx a multiple of 4) to every rank's
// buffer: one 16-byte store per rank where the destination is 16-byte
// aligned, so that a warp's stores cross NVLink as whole 128-byte lines.
__device__ __forceinline__ void gather_store4(const TGKvAttnParams& p, uint64_t idx, float4 v) {
    for (uint32_t r = 0; r < p.gather_world; ++r) {
        float* d = p.gather_out[r] + p.gather_base + idx;
        if ((reinterpret_cast<uintptr_t>(d) & 15) == 0) {
            *reinterpret_cast<float4*>(d) = v;
        } else {
            d[0] = v.x;
            d[1] = v.y;
            d[2] = v.z;
            d[3] = v.w;
        }
    }
}

// After the CTA's 128 consumer threads stored a segment's outputs to every
// rank: system fence per thread, then one arrival per rank.
__device__ __noinline__ void gather_signal(const TGKvAttnParams& p, int tid) {
    __threadfence_system();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (tid == 0)
        for (uint32_t r = 0; r < p.gather_world; ++r) atomicAdd_system(p.gather_flag[r], 1u);
}

// Merge the nparts partials of one segment (slots first .. first+nparts-1;
// this CTA finished last).  The merge sits on the launch's critical path and
// is L2-latency bound, so it is built around few dependent round trips:
//  - the first batch of partial outputs is requested before anything else;
//  - one pass loads every (m, l) pair, reduces the per-head maxima and keeps
//    the pairs in the idle K/V ring (sm_ml), where the factors
//    exp2(m - M) then replace m in place;
//  - the weighted sums read one float4 of a partial per thread (thread v of
//    NV = GT*HD/4 vectors; 128/NV groups take every (128/NV)-th partial),
//    kB partials per step, so 128 * kB * 16 bytes are in flight per CTA.
// Segments of more than CAP partials reload the pairs block by block.
// Kept out of line so the streaming loop keeps its registers.
// out_slot: ~0u writes the segment's outputs (and its gather); any other
// value writes the merged, still unnormalised partial (O, and per head the
// maximum and sum) to that partial slot, for the second level of a
// two-level merge.
template <int GT, int HD, int CAP>
__device__ __noinline__ void combine_segment(const TGKvAttnParams& p, uint32_t first,
                                             uint32_t nparts, uint64_t row, uint32_t head0,
                                             float2* sm_ml, float4* sm_acc, float* sm_red,
                                             int tid, int lane, int warp, uint32_t out_slot) {
    constexpr int NV = GT * HD / 4;            // float4 per partial output
    constexpr int G = 128 / NV;                // groups of threads over the partials
    constexpr int kB = HD > 128 ? 16 : 24;     // partials per thread and step (24: a
                                               // segment of up to 24 chunks merges in one
                                               // round trip of loads)
    constexpr int kMl = 8;                     // (m, l) pairs per thread and step
    static_assert(NV <= 128 && 128 % NV == 0, "partial vectors");
    const int v = tid % NV, g = tid / NV;
    const int h = (v * 4) / HD;                 // head of this thread's vector
    const int hm = tid % GT;                    // head of this thread's (m, l) pairs
    const float4* po = reinterpret_cast<const float4*>(p.part_o) + (uint64_t)first * NV + v;
    const float2* pml = reinterpret_cast<const float2*>(p.part_ml) + (uint64_t)first * GT;
    const uint32_t nb0 = min((uint32_t)CAP, nparts);

    // first step of block 0's weighted sums, in flight during the pair pass
    float4 x[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
        const uint32_t c = (uint32_t)(g + u * G);
        x[u] = c < nb0 ? __ldcg(po + (uint64_t)c * NV) : make_float4(0.f, 0.f, 0.f, 0.f);
    }

    // ---- per-head maxima over all pairs; block 0's pairs stay in shared memory
    const uint32_t ne = nparts * GT;
    float mloc = -INFINITY;
    for (uint32_t e0 = 0; e0 < ne; e0 += 128 * kMl) {
        float2 y[kMl];
#pragma unroll
        for (int k = 0; k < kMl; ++k) {
            const uint32_t e = e0 + (uint32_t)(k * 128 + tid);
            y[k] = e < ne ? __ldcg(pml + e) : make_float2(-INFINITY, 0.f);
        }
#pragma unroll
        for (int k = 0; k < kMl; ++k) {
            const uint32_t e = e0 + (uint32_t)(k * 128 + tid);
            mloc = fmaxf(mloc, y[k].x);
            if (e < nb0 * GT) sm_ml[e] = y[k];
        }
    }
#pragma unroll
    for (int o = 16; o >= GT; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
    if (lane < GT) sm_red[(warp * GT + lane) * 2] = mloc;
    consumer_bar();
    float Mh = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) Mh = fmaxf(Mh, sm_red[(w * GT + hm) * 2]);

    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float lsum = 0.f;
    for (uint32_t b0 = 0; b0 < nparts; b0 += CAP) {
        const uint32_t nb = min((uint32_t)CAP, nparts - b0);
        if (b0) {                                  // later blocks: pairs from L2 again
            consumer_bar();                        // the previous block's factors are used
            for (uint32_t e = tid; e < nb * GT; e += 128) sm_ml[e] = __ldcg(pml + (uint64_t)b0 * GT + e);
        }
        // factors in place of m (each thread rewrites only the pairs it owns)
        for (uint32_t e = tid; e < nb * GT; e += 128) {
            const float2 ml = sm_ml[e];
            const float f = (ml.x == -INFINITY) ? 0.f : exp2f(ml.x - Mh);
            lsum += ml.y * f;
            sm_ml[e].x = f;
        }
        consumer_bar();
        for (uint32_t c0 = 0; c0 < nb; c0 += (uint32_t)(G * kB)) {
            if (b0 || c0) {
#pragma unroll
                for (int u = 0; u < kB; ++u) {
                    const uint32_t c = c0 + (uint32_t)(g + u * G);
                    x[u] = c < nb ? __ldcg(po + (uint64_t)(b0 + c) * NV)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int u = 0; u < kB; ++u) {
                const uint32_t c = c0 + (uint32_t)(g + u * G);
                const float f = c < nb ? sm_ml[c * GT + h].x : 0.f;
                acc.x += x[u].x * f;
                acc.y += x[u].y * f;
                acc.z += x[u].z * f;
                acc.w += x[u].w * f;
            }
        }
    }

    // ---- totals: l per head over threads and warps, outputs over groups
#pragma unroll
    for (int o = 16; o >= GT; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane < GT) sm_red[(warp * GT + lane) * 2 + 1] = lsum;
    if (G > 1) sm_acc[g * NV + v] = acc;
    consumer_bar();
    if (g == 0) {
#pragma unroll
        for (int k = 1; k < G; ++k) {
            const float4 a = sm_acc[k * NV + v];
            acc.x += a.x; acc.y += a.y; acc.z += a.z; acc.w += a.w;
        }
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) L += sm_red[(w * GT + h) * 2 + 1];
        if (out_slot != ~0u) {
            reinterpret_cast<float4*>(p.part_o)[(uint64_t)out_slot * NV + v] = acc;
            if ((v * 4) % HD == 0) {                // one thread per head: (M, L)
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm_red[(w * GT + h) * 2]);
                reinterpret_cast<float2*>(p.part_ml)[(uint64_t)out_slot * GT + h] =
                    make_float2(M, L);
            }
        } else {
            const bool any = L > 0.f;
            const float o[4] = {any ? acc.x / L : 0.f, any ? acc.y / L : 0.f,
                                any ? acc.z / L : 0.f, any ? acc.w / L : 0.f};
            const uint64_t base = row + (uint64_t)(head0 + h) * HD + (v * 4) % HD;
#pragma unroll
            for (int k = 0; k < 4; ++k) p.out[base + k] = o[k];
            if (p.gather_world) gather_store4(p, base, make_float4(o[0], o[1], o[2], o[3]));
        }
    }
    if (out_slot == ~0u && p.gather_world) gather_signal(p, tid);
}

// After this CTA has written the partial of chunk u (segment ck, arrival
// counter cidx): the CTA that completes the segment merges it.  Segments of
// more than p.two_level_min chunks merge in two levels, so that no single
// CTA walks hundreds of partials (one KV head of a 131072-position context
// on a GPU is one segment of ~300 chunks): the last chunk of each group of
// 16 to finish merges the group into a partial slot, and the last group to
// finish merges those.  Called by the 128 threads of named barrier 1; flag
// [0] is set when a wait gave up (the ring is then not idle and nothing is
// merged), flag[1] is scratch.  Returns true on the CTA that finished the
// segment (its counters are reset).
template <int GT, int HD, int CAP>
__device__ __forceinline__ bool merge_segment(const TGKvAttnParams& p, const Chunk& ck,
                                              uint32_t u, uint64_t cidx, uint64_t row,
                                              uint32_t head0, float2* sm_ml, float4* sm_acc,
                                              float* sm_red, volatile int* flag, int tid,
                                              int lane, int warp) {
    constexpr uint32_t kGroup = 16;
    __threadfence();
    consumer_bar();
    uint32_t parts = ck.nch, src = ck.first;
    if (p.two_level_min && ck.nch > p.two_level_min) {
        const uint32_t gi = (u - ck.first) / kGroup, g0 = gi * kGroup;
        const uint32_t gsz = min(kGroup, ck.nch - g0);
        const uint64_t gidx = (uint64_t)p.gctr_base + ck.first + gi;
        if (tid == 0) flag[1] = atomicAdd(&p.counters[gidx], 1u) == gsz - 1 ? 1 : 0;
        consumer_bar();
        if (!flag[1]) return false;
        __threadfence();
        if (!flag[0])
            combine_segment<GT, HD, CAP>(p, ck.first + g0, gsz, row, head0, sm_ml, sm_acc, sm_red,
                                         tid, lane, warp, p.l1_base + ck.first + gi);
        if (tid == 0) p.counters[gidx] = 0u;
        __threadfence();
        consumer_bar();
        parts = (ck.nch + kGroup - 1) / kGroup;
        src = p.l1_base + ck.first;
    }
    if (tid == 0) flag[1] = atomicAdd(&p.counters[cidx], 1u) == parts - 1 ? 1 : 0;
    consumer_bar();
    if (!flag[1]) return false;
    __threadfence();
    if (!flag[0])                                  // the ring is idle unless a wait gave up
        combine_segment<GT, HD, CAP>(p, src, parts, row, head0, sm_ml, sm_acc, sm_red, tid, lane,
                                     warp, ~0u);
    if (tid == 0) p.counters[cidx] = 0u;
    return true;
}

template <int DT, int HD, int GT>
__global__ void __launch_bounds__(kThreads, 2)
attention_kernel(const __grid_constant__ TGKvAttnParams p) {
    using C = AttnCfg<DT, HD, GT>;
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = full + C::NSTAGE;
    float* sm_p = reinterpret_cast<float*>(smem + C::OFF_P);          // [4][32]
    float* sm_alpha = reinterpret_cast<float*>(smem + C::OFF_ALPHA);  // [4][4]
    float* sm_co = reinterpret_cast<float*>(smem + C::OFF_CO);        // [4][GT][HD]
    float* sm_cml = reinterpret_cast<float*>(smem + C::OFF_CML);      // [4][GT][2]
    float* sm_red = reinterpret_cast<float*>(smem + C::OFF_RED);      // [4][GT][2]
    int* sm_flag = reinterpret_cast<int*>(smem + C::OFF_FLAG);        // [0] abort, [1] last

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t u = blockIdx.x;                // this CTA's chunk
    const Chunk ck = decode_chunk(p, u);
    const int ntiles = (int)((ck.pos1 - ck.pos0 + kTile - 1) / kTile);

    if (tid == 0) {
        for (int s = 0; s < C::NSTAGE; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        sm_flag[0] = 0;
        sm_flag[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // A one-cache launch's tensor map was written when the cache was made (or
    // sits in the parameters): its descriptor is fetched while the previous
    // kernel finishes.
    if (!p.caches && warp == kConsumerWarps && lane == 0)
        prefetch_tmap(p.cache0.tmap ? p.cache0.tmap : reinterpret_cast<uint64_t>(&p.tmap0));
    // Programmatic dependent launch: everything above overlaps the previous
    // kernel on the stream; nothing below reads global memory written by the
    // previous kernels before they are done.
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == kConsumerWarps) {
        const TGKvCacheDesc cd = p.caches ? p.caches[ck.item * p.cache_stride] : p.cache0;
        if (p.k_new && ck.pos1 == p.n_pos[ck.item]) {
            // ---------------- fused append: the chunk that ends at the newest
            // position first stores this KV head's slice of the new K and V
            // row (fp32 -> cache type), then makes the stores visible to the
            // TMA reads below.  Every head subset's CTA writes the same bytes.
            const uint64_t kv_dim = (uint64_t)p.n_kv_heads * HD;
            const uint64_t src = (uint64_t)(p.item_base + ck.item) * kv_dim + ck.kvh * HD;
            const uint64_t dst = (uint64_t)(ck.pos1 - 1) * kv_dim + ck.kvh * HD;
            const uint64_t vofs = (uint64_t)cd.max_seq * kv_dim;
            for (int e = lane; e < HD; e += 32) {
                const float kx = p.k_new[src + e], vx = p.v_new[src + e];
                if constexpr (DT == 0) {
                    float* c = reinterpret_cast<float*>(cd.base);
                    c[dst + e] = kx;
                    c[vofs + dst + e] = vx;
                } else {
                    uint16_t* c = reinterpret_cast<uint16_t*>(cd.base);
                    c[dst + e] = f32_to_bf16_rne(kx);
                    c[vofs + dst + e] = f32_to_bf16_rne(vx);
                }
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
            __syncwarp();
        }
        // ---------------- producer: one tiled TMA box of K and one of V per
        // stage (32 rows of this KV head; rows past max_seq arrive as 0)
        if (lane == 0 && !p.stall_loads) {
            const uint64_t tmap = cd.tmap ? cd.tmap : reinterpret_cast<uint64_t>(&p.tmap0);
            prefetch_tmap(tmap);
            const int x = (int)(ck.kvh * HD);
            int issued = 0;
            for (int t = 0; t < ntiles; ++t) {
                const int s = t % C::NSTAGE;
                if (t >= C::NSTAGE && !mbar_wait(&empty[s], ((t / C::NSTAGE) - 1) & 1)) {
                    atomicExch(p.err, kErrEmptyTimeout);
                    sm_flag[0] = 1;
                    break;
                }
                const int row0 = (int)(ck.pos0 + (uint32_t)t * kTile);
                unsigned char* st = smem + s * C::STAGE;
                mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * kTile * C::RB));
                tma_load_3d(st, tmap, x, row0, 0, &full[s]);
                tma_load_3d(st + kTile * C::RB, tmap, x, row0, 1, &full[s]);
                ++issued;
            }
            // Keep the CTA alive until its last stages have landed, so that
            // consumers that gave up early never leave copies in flight into
            // shared memory.  No later tile reuses these stages, so each
            // barrier stays in the phase its last copy completed.
            for (int t = issued > C::NSTAGE ? issued - C::NSTAGE : 0; t < issued; ++t)
                if (!mbar_wait(&full[t % C::NSTAGE], (t / C::NSTAGE) & 1))
                    atomicExch(p.err, kErrFullTimeout);
        }
        return;
    }

    // ---------------- consumers
    const int g = lane >> 3, j = lane & 7;
    const int r_me = (lane >> 2) & 1;
    const int h_me = (lane & 3) / C::HSTEP;
    const bool canon = (lane & (C::HSTEP - 1)) == 0;
    const uint32_t group = p.n_heads / p.n_kv_heads;
    const uint32_t head0 = ck.kvh * group + ck.sub * GT;
    const uint64_t row = (uint64_t)(p.item_base + ck.item) * p.n_heads * HD;

    float2 q2[GT][C::NP];
#pragma unroll
    for (int h = 0; h < GT; ++h) {
        const float* qh = p.q + row + (uint64_t)(head0 + h) * HD;
#pragma unroll
        for (int i = 0; i < C::NP; ++i) {
            const float2 x = *reinterpret_cast<const float2*>(qh + elem_of<DT, HD, GT>(j, i));
            q2[h][i] = make_float2(x.x * p.qscale, x.y * p.qscale);
        }
    }
    float2 o2[GT][C::NP];
#pragma unroll
    for (int h = 0; h < GT; ++h)
#pragma unroll
        for (int i = 0; i < C::NP; ++i) o2[h][i] = make_float2(0.f, 0.f);
    float m_run = -INFINITY, l_lane = 0.f;

    for (int t = 0; t < ntiles; ++t) {
        const int s = t % C::NSTAGE;
        // the warp leaves together: a lane that saw the stage complete while
        // another gave up must not go on to the shuffles below alone
        if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (t / C::NSTAGE) & 1))) {
            if (lane == 0) { atomicExch(p.err, kErrFullTimeout); sm_flag[0] = 1; }
            break;
        }
        const unsigned char* kt = smem + s * C::STAGE;
        const unsigned char* vt = kt + kTile * C::RB;
        const uint32_t tpos = ck.pos0 + (uint32_t)t * kTile;

        // scores of rows w*8 + r*4 + g for r = 0, 1 and all GT heads
        float sc[2 * GT];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float2 k2[C::NP];
            load_row<DT, HD, GT>(kt + (warp * 8 + r * 4 + g) * C::RB, j, k2);
#pragma unroll
            for (int h = 0; h < GT; ++h) {
                float2 acc = make_float2(0.f, 0.f);
#pragma unroll
                for (int i = 0; i < C::NP; ++i) acc = ffma2(q2[h][i], k2[i], acc);
                sc[r * GT + h] = acc.x + acc.y;
            }
        }
        float sv = group_transpose_reduce<2 * GT>(sc, lane);
        const bool valid = tpos + (uint32_t)(warp * 8 + r_me * 4 + g) < ck.pos1;
        sv = valid ? sv : -INFINITY;

        float tm = sv;
        tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 4));
        tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 8));
        tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 16));
        // Lazy rescale: the running maximum only moves when a score exceeds
        // it by more than 2^8, so exp2(score - m_run) stays <= 256.
        const bool need = tm > m_run + 8.f;
        if (__any_sync(0xffffffffu, need)) {
            const float m_new = fmaxf(m_run, tm);
            const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m_run - m_new);
            m_run = m_new;
            l_lane *= alpha;
            if (g == 0 && r_me == 0 && canon) sm_alpha[warp * 4 + h_me] = alpha;
            __syncwarp();
#pragma unroll
            for (int h = 0; h < GT; ++h) {
                const float a = sm_alpha[warp * 4 + h];
#pragma unroll
                for (int i = 0; i < C::NP; ++i) {
                    o2[h][i].x *= a;
                    o2[h][i].y *= a;
                }
            }
        }
        const float pv = (sv == -INFINITY) ? 0.f : exp2f(sv - m_run);
        if (canon) l_lane += pv;
        sm_p[warp * 32 + lane] = pv;
        __syncwarp();

        const bool tail = tpos + kTile > ck.pos1;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int rw = warp * 8 + r * 4 + g;
            float2 v2[C::NP];
            load_row<DT, HD, GT>(vt + rw * C::RB, j, v2);
            if (tail && tpos + (uint32_t)rw >= ck.pos1) {
#pragma unroll
                for (int i = 0; i < C::NP; ++i) v2[i] = make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int h = 0; h < GT; ++h) {
                const float ph = sm_p[warp * 32 + g * 8 + r * 4 + h * C::HSTEP];
                const float2 p2 = make_float2(ph, ph);
#pragma unroll
                for (int i = 0; i < C::NP; ++i) o2[h][i] = ffma2(p2, v2[i], o2[h][i]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    // the streaming is over: the next kernel on the stream may start launching
    if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // ---- warp totals: O over the four row groups, l over lanes of a head
#pragma unroll
    for (int h = 0; h < GT; ++h)
#pragma unroll
        for (int i = 0; i < C::NP; ++i) {
            o2[h][i].x += __shfl_xor_sync(0xffffffffu, o2[h][i].x, 8);
            o2[h][i].y += __shfl_xor_sync(0xffffffffu, o2[h][i].y, 8);
            o2[h][i].x += __shfl_xor_sync(0xffffffffu, o2[h][i].x, 16);
            o2[h][i].y += __shfl_xor_sync(0xffffffffu, o2[h][i].y, 16);
        }
    if (C::HSTEP >= 2) l_lane += __shfl_xor_sync(0xffffffffu, l_lane, 1);
    if (C::HSTEP >= 4) l_lane += __shfl_xor_sync(0xffffffffu, l_lane, 2);
    l_lane += __shfl_xor_sync(0xffffffffu, l_lane, 4);
    l_lane += __shfl_xor_sync(0xffffffffu, l_lane, 8);
    l_lane += __shfl_xor_sync(0xffffffffu, l_lane, 16);

    if (lane < 8) {
#pragma unroll
        for (int h = 0; h < GT; ++h)
#pragma unroll
            for (int i = 0; i < C::NP; ++i) {
                float* dst = sm_co + (warp * GT + h) * HD + elem_of<DT, HD, GT>(j, i);
                dst[0] = o2[h][i].x;
                dst[1] = o2[h][i].y;
            }
    }
    if (g == 0 && r_me == 0 && canon) {
        sm_cml[(warp * GT + h_me) * 2 + 0] = m_run;
        sm_cml[(warp * GT + h_me) * 2 + 1] = l_lane;
    }
    consumer_bar();

    // ---- merge the four warps; write the output or this chunk's partial
    const bool whole = ck.nch == 1;
    for (int idx = tid; idx < GT * HD; idx += 128) {
        const int h = idx / HD, d = idx % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm_cml[(w * GT + h) * 2]);
        float O = 0.f, L = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
            const float mw = sm_cml[(w * GT + h) * 2];
            const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
            O += sm_co[(w * GT + h) * HD + d] * f;
            L += sm_cml[(w * GT + h) * 2 + 1] * f;
        }
        if (whole) {
            const float o = (L > 0.f) ? O / L : 0.f;
            p.out[row + (uint64_t)(head0 + h) * HD + d] = o;
            if (p.gather_world) gather_store(p, row + (uint64_t)(head0 + h) * HD + d, o);
        } else {
            p.part_o[((uint64_t)u * GT + h) * HD + d] = O;
            if (d == 0) {
                p.part_ml[((uint64_t)u * GT + h) * 2 + 0] = M;
                p.part_ml[((uint64_t)u * GT + h) * 2 + 1] = L;
            }
        }
    }
    if (whole) {
        if (p.gather_world) gather_signal(p, tid);
        return;
    }

    // ---- the chunk that completes the segment merges it
    const uint64_t cidx = (uint64_t)(p.item_base + ck.item) * (p.n_sub * p.n_kv_heads) + ck.seg;
    merge_segment<GT, HD, C::ML_CAP>(p, ck, u, cidx, row, head0, reinterpret_cast<float2*>(smem),
                                     reinterpret_cast<float4*>(smem + C::OFF_ACC), sm_red, sm_flag,
                                     tid, lane, warp);
}

}  // namespace tgkv

namespace tgkv {

// ------------------------------------------------------------ append
// One thread moves 8 consecutive elements of one K or V row (blockIdx.y picks
// K or V): two 16-byte loads of fp32, one or two 16-byte stores.
// Launched as a programmatic dependent itself: it may start while the
// previous kernel finishes, but writes nothing before that kernel has
// completed (an LCP re-append overwrites rows the last attention read).  The
// attention launched next may start its setup right away; it reads nothing
// before this grid has completed.
template <int DT>
__global__ void __launch_bounds__(256) append_kernel(const __grid_constant__ TGKvAppendParams p) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint64_t vec_per_row = p.kv_dim / 8;
    const uint64_t rows = (uint64_t)p.n_items * p.rows_per_item;
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= rows * vec_per_row) return;
    const int which = blockIdx.y;                       // 0 = K, 1 = V
    const uint64_t row = t / vec_per_row, e = (t % vec_per_row) * 8;
    const uint32_t item = (uint32_t)(row / p.rows_per_item);
    const uint32_t r = (uint32_t)(row % p.rows_per_item);
    const float* src = (which ? p.v : p.k) + row * p.kv_dim + e;
    const float4 a = *reinterpret_cast<const float4*>(src);
    const float4 b = *reinterpret_cast<const float4*>(src + 4);
    const TGKvCacheDesc cd = p.caches ? p.caches[item * p.cache_stride] : p.cache0;
    const uint64_t pos = (uint64_t)p.pos[item] + r;
    const uint64_t elem = (uint64_t)which * cd.max_seq * p.kv_dim + pos * p.kv_dim + e;
    if constexpr (DT == 0) {
        float* dst = reinterpret_cast<float*>(cd.base) + elem;
        *reinterpret_cast<float4*>(dst) = a;
        *reinterpret_cast<float4*>(dst + 4) = b;
    } else {
        uint4 w;
        w.x = (uint32_t)f32_to_bf16_rne(a.x) | ((uint32_t)f32_to_bf16_rne(a.y) << 16);
        w.y = (uint32_t)f32_to_bf16_rne(a.z) | ((uint32_t)f32_to_bf16_rne(a.w) << 16);
        w.z = (uint32_t)f32_to_bf16_rne(b.x) | ((uint32_t)f32_to_bf16_rne(b.y) << 16);
        w.w = (uint32_t)f32_to_bf16_rne(b.z) | ((uint32_t)f32_to_bf16_rne(b.w) << 16);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(cd.base) + elem) = w;
    }
}

// ------------------------------------------------------------ rope + append
// shaders/rope.comp semantics: thread = (token, head, pair).  Q of every head
// is rotated into qout; heads below n_kv_heads also rotate K and copy V into
// the cache at position start_pos + token.  The rotation is evaluated as the
// reference engine's gcc -mfma build evaluates src/tgai_engine.c:3480-3481:
// x0*c - x1*s == fma(x0, c, -(x1*s)), x0*s + x1*c == fma(x0, s, x1*c).
__device__ __forceinline__ float2 rotate_pair(float x0, float x1, float c, float s) {
    return make_float2(__fmaf_rn(x0, c, -__fmul_rn(x1, s)), __fmaf_rn(x0, s, __fmul_rn(x1, c)));
}

template <int DT>
__global__ void __launch_bounds__(256) rope_append_kernel(const __grid_constant__ TGKvRopeParams p) {
    const uint32_t half = p.head_dim >> 1;
    const uint64_t total = (uint64_t)p.n_tokens * p.n_heads * half;
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= total) return;
    const uint32_t pair = (uint32_t)(gid % half);
    const uint32_t head = (uint32_t)((gid / half) % p.n_heads);
    const uint32_t tok = (uint32_t)(gid / ((uint64_t)half * p.n_heads));
    const uint64_t q_dim = (uint64_t)p.n_heads * p.head_dim;
    const uint64_t kv_dim = (uint64_t)p.n_kv_heads * p.head_dim;
    const uint64_t stride = q_dim + 2 * kv_dim;
    const uint64_t pos = (uint64_t)p.start_pos + tok;
    const float c = p.cs[pos * half + pair], s = p.sn[pos * half + pair];
    const uint32_t i0 = pair * 2;
    const float* row = p.qkv + tok * stride;
    const float2 q = rotate_pair(row[head * p.head_dim + i0], row[head * p.head_dim + i0 + 1], c, s);
    p.qout[tok * q_dim + head * p.head_dim + i0] = q.x;
    p.qout[tok * q_dim + head * p.head_dim + i0 + 1] = q.y;
    if (head < p.n_kv_heads) {
        const float* kr = row + q_dim + head * p.head_dim + i0;
        const float* vr = row + q_dim + kv_dim + head * p.head_dim + i0;
        const float2 k = rotate_pair(kr[0], kr[1], c, s);
        const uint64_t ko = pos * kv_dim + head * p.head_dim + i0;
        const uint64_t vo = (uint64_t)p.max_seq * kv_dim + ko;
        if constexpr (DT == 0) {
            float* kv = reinterpret_cast<float*>(p.kvc);
            kv[ko] = k.x; kv[ko + 1] = k.y;
            kv[vo] = vr[0]; kv[vo + 1] = vr[1];
        } else {
            uint32_t* kv = reinterpret_cast<uint32_t*>(p.kvc);
            kv[ko / 2] = (uint32_t)f32_to_bf16_rne(k.x) | ((uint32_t)f32_to_bf16_rne(k.y) << 16);
            kv[vo / 2] = (uint32_t)f32_to_bf16_rne(vr[0]) | ((uint32_t)f32_to_bf16_rne(vr[1]) << 16);
        }
    }
}

// Launched with programmatic stream serialization (PDL) unless TGKV_PDL=0:
// the kernel waits (griddepcontrol.wait) before its first global access, so
// overlapping its launch with the previous kernel is safe.
template <int DT, int HD, int GT>
int launch_attn(const TGKvAttnParams* p, uint32_t grid, cudaStream_t st) {
    using C = AttnCfg<DT, HD, GT>;
    static bool configured = false;                 // benign race: same value
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel<DT, HD, GT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return (int)e;
        configured = true;
    }
    static const bool pdl = [] {
        const char* e = getenv("TGKV_PDL");
        return !(e && e[0] == '0');
    }();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, attention_kernel<DT, HD, GT>, *p);
}

}  // namespace tgkv

#include "tgkv_decode_tc.cuh"

namespace tgkv {
template <int GT>
int launch_attn_tc(const TGKvAttnParams* p, uint32_t grid, cudaStream_t st) {
    static bool configured = false;                 // benign race: same value
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel<GT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)tc::SMEM_BYTES);
        if (e != cudaSuccess) return (int)e;
        configured = true;
    }
    static const bool pdl = [] {
        const char* e = getenv("TGKV_PDL");
        return !(e && e[0] == '0');
    }();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = tc::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, attention_tc_kernel<GT>, *p);
}
}  // namespace tgkv

extern "C" int tgkv_launch_attention_tc(const TGKvAttnParams* p, uint32_t g_tile, uint32_t grid,
                                        void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    switch (g_tile) {
    case 1: return tgkv::launch_attn_tc<1>(p, grid, st);
    case 2: return tgkv::launch_attn_tc<2>(p, grid, st);
    case 4: return tgkv::launch_attn_tc<4>(p, grid, st);
    default: return (int)cudaErrorInvalidValue;
    }
}

extern "C" uint32_t tgkv_attention_g_tile(uint32_t head_dim, uint32_t group) {
    // Largest of 4, 2, 1 that divides the group and fits the register budget
    // (query and output slices of GT heads per lane).
    const uint32_t cap = head_dim >= 256 ? 2u : 4u;
    for (uint32_t gt = cap; gt > 1; gt >>= 1)
        if (group % gt == 0) return gt;
    return 1u;
}

extern "C" int tgkv_attention_supported(int dtype, uint32_t head_dim) {
    if (dtype == 0) return head_dim == 32 || head_dim == 64 || head_dim == 128;
    if (dtype == 1) return head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256;
    return 0;
}

#define TGKV_ATTN_CASE(DT, HD, GT)                                             \
    if (dtype == DT && head_dim == HD && g_tile == GT)                         \
        return tgkv::launch_attn<DT, HD, GT>(p, grid, st);

extern "C" int tgkv_launch_attention(const TGKvAttnParams* p, int dtype, uint32_t head_dim,
                                     uint32_t g_tile, uint32_t grid, void* stream) {
    cudaStream_t st = (cudaStream_t)stream;
    if (grid == 0) return 0;
    TGKV_ATTN_CASE(0, 32, 1) TGKV_ATTN_CASE(0, 32, 2) TGKV_ATTN_CASE(0, 32, 4)
    TGKV_ATTN_CASE(0, 64, 1) TGKV_ATTN_CASE(0, 64, 2) TGKV_ATTN_CASE(0, 64, 4)
    TGKV_ATTN_CASE(0, 128, 1) TGKV_ATTN_CASE(0, 128, 2) TGKV_ATTN_CASE(0, 128, 4)
    TGKV_ATTN_CASE(1, 32, 1) TGKV_ATTN_CASE(1, 32, 2) TGKV_ATTN_CASE(1, 32, 4)
    TGKV_ATTN_CASE(1, 64, 1) TGKV_ATTN_CASE(1, 64, 2) TGKV_ATTN_CASE(1, 64, 4)
    TGKV_ATTN_CASE(1, 128, 1) TGKV_ATTN_CASE(1, 128, 2) TGKV_ATTN_CASE(1, 128, 4)
    TGKV_ATTN_CASE(1, 256, 1) TGKV_ATTN_CASE(1, 256, 2)
    return (int)cudaErrorInvalidValue;
}

extern "C" int tgkv_launch_append(const TGKvAppendParams* p, int dtype, void* stream) {
    const uint64_t vecs = (uint64_t)p->n_items * p->rows_per_item * (p->kv_dim / 8);
    if (vecs == 0) return 0;
    if (p->kv_dim % 8) return (int)cudaErrorInvalidValue;
    static const bool pdl = [] {
        const char* e = getenv("TGKV_PDL");
        return !(e && e[0] == '0');
    }();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((vecs + 255) / 256), 2);
    cfg.blockDim = dim3(256);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    if (dtype == 0) return (int)cudaLaunchKernelEx(&cfg, tgkv::append_kernel<0>, *p);
    return (int)cudaLaunchKernelEx(&cfg, tgkv::append_kernel<1>, *p);
}

namespace tgkv {
// Launched as a programmatic dependent of the attention: it starts spinning
// once the attention's CTAs have streamed their tiles (every rank's arrivals
// come from the attention's last, merging CTAs), so its launch overlaps the
// merges; it waits for the attention itself only at its end, so the next
// kernel, which waits for this one, also follows the attention.
__global__ void gather_wait_kernel(const uint32_t* flag, uint32_t target, int32_t* err) {
    if (threadIdx.x == 0) {
        const unsigned long long t0 = global_ns();
        for (;;) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
            if ((int32_t)(v - target) >= 0) break;
            if (global_ns() - t0 > kWaitLimitNs) {
                atomicExch(err, kErrGatherTimeout);
                break;
            }
            __nanosleep(64);
        }
    }
    __syncwarp();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
}  // namespace tgkv

extern "C" int tgkv_launch_gather_wait(const uint32_t* flag, uint32_t target, int32_t* err,
                                       void* stream) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = tgkv::pdl_enabled() ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, tgkv::gather_wait_kernel, flag, target, err);
}

namespace tgkv {
// Up to three page-locked host arrays (device-mapped pointers) copied into
// one device buffer back to back.  Every thread issues all its loads before
// any store, so the PCIe round trip is paid once.  Launched as a programmatic
// dependent that waits for nothing before its copies (the inputs are host
// data), it overlaps the previous kernel's tail; it waits for that kernel at
// its end, so a kernel waiting for this one also follows the previous one.
__global__ void __launch_bounds__(256) stage_host_kernel(const float4* __restrict__ a,
                                                         uint32_t na, const float4* __restrict__ b,
                                                         uint32_t nb, const float4* __restrict__ c,
                                                         uint32_t nc, float4* dst) {
    constexpr int kPer = 8;
    const uint32_t n = na + nb + nc;
    for (uint32_t base = blockIdx.x * 256u * kPer; base < n; base += gridDim.x * 256u * kPer) {
        float4 v[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const uint32_t i = base + u * 256u + threadIdx.x;
            v[u] = i < na ? a[i] : i < na + nb ? b[i - na] : i < n ? c[i - na - nb]
                                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const uint32_t i = base + u * 256u + threadIdx.x;
            if (i < n) dst[i] = v[u];
        }
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
}  // namespace tgkv

extern "C" int tgkv_launch_stage_host(const void* a, uint64_t na, const void* b, uint64_t nb,
                                      const void* c, uint64_t nc, void* dst, void* stream) {
    const uint64_t n4 = (na + nb + nc) / 16;
    if (!n4) return 0;
    uint64_t blocks = (n4 + 256 * 8 - 1) / (256 * 8);
    if (blocks > 148) blocks = 148;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = tgkv::pdl_enabled() ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, tgkv::stage_host_kernel,
                                   static_cast<const float4*>(a), (uint32_t)(na / 16),
                                   static_cast<const float4*>(b), (uint32_t)(nb / 16),
                                   static_cast<const float4*>(c), (uint32_t)(nc / 16),
                                   static_cast<float4*>(dst));
}

extern "C" int tgkv_launch_rope_append(const TGKvRopeParams* p, void* stream) {
    const uint64_t total = (uint64_t)p->n_tokens * p->n_heads * (p->head_dim / 2);
    if (total == 0) return 0;
    const unsigned grid = (unsigned)((total + 255) / 256);
    if (p->dtype == 0)
        tgkv::rope_append_kernel<0><<<grid, 256, 0, (cudaStream_t)stream>>>(*p);
    else
        tgkv::rope_append_kernel<1><<<grid, 256, 0, (cudaStream_t)stream>>>(*p);
    return (int)cudaGetLastError();
}

// ------------------------------------------------------------ no-allocation
// tg_kv_attention_static: the split-sequence attention for callers that may
// not allocate device memory -- code running where cudaMalloc is off limits
// (inside a host allocator hook, a real-time decode thread with a fixed memory
// budget, or an engine that hands this library only its own buffers).  Its
// scratch (the CTA partials, the arrival counters and an error word) lives in
// the file-scope device array below: 4 MiB that every GPU which loads this
// library holds until the process exits.  The cache's TMA tensor map travels
// in the kernel's parameter block, so a call copies nothing from the host.
extern "C" void tgkv_set_last_error(const char* msg);   // tgai_kv_cache.c

namespace tgkv {
namespace staticmem {

constexpr size_t kBytes = 4u << 20;
constexpr size_t kOffErr = 0;         // bounded-wait error word, kept until read
constexpr size_t kOffCounters = 256;  // arrival counters, then partials
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kBytes];

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_mu;
unsigned char* g_addr[kMaxDevices];   // device address of g_scratch, per device
int g_sms[kMaxDevices];
EncodeTiledFn g_encode = nullptr;
int g_stall_calls = 0;                // failure injection: calls left to stall

// 1 if this call is to launch with its loads stalled (failure injection).
uint32_t take_stall() {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_stall_calls <= 0) return 0;
    --g_stall_calls;
    return 1;
}

int fail(const char* fmt, ...) {
    char msg[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, sizeof(msg), fmt, ap);
    va_end(ap);
    tgkv_set_last_error(msg);
    return 0;
}

// Per-device set-up on the first call made with that device current: the
// array's device address (host code only sees a stand-in symbol) and the SM
// count used by the split planner.
bool setup(int dev) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_addr[dev]) return true;
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
    if (e != cudaSuccess || !ptr) {
        fail("tg_kv_attention_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        return false;
    }
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
        fail("tg_kv_attention_static: SM count query failed: %s", cudaGetErrorString(e));
        return false;
    }
    if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
                cudaSuccess || !fn) {
            fail("tg_kv_attention_static: cuTensorMapEncodeTiled unavailable");
            return false;
        }
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    g_sms[dev] = sms;
    g_addr[dev] = static_cast<unsigned char*>(ptr);
    return true;
}

}  // namespace staticmem
}  // namespace tgkv

extern "C" __attribute__((visibility("default"))) int tg_kv_attention_static(
    const void* kvc, int dtype, uint32_t max_seq, uint32_t n_kv_heads, uint32_t head_dim,
    uint32_t kv_len, const float* q, float* out, uint32_t n_heads, uint32_t n_q, void* stream) {
    using namespace tgkv::staticmem;
    if (!kvc || !q || !out) return fail("tg_kv_attention_static: null pointer");
    if (!tgkv_attention_supported(dtype, head_dim))
        return fail("tg_kv_attention_static: no kernel for dtype %d head_dim %u", dtype, head_dim);
    if (n_kv_heads == 0 || n_heads == 0 || n_heads % n_kv_heads)
        return fail("tg_kv_attention_static: n_heads %u is not a multiple of n_kv_heads %u",
                    n_heads, n_kv_heads);
    if (kv_len > max_seq || n_q == 0 || n_q > kv_len)
        return fail("tg_kv_attention_static: need 1 <= n_q (%u) <= kv_len (%u) <= max_seq (%u)",
                    n_q, kv_len, max_seq);
    if (n_q > TGKV_MAX_ITEMS)
        return fail("tg_kv_attention_static: n_q %u above the limit of %u query rows", n_q,
                    (unsigned)TGKV_MAX_ITEMS);
    const uint64_t es = dtype == 1 ? 2 : 4;
    const uint64_t kv_dim = (uint64_t)n_kv_heads * head_dim;
    if (((uintptr_t)kvc & 15u) || (((uintptr_t)q | (uintptr_t)out) & 7u))
        return fail("tg_kv_attention_static: kvc must be 16-byte and q/out 8-byte aligned");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail("tg_kv_attention_static: no usable current device");
    if (!setup(dev)) return 0;

    // Split plan: the rule tg_cuda_kv_attention uses (tgkv_pick_chunk).
    const uint32_t group = n_heads / n_kv_heads;
    const uint32_t gt = tgkv_attention_g_tile(head_dim, group);
    const uint32_t n_sub = group / gt;
    TGKvAttnParams p;                     // ~8 KB on the stack: no heap, no device memory
    memset(&p, 0, offsetof(TGKvAttnParams, n_pos));
    for (uint32_t t = 0; t < n_q; ++t) p.n_pos[t] = kv_len - n_q + t + 1;
    const uint64_t chunk = tgkv_pick_chunk(p.n_pos, n_q, n_kv_heads * n_sub, (uint32_t)g_sms[dev]);
    uint64_t n_chunks = 0;
    for (uint32_t t = 0; t < n_q; ++t) {
        const uint32_t np = p.n_pos[t];
        p.chunk_prefix[t] = (uint32_t)n_chunks;
        n_chunks += (uint64_t)((np + chunk - 1) / chunk) * n_kv_heads * n_sub;
    }
    if (n_chunks > 0x7fffffffu) return fail("tg_kv_attention_static: too many chunks");
    p.chunk_prefix[n_q] = (uint32_t)n_chunks;
    const uint64_t counters = ((uint64_t)n_q * n_kv_heads * n_sub * 4 + 255) / 256 * 256;
    const uint64_t part_o = (n_chunks * gt * head_dim * 4 + 255) / 256 * 256;
    const uint64_t need = kOffCounters + counters + part_o + n_chunks * gt * 2 * 4;
    if (need > kBytes)
        return fail("tg_kv_attention_static: needs %llu bytes of scratch, above the static "
                    "limit of %llu bytes (4 MiB); use tg_kv_attention or fewer query rows",
                    (unsigned long long)need, (unsigned long long)kBytes);
    const uint32_t grid = (uint32_t)n_chunks;

    // The cache's tensor map travels in the kernel's parameter block (tmap0);
    // only the arrival counters are cleared on the stream, since the
    // previous call's contents are still in the array.  The error word is
    // left alone: it keeps a failed call's code until
    // tg_kv_attention_static_error() has returned it.
    cuuint64_t dims[3] = {kv_dim, max_seq, 2};
    cuuint64_t strides[2] = {kv_dim * es, (uint64_t)max_seq * kv_dim * es};
    cuuint32_t box[3] = {head_dim, TGKV_TILE, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(&p.tmap0, dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                          3, const_cast<void*>(kvc), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail("tg_kv_attention_static: cuTensorMapEncodeTiled failed (%d)", (int)r);
    unsigned char* base = g_addr[dev];
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaMemsetAsync(base + kOffCounters, 0, counters, st);
    if (e != cudaSuccess)
        return fail("tg_kv_attention_static: clearing the counters failed: %s",
                    cudaGetErrorString(e));

    p.caches = nullptr;
    p.cache0.base = (uint64_t)(uintptr_t)kvc;
    p.cache0.max_seq = max_seq;
    p.cache0.tmap = 0;                     // the kernel uses p.tmap0
    p.q = q;
    p.out = out;
    p.counters = reinterpret_cast<uint32_t*>(base + kOffCounters);
    p.part_o = reinterpret_cast<float*>(base + kOffCounters + counters);
    p.part_ml = reinterpret_cast<float*>(base + kOffCounters + counters + part_o);
    p.err = reinterpret_cast<int32_t*>(base + kOffErr);
    p.cache_stride = 0;
    p.n_items = n_q;
    p.n_heads = n_heads;
    p.n_kv_heads = n_kv_heads;
    p.n_sub = n_sub;
    p.chunk = (uint32_t)chunk;
    p.qscale = (1.0f / sqrtf((float)head_dim)) * 1.4426950408889634f;
    p.item_base = 0;
    p.stall_loads = take_stall();
    const int rc = tgkv_launch_attention(&p, dtype, head_dim, gt, grid, stream);
    if (rc != 0)
        return fail("tg_kv_attention_static: launch failed: %s",
                    cudaGetErrorString((cudaError_t)rc));
    return 1;
}

// The error word of the static array on the current device: 0 when every
// call so far finished its waits, else the code of a wait that ran out.
// Waits for `stream` first; clears the word once it has been returned.
extern "C" __attribute__((visibility("default"))) int tg_kv_attention_static_error(void* stream) {
    using namespace tgkv::staticmem;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    unsigned char* base;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        base = g_addr[dev];
    }
    if (!base) return 0;                  // no call was made on this device
    cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
    int32_t v = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&v, base + kOffErr, sizeof(v), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && v) e = cudaMemset(base + kOffErr, 0, sizeof(v));
    if (e != cudaSuccess) {
        fail("tg_kv_attention_static_error: %s", cudaGetErrorString(e));
        return -1;
    }
    return v;
}

// Failure injection for tests: the next n_calls calls of
// tg_kv_attention_static launch with the producer issuing no loads, so each
// of their waits runs out after its bound (about 2 s) and records its code.
extern "C" __attribute__((visibility("default"))) void tg_kv_attention_static_inject_stall(
    int n_calls) {
    using namespace tgkv::staticmem;
    std::lock_guard<std::mutex> lock(g_mu);
    g_stall_calls = n_calls > 0 ? n_calls : 0;
}
