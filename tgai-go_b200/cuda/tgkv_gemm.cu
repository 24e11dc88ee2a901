// tgkv_gemm.cu -- fp32 GEMM on the sm_100a tensor cores at fp32-product
// accuracy, for the forward's prefill projections (the reference bridge runs
// them as cublasSgemm, cuda/tgai_cuda.cu:473-479).
//
//   out[M][N] (+)= A[M][K] . W[N][K]^T
//
// Both operands arrive split in two: big = the value rounded to tf32 (10
// mantissa bits, low 13 bits zero) and small = value - big (exact in fp32).
// The product is A_big.W_big + A_big.W_small + A_small.W_big; the dropped
// A_small.W_small term is below 2^-22 of |a||w|, and the tf32 rounding the
// tensor core applies to `small` costs about as much, so every product is
// good to about 2^-21.  One pipeline stage holds all four tiles of a k-block
// (A_big, A_small, W_big, W_small), each loaded once, and the MMA thread
// issues the three products from it.  The tensor core's fp32 accumulation
// truncates at every step, relative to the accumulator's magnitude, so the
// two small cross terms go to an accumulator of their own (about 2^-11 of
// the result) and the big products are dealt round-robin over the rest of
// TMEM (512 / BN - 1 accumulators); the epilogue adds them in IEEE fp32, so
// every accumulator sees a fraction of the steps at a fraction of the
// magnitude.
//
// One CTA (128 threads) per 128 x BN output tile.  Lane 0 of warp 0 moves
// 128x32 (A) and BNx32 (W) fp32 tiles with 128-byte-swizzled tiled TMA into
// a ring of stages (mbarrier completion); lane 0 of warp 1 issues
// tcgen05.mma kind::tf32 (M = 128, N = BN, K = 8; twelve per k-block) into
// TMEM accumulators and releases each stage with tcgen05.commit; then all
// four warps read their 32 TMEM lanes (rows) and store or accumulate the
// output rows.  Rows past M and columns past N arrive as zeros (TMA bounds)
// and are not stored.  Every wait is bounded (about 2 s): on expiry the
// kernel records an error code, lets its own copies land and MMAs finish,
// frees its TMEM and stores nothing.

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>
#include <mutex>

#include "tgkv_forward.h"
#include "tgkv_ptx.cuh"

namespace tgkv {
namespace gemm {

constexpr int kErrFull = 1, kErrEmpty = 2, kErrDone = 3;
constexpr int kBM = 128, kBK = 32;            // rows per tile, fp32 elements per k-block
constexpr int kABytes = kBM * kBK * 4;        // 16 KB

template <int BN>
struct Cfg {
    static constexpr int BBytes = BN * kBK * 4;
    // a stage: A_big, A_small, W_big, W_small of one k-block
    static constexpr int OffAs = kABytes, OffWb = 2 * kABytes, OffWs = 2 * kABytes + BBytes;
    static constexpr int Stage = 2 * kABytes + 2 * BBytes;
    static constexpr int NStage = (196608 / Stage) > 8 ? 8 : (196608 / Stage);
    static constexpr int OffBar = NStage * Stage;
    static constexpr int Smem = OffBar + (2 * NStage + 2) * 8 + 16 + 1024;   // + alignment slack
    static constexpr int NAcc = 512 / BN;              // accumulators: all 512 TMEM columns,
    static constexpr int NBig = NAcc - 1;              //   the first for the cross terms
    static constexpr uint32_t TmemCols = 512;
};

// Instruction descriptor, kind::tf32: D f32 (bits 4-5 = 1), A and B tf32
// (format 2 in bits 7-9 and 10-12), both K-major, N >> 3 at 17, M >> 4 at 24.
__host__ __device__ constexpr uint32_t idesc_tf32(uint32_t m, uint32_t n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

template <int BN>
__global__ void __launch_bounds__(128, 1) gemm_tf32x3_kernel(const __grid_constant__ TGGemmParams p) {
    using C = Cfg<BN>;
    extern __shared__ unsigned char smem_raw[];
    // 128-byte swizzled tiles want 1024-byte aligned stage bases
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OffBar);
    uint64_t* empty = full + C::NStage;
    uint64_t* done = empty + C::NStage;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t n0 = blockIdx.x * BN, m0 = blockIdx.y * kBM;
    const int nkb = (int)((p.K + kBK - 1) / kBK);
    const int total = nkb;

    if (tid == 0) {
        for (int s = 0; s < C::NStage; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.a_big)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.w_big)) : "memory");
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the inputs come from the kernels before this one on the stream
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // this CTA's rows: the whole A (plain), or its group's packed rows
    uint32_t M = p.M, a_row0 = 0, w_row0 = 0;
    if (p.group_count) {
        M = p.group_count[blockIdx.z];
        a_row0 = p.group_off[blockIdx.z];
        w_row0 = blockIdx.z * p.N;
    }
    const bool active = m0 < M;               // CTA-uniform

    if (!active) {
        // a tile past its group's rows: nothing to load, multiply or store
    } else if (warp == 0 && lane == 0) {
        // ---------------- producer
        int issued = 0;
        for (int kb = 0; kb < total; ++kb) {
            const int s = kb % C::NStage;
            if (kb >= C::NStage && !mbar_wait(&empty[s], ((kb / C::NStage) - 1) & 1)) {
                atomicExch(p.err, kErrEmpty);
                *abort_flag = 1;
                break;
            }
            if (*reinterpret_cast<volatile int*>(abort_flag)) break;
            const int kx = kb * kBK;
            unsigned char* st = smem + s * C::Stage;
            mbar_arrive_expect_tx(&full[s], (uint32_t)C::Stage);
            tma_load_2d(st, &p.a_big, kx, (int)(a_row0 + m0), &full[s]);
            tma_load_2d(st + C::OffAs, &p.a_small, kx, (int)(a_row0 + m0), &full[s]);
            tma_load_2d(st + C::OffWb, &p.w_big, kx, (int)(w_row0 + n0), &full[s]);
            tma_load_2d(st + C::OffWs, &p.w_small, kx, (int)(w_row0 + n0), &full[s]);
            ++issued;
        }
        // the last stages' copies land before this thread may leave
        for (int kb = issued > C::NStage ? issued - C::NStage : 0; kb < issued; ++kb)
            if (!mbar_wait(&full[kb % C::NStage], (kb / C::NStage) & 1))
                atomicExch(p.err, kErrFull);
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issue
        constexpr uint32_t idesc = idesc_tf32(kBM, BN);
        for (int kb = 0; kb < total; ++kb) {
            const int s = kb % C::NStage;
            if (!mbar_wait(&full[s], (kb / C::NStage) & 1)) {
                atomicExch(p.err, kErrFull);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t ab = smem_addr(smem + s * C::Stage);
            const uint32_t as = ab + C::OffAs, wb = ab + C::OffWb, ws = ab + C::OffWs;
            const uint32_t big = tmem + (uint32_t)((1 + kb % C::NBig) * BN);
#pragma unroll
            for (int k = 0; k < kBK / 8; ++k) {        // K = 8 tf32 = 32 bytes per MMA
                const uint64_t dab = umma_desc_sw128(ab + 32 * k, 16, 1024);
                const uint64_t dwb = umma_desc_sw128(wb + 32 * k, 16, 1024);
                umma_tf32(tmem, umma_desc_sw128(as + 32 * k, 16, 1024), dwb, idesc,
                          (kb > 0) || (k > 0));
                umma_tf32(tmem, dab, umma_desc_sw128(ws + 32 * k, 16, 1024), idesc, 1u);
                umma_tf32(big, dab, dwb, idesc, (kb >= C::NBig) || (k > 0));
            }
            umma_commit(&empty[s]);                    // the stage is free once these are done
        }
        umma_commit(done);                             // every MMA issued so far is done
    }
    __syncwarp();

    // ---------------- epilogue: warp w holds rows m0 + 32w .. + 31
    const bool ok = !active || mbar_wait(done, 0);
    if (!ok && lane == 0) atomicExch(p.err, kErrDone);
    tc_fence_after();
    // let the next kernel on the stream start its prologue
    if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bool store = active && ok && !*reinterpret_cast<volatile int*>(abort_flag);
    const uint32_t row = m0 + 32 * warp + lane;
    const uint32_t orow_i = !p.group_count ? row
                            : p.out_rows ? (row < M ? p.out_rows[a_row0 + row] : 0u)
                                         : a_row0 + row;
    float* orow = p.out + (uint64_t)orow_i * p.ldo;
    const bool vec = (p.ldo % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.out) & 15) == 0);
    const int n_acc = 1 + (total < C::NBig ? total : C::NBig);   // accumulators written
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
        const uint32_t col0 = n0 + 32 * c;
        if (col0 >= p.N || !active) break;             // warp-uniform
        uint32_t r[32];
        const uint32_t t = tmem + ((uint32_t)(32 * warp) << 16) + 32 * c;
        tmem_ld32(t, r);
        tmem_wait_ld(r);
#pragma unroll 1
        for (int a = 1; a < n_acc; ++a) {
            uint32_t q[32];
            tmem_ld32(t + (uint32_t)(a * BN), q);
            tmem_wait_ld(q);
#pragma unroll
            for (int j = 0; j < 32; ++j)
                r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(q[j]));
        }
        if (!store || row >= M) continue;
        if (vec && col0 + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                       __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                float4* dst = reinterpret_cast<float4*>(orow + col0 + j);
                if (p.accumulate) {
                    const float4 o = *dst;
                    v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
                }
                *dst = v;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                if (col0 + j < p.N) {
                    const float v = __uint_as_float(r[j]);
                    orow[col0 + j] = p.accumulate ? orow[col0 + j] + v : v;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, C::TmemCols);
}

// big = x rounded to tf32 (nearest, ties away from zero), small = x - big.
__global__ void split_tf32_kernel(const float* __restrict__ x, uint64_t ldx, float* big,
                                  float* small, uint64_t ldo, uint32_t rows, uint32_t cols) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint64_t n = (uint64_t)rows * cols;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / cols, c = i % cols;
        const float v = x[r * ldx + c];
        uint32_t b;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(b) : "f"(v));
        const float bf = __uint_as_float(b);
        big[r * ldo + c] = bf;
        small[r * ldo + c] = v - bf;
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::once_flag g_once;
EncodeTiledFn g_encode = nullptr;
int g_attr_done[64];
std::mutex g_mu;

// 2-D map over rows x cols fp32 (row stride ld elements), box 32 x box_rows,
// 128-byte swizzle.
bool encode(CUtensorMap* m, const float* base, uint64_t ld, uint32_t rows, uint32_t cols,
            uint32_t box_rows) {
    std::call_once(g_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess)
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    });
    if (!g_encode) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 4};
    cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
int launch(const TGGemmParams* p, void* stream) {
    using C = Cfg<BN>;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lock(g_mu);
        const int bit = BN == 128 ? 1 : 2;
        if (dev >= 0 && dev < 64 && !(g_attr_done[dev] & bit)) {
            const cudaError_t e = cudaFuncSetAttribute(
                gemm_tf32x3_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::Smem);
            if (e != cudaSuccess) return (int)e;
            g_attr_done[dev] |= bit;
        }
    }
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = p->group_count
                      ? dim3((p->N + BN - 1) / BN, (p->max_rows + kBM - 1) / kBM, p->groups)
                      : dim3((p->N + BN - 1) / BN, (p->M + kBM - 1) / kBM, 1);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.dynamicSmemBytes = C::Smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&cfg, gemm_tf32x3_kernel<BN>, *p);
}

}  // namespace gemm
}  // namespace tgkv

extern "C" int tgkv_gemm_encode(TGGemmParams* p, const float* a_big, const float* a_small,
                                uint64_t lda, const float* w_big, const float* w_small,
                                uint64_t ldw, float* out, uint64_t ldo, uint32_t M, uint32_t N,
                                uint32_t K, int accumulate, int32_t* err) {
    using namespace tgkv::gemm;
    memset(p, 0, sizeof(*p));
    if (!M || !N || !K || (K % 4) || (lda % 4) || (ldw % 4) || ldo < N || !err) return 0;
    const uint32_t bn = tgkv_gemm_bn(M, N);
    if (!encode(&p->a_big, a_big, lda, M, K, kBM) || !encode(&p->a_small, a_small, lda, M, K, kBM) ||
        !encode(&p->w_big, w_big, ldw, N, K, bn) || !encode(&p->w_small, w_small, ldw, N, K, bn))
        return 0;
    p->out = out;
    p->ldo = ldo;
    p->M = M;
    p->N = N;
    p->K = K;
    p->accumulate = accumulate;
    p->err = err;
    return 1;
}

extern "C" uint32_t tgkv_gemm_bn(uint32_t M, uint32_t N) {
    // 128-wide tiles unless they would leave most SMs idle
    const uint64_t tiles = (uint64_t)((N + 127) / 128) * ((M + 127) / 128);
    return tiles >= 74 ? 128u : 64u;
}

static uint32_t launch_bn(const TGGemmParams* p) {
    return p->group_count ? tgkv_gemm_bn(p->max_rows * p->groups, p->N) : tgkv_gemm_bn(p->M, p->N);
}

extern "C" int tgkv_gemm_launch(const TGGemmParams* p, void* stream) {
    return launch_bn(p) == 128 ? tgkv::gemm::launch<128>(p, stream)
                               : tgkv::gemm::launch<64>(p, stream);
}

extern "C" int tgkv_gemm_encode_grouped(TGGemmParams* p, const float* a_big, const float* a_small,
                                        uint32_t a_rows, const float* w_big, const float* w_small,
                                        uint32_t groups, uint32_t N, uint32_t K, float* out,
                                        uint64_t ldo, const uint32_t* group_count,
                                        const uint32_t* group_off, const uint32_t* out_rows,
                                        uint32_t max_rows, int32_t* err) {
    using namespace tgkv::gemm;
    memset(p, 0, sizeof(*p));
    if (!a_rows || !groups || !N || !K || (K % 4) || ldo < N || !err || !group_count ||
        !group_off || !max_rows || (uint64_t)groups * N > 0x7fffffffu)
        return 0;
    p->group_count = group_count;
    p->group_off = group_off;
    p->out_rows = out_rows;
    p->groups = groups;
    p->max_rows = max_rows;
    p->N = N;
    const uint32_t bn = launch_bn(p);
    if (!encode(&p->a_big, a_big, K, a_rows, K, kBM) ||
        !encode(&p->a_small, a_small, K, a_rows, K, kBM) ||
        !encode(&p->w_big, w_big, K, groups * N, K, bn) ||
        !encode(&p->w_small, w_small, K, groups * N, K, bn))
        return 0;
    p->out = out;
    p->ldo = ldo;
    p->M = max_rows;
    p->K = K;
    p->accumulate = 0;
    p->err = err;
    return 1;
}

namespace tgkv {
namespace gemm {

__device__ __forceinline__ void split1(float v, float& b, float& s) {
    uint32_t u;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(v));
    b = __uint_as_float(u);
    s = v - b;
}

// Packed row r: the expert e with off[e] <= r < off[e] + counts[e] (off the
// prefix sums, each CTA computes them; at most 16 experts), slot i = r -
// off[e], pair q = lists[e * seq * na + i], token q / na.  One CTA per 8
// rows, a warp per row.
__global__ void __launch_bounds__(256) moe_pack_kernel(const uint32_t* counts,
                                                       const uint32_t* lists, const float* x,
                                                       uint32_t d, uint32_t seq, uint32_t ne,
                                                       uint32_t na, float* a_big, float* a_small,
                                                       uint32_t* offs, uint32_t* rows) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __shared__ uint32_t s_off[17];
    if (threadIdx.x == 0) {
        uint32_t o = 0;
        for (uint32_t e = 0; e < ne; ++e) {
            s_off[e] = o;
            o += counts[e];
        }
        s_off[ne] = o;
        if (blockIdx.x == 0)
            for (uint32_t e = 0; e < ne; ++e) offs[e] = s_off[e];
    }
    __syncthreads();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * 8 + warp;
    if (r < s_off[ne]) {
        uint32_t e = 0;
        while (e + 1 < ne && s_off[e + 1] <= r) ++e;
        const uint32_t q = lists[(uint64_t)e * seq * na + (r - s_off[e])];
        if (lane == 0) rows[r] = q;
        const float4* src = reinterpret_cast<const float4*>(x + (uint64_t)(q / na) * d);
        float4* db = reinterpret_cast<float4*>(a_big + (uint64_t)r * d);
        float4* ds = reinterpret_cast<float4*>(a_small + (uint64_t)r * d);
        for (uint32_t i = lane; i < d / 4; i += 32) {
            const float4 v = src[i];
            float4 b, sm;
            split1(v.x, b.x, sm.x);
            split1(v.y, b.y, sm.y);
            split1(v.z, b.z, sm.z);
            split1(v.w, b.w, sm.w);
            db[i] = b;
            ds[i] = sm;
        }
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__global__ void __launch_bounds__(256) moe_silu_kernel(const float* ab, const uint32_t* counts,
                                                       uint32_t ne, uint32_t dff, float* h_big,
                                                       float* h_small) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    uint32_t n = 0;
    for (uint32_t e = 0; e < ne; ++e) n += counts[e];
    const uint64_t total = (uint64_t)n * dff;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / dff, j = i % dff;
        const float a = ab[r * 2 * dff + j], b = ab[r * 2 * dff + dff + j];
        const float h = (a / (1.0f + expf(-a))) * b;        // the expert FFN's SiLU, no clamp
        float hb, hs;
        split1(h, hb, hs);
        h_big[r * dff + j] = hb;
        h_small[r * dff + j] = hs;
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

int launch_simple(const void* fn, dim3 grid, void** args, void* stream) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace gemm
}  // namespace tgkv

extern "C" int tgkv_moe_pack_split(const uint32_t* counts, const uint32_t* lists, const float* x,
                                   uint32_t d, uint32_t seq, uint32_t ne, uint32_t na,
                                   float* a_big, float* a_small, uint32_t* offs, uint32_t* rows,
                                   void* stream) {
    if (!ne || ne > 16 || d % 4 || !seq || !na) return (int)cudaErrorInvalidValue;
    const uint32_t max_rows = seq * na;
    void* args[] = {&counts, &lists, &x, &d, &seq, &ne, &na, &a_big, &a_small, &offs, &rows};
    return tgkv::gemm::launch_simple((const void*)tgkv::gemm::moe_pack_kernel,
                                     dim3((max_rows + 7) / 8), args, stream);
}

extern "C" int tgkv_moe_silu_split(const float* ab, const uint32_t* counts, uint32_t ne,
                                   uint32_t max_rows, uint32_t dff, float* h_big, float* h_small,
                                   void* stream) {
    if (!ne || ne > 16 || !dff) return (int)cudaErrorInvalidValue;
    uint64_t blocks = ((uint64_t)max_rows * dff + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    void* args[] = {&ab, &counts, &ne, &dff, &h_big, &h_small};
    return tgkv::gemm::launch_simple((const void*)tgkv::gemm::moe_silu_kernel,
                                     dim3((unsigned)blocks), args, stream);
}

extern "C" int tgkv_split_tf32(const float* x, uint64_t ldx, float* big, float* small,
                               uint64_t ldo, uint32_t rows, uint32_t cols, void* stream) {
    const uint64_t n = (uint64_t)rows * cols;
    if (!n) return 0;
    uint64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3((unsigned)blocks, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return (int)cudaLaunchKernelEx(&cfg, tgkv::gemm::split_tf32_kernel, x, ldx, big, small, ldo,
                                   rows, cols);
}
