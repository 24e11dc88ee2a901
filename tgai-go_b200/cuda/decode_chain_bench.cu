// decode_chain_bench.cu -- live per-launch time of the whole-model decode
// kernels (tgkv_forward.cu) and of the decode attention, each launched 28
// times in a row as programmatic dependents over 28 layers' weights, so that
// no launch finds its weights in L2.  CUDA events around each chain of 28
// launches; the best and the mean of 10 chains, after 3 untimed chains and a
// 256 MB write between chains.
//
// Shapes: the V2.7-shaped MoE of bench.py --workload fwd (d_model 1536,
// 12 query / 4 KV heads of 128, 8 experts top-2 of d_ff 2560, vocab 32000),
// one decode token at context 541.  With --floors it first times a plain read
// kernel (16-byte loads, one warp per 6 KB row) over the same byte counts and
// grid sizes: the floor a launch of that many bytes has in such a chain.
//
//   make -C tgai-go_b200 decode_chain_bench
//   tgai-go_b200/_build/decode_chain_bench [--floors]
#include "tgkv_forward.cu"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "tgai_backend.h"
#include "tgai_kv_cache.h"

namespace {

constexpr uint32_t kD = 1536, kQDim = 1536, kKvDim = 512, kHd = 128, kDff = 2560, kNe = 8,
                   kNa = 2, kMaxSeq = 2048, kLayers = 28, kVocab = 32000, kPos = 540;

__global__ void fill_kernel(float* p, uint64_t n, uint32_t seed, float scale) {
    for (uint64_t i = blockIdx.x * 256ull + threadIdx.x; i < n; i += gridDim.x * 256ull) {
        uint32_t h = (uint32_t)i * 2654435761u ^ seed;
        h ^= h >> 13;
        h *= 0x5bd1e995u;
        h ^= h >> 15;
        p[i] = ((h & 0xffff) / 65536.0f - 0.5f) * scale;
    }
}

float* dev_fill(uint64_t n, uint32_t seed, float scale) {
    float* p = nullptr;
    if (cudaMalloc(&p, n * 4) != cudaSuccess) {
        fprintf(stderr, "cudaMalloc of %llu floats failed\n", (unsigned long long)n);
        exit(1);
    }
    fill_kernel<<<1184, 256>>>(p, n, seed, scale);
    return p;
}

// Reads nrows rows of K floats (one warp per row, kU 16-byte loads per lane in
// flight) and keeps the sum only so that the loads are not removed.
template <int kU>
__global__ void __launch_bounds__(256) read_kernel(const float* __restrict__ w, uint32_t nrows,
                                                   uint32_t K, float* out) {
    pdl_wait();
    pdl_trigger();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float s = 0.f;
    for (uint32_t n = blockIdx.x * 8 + warp; n < nrows; n += gridDim.x * 8) {
        const float* r = w + (uint64_t)n * K;
        for (uint32_t i0 = lane * 4; i0 < K; i0 += kU * 128) {
            float4 v[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u)
                v[u] = i0 + u * 128 < K ? __ldg(reinterpret_cast<const float4*>(r + i0 + u * 128))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int u = 0; u < kU; ++u) s += (v[u].x + v[u].y) + (v[u].z + v[u].w);
        }
    }
    if (s == 1234.5f) out[0] = s;
}

struct LayerW {
    float *wqkv, *bqkv, *wo, *w12, *w3, *router, *ln1, *ln2;
};

}  // namespace

int main(int argc, char** argv) {
    const bool floors = argc > 1 && strcmp(argv[1], "--floors") == 0;
    std::vector<LayerW> L(kLayers);
    for (uint32_t l = 0; l < kLayers; l++) {
        L[l].wqkv = dev_fill((uint64_t)(kQDim + 2 * kKvDim) * kD, 1 + l, 0.05f);
        L[l].bqkv = dev_fill(kQDim + 2 * kKvDim, 100 + l, 0.01f);
        L[l].wo = dev_fill((uint64_t)kD * kQDim, 200 + l, 0.05f);
        L[l].w12 = dev_fill((uint64_t)kNe * 2 * kDff * kD, 300 + l, 0.05f);
        L[l].w3 = dev_fill((uint64_t)kNe * kD * kDff, 400 + l, 0.05f);
        L[l].router = dev_fill((uint64_t)kNe * kD, 500 + l, 0.5f);
        L[l].ln1 = dev_fill(kD, 600 + l, 2.0f);
        L[l].ln2 = dev_fill(kD, 700 + l, 2.0f);
    }
    float* emb = dev_fill((uint64_t)kVocab * kD, 9, 0.05f);
    float* fnorm = dev_fill(kD, 10, 2.0f);
    float* x = dev_fill(kD * 4, 11, 1.0f);
    float* q = dev_fill(kQDim * 4, 12, 1.0f);
    float* attn = dev_fill(kQDim * 4, 13, 1.0f);
    float* h = dev_fill(kDff * 8, 14, 1.0f);
    float* cs = dev_fill((uint64_t)kMaxSeq * kHd / 2, 16, 1.0f);
    float* sn = dev_fill((uint64_t)kMaxSeq * kHd / 2, 17, 1.0f);
    float* logits = dev_fill(kVocab, 18, 1.0f);
    float* top_w = nullptr;
    int32_t* top_ids = nullptr;
    float* flush = nullptr;
    if (cudaMalloc(&top_w, 64) || cudaMalloc(&top_ids, 64) || cudaMalloc(&flush, 256 << 20)) {
        fprintf(stderr, "cudaMalloc failed\n");
        return 1;
    }
    cudaMemset(top_ids, 0, 64);
    cudaMemset(top_w, 0, 64);
    if (!tg_be_select("cuda")) {
        fprintf(stderr, "no CUDA backend\n");
        return 1;
    }
    std::vector<TGKvCache*> kc(kLayers);
    for (uint32_t l = 0; l < kLayers; l++) {
        kc[l] = tg_kv_create(kMaxSeq, kKvDim / kHd, kHd);
        if (!kc[l]) {
            fprintf(stderr, "tg_kv_create: %s\n", tg_kv_last_error());
            return 1;
        }
        tg_kv_advance(kc[l], kPos + 1);
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return 1;
    cudaStream_t st;
    cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    // a first routing so that the W3 launches read valid expert ids
    tgkv_fwd_dec_moe_w12(x, L[0].ln2, L[0].router, nullptr, L[0].w12, top_ids, top_w, h, 1, kD,
                         kDff, kNe, kNa, nullptr, st);

    int failed = 0;
    auto run = [&](const char* name, auto launch) {
        for (int rep = 0; rep < 3; rep++)
            for (uint32_t l = 0; l < kLayers; l++) failed |= launch(l) != 0;
        cudaStreamSynchronize(st);
        float best = 1e30f, tot = 0.f;
        for (int rep = 0; rep < 10; rep++) {
            cudaMemsetAsync(flush, rep, 256 << 20, st);
            cudaEventRecord(e0, st);
            for (uint32_t l = 0; l < kLayers; l++) failed |= launch(l) != 0;
            cudaEventRecord(e1, st);
            cudaEventSynchronize(e1);
            float ms = 0.f;
            cudaEventElapsedTime(&ms, e0, e1);
            best = ms < best ? ms : best;
            tot += ms;
        }
        const cudaError_t err = cudaGetLastError();
        failed |= err != cudaSuccess;
        printf("%-34s %8.2f us per launch (best of 10 chains)  %8.2f mean  %s\n", name,
               best * 1000.f / kLayers, tot * 100.f / kLayers, cudaGetErrorString(err));
    };

    if (floors) {
        const uint64_t rows_per_layer = 65536;   // 403 MB of 1536-float rows per layer
        float* big = dev_fill((uint64_t)kLayers * rows_per_layer * kD, 77, 1.0f);
        cudaDeviceSynchronize();
        struct F { const char* name; uint32_t rows, grid; };
        const F fl[] = {{"read 15.7 MB, 160 CTAs", 2560, 160},  {"read 15.7 MB, 320 CTAs", 2560, 320},
                        {"read 9.4 MB, 192 CTAs", 1536, 192},   {"read 63 MB, 640 CTAs", 10240, 640},
                        {"read 63 MB, 1280 CTAs", 10240, 1280}, {"read 63 MB, 296 CTAs", 10240, 296},
                        {"read 403 MB, 592 CTAs", 65536, 592}};
        for (const F& f : fl)
            run(f.name, [&](uint32_t l) {
                return launch_pdl(read_kernel<8>, dim3(f.grid), 0, st,
                                  big + (uint64_t)l * rows_per_layer * kD, f.rows, kD, logits);
            });
        cudaFree(big);
    }
    run("attention (fp32 cache, L 541)", [&](uint32_t l) {
        return tg_kv_attention(kc[l], q, attn, kQDim / kHd, 1, st) ? 0 : 1;
    });
    run("qkv + rope + append", [&](uint32_t l) {
        return tgkv_fwd_dec_qkv_rope(L[l].wqkv, x, L[l].ln1, L[l].bqkv, cs, sn, q,
                                     (float*)tg_kv_device_handle(kc[l]), 1, kD, kQDim, kKvDim, kHd,
                                     kPos, kMaxSeq, nullptr, 0, st);
    });
    run("out projection + residual", [&](uint32_t l) {
        return tgkv_fwd_dec_gemv(1, L[l].wo, attn, kQDim, nullptr, nullptr, x, kD, 1, kD, kQDim, 0,
                                 nullptr, 0, st);
    });
    run("router + experts W1/W2", [&](uint32_t l) {
        return tgkv_fwd_dec_moe_w12(x, L[l].ln2, L[l].router, nullptr, L[l].w12, top_ids, top_w, h,
                                    1, kD, kDff, kNe, kNa, nullptr, st);
    });
    run("experts W3 + combine", [&](uint32_t l) {
        return tgkv_fwd_dec_w3_combine(L[l].w3, h, top_ids, top_w, x, 1, kD, kDff, kNe, kNa,
                                       nullptr, 0, st);
    });
    run("layer (5 launches)", [&](uint32_t l) {
        int e = tgkv_fwd_dec_qkv_rope(L[l].wqkv, x, L[l].ln1, L[l].bqkv, cs, sn, q,
                                      (float*)tg_kv_device_handle(kc[l]), 1, kD, kQDim, kKvDim,
                                      kHd, kPos, kMaxSeq, nullptr, 0, st);
        e |= tg_kv_attention(kc[l], q, attn, kQDim / kHd, 1, st) ? 0 : 1;
        e |= tgkv_fwd_dec_gemv(1, L[l].wo, attn, kQDim, nullptr, nullptr, x, kD, 1, kD, kQDim, 0,
                               nullptr, 0, st);
        e |= tgkv_fwd_dec_moe_w12(x, L[l].ln2, L[l].router, nullptr, L[l].w12, top_ids, top_w, h,
                                  1, kD, kDff, kNe, kNa, nullptr, st);
        e |= tgkv_fwd_dec_w3_combine(L[l].w3, h, top_ids, top_w, x, 1, kD, kDff, kNe, kNa, nullptr,
                                     0, st);
        return e;
    });
    // one LM head per chain: the printed time is per layer-slot, x 28 per launch
    run("LM head / 28", [&](uint32_t l) {
        return l ? 0 : tgkv_fwd_dec_gemv(0, emb, x, kD, fnorm, nullptr, logits, kVocab, 1, kVocab,
                                         kD, 0, nullptr, 0, st);
    });
    for (TGKvCache* c : kc) tg_kv_destroy(c);
    return failed;
}
