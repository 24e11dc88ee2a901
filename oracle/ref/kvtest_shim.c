/* kvtest_shim.c -- compiles the reference's KV-cache GPU test
 * (tests/test_kv_cache_gpu.c) UNMODIFIED, with its main() renamed, so that its
 * double-precision cpu_attention (test_kv_cache_gpu.c:21-54) can produce golden
 * outputs.  The Vulkan symbols it references stay unresolved and are never
 * called (the library is opened with RTLD_LAZY).  TEST INFRASTRUCTURE ONLY. */
#define main tgref_kvtest_main
#include "test_kv_cache_gpu.c"
#undef main

void tgref_cpu_attention_kvtest(const float* q, const float* kv, float* out,
                                int nh, int nkvh, int hd, int n_kv, int pos,
                                int max_seq) {
    cpu_attention(q, kv, out, nh, nkvh, hd, n_kv, pos, max_seq);
}
