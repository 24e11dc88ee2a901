/* attntest_shim.c -- compiles the reference's attention kernel test
 * (tests/test_vk_attn_moe.c) UNMODIFIED, main() renamed, to expose its
 * double-precision cpu_attention (test_vk_attn_moe.c:38-73).  Vulkan symbols
 * stay unresolved and uncalled (RTLD_LAZY).  TEST INFRASTRUCTURE ONLY. */
#define main tgref_attntest_main
#include "test_vk_attn_moe.c"
#undef main

void tgref_cpu_attention_attntest(const float* q, const float* kvc, float* out,
                                  int nh, int nkvh, int hd, int n_kv, int pos,
                                  int max_seq) {
    cpu_attention(q, kvc, out, nh, nkvh, hd, n_kv, pos, max_seq);
}
