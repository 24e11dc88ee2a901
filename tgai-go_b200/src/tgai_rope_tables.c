/* tgai_rope_tables.c -- RoPE cos/sin tables for TGBackend.rope, including the
 * engine's context extension (NTK-by-parts with the YaRN attention
 * temperature), so the rotated K written into the cache is bit-identical to
 * the engine's own rope() (src/tgai_engine.c:3404-3460).
 *
 * The engine evaluates the table entries inside its rotation loop; this file
 * evaluates the same float expressions once per (position, pair).  Where the
 * reference's gcc -mfma build fuses a multiply into an add, the fused form is
 * written out with fmaf() (compiled with -ffp-contract=off), so the tables do
 * not depend on this compiler's contraction choices.
 */
#include "tgai_kv_cache.h"

#include <math.h>
#include <stddef.h>

/* src/tgai_engine.c:3370-3376 */
static float yarn_ramp(float low, float high, int j) {
    if (high <= low) return 0.0f;
    float y = ((float)j - low) / (high - low);
    if (y < 0.0f) y = 0.0f;
    if (y > 1.0f) y = 1.0f;
    return 1.0f - y;
}

int tg_kv_rope_tables(float theta, uint32_t head_dim, uint32_t pos0, uint32_t n_pos,
                      uint32_t extend_ctx, uint32_t max_seq_len, float* cos_out,
                      float* sin_out, float* mscale_out) {
    if (head_dim == 0 || (head_dim & 1) || !cos_out || !sin_out) return 0;
    const int d_k = (int)head_dim;
    int use_ntk = (extend_ctx > max_seq_len && max_seq_len > 0);
    float inv_scale = 1.0f, dim_high = 0.0f, dim_low = 0.0f, yarn_mscale = 1.0f;
    if (use_ntk) {                                   /* tgai_engine.c:3413-3436 */
        const float scale = (float)extend_ctx / (float)max_seq_len;
        inv_scale = 1.0f / scale;
        yarn_mscale = fmaf(0.1f, logf(scale), 1.0f);
        if (yarn_mscale < 1.0f) yarn_mscale = 1.0f;
        const float alpha_slow = 1.0f, beta_fast = 32.0f, two_pi = 6.2831853f;
        const float log_theta = logf(theta);
        if (log_theta > 0.0f) {
            const float L = (float)max_seq_len;
            const float half_dk = (float)d_k / 2.0f;
            dim_high = half_dk * logf(L / (two_pi * beta_fast)) / log_theta;
            dim_low = half_dk * logf(L / (two_pi * alpha_slow)) / log_theta;
            if (dim_high > dim_low) {
                const float t = dim_high;
                dim_high = dim_low;
                dim_low = t;
            }
        } else {
            use_ntk = 0;
        }
    }
    if (mscale_out) *mscale_out = use_ntk ? yarn_mscale : 1.0f;
    const int half = d_k / 2;
    for (int i = 0; i < d_k; i += 2) {               /* tgai_engine.c:3446-3459 */
        const float freq_extrap = 1.0f / powf(theta, (float)i / d_k);
        float freq = freq_extrap;
        if (use_ntk) {
            const float ramp = yarn_ramp(dim_high, dim_low, i / 2);
            const float freq_interp = freq_extrap * inv_scale;
            freq = fmaf(freq_interp, 1.0f - ramp, freq_extrap * ramp);
        }
        for (uint32_t t = 0; t < n_pos; t++) {
            const float angle = (float)(pos0 + t) * freq;
            cos_out[(size_t)t * half + i / 2] = cosf(angle);
            sin_out[(size_t)t * half + i / 2] = sinf(angle);
        }
    }
    return 1;
}
