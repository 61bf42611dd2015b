// rope_table.cpp -- host-side RoPE cos/sin table, built once per handle.
//
// Follows ggml's CPU rope cache (ggml_rope_cache_init + rope_yarn, as called
// by ggml_rope_ext from src/models/qwen3.cpp:505-514 with Qwen3Hparams'
// freq_base 1e6, freq_scale 1, ext_factor 1, attn_factor 1, beta_fast 32,
// beta_slow 1 and n_ctx_orig = n_ctx, qwen3.h:45-50): theta starts at the
// position as a float and is multiplied by powf(base, -2/n_dims) once per
// pair; the YaRN ramp mixes interpolated and extrapolated angles.  Compiled
// with -ffp-contract=off so each product and sum is rounded separately, as in
// ggml's scalar code; the device kernel reads this table instead of
// evaluating sin/cos itself so that rotated K rows match the reference's
// float arithmetic bit for bit.
#include <cmath>

#include "internal.h"

namespace nvattn {
namespace {

float yarn_corr_dim(int n_dims, int n_ctx_orig, float n_rot, float base) {
  return n_dims * logf(n_ctx_orig / (n_rot * 2 * (float)M_PI)) / (2 * logf(base));
}

float yarn_ramp(float low, float high, int i0) {
  const float y = (i0 / 2 - low) / std::fmax(0.001f, high - low);
  return 1 - std::fmin(1.0f, std::fmax(0.0f, y));
}

}  // namespace

void build_rope_table(const nvattn_config& cfg, int n_pos, float* table) {
  const int n_dims = cfg.head_dim;
  float corr[2];
  {
    const float start = floorf(yarn_corr_dim(n_dims, cfg.rope_n_ctx_orig, cfg.rope_beta_fast,
                                             cfg.rope_theta));
    const float end =
        ceilf(yarn_corr_dim(n_dims, cfg.rope_n_ctx_orig, cfg.rope_beta_slow, cfg.rope_theta));
    corr[0] = std::fmax(0.0f, start);
    corr[1] = std::fmin((float)(n_dims - 1), end);
  }
  const float theta_scale = powf(cfg.rope_theta, -2.0f / n_dims);
  const int half = n_dims / 2;
  for (int pos = 0; pos < n_pos; ++pos) {
    float* row = table + (long long)pos * n_dims;  // [cos x half | sin x half]
    float theta_extrap = (float)pos;
    for (int i0 = 0; i0 < n_dims; i0 += 2) {
      const float theta_interp = cfg.rope_freq_scale * theta_extrap;
      float theta = theta_interp;
      float mscale = cfg.rope_attn_factor;
      if (cfg.rope_ext_factor != 0.0f) {
        const float ramp_mix = yarn_ramp(corr[0], corr[1], i0) * cfg.rope_ext_factor;
        theta = theta_interp * (1 - ramp_mix) + theta_extrap * ramp_mix;
        mscale *= 1.0f + 0.1f * logf(1.0f / cfg.rope_freq_scale);
      }
      row[i0 / 2] = cosf(theta) * mscale;
      row[half + i0 / 2] = sinf(theta) * mscale;
      theta_extrap *= theta_scale;
    }
  }
}

}  // namespace nvattn
