// row_math.cuh -- the per-head row arithmetic of the fused q/k RMSNorm +
// NEOX RoPE + BF16 store, shared by the KV-store kernels (kv_store.cu) and
// the fused decode step (decode.cu) so that both produce the same bits.
//
// Eight lanes own a 128-element head row: lane l holds elements [8l, 8l+8)
// and their NEOX partners [64+8l, 64+8l+8).  Every floating-point operation
// here is an explicit rounding intrinsic or a packed instruction in inline
// PTX, so no multiply-add contraction can change a result whatever the
// including file's -fmad setting (see kv_store.cu for the bit-exactness
// argument against ggml's CPU path).
#pragma once

#include "common.cuh"

namespace nvattn {
namespace rowmath {

constexpr int kD = 128;
constexpr int kHalf = kD / 2;
constexpr int kLanesPerRow = 8;
constexpr int kPer = kHalf / kLanesPerRow;  // 8 elements per lane per half

// Per-lane norm weights of one row kind (16 bf16, packed in pairs) and
// whether they are small enough (|w| < 2^120, finite) that a finite input
// row cannot produce a NaN.
struct LaneWeights {
  uint32_t w[kPer];
  bool tame;
};

__device__ __forceinline__ void load_weights(const uint16_t* wsrc, int l8, LaneWeights& lw) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(wsrc + kPer * l8));
  const uint4 b = __ldg(reinterpret_cast<const uint4*>(wsrc + kHalf + kPer * l8));
  const uint32_t u[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  bool tame = true;
#pragma unroll
  for (int e = 0; e < kPer; ++e) {
    lw.w[e] = u[e];
    // bf16 magnitude bits < 0x7b80 <=> |w| < 2^120 (inf and NaN excluded)
    tame = tame && (u[e] & 0x7fffu) < 0x7b80u && ((u[e] >> 16) & 0x7fffu) < 0x7b80u;
  }
  lw.tame = tame;
}

// RMSNorm scale 1/sqrt(mean(x^2) + eps) of the group's row, bit-exact with
// ggml's double accumulation.  Warp-collective: every lane of the warp calls
// it (rows that are not normed pass norm_row = false).  `finite` tells
// whether the whole row is finite (sum of squares finite).
__device__ __forceinline__ float rms_scale(const float (&x)[2 * kPer], bool norm_row, float eps,
                                           bool& finite) {
  if (__all_sync(0xffffffffu, !norm_row)) {
    // a warp of v rows: only finiteness is needed
    uint32_t m = 0;
#pragma unroll
    for (int e = 0; e < 2 * kPer; ++e) m = max(m, __float_as_uint(x[e]) & 0x7fffffffu);
    finite = m < 0x7f800000u;
    return 1.0f;
  }
  // The lane's 16 squares summed in double into four accumulators.  A
  // positive normal float widens to double by its bits (exponent re-biased
  // from 127 to 1023, mantissa shifted up 29 places), which spares the slow
  // conversion instruction; a warp with a zero, subnormal or non-finite
  // square redoes the sums with the conversion.
  float sq[2 * kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const uint64_t x2 = pack2(x[2 * k], x[2 * k + 1]);
    unpack2(fmul2(x2, x2), sq[2 * k], sq[2 * k + 1]);
  }
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  uint32_t odd = 0;
#pragma unroll
  for (int e = 0; e < 2 * kPer; ++e) {
    const uint32_t u = __float_as_uint(sq[e]);
    odd |= (u >> 23) - 1u >= 254u;  // exponent field 0 or 255, or the sign set
    acc[e & 3] = __dadd_rn(acc[e & 3],
                           __hiloint2double((int)((u >> 3) + 0x38000000u), (int)(u << 29)));
  }
  if (__any_sync(0xffffffffu, odd != 0)) {
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = 0.0;
#pragma unroll
    for (int e = 0; e < 2 * kPer; ++e) acc[e & 3] = __dadd_rn(acc[e & 3], (double)sq[e]);
  }
  double s = __dadd_rn(__dadd_rn(acc[0], acc[1]), __dadd_rn(acc[2], acc[3]));
#pragma unroll
  for (int o = kLanesPerRow / 2; o >= 1; o >>= 1)
    s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o, kLanesPerRow));
  finite = s <= 1.7976931348623157e308;  // false for inf and NaN

  // sum / 128 is exact as a multiplication by 2^-7 (no double division).
  constexpr double kInvD = 1.0 / kD;
  static_assert(kD == 128, "1/kD must be a power of two");
  // Rounding d = sum/128 to float drops the low 29 of its 52 mantissa bits;
  // d sits near a float rounding boundary when those bits are within 512
  // double ulps (> 2^-44 relative) of one half.  Any order of summing 128
  // non-negative terms in double is within 127 u S of the exact sum S (u =
  // 2^-53), so this order and ggml's sequential one differ by at most
  // 2^-45 S: outside the margin both round to the same float.  Outside the
  // normal float range the exact sum is always redone.
  const double dm = s * kInvD;
  const int hi = __double2hiint(dm);
  const int ex = (hi >> 20) & 0x7ff;
  const int dropped = __double2loint(dm) & 0x1fffffff;
  const bool ambiguous =
      norm_row && (abs(dropped - 0x10000000) <= 512 || ex < 1023 - 126 || ex > 1023 + 127);
  if (__any_sync(0xffffffffu, ambiguous)) {
    // ggml's order: elements 0..63 (lanes 0..7, first halves), then 64..127.
    double seq = 0.0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      for (int srcl = 0; srcl < kLanesPerRow; ++srcl) {
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          const float v = __shfl_sync(0xffffffffu, x[h * kPer + e], srcl, kLanesPerRow);
          seq = __dadd_rn(seq, (double)__fmul_rn(v, v));
        }
      }
    }
    s = seq;
  }
  if (!norm_row) return 1.0f;
  const float mean = __double2float_rn(s * kInvD);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// y = (x * scale) * w, then the NEOX rotation (element i with i+64):
//   y_i' = y_i*cos - y_{i+64}*sin,  y_{i+64}' = y_i*sin + y_{i+64}*cos.
__device__ __forceinline__ void norm_rope(float (&x)[2 * kPer], float scale,
                                          const float (&w)[2 * kPer], const float (&c)[kPer],
                                          const float (&sn)[kPer]) {
  const uint64_t sc = pack2(scale, scale);
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const uint64_t y =
        fmul2(fmul2(pack2(x[2 * k], x[2 * k + 1]), sc), pack2(w[2 * k], w[2 * k + 1]));
    unpack2(y, x[2 * k], x[2 * k + 1]);
  }
  // Packed products, scalar .rn sums: ptxas fuses a packed mul.rn.f32x2
  // with a following packed add/sub into an FMA (even under -fmad=false),
  // which would skip the rounding of one product.
#pragma unroll
  for (int k = 0; k < kPer / 2; ++k) {
    const uint64_t x0 = pack2(x[2 * k], x[2 * k + 1]);
    const uint64_t x1 = pack2(x[kPer + 2 * k], x[kPer + 2 * k + 1]);
    const uint64_t cc = pack2(c[2 * k], c[2 * k + 1]);
    const uint64_t ss = pack2(sn[2 * k], sn[2 * k + 1]);
    float x0c[2], x1s[2], x0s[2], x1c[2];
    unpack2(fmul2(x0, cc), x0c[0], x0c[1]);
    unpack2(fmul2(x1, ss), x1s[0], x1s[1]);
    unpack2(fmul2(x0, ss), x0s[0], x0s[1]);
    unpack2(fmul2(x1, cc), x1c[0], x1c[1]);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      x[2 * k + j] = __fsub_rn(x0c[j], x1s[j]);
      x[kPer + 2 * k + j] = __fadd_rn(x0s[j], x1c[j]);
    }
  }
}

// Eight floats -> f16, round to nearest even (ggml_fp32_to_fp16's rounding
// for every finite value; overflow gives inf, as there).
__device__ __forceinline__ uint4 pack8_f16(const float* y) {
  return make_uint4(cvt_f16x2(y[0], y[1]), cvt_f16x2(y[2], y[3]), cvt_f16x2(y[4], y[5]),
                    cvt_f16x2(y[6], y[7]));
}

__device__ __forceinline__ uint4 pack8_bf16(const float* y, bool nan_rule) {
  uint4 a;
  if (!nan_rule) {
    a.x = cvt_bf16x2(y[0], y[1]);
    a.y = cvt_bf16x2(y[2], y[3]);
    a.z = cvt_bf16x2(y[4], y[5]);
    a.w = cvt_bf16x2(y[6], y[7]);
  } else {
    a.x = pack_bf16x2(y[0], y[1]);
    a.y = pack_bf16x2(y[2], y[3]);
    a.z = pack_bf16x2(y[4], y[5]);
    a.w = pack_bf16x2(y[6], y[7]);
  }
  return a;
}

// Streaming loads (evict-first): every input byte is read once.  Plain
// coherent loads, because q_out may alias q (a row is read before the same
// lanes write it).
__device__ __forceinline__ void load_row(const float* src, int l8, float (&x)[2 * kPer]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float4* s4 = reinterpret_cast<const float4*>(src + h * kHalf + kPer * l8);
    const float4 a = __ldcs(s4), b = __ldcs(s4 + 1);
    x[h * kPer + 0] = a.x; x[h * kPer + 1] = a.y; x[h * kPer + 2] = a.z; x[h * kPer + 3] = a.w;
    x[h * kPer + 4] = b.x; x[h * kPer + 5] = b.y; x[h * kPer + 6] = b.z; x[h * kPer + 7] = b.w;
  }
}

}  // namespace rowmath
}  // namespace nvattn
