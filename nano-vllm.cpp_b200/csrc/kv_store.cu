// kv_store.cu -- fused per-head q/k RMSNorm + NEOX RoPE + paged BF16 KV store.
//
// Replaces, for one layer, the reference's graph ops BuildNorm(q/k) +
// ggml_rope_ext (src/models/qwen3.cpp:497-514, 627-641) and the host loops
// StorePrefillKV / AppendDecodeKV + WriteKVToCache
// (src/engine/model_runner.cpp:248-296, 380-415; src/models/qwen3.cpp:411-422).
//
// Eight lanes own a 128-element head row.  Lane l holds elements
// [8l, 8l+8) and their NEOX partners [64+8l, 64+8l+8), so the rotation needs
// no shuffle and each lane needs only 8 (cos, sin) pairs.  Each half is two
// 16-byte loads and one 16-byte bf16 store.  An 8-lane group walks
// `rows_per_group` consecutive rows of the flattened [token][Hq q | Hkv k |
// Hkv v] row list, reloads the norm weights only when the row kind changes
// and the (cos, sin) pairs only when the token changes, and prefetches
// the next row's input while it works on the current one.
//
// Bit-exactness with the reference's ggml CPU path:
//  * RMSNorm: ggml sums float squares in double in index order, rounds
//    mean = sum/128 to float, scale = 1/sqrtf(mean+eps), y = (x*scale)*w.
//    Here the squares are summed in double by an 8-lane tree.  The tree and
//    the sequential sum both lie within 2^-45*sum of the exact sum, so the
//    float mean can only differ when sum/128 lies within that distance of a
//    float rounding boundary.  That case is detected (both ends of the
//    interval are rounded) and the warp then redoes the sum in ggml's exact
//    index order.
//  * RoPE: cos/sin come from the host-built table (ggml's float recurrence);
//    the rotation uses separately rounded products (no FMA contraction).
//  * Store: ggml_compute_fp32_to_bf16 rounding.
#include "common.cuh"
#include "internal.h"

namespace nvattn {
namespace {

constexpr int kD = 128;
constexpr int kHalf = kD / 2;
constexpr int kLanesPerRow = 8;
constexpr int kPer = kHalf / kLanesPerRow;  // 8 elements per lane per half
constexpr int kThreads = 256;
constexpr int kGroupsPerBlock = kThreads / kLanesPerRow;
constexpr int kMaxRowsPerGroup = 8;

struct KvStoreParams {
  int n_tokens, Hq, Hkv, layer, max_position, rows_per_group;
  int total_rows;
  long long n_slots;
  float eps;
  const float* q;
  const float* k;
  const float* v;
  const uint16_t* qw;
  const uint16_t* kw;
  const int32_t* positions;
  const int32_t* slots;
  const float2* rope;  // [max_position][64] (cos, sin)
  void* q_out;
  uint16_t* k_cache;
  uint16_t* v_cache;
  DeviceStatus* status;
};

__device__ __forceinline__ uint4 pack8_bf16(const float* y) {
  uint4 a;
  a.x = pack_bf16x2(y[0], y[1]);
  a.y = pack_bf16x2(y[2], y[3]);
  a.z = pack_bf16x2(y[4], y[5]);
  a.w = pack_bf16x2(y[6], y[7]);
  return a;
}

// Input row of flattened row (t, rr): q, k or v head row.
__device__ __forceinline__ const float* row_src(const KvStoreParams& p, int t, int rr) {
  if (rr < p.Hq) return p.q + ((long long)t * p.Hq + rr) * kD;
  if (rr < p.Hq + p.Hkv) return p.k + ((long long)t * p.Hkv + (rr - p.Hq)) * kD;
  return p.v + ((long long)t * p.Hkv + (rr - p.Hq - p.Hkv)) * kD;
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

template <bool kQOutBf16>
__global__ void __launch_bounds__(kThreads, 3) kv_store_qk_norm_rope_kernel(KvStoreParams p) {
  const int l8 = threadIdx.x & 7;  // lane within the row's 8-lane group
  const int rows_per_token = p.Hq + 2 * p.Hkv;
  const int group = blockIdx.x * kGroupsPerBlock + (threadIdx.x >> 3);
  const int row0 = group * p.rows_per_group;

  // Groups past the last row redo it (so every lane joins the shuffles) and
  // store nothing.
  int row = min(row0, p.total_rows - 1);
  int t = row / rows_per_token;
  int rr = row - t * rows_per_token;
  float xn[2 * kPer];
  load_row(row_src(p, t, rr), l8, xn);

  int cur_t = -1, pos = 0, cur_kind = -1;
  bool pos_ok = false;
  float c[kPer], sn[kPer];
  uint4 w[2];  // norm weights of this lane's 16 elements (packed bf16 pairs)

  for (int it = 0; it < p.rows_per_group; ++it) {
    const bool valid = row0 + it < p.total_rows;
    const int t_row = t, rr_row = rr;
    float x[2 * kPer];
#pragma unroll
    for (int e = 0; e < 2 * kPer; ++e) x[e] = xn[e];
    // advance to (and prefetch) the next row
    if (it + 1 < p.rows_per_group && row0 + it + 1 < p.total_rows) {
      if (++rr == rows_per_token) { rr = 0; ++t; }
      load_row(row_src(p, t, rr), l8, xn);
    }
    const int kind = rr_row < p.Hq ? 0 : (rr_row < p.Hq + p.Hkv ? 1 : 2);

    if (t_row != cur_t) {
      cur_t = t_row;
      pos = p.positions[t_row];
      pos_ok = pos >= 0 && pos < p.max_position;
      if (pos_ok) {
        const float4* cs =
            reinterpret_cast<const float4*>(p.rope + (long long)pos * kHalf + kPer * l8);
#pragma unroll
        for (int j = 0; j < kPer / 2; ++j) {
          const float4 a = __ldg(cs + j);
          c[2 * j] = a.x; sn[2 * j] = a.y; c[2 * j + 1] = a.z; sn[2 * j + 1] = a.w;
        }
      }
    }

    // ---- RMSNorm (q and k rows; v rows compute it too and discard it) ----
    double s = 0.0;
#pragma unroll
    for (int e = 0; e < 2 * kPer; ++e) s = __dadd_rn(s, (double)__fmul_rn(x[e], x[e]));
#pragma unroll
    for (int o = kLanesPerRow / 2; o >= 1; o >>= 1)
      s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o, kLanesPerRow));

    // sum / 128 is exact as a multiplication by 2^-7 (no double division).
    constexpr double kInvD = 1.0 / kD;
    static_assert(kD == 128, "1/kD must be a power of two");
    const double delta = s * 0x1p-44;
    const bool ambiguous = kind != 2 && __double2float_rn((s - delta) * kInvD) !=
                                            __double2float_rn((s + delta) * kInvD);
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

    if (valid && !pos_ok) record_error(p.status, NVATTN_ERR_OUT_OF_RANGE, 1, pos);
    const bool ok = valid && pos_ok;
    if (kind != 2) {
      const float mean = __double2float_rn(s * kInvD);
      const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
      if (kind != cur_kind) {
        cur_kind = kind;
        const uint16_t* wp = (kind == 0 ? p.qw : p.kw) + kPer * l8;
        w[0] = __ldg(reinterpret_cast<const uint4*>(wp));
        w[1] = __ldg(reinterpret_cast<const uint4*>(wp + kHalf));
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t w4[4] = {w[h].x, w[h].y, w[h].z, w[h].w};
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          const float wf = (e & 1) ? bf16hi_to_f32(w4[e >> 1]) : bf16lo_to_f32(w4[e >> 1]);
          x[h * kPer + e] = __fmul_rn(__fmul_rn(x[h * kPer + e], scale), wf);
        }
      }
      // ---- NEOX RoPE: element i pairs with i+64 ----
      if (ok) {
#pragma unroll
        for (int e = 0; e < kPer; ++e) {
          const float x0 = x[e], x1 = x[kPer + e];
          x[e] = __fsub_rn(__fmul_rn(x0, c[e]), __fmul_rn(x1, sn[e]));
          x[kPer + e] = __fadd_rn(__fmul_rn(x0, sn[e]), __fmul_rn(x1, c[e]));
        }
      }
    }
    if (!ok) continue;

    // ---- stores ----
    if (kind == 0) {
      const long long off = ((long long)t_row * p.Hq + rr_row) * kD + kPer * l8;
      if (kQOutBf16) {
        uint16_t* o = static_cast<uint16_t*>(p.q_out) + off;
        *reinterpret_cast<uint4*>(o) = pack8_bf16(x);
        *reinterpret_cast<uint4*>(o + kHalf) = pack8_bf16(x + kPer);
      } else {
        float* o = static_cast<float*>(p.q_out) + off;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float4* o4 = reinterpret_cast<float4*>(o + h * kHalf);
          o4[0] = make_float4(x[h * kPer], x[h * kPer + 1], x[h * kPer + 2], x[h * kPer + 3]);
          o4[1] = make_float4(x[h * kPer + 4], x[h * kPer + 5], x[h * kPer + 6], x[h * kPer + 7]);
        }
      }
      continue;
    }
    const int slot = p.slots[t_row];
    if (slot < 0) continue;
    if ((long long)slot >= p.n_slots) {
      record_error(p.status, NVATTN_ERR_OUT_OF_RANGE, 2, slot);
      continue;
    }
    const int head = kind == 1 ? rr_row - p.Hq : rr_row - p.Hq - p.Hkv;
    uint16_t* dst = (kind == 1 ? p.k_cache : p.v_cache) +
                    (((long long)p.layer * p.n_slots + slot) * p.Hkv + head) * kD + kPer * l8;
    *reinterpret_cast<uint4*>(dst) = pack8_bf16(x);
    *reinterpret_cast<uint4*>(dst + kHalf) = pack8_bf16(x + kPer);
  }
}

}  // namespace

nvattn_status launch_kv_store(nvattn_handle* h, int layer, int n_tokens, const float* q,
                              const float* k, const float* v, const uint16_t* qw,
                              const uint16_t* kw, const int32_t* positions,
                              const int32_t* slots, void* q_out, nvattn_dtype q_out_dtype,
                              uint16_t* k_cache, uint16_t* v_cache, cudaStream_t stream) {
  if (n_tokens == 0) return NVATTN_OK;
  KvStoreParams p;
  p.n_tokens = n_tokens;
  p.Hq = h->cfg.n_q_heads;
  p.Hkv = h->cfg.n_kv_heads;
  p.layer = layer;
  p.max_position = h->cfg.max_position;
  p.n_slots = h->n_slots;
  p.eps = h->cfg.rms_eps;
  p.q = q; p.k = k; p.v = v; p.qw = qw; p.kw = kw;
  p.positions = positions;
  p.slots = slots;
  p.rope = reinterpret_cast<const float2*>(h->rope_table_dev);
  p.q_out = q_out;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.status = h->status_dev;
  const long long rows = (long long)n_tokens * (p.Hq + 2 * p.Hkv);
  if (rows > 0x7fffffffLL - kMaxRowsPerGroup * kGroupsPerBlock) return NVATTN_ERR_INVALID_ARG;
  p.total_rows = (int)rows;
  // Enough groups for about four resident blocks per SM; beyond that each
  // group takes more rows so the per-token loads are shared.
  const long long per_wave = (long long)h->sm_count * 4 * kGroupsPerBlock;
  p.rows_per_group = (int)std::max(1LL, std::min<long long>(kMaxRowsPerGroup, rows / per_wave));
  const long long groups = (rows + p.rows_per_group - 1) / p.rows_per_group;
  const long long blocks = (groups + kGroupsPerBlock - 1) / kGroupsPerBlock;
  if (q_out_dtype == NVATTN_DTYPE_BF16)
    kv_store_qk_norm_rope_kernel<true><<<(unsigned)blocks, kThreads, 0, stream>>>(p);
  else
    kv_store_qk_norm_rope_kernel<false><<<(unsigned)blocks, kThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace nvattn
