// kv_store.cu -- fused per-head q/k RMSNorm + NEOX RoPE + paged BF16 KV store.
//
// Replaces, for one layer, the reference's graph ops BuildNorm(q/k) +
// ggml_rope_ext (src/models/qwen3.cpp:497-514, 627-641) and the host loops
// StorePrefillKV / AppendDecodeKV + WriteKVToCache
// (src/engine/model_runner.cpp:248-296, 380-415; src/models/qwen3.cpp:411-422).
//
// Eight lanes own one 128-element head row (16 elements per lane: four
// 16-byte loads, two 16-byte bf16 stores); a warp handles four rows.  Rows are
// ordered per token as [Hq q rows | Hkv k rows | Hkv v rows].
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
constexpr int kLanesPerRow = 8;
constexpr int kElems = kD / kLanesPerRow;  // 16 per lane
constexpr int kThreads = 256;
constexpr int kRowsPerBlock = kThreads / kLanesPerRow;

struct KvStoreParams {
  int n_tokens, Hq, Hkv, layer, max_position;
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

__device__ __forceinline__ void store16_bf16(uint16_t* dst, const float (&y)[kElems]) {
  uint4 a, b;
  a.x = pack_bf16x2(y[0], y[1]);
  a.y = pack_bf16x2(y[2], y[3]);
  a.z = pack_bf16x2(y[4], y[5]);
  a.w = pack_bf16x2(y[6], y[7]);
  b.x = pack_bf16x2(y[8], y[9]);
  b.y = pack_bf16x2(y[10], y[11]);
  b.z = pack_bf16x2(y[12], y[13]);
  b.w = pack_bf16x2(y[14], y[15]);
  reinterpret_cast<uint4*>(dst)[0] = a;
  reinterpret_cast<uint4*>(dst)[1] = b;
}

template <bool kQOutBf16>
__global__ void __launch_bounds__(kThreads) kv_store_qk_norm_rope_kernel(KvStoreParams p) {
  const int lane = threadIdx.x & 31;
  const int l8 = lane & 7;  // lane within the row's 8-lane group
  const int rows_per_token = p.Hq + 2 * p.Hkv;
  const long long total_rows = (long long)p.n_tokens * rows_per_token;
  const long long row_g = (long long)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 3);
  const bool valid = row_g < total_rows;
  // Groups past the last row redo it (so every lane joins the shuffles) and
  // store nothing.
  const long long row = valid ? row_g : total_rows - 1;
  const int t = (int)(row / rows_per_token);
  const int rr = (int)(row % rows_per_token);
  int kind, head;
  const float* src;
  if (rr < p.Hq) {
    kind = 0; head = rr;
    src = p.q + ((long long)t * p.Hq + head) * kD;
  } else if (rr < p.Hq + p.Hkv) {
    kind = 1; head = rr - p.Hq;
    src = p.k + ((long long)t * p.Hkv + head) * kD;
  } else {
    kind = 2; head = rr - p.Hq - p.Hkv;
    src = p.v + ((long long)t * p.Hkv + head) * kD;
  }

  // Plain loads: q_out may alias q (each row is read before it is written,
  // by the same lanes).
  float x[kElems];
#pragma unroll
  for (int i = 0; i < kElems / 4; ++i) {
    const float4 a = reinterpret_cast<const float4*>(src + kElems * l8)[i];
    x[4 * i] = a.x; x[4 * i + 1] = a.y; x[4 * i + 2] = a.z; x[4 * i + 3] = a.w;
  }

  // ---- RMSNorm (q and k rows) ----
  float sq[kElems];
  double s = 0.0;
#pragma unroll
  for (int e = 0; e < kElems; ++e) {
    sq[e] = __fmul_rn(x[e], x[e]);
    s = __dadd_rn(s, (double)sq[e]);
  }
#pragma unroll
  for (int o = kLanesPerRow / 2; o >= 1; o >>= 1)
    s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o, kLanesPerRow));

  // sum / 128 is exact as a multiplication by 2^-7 (no double division).
  constexpr double kInvD = 1.0 / kD;
  static_assert(kD == 128, "1/kD must be a power of two");
  const double delta = s * 0x1p-44;
  const bool ambiguous =
      kind != 2 && __double2float_rn((s - delta) * kInvD) != __double2float_rn((s + delta) * kInvD);
  if (__any_sync(0xffffffffu, ambiguous)) {
    // ggml's order: element 0, 1, ..., 127 of this group's row.
    double seq = 0.0;
    for (int srcl = 0; srcl < kLanesPerRow; ++srcl) {
#pragma unroll
      for (int e = 0; e < kElems; ++e) {
        const float v = __shfl_sync(0xffffffffu, sq[e], srcl, kLanesPerRow);
        seq = __dadd_rn(seq, (double)v);
      }
    }
    s = seq;
  }
  const float mean = __double2float_rn(s * kInvD);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));

  float y[kElems];
  if (kind != 2) {
    const uint4* wp = reinterpret_cast<const uint4*>((kind == 0 ? p.qw : p.kw) + kElems * l8);
    const uint4 w0 = __ldg(wp), w1 = __ldg(wp + 1);
    const uint32_t w8[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int e = 0; e < kElems; ++e) {
      const float w = (e & 1) ? bf16hi_to_f32(w8[e >> 1]) : bf16lo_to_f32(w8[e >> 1]);
      y[e] = __fmul_rn(__fmul_rn(x[e], scale), w);
    }
  } else {
#pragma unroll
    for (int e = 0; e < kElems; ++e) y[e] = x[e];
  }

  // ---- NEOX RoPE: element i pairs with i+64 (lane l8 pairs with l8^4) ----
  float partner[kElems];
#pragma unroll
  for (int e = 0; e < kElems; ++e)
    partner[e] = __shfl_xor_sync(0xffffffffu, y[e], kLanesPerRow / 2, kLanesPerRow);

  const int pos = p.positions[t];
  bool ok = valid;
  if (valid && (pos < 0 || pos >= p.max_position)) {
    record_error(p.status, NVATTN_ERR_OUT_OF_RANGE, 1, pos);
    ok = false;
  }
  if (kind != 2 && ok) {
    const float4* cs =
        reinterpret_cast<const float4*>(p.rope + (long long)pos * (kD / 2) + kElems * (l8 & 3));
    float c[kElems], sn[kElems];
#pragma unroll
    for (int j = 0; j < kElems / 2; ++j) {
      const float4 a = __ldg(cs + j);
      c[2 * j] = a.x; sn[2 * j] = a.y; c[2 * j + 1] = a.z; sn[2 * j + 1] = a.w;
    }
    if (l8 < 4) {
#pragma unroll
      for (int e = 0; e < kElems; ++e)
        y[e] = __fsub_rn(__fmul_rn(y[e], c[e]), __fmul_rn(partner[e], sn[e]));
    } else {
#pragma unroll
      for (int e = 0; e < kElems; ++e)
        y[e] = __fadd_rn(__fmul_rn(partner[e], sn[e]), __fmul_rn(y[e], c[e]));
    }
  }
  if (!ok) return;

  // ---- stores ----
  if (kind == 0) {
    const long long off = ((long long)t * p.Hq + head) * kD + kElems * l8;
    if (kQOutBf16) {
      store16_bf16(static_cast<uint16_t*>(p.q_out) + off, y);
    } else {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(p.q_out) + off);
#pragma unroll
      for (int i = 0; i < kElems / 4; ++i)
        o[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
    }
    return;
  }
  const int slot = p.slots[t];
  if (slot < 0) return;
  if ((long long)slot >= p.n_slots) {
    record_error(p.status, NVATTN_ERR_OUT_OF_RANGE, 2, slot);
    return;
  }
  uint16_t* cache = kind == 1 ? p.k_cache : p.v_cache;
  store16_bf16(cache + (((long long)p.layer * p.n_slots + slot) * p.Hkv + head) * kD + kElems * l8,
               y);
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
  const long long blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  if (blocks > 0x7fffffffLL) return NVATTN_ERR_INVALID_ARG;
  if (q_out_dtype == NVATTN_DTYPE_BF16)
    kv_store_qk_norm_rope_kernel<true><<<(unsigned)blocks, kThreads, 0, stream>>>(p);
  else
    kv_store_qk_norm_rope_kernel<false><<<(unsigned)blocks, kThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace nvattn
