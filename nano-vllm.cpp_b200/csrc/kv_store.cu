// kv_store.cu -- fused per-head q/k RMSNorm + NEOX RoPE + paged BF16 KV store.
//
// Replaces, for one layer, the reference's graph ops BuildNorm(q/k) +
// ggml_rope_ext (src/models/qwen3.cpp:497-514, 627-641) and the host loops
// StorePrefillKV / AppendDecodeKV + WriteKVToCache
// (src/engine/model_runner.cpp:248-296, 380-415; src/models/qwen3.cpp:411-422).
//
// Eight lanes own a 128-element head row.  Lane l holds elements
// [8l, 8l+8) and their NEOX partners [64+8l, 64+8l+8), so the rotation needs
// no shuffle and each lane needs only 8 cos and 8 sin values.  Each half
// leaves as one 16-byte bf16 store.  The arithmetic runs on packed f32x2
// instructions for the products; the rotation's sums of two products are
// scalar .rn adds.
//
// Two kernels share that row math:
//  * kv_store_staged_kernel (large batches): one persistent CTA per SM.  A
//    producer warp streams chunks of whole tokens -- their q, k and v rows
//    (three contiguous ranges) and each token's cos/sin row -- into a ring of
//    shared-memory stages with bulk async copies, so ~150 KB per SM are in
//    flight without holding registers.  The number of consumer warps is
//    chosen per model so that each stage's rows split evenly over them (four
//    rows per warp per pass, no idle groups).
//  * kv_store_rows_kernel (small batches, e.g. one decode token per
//    sequence): each 8-lane group walks a short run of consecutive rows with
//    register loads and a one-row prefetch.
//
// Bit-exactness with the reference's ggml CPU path:
//  * RMSNorm: ggml sums float squares in double in index order, rounds
//    mean = sum/128 to float, scale = 1/sqrtf(mean+eps), y = (x*scale)*w.
//    Here the squares are summed in double by a tree.  The tree and the
//    sequential sum both lie within 2^-45*sum of the exact sum, so the float
//    mean can only differ when sum/128 lies within that distance of a float
//    rounding boundary.  That case is detected (both ends of the interval are
//    rounded) and the warp then redoes the sum in ggml's exact index order.
//  * RoPE: cos/sin come from the host-built table (ggml's float recurrence);
//    the rotation uses separately rounded products (packed products, scalar
//    .rn sums, which ptxas does not contract into an FMA).
//  * Store: ggml_compute_fp32_to_bf16 rounding.  For finite values that is
//    round-to-nearest-even, i.e. cvt.rn.bf16x2.f32; a row that may hold a NaN
//    (non-finite input, or norm weights of magnitude >= 2^120) takes ggml's
//    bit rule instead, which keeps the NaN payload.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "internal.h"
#include "row_math.cuh"

namespace nvattn {
namespace {

using namespace rowmath;  // kD, kHalf, kLanesPerRow, kPer and the row functions
constexpr int kRowBytes = kD * 4;
constexpr int kThreads = 256;
constexpr int kGroupsPerBlock = kThreads / kLanesPerRow;
constexpr int kMaxRowsPerGroup = 8;

// staged kernel
constexpr int kMinConsumerWarps = 8;
constexpr int kMaxConsumerWarps = 20;
constexpr int kStageMaxThreads = (kMaxConsumerWarps + 1) * 32;
constexpr int kMaxStages = 8;
constexpr int kMaxTokensPerStage = 32;  // one producer lane per token
constexpr int kStageHeader = 4096;      // barriers, flags, per-stage positions/slots
constexpr int kStageMaxBytes = 56 * 1024;
constexpr int kStageSmemBudget = 227 * 1024;

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
  const float* rope;  // [max_position][cos x 64 | sin x 64]
  void* q_out;
  uint16_t* k_cache;
  uint16_t* v_cache;
  uint16_t* k_rows;  // nullable: f16 copies of the stored K rows, [n_tokens][Hkv][128]
  uint16_t* v_rows;  // nullable: f16 copies of the V rows
  DeviceStatus* status;
};

// q_out element types (template argument of the row kernels).
constexpr int kQOutF32 = 0, kQOutBf16 = 1, kQOutF16 = 2;

// Writes the finished row: q rows to q_out, k/v rows to slot_mapping[t] of
// the cache (slot < 0: not stored; slot >= n_slots: reported).
template <int kQOut>
__device__ __forceinline__ void store_row(const KvStoreParams& p, const float (&x)[2 * kPer],
                                          int t, int rr, int kind, int slot, bool nan_rule,
                                          int l8) {
  if (kind == 0) {
    const long long off = ((long long)t * p.Hq + rr) * kD + kPer * l8;
    if (kQOut == kQOutBf16) {
      uint16_t* o = static_cast<uint16_t*>(p.q_out) + off;
      *reinterpret_cast<uint4*>(o) = pack8_bf16(x, nan_rule);
      *reinterpret_cast<uint4*>(o + kHalf) = pack8_bf16(x + kPer, nan_rule);
    } else if (kQOut == kQOutF16) {
      uint16_t* o = static_cast<uint16_t*>(p.q_out) + off;
      *reinterpret_cast<uint4*>(o) = pack8_f16(x);
      *reinterpret_cast<uint4*>(o + kHalf) = pack8_f16(x + kPer);
    } else {
      float* o = static_cast<float*>(p.q_out) + off;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float4* o4 = reinterpret_cast<float4*>(o + h * kHalf);
        o4[0] = make_float4(x[h * kPer], x[h * kPer + 1], x[h * kPer + 2], x[h * kPer + 3]);
        o4[1] = make_float4(x[h * kPer + 4], x[h * kPer + 5], x[h * kPer + 6], x[h * kPer + 7]);
      }
    }
    return;
  }
  const int head = kind == 1 ? rr - p.Hq : rr - p.Hq - p.Hkv;
  uint16_t* rows = kind == 1 ? p.k_rows : p.v_rows;
  if (rows != nullptr) {
    // The step's own row as the reference's attention sees it: the graph's
    // f32 value cast to F16 (round to nearest even).
    uint16_t* o = rows + ((long long)t * p.Hkv + head) * kD + kPer * l8;
    *reinterpret_cast<uint4*>(o) = pack8_f16(x);
    *reinterpret_cast<uint4*>(o + kHalf) = pack8_f16(x + kPer);
  }
  if (slot < 0) return;
  if ((long long)slot >= p.n_slots) {
    record_error(p.status, NVATTN_ERR_OUT_OF_RANGE, 2, slot);
    return;
  }
  uint16_t* dst = (kind == 1 ? p.k_cache : p.v_cache) +
                  (((long long)p.layer * p.n_slots + slot) * p.Hkv + head) * kD + kPer * l8;
  *reinterpret_cast<uint4*>(dst) = pack8_bf16(x, nan_rule);
  *reinterpret_cast<uint4*>(dst + kHalf) = pack8_bf16(x + kPer, nan_rule);
}

// Norm, rotate and store one row (x already loaded; every lane of the warp
// calls this, `active` false for padding rows).  get_w(w) and get_cs(c, sn)
// supply the lane's norm weights and cos/sin values; they run after the
// norm's dependency chain so the values are live only where they are used.
template <int kQOut, class GetW, class GetCs>
__device__ __forceinline__ void finish_row(const KvStoreParams& p, float (&x)[2 * kPer],
                                           bool active, int t, int rr, int kind, int pos,
                                           bool pos_ok, int slot, GetW get_w, bool w_tame,
                                           GetCs get_cs, int l8) {
  bool finite;
  const float scale = rms_scale(x, kind != 2, p.eps, finite);
  if (!active) return;
  if (!pos_ok) {
    record_error(p.status, NVATTN_ERR_OUT_OF_RANGE, 1, pos);
    return;
  }
  bool nan_rule = !finite;
  if (kind != 2) {
    float w[2 * kPer], c[kPer], sn[kPer];
    get_w(w);
    get_cs(c, sn);
    norm_rope(x, scale, w, c, sn);
    nan_rule = nan_rule || !w_tame;
  }
  store_row<kQOut>(p, x, t, rr, kind, slot, nan_rule, l8);
}

// Input row of flattened row (t, rr): q, k or v head row.
__device__ __forceinline__ const float* row_src(const KvStoreParams& p, int t, int rr) {
  if (rr < p.Hq) return p.q + ((long long)t * p.Hq + rr) * kD;
  if (rr < p.Hq + p.Hkv) return p.k + ((long long)t * p.Hkv + (rr - p.Hq)) * kD;
  return p.v + ((long long)t * p.Hkv + (rr - p.Hq - p.Hkv)) * kD;
}

// kOneRow: every group stores one row (rows_per_group == 1), so nothing is
// prefetched and three blocks fit on an SM; otherwise the group prefetches
// its next row while it finishes the current one, two blocks per SM.
template <int kQOut, bool kOneRow>
__global__ void __launch_bounds__(kThreads, kOneRow ? 3 : 2) kv_store_rows_kernel(KvStoreParams p) {
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
  LaneWeights lw;

  const int n_rows = kOneRow ? 1 : p.rows_per_group;
  for (int it = 0; it < n_rows; ++it) {
    const bool valid = row0 + it < p.total_rows;
    const int t_row = t, rr_row = rr;
    float x[2 * kPer];
#pragma unroll
    for (int e = 0; e < 2 * kPer; ++e) x[e] = xn[e];
    // advance to (and prefetch) the next row
    if (!kOneRow && it + 1 < n_rows && row0 + it + 1 < p.total_rows) {
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
            reinterpret_cast<const float4*>(p.rope + (long long)pos * kD + kPer * l8);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float4 a = __ldg(cs + j), b = __ldg(cs + kHalf / 4 + j);
          c[4 * j] = a.x; c[4 * j + 1] = a.y; c[4 * j + 2] = a.z; c[4 * j + 3] = a.w;
          sn[4 * j] = b.x; sn[4 * j + 1] = b.y; sn[4 * j + 2] = b.z; sn[4 * j + 3] = b.w;
        }
      }
    }
    if (kind != 2 && kind != cur_kind) {
      cur_kind = kind;
      load_weights(kind == 0 ? p.qw : p.kw, l8, lw);
    }
    const int slot = (valid && kind != 0) ? p.slots[t_row] : 0;
    finish_row<kQOut>(p, x, valid, t_row, rr_row, kind, pos, pos_ok, slot,
                          [&](float (&w)[2 * kPer]) {
#pragma unroll
                            for (int e = 0; e < kPer; ++e) {
                              w[2 * e] = bf16lo_to_f32(lw.w[e]);
                              w[2 * e + 1] = bf16hi_to_f32(lw.w[e]);
                            }
                          },
                          lw.tame,
                          [&](float (&cc)[kPer], float (&ss)[kPer]) {
#pragma unroll
                            for (int e = 0; e < kPer; ++e) {
                              cc[e] = c[e];
                              ss[e] = sn[e];
                            }
                          },
                          l8);
  }
}

struct StagedPlan {
  int tokens_per_stage;  // whole tokens per shared-memory stage (nt)
  int consumer_warps;    // W; the producer is warp W
  int passes;            // ceil(nt * rows_per_token / (4 W)): four rows per warp per pass
  int n_stages;          // ring depth
  int stage_bytes;
  int n_chunks;          // ceil(n_tokens / nt)
};

// Reads 8 consecutive floats (chunks 2*l8 and 2*l8+1 of a 64-float half row)
// from shared memory.  The eight lanes' 32-byte pieces span 256 bytes, a
// two-way bank conflict; shared-memory bandwidth has the room, and swapping
// the chunk order per lane would cost more issue slots (selects) than the
// conflict costs.
__device__ __forceinline__ void lds_lane8(const float4* half_row, int l8, float* out) {
  const float4 a = half_row[2 * l8];
  const float4 b = half_row[2 * l8 + 1];
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}

// Norm weights in shared memory as floats, laid out [kind][j][lane l8][4] so
// that load j of the eight lanes reads 128 contiguous bytes.  Lane l8's
// floats f = 0..15 are elements 8*l8 + f (f < 8) and 64 + 8*l8 + (f - 8).
constexpr int kWeightsOffset = 256 + kMaxStages * 2 * kMaxTokensPerStage * 4;
__device__ __forceinline__ int lane_weight_slot(int el) {
  const int l8 = (el & 63) >> 3;
  const int f = (el & 7) + (el >= 64 ? 8 : 0);
  return ((f >> 2) * 8 + l8) * 4 + (f & 3);
}

// Stage layout (nt tokens, rows_per_token = Hq + 2 Hkv):
//   [nt*Hq q rows][nt*Hkv k rows][nt*Hkv v rows][nt cos/sin rows], each row
//   512 bytes; the q, k and v ranges are each one contiguous bulk copy.
// The header holds the ring's barriers and, per stage, the chunk's positions
// and slots (written by the producer warp before it arms the stage, so the
// consumers never wait on a global load).
template <int kQOut>
__global__ void __launch_bounds__(kStageMaxThreads, 1)
    kv_store_staged_kernel(KvStoreParams p, StagedPlan plan) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  int* abort_flag = reinterpret_cast<int*>(empty + kMaxStages);
  int* skip = abort_flag + 1;
  int* meta = reinterpret_cast<int*>(smem + 256);  // [stage][pos | slot][kMaxTokensPerStage]
  float* wsm = reinterpret_cast<float*>(smem + kWeightsOffset);  // [2][128]
  int* wild = skip + 1;  // [2]: some weight of q / k is not tame
  uint8_t* stages = smem + kStageHeader;
  static_assert(kWeightsOffset + 2 * kD * 4 <= kStageHeader, "header");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = plan.consumer_warps;
  const int nt = plan.tokens_per_stage;
  const int rpt = p.Hq + 2 * p.Hkv;
  if (threadIdx.x == 0) {
    for (int b = 0; b < plan.n_stages; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], W);
    }
    *abort_flag = 0;
    *skip = timeout_recorded(p.status) ? 1 : 0;
    wild[0] = wild[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 2 * kD; idx += blockDim.x) {
    const int kind = idx / kD, el = idx % kD;
    const uint32_t b = (kind == 0 ? p.qw : p.kw)[el];
    wsm[kind * kD + lane_weight_slot(el)] = __uint_as_float(b << 16);
    if ((b & 0x7fffu) >= 0x7b80u) wild[kind] = 1;  // |w| >= 2^120, inf or NaN
  }
  __syncthreads();
  if (*skip) return;

  if (warp == W) {
    // ---- producer warp: lane j handles token j of the chunk; lane 0 issues
    // the three row-range copies.  The next chunk's positions and slots are
    // loaded while this one is set up, off the critical path. ----
    const uint64_t pol = l2_policy_evict_first();
    int npos = 0, nslot = -1;
    auto fetch = [&](int chk) {
      const int t = chk * nt + lane;
      if (chk < plan.n_chunks && lane < nt && t < p.n_tokens) {
        npos = p.positions[t];
        nslot = p.slots[t];
      }
    };
    fetch(blockIdx.x);
    int it = 0;
    for (int ch = blockIdx.x; ch < plan.n_chunks; ch += gridDim.x, ++it) {
      const int pos = npos, slot = nslot;
      fetch(ch + gridDim.x);
      const int buf = it % plan.n_stages;
      const int use = it / plan.n_stages;
      bool ok = true;
      if (use > 0) ok = mbar_wait(&empty[buf], (use - 1) & 1, p.status, 50, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      const int t0 = ch * nt;
      const int ntc = min(nt, p.n_tokens - t0);
      const bool cs_valid = lane < ntc && pos >= 0 && pos < p.max_position;
      if (lane < ntc) {
        meta[(buf * 2 + 0) * kMaxTokensPerStage + lane] = pos;
        meta[(buf * 2 + 1) * kMaxTokensPerStage + lane] = slot;
      }
      const uint32_t n_cs = __popc(__ballot_sync(0xffffffffu, cs_valid));
      __syncwarp();  // the meta stores precede lane 0's arrive (release)
      uint8_t* st = stages + (size_t)buf * plan.stage_bytes;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[buf], (uint32_t)(ntc * rpt + n_cs) * kRowBytes);
        bulk_load(st, p.q + (long long)t0 * p.Hq * kD, ntc * p.Hq * kRowBytes, &full[buf], pol);
        bulk_load(st + nt * p.Hq * kRowBytes, p.k + (long long)t0 * p.Hkv * kD,
                  ntc * p.Hkv * kRowBytes, &full[buf], pol);
        bulk_load(st + nt * (p.Hq + p.Hkv) * kRowBytes, p.v + (long long)t0 * p.Hkv * kD,
                  ntc * p.Hkv * kRowBytes, &full[buf], pol);
      }
      __syncwarp();  // the stage is armed before any cos/sin copy lands
      if (cs_valid)
        bulk_load(st + (nt * rpt + lane) * kRowBytes, p.rope + (long long)pos * kD, kRowBytes,
                  &full[buf], pol);
    }
    // Drain: the CTA must not exit with copies in flight (they only matter
    // when the consumers gave up on a wait; otherwise these return at once).
    const int issued = it;
    if (lane == 0) {
      for (int b = 0; b < plan.n_stages && b < issued; ++b) {
        const int last = b + ((issued - 1 - b) / plan.n_stages) * plan.n_stages;
        mbar_wait(&full[b], (last / plan.n_stages) & 1, p.status, 51);
      }
    }
    return;
  }

  // ---- consumers: in pass kk, warp w's four groups take stage rows
  // 4 (kk W + w) .. +3 (consecutive rows, usually one token).  A row's place
  // in the stage does not depend on the stage, so pass 0's geometry is
  // computed once. ----
  const int l8 = lane & 7;
  const int stage_rows = nt * rpt;
  struct Geom {
    int i, tl, rr, kind, srow;
  };
  auto geom = [&](int kk) {
    Geom g;
    g.i = 4 * (kk * W + warp) + (lane >> 3);
    const int ic = min(g.i, stage_rows - 1);  // padding rows read a real row
    g.tl = ic / rpt;
    g.rr = ic - g.tl * rpt;
    if (g.rr < p.Hq) {
      g.kind = 0; g.srow = g.tl * p.Hq + g.rr;
    } else if (g.rr < p.Hq + p.Hkv) {
      g.kind = 1; g.srow = nt * p.Hq + g.tl * p.Hkv + (g.rr - p.Hq);
    } else {
      g.kind = 2; g.srow = nt * (p.Hq + p.Hkv) + g.tl * p.Hkv + (g.rr - p.Hq - p.Hkv);
    }
    return g;
  };
  const Geom g0 = geom(0);

  int it = 0;
  for (int ch = blockIdx.x; ch < plan.n_chunks; ch += gridDim.x, ++it) {
    const int buf = it % plan.n_stages;
    const bool got = mbar_wait(&full[buf], (it / plan.n_stages) & 1, p.status, 52, abort_flag);
    if (!__all_sync(0xffffffffu, got)) break;
    const int t0 = ch * nt;
    const int rows = min(nt, p.n_tokens - t0) * rpt;
    const uint8_t* st = stages + (size_t)buf * plan.stage_bytes;
    const int* mpos = meta + (buf * 2 + 0) * kMaxTokensPerStage;
    const int* mslot = meta + (buf * 2 + 1) * kMaxTokensPerStage;
    for (int kk = 0; kk < plan.passes; ++kk) {
      const Geom g = kk == 0 ? g0 : geom(kk);
      const bool active = g.i < rows;
      const float4* r4 = reinterpret_cast<const float4*>(st + g.srow * kRowBytes);
      float x[2 * kPer];
      lds_lane8(r4, l8, x);
      lds_lane8(r4 + kHalf / 4, l8, x + kPer);
      const int pos = mpos[g.tl];
      const bool pos_ok = pos >= 0 && pos < p.max_position;
      const float4* cs4 = reinterpret_cast<const float4*>(st + (stage_rows + g.tl) * kRowBytes);
      const float4* w4 = reinterpret_cast<const float4*>(wsm + (g.kind == 0 ? 0 : kD)) + l8;
      finish_row<kQOut>(
          p, x, active, t0 + g.tl, g.rr, g.kind, pos, pos_ok, mslot[g.tl],
          [&](float (&w)[2 * kPer]) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 v = w4[8 * j];
              w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
            }
          },
          !wild[g.kind == 0 ? 0 : 1],
          [&](float (&cc)[kPer], float (&ss)[kPer]) {
            lds_lane8(cs4, l8, cc);
            lds_lane8(cs4 + kHalf / 4, l8, ss);
          },
          l8);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[buf]);
  }
}

// Picks the stage size and consumer-warp count: among stages of whole tokens
// up to kStageMaxBytes whose rows split into passes of four rows per warp
// with no remainder, the one with the most consumer warps (more warps hide
// the latency of the norm's dependency chain), then the fewest tokens.
// Without an exact split: 16 warps and a partly idle last pass.
StagedPlan plan_staged(int n_tokens, int Hq, int Hkv) {
  const int rpt = Hq + 2 * Hkv;
  const int token_bytes = (rpt + 1) * kRowBytes;
  StagedPlan s{};
  for (int nt = 1; nt <= kMaxTokensPerStage; ++nt) {
    const int sb = nt * token_bytes;
    if (sb > kStageMaxBytes && nt > 1) break;
    const int rows = nt * rpt;
    if (rows % 4) continue;
    const int quads = rows / 4;
    int W = 0;
    for (int w = kMaxConsumerWarps; w >= kMinConsumerWarps && !W; --w)
      if (quads % w == 0) W = w;
    if (W > s.consumer_warps) s = StagedPlan{nt, W, quads / W, 0, sb, 0};
  }
  if (!s.tokens_per_stage) {
    s.tokens_per_stage =
        std::min(kMaxTokensPerStage, std::max(1, kStageMaxBytes / 2 / token_bytes));
    s.consumer_warps = 16;
    s.stage_bytes = s.tokens_per_stage * token_bytes;
    s.passes = (s.tokens_per_stage * rpt + 63) / 64;
  }
  s.n_stages = std::min(kMaxStages, (kStageSmemBudget - kStageHeader) / s.stage_bytes);
  s.n_chunks = (n_tokens + s.tokens_per_stage - 1) / s.tokens_per_stage;
  return s;
}

template <int kQOut>
nvattn_status launch_staged(const KvStoreParams& p, const StagedPlan& plan, int sm_count,
                            cudaStream_t stream) {
  // (atomic: handles on different threads may launch at the same time)
  static std::atomic<unsigned long long> attr_set_mask{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVATTN_ERR_CUDA;
  if (dev >= 64 || !(attr_set_mask.load(std::memory_order_relaxed) & (1ull << dev))) {
    if (cudaFuncSetAttribute(kv_store_staged_kernel<kQOut>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kStageSmemBudget) != cudaSuccess)
      return NVATTN_ERR_CUDA;
    if (dev < 64) attr_set_mask.fetch_or(1ull << dev, std::memory_order_relaxed);
  }
  const int grid = std::min(sm_count, plan.n_chunks);
  const size_t smem = kStageHeader + (size_t)plan.n_stages * plan.stage_bytes;
  kv_store_staged_kernel<kQOut>
      <<<grid, (plan.consumer_warps + 1) * 32, smem, stream>>>(p, plan);
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace

nvattn_status launch_kv_store(nvattn_handle* h, int layer, int n_tokens, const float* q,
                              const float* k, const float* v, const uint16_t* qw,
                              const uint16_t* kw, const int32_t* positions,
                              const int32_t* slots, void* q_out, nvattn_dtype q_out_dtype,
                              uint16_t* k_cache, uint16_t* v_cache, uint16_t* k_rows,
                              uint16_t* v_rows, cudaStream_t stream) {
  if (n_tokens == 0) return NVATTN_OK;
  KvStoreParams p = {};
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
  p.rope = h->rope_table_dev;
  p.q_out = q_out;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.k_rows = k_rows;
  p.v_rows = v_rows;
  p.status = h->status_dev;
  const long long rows = (long long)n_tokens * (p.Hq + 2 * p.Hkv);
  if (rows > 0x7fffffffLL - kMaxRowsPerGroup * kGroupsPerBlock) return NVATTN_ERR_INVALID_ARG;
  p.total_rows = (int)rows;
  const int q_kind = q_out_dtype == NVATTN_DTYPE_BF16  ? kQOutBf16
                     : q_out_dtype == NVATTN_DTYPE_F16 ? kQOutF16
                                                       : kQOutF32;

  // Large batches: bulk-copy staging (at least four stages per CTA so the
  // ring pipelines).  Small batches: the register-row kernel, which spreads
  // a few thousand rows over every SM.
  const StagedPlan plan = plan_staged(n_tokens, p.Hq, p.Hkv);
  if (plan.n_stages >= 3 && plan.n_chunks >= 4 * h->sm_count) {
    p.rows_per_group = 0;
    switch (q_kind) {
      case kQOutBf16: return launch_staged<kQOutBf16>(p, plan, h->sm_count, stream);
      case kQOutF16: return launch_staged<kQOutF16>(p, plan, h->sm_count, stream);
      default: return launch_staged<kQOutF32>(p, plan, h->sm_count, stream);
    }
  }
  // One wave: as many groups as the resident blocks hold (the occupancy of
  // each form is queried once per device), each group taking as many
  // consecutive rows as that needs -- a second, partial wave would double
  // the latency of a decode step's store.  Batches that fit one row per
  // group in the one-row form's wave (three blocks per SM) take it.
  static std::atomic<int> rows_blocks_per_sm[64][2];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVATTN_ERR_CUDA;
  int per_sm[2] = {0, 0};
  for (int one = 0; one < 2; ++one) {
    per_sm[one] = dev < 64 ? rows_blocks_per_sm[dev][one].load(std::memory_order_relaxed) : 0;
    if (per_sm[one] <= 0) {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
              &per_sm[one],
              one ? kv_store_rows_kernel<kQOutF32, true> : kv_store_rows_kernel<kQOutF32, false>,
              kThreads, 0) != cudaSuccess)
        return NVATTN_ERR_CUDA;
      per_sm[one] = std::max(1, per_sm[one]);
      if (dev < 64) rows_blocks_per_sm[dev][one].store(per_sm[one], std::memory_order_relaxed);
    }
  }
  const bool one_row = rows <= (long long)h->sm_count * per_sm[1] * kGroupsPerBlock;
  const long long per_wave = (long long)h->sm_count * per_sm[one_row ? 1 : 0] * kGroupsPerBlock;
  p.rows_per_group =
      (int)std::max(1LL, std::min<long long>(kMaxRowsPerGroup, (rows + per_wave - 1) / per_wave));
  const long long groups = (rows + p.rows_per_group - 1) / p.rows_per_group;
  const unsigned blocks = (unsigned)((groups + kGroupsPerBlock - 1) / kGroupsPerBlock);
  auto launch = [&](auto kernel) { kernel<<<blocks, kThreads, 0, stream>>>(p); };
  switch (q_kind) {
    case kQOutBf16:
      one_row ? launch(kv_store_rows_kernel<kQOutBf16, true>)
              : launch(kv_store_rows_kernel<kQOutBf16, false>);
      break;
    case kQOutF16:
      one_row ? launch(kv_store_rows_kernel<kQOutF16, true>)
              : launch(kv_store_rows_kernel<kQOutF16, false>);
      break;
    default:
      one_row ? launch(kv_store_rows_kernel<kQOutF32, true>)
              : launch(kv_store_rows_kernel<kQOutF32, false>);
  }
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace nvattn
