// decode.cu -- paged GQA split-KV decode attention over the BF16 block cache,
// on the tcgen05 tensor cores (sm_100a).
//
// Replaces the reference's decode attention path: LoadHistoryKV's per-token
// gather through block_table + bf16->f32 + reorder (src/engine/
// model_runner.cpp:300-376), FillVarlenMask (:219-243), the graph concat /
// pad / permute (src/models/qwen3.cpp:648-661) and BuildAttention's
// ggml_flash_attn_ext (qwen3.cpp:377-405).  The reference attends every query
// row over all sequences' concatenated history (O(B * sum L)); here each
// (sequence, kv head) reads only its own blocks, once, for all its GQA heads.
//
// Grid (split, kv head, sequence); a split is a run of split_tokens tokens.
// 128-token K and V tiles (32 KiB each, two TMA boxes {64, 1, 128} with
// 128-byte swizzle over the cache viewed as [layer*slot][kv head][128])
// stream through a 3-slot ring; two CTAs share an SM.
//   warp 0      TMA producer.
//   warp 1      TMEM allocation; one lane issues the MMAs:
//                 S^T = K Q^T   M = 128 tokens, N = 16, K = 128 dims
//                 O^T += V^T P^T M = 128 dims, N = 16, K = 128 tokens
//               N holds the G query heads twice: bf16(q) in columns [0, G)
//               and the bf16 remainder q - bf16(q) in [G, 2G) (zero above),
//               so S carries ~16 significant bits of q; P^T is split the
//               same way.  The padding to N = 16 makes the split free.
//   warps 2-5   thread = token of the tile (S^T lane) and = head dim (O^T
//               lane): per-head tile max by shuffles + shared memory, online
//               softmax in the log2 domain with lazy O rescaling (only when a
//               head's max grows by more than 2^8), per-thread partial row
//               sums reduced once per split, P^T written to shared memory in
//               the UMMA operand layout.
// A split writes either the final row (single split) or its (m, l, O)
// partial; the last split CTA of a (sequence, kv head) to finish -- found by
// an atomic ticket per (sequence, kv head), which that CTA re-arms to zero --
// merges the partials and writes the rows, so a decode is one launch.
//
// The fused step (nvattn_paged_decode_step on grids up to 32 CTAs per SM)
// also does the step's q/k RMSNorm + NEOX RoPE and the store of the new K/V
// row, so a decode step is one launch instead of the store kernel plus this
// one: warps 2-5 of every CTA norm and rotate the CTA's G query rows (eight
// lanes per row, the KV store's bit-exact row arithmetic from row_math.cuh)
// into shared memory, and the CTA whose split holds position ctx-1 -- the
// only one that reads it -- also writes the new K and V rows to the cache,
// fences them to the async proxy and releases its producer, which loads the
// tile holding that position only afterwards.  Larger grids run the step as
// the store kernel and the plain kernel (launch_paged_decode_step).
#include <atomic>
#include <functional>
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "row_math.cuh"

namespace nvattn {
namespace {

constexpr int kD = 128;
constexpr int kTile = 128;  // tokens per KV tile
constexpr int kSlots = 3;
constexpr int kThreads = 6 * 32;
constexpr int kHalfBytes = 128 * 64 * 2;  // one 128-row x 64-column bf16 box: 16 KiB
constexpr int kN = 16;                    // MMA N: heads x {hi, lo}, zero padded
constexpr uint32_t kTmemCols = 64;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct DecodeParams {
  int Hq, Hkv, layer, block_size, max_blocks, split_tokens, max_splits;
  int max_context;  // host bound on context_lens (<= max_blocks * block_size)
  long long n_slots, num_blocks;
  float scale_log2;  // softmax scale * log2(e)
  const float* q;
  const int32_t* block_tables;
  const int32_t* context_lens;
  float* out;
  float* ws_o;
  float* ws_ml;
  int* tickets;  // [n_seqs][Hkv] split tickets, zero between launches
  DeviceStatus* status;
  // fused step only: q above is the raw projection [n_seqs][Hq][128]
  const float* k_new;  // raw k, v rows [n_seqs][Hkv][128]
  const float* v_new;
  const uint16_t* qw;  // RMSNorm weights, bf16 [128]
  const uint16_t* kw;
  const int32_t* positions;
  const int32_t* slots;
  const float* rope;  // [max_position][cos x 64 | sin x 64]
  int max_position;
  float eps;
  uint16_t* k_cache;
  uint16_t* v_cache;
  // all-gather over peer memory: every final output row is also stored at
  // the same offset from each g_dst[p] (g_n ranks; 0 = no gather)
  float* g_dst[nvattn_handle::kMaxGatherRanks];
  int g_n;
  // ...and the step's release/wait (g_done != null): the CTA whose add takes
  // this rank's final-row count g_done to g_done_target (the last CTA of the
  // launch to write final rows) adds one to every rank's counter g_flag[p]
  // and waits until its own counter g_own_flag reaches g_flag_target
  uint32_t* g_flag[nvattn_handle::kMaxGatherRanks];
  const uint32_t* g_own_flag;
  unsigned* g_done;
  unsigned g_done_target;
  uint32_t g_flag_target;
};

// Releases this rank's rows of a gather step to every rank (a sequentially
// consistent system fence, then a system-scope release add on each rank's
// counter) and waits until this rank's counter shows every rank's rows of
// the step.  Bounded: after kWaitLimitNs it records NVATTN_ERR_TIMEOUT
// (detail = the count reached) and returns.
__device__ void gather_release_wait(uint32_t* const* flag, int n, const uint32_t* own,
                                    uint32_t target, DeviceStatus* status) {
  asm volatile("fence.sc.sys;" ::: "memory");
  for (int p = 0; p < n; ++p)
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(flag[p]) : "memory");
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(own) : "memory");
    if ((int)(v - target) >= 0) return;
    if ((it & 63u) == 63u && global_timer_ns() - t0 > kWaitLimitNs) {
      record_error(status, NVATTN_ERR_TIMEOUT, 80, (long long)v);
      return;
    }
    __nanosleep(64);
  }
}

template <int G>
struct __align__(1024) DecodeSmem {
  uint16_t kv[kSlots][2][kTile * 64];  // [slot][d half][token][64]
  uint16_t qt[2][kN * 64];             // Q^T operand: [d half][row][64]
  uint16_t pt[2][kN * 64];             // P^T operand: [token half][row][64]
  float red[2][4][kN];                 // per-warp tile maxima (double-buffered)
  float red_sum[4][kN];
  float qf[G][128];                    // fused step: the normed, rotated q rows
  uint64_t full[kSlots], empty[kSlots];
  uint64_t q_ready, s_full[2], p_full, o_done;
  uint64_t kv_stored;                  // fused step: the new K/V row is in the cache
  uint32_t tmem_base;
  int abort_flag;  // raised by the first wait that times out
  int last_split;  // this CTA merges the (sequence, kv head)'s partials
};

__device__ __forceinline__ int ring_slot(int idx) { return idx % kSlots; }
__device__ __forceinline__ uint32_t ring_parity(int idx) { return (uint32_t)(idx / kSlots) & 1u; }

// Byte offset of element (row n, column c) of a K-major, 128-byte-swizzled
// operand region of 64 columns: rows at 128 B, 16-byte chunks XOR row % 8.
__device__ __forceinline__ int sw128_offset(int n, int c) {
  return n * 128 + ((((c >> 3) ^ n) & 7) << 4) + (c & 7) * 2;
}

__device__ __forceinline__ uint16_t bf16_rn(float x) {
  return (uint16_t)(cvt_bf16x2(x, 0.0f) & 0xffffu);
}

// Fused step, warps 2-5 (128 threads = 16 groups of eight lanes): group g <
// G norms and rotates q row kvh*G + g into sm.qf[g]; in the CTA that stores
// (store_here) group G does the K row and group G+1 the V row and writes
// them to slot_mapping[seq] as the KV store does (positions outside the RoPE
// table and slots outside the cache reported, slot -1 skipped), and a slot
// that is not the block table's slot of position ctx-1 is reported (the
// attention would not read the new row there).  Every warp calls the
// warp-collective norm; the warps end on a barrier over the four.  (Issuing
// these loads before the CTA's barrier and TMEM set-up was measured slower.)
template <int G>
__device__ __forceinline__ void fused_rows(DecodeSmem<G>& sm, const DecodeParams& prm, int seq,
                                           int kvh, int ctx, bool store_here, int lane) {
  using namespace rowmath;
  const int tq = (int)threadIdx.x - 64;  // 0..127
  const int grp = tq >> 3, l8 = tq & 7;
  const int kind = grp < G ? 0 : (store_here && grp == G) ? 1 : (store_here && grp == G + 1) ? 2 : -1;
  const float* src = kind == 0   ? prm.q + ((long long)seq * prm.Hq + kvh * G + grp) * kD
                     : kind == 1 ? prm.k_new + ((long long)seq * prm.Hkv + kvh) * kD
                     : kind == 2 ? prm.v_new + ((long long)seq * prm.Hkv + kvh) * kD
                                 : nullptr;
  float x[2 * kPer];
  if (src != nullptr) {
    load_row(src, l8, x);
  } else {
#pragma unroll
    for (int e = 0; e < 2 * kPer; ++e) x[e] = 0.0f;
  }
  const bool normed = kind == 0 || kind == 1;
  // The RoPE row of position ctx-1 -- the new token's position in a decode
  // step -- and the norm weights load beside the row, not after the
  // position arrives; a step whose position differs reloads the RoPE row.
  const int pos_guess = min(max(ctx - 1, 0), prm.max_position - 1);
  float c[kPer], sn[kPer];
  auto load_rope = [&](int p) {
    const float4* cs = reinterpret_cast<const float4*>(prm.rope + (long long)p * kD + kPer * l8);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float4 a = __ldg(cs + j), b = __ldg(cs + kHalf / 4 + j);
      c[4 * j] = a.x; c[4 * j + 1] = a.y; c[4 * j + 2] = a.z; c[4 * j + 3] = a.w;
      sn[4 * j] = b.x; sn[4 * j + 1] = b.y; sn[4 * j + 2] = b.z; sn[4 * j + 3] = b.w;
    }
  };
  LaneWeights lw;
  if (normed) {
    load_rope(pos_guess);
    load_weights(kind == 0 ? prm.qw : prm.kw, l8, lw);
  }
  const int pos = prm.positions[seq];
  const bool pos_ok = pos >= 0 && pos < prm.max_position;
  bool finite;
  const float scale = rms_scale(x, normed, prm.eps, finite);
  bool nan_rule = !finite;
  if (normed && pos_ok) {
    if (pos != pos_guess) load_rope(pos);
    float w[2 * kPer];
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
      w[2 * e] = bf16lo_to_f32(lw.w[e]);
      w[2 * e + 1] = bf16hi_to_f32(lw.w[e]);
    }
    norm_rope(x, scale, w, c, sn);
    nan_rule = nan_rule || !lw.tame;
  }
  if (kind >= 0 && !pos_ok && l8 == 0) record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 26, pos);
  if (kind == 0) {
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
      sm.qf[grp][kPer * l8 + e] = pos_ok ? x[e] : 0.0f;
      sm.qf[grp][kHalf + kPer * l8 + e] = pos_ok ? x[kPer + e] : 0.0f;
    }
  } else if (kind > 0 && pos_ok) {
    const int slot = prm.slots[seq];
    if (slot >= 0) {
      if ((long long)slot >= prm.n_slots) {
        if (l8 == 0) record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 27, slot);
      } else {
        if (kind == 1 && l8 == 0 && ctx > 0) {
          const int p = ctx - 1;
          const long long want =
              (long long)prm.block_tables[(long long)seq * prm.max_blocks + p / prm.block_size] *
                  prm.block_size + p % prm.block_size;
          if (want != slot) record_error(prm.status, NVATTN_ERR_INVALID_ARG, 28, slot);
        }
        uint16_t* dst = (kind == 1 ? prm.k_cache : prm.v_cache) +
                        (((long long)prm.layer * prm.n_slots + slot) * prm.Hkv + kvh) * kD +
                        kPer * l8;
        *reinterpret_cast<uint4*>(dst) = pack8_bf16(x, nan_rule);
        *reinterpret_cast<uint4*>(dst + kHalf) = pack8_bf16(x + kPer, nan_rule);
      }
    }
  }
  if (store_here) {
    // The row's generic-proxy stores reach L2 and are ordered before the
    // producer's TMA (async proxy) load of the same tile.
    __threadfence();
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.kv_stored);
  }
  named_barrier_sync(1, 128);  // sm.qf complete
}

template <int G, bool kFused>
__global__ void __launch_bounds__(kThreads, 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, DecodeParams prm) {
  static_assert(2 * G <= kN, "GQA group too large for N = 16");
  extern __shared__ uint8_t smem_raw[];
  DecodeSmem<G>& sm = *reinterpret_cast<DecodeSmem<G>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int ctx = prm.context_lens[seq];
  const int t_begin = split * prm.split_tokens;
  if (ctx < 0 || ctx > prm.max_context) {
    // A length outside [0, max_context_len] would index past the block table
    // row or the grid; flag it and attend over the clamped range.
    if (threadIdx.x == 0 && split == 0) record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 10, ctx);
    ctx = ctx < 0 ? 0 : prm.max_context;
  }
  if (t_begin >= ctx && split > 0) return;  // nothing for this split
  const int n_splits = ctx > 0 ? (ctx + prm.split_tokens - 1) / prm.split_tokens : 1;
  if (timeout_recorded(prm.status)) {
    // An earlier launch timed out: skip the work, but keep the ticket count
    // right so the last split still re-arms it.
    if (threadIdx.x == 0 && n_splits > 1) {
      int* tk = prm.tickets + (long long)seq * prm.Hkv + kvh;
      if (atomicAdd(tk, 1) == n_splits - 1) atomicExch(tk, 0);
    }
    return;
  }
  const int t_end = min(ctx, t_begin + prm.split_tokens);
  const int n_tiles = t_end > t_begin ? (t_end - t_begin + kTile - 1) / kTile : 0;
  volatile int* abort_flag = &sm.abort_flag;
  // fused step: this split holds position ctx-1 (split 0 for an empty
  // context) and stores the new K/V row
  const bool store_here = kFused && split == (ctx > 0 ? (ctx - 1) / prm.split_tokens : 0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    mbar_init(&sm.q_ready, 4);
    mbar_init(&sm.s_full[0], 1);
    mbar_init(&sm.s_full[1], 1);
    mbar_init(&sm.p_full, 4);
    mbar_init(&sm.o_done, 1);
    mbar_init(&sm.kv_stored, 4);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const uint64_t policy = l2_policy_evict_first();
      const int n_loads = 2 * n_tiles;
      long long bid = 0;
      for (int idx = 0; idx < n_loads; ++idx) {
        const int slot = ring_slot(idx);
        if (idx >= kSlots)
          mbar_wait(&sm.empty[slot], ring_parity(idx) ^ 1u, prm.status, abort_flag, 11);
        // the last tile holds position ctx-1: load it after the new row is stored
        if (store_here && idx == 2 * (n_tiles - 1))
          mbar_wait(&sm.kv_stored, 0, prm.status, abort_flag, 24);
        const int tok = t_begin + (idx >> 1) * kTile;
        if ((idx & 1) == 0) {
          bid = prm.block_tables[(long long)seq * prm.max_blocks + tok / prm.block_size];
          if (bid < 0 || bid >= prm.num_blocks) {
            record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 12, bid);
            bid = 0;  // keep the pipeline flowing; the result is flagged invalid
          }
        }
        const int row = (int)((long long)prm.layer * prm.n_slots + bid * prm.block_size +
                              tok % prm.block_size);
        const CUtensorMap* map = (idx & 1) ? &tm_v : &tm_k;
        mbar_arrive_expect_tx(&sm.full[slot], 2 * kHalfBytes);
        tma_load_3d_hint(sm.kv[slot][0], map, &sm.full[slot], 0, kvh, row, policy);
        tma_load_3d_hint(sm.kv[slot][1], map, &sm.full[slot], 64, kvh, row, policy);
      }
      if constexpr (!kFused) {
        // The decode launch of a step run as two launches makes the fused
        // kernel's slot check: the stored row must be the one that position
        // ctx-1 is read from.  This split's last tile holds ctx-1, and a
        // 128-token tile never crosses a block, so bid is that block.
        if (prm.slots != nullptr && kvh == 0 && n_tiles > 0 && t_end == ctx) {
          const int pos = prm.positions[seq], slot = prm.slots[seq];
          if (pos >= 0 && pos < prm.max_position && slot >= 0 && (long long)slot < prm.n_slots &&
              bid * prm.block_size + (ctx - 1) % prm.block_size != slot)
            record_error(prm.status, NVATTN_ERR_INVALID_ARG, 28, slot);
        }
      }
      // Drain: the last load of every slot has landed before the CTA exits.
      for (int idx = max(0, n_loads - kSlots); idx < n_loads; ++idx)
        mbar_wait(&sm.full[ring_slot(idx)], ring_parity(idx), prm.status, 14);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16_f32(kTile, kN, 0, 0);
      constexpr uint32_t idesc_o = umma_idesc_bf16_f32(kD, kN, 1, 0);
      mbar_wait(&sm.q_ready, 0, prm.status, abort_flag, 15);
      auto issue_s = [&](int j) {
        const int slot = ring_slot(2 * j);
        mbar_wait(&sm.full[slot], ring_parity(2 * j), prm.status, abort_flag, 16);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const uint32_t koff = (uint32_t)(k & 3) * 32;
          const uint64_t a = umma_desc_sw128(smem_u32(sm.kv[slot][k >> 2]) + koff, 16, 1024);
          const uint64_t b = umma_desc_sw128(smem_u32(sm.qt[k >> 2]) + koff, 16, 1024);
          umma_bf16(tmem + (j & 1) * kN, a, b, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full[j & 1]);
        umma_commit(&sm.empty[slot]);
      };
      issue_s(0);
      for (int j = 0; j < n_tiles; ++j) {
        if (j + 1 < n_tiles) issue_s(j + 1);
        const int vslot = ring_slot(2 * j + 1);
        mbar_wait(&sm.p_full, j & 1, prm.status, abort_flag, 17);
        mbar_wait(&sm.full[vslot], ring_parity(2 * j + 1), prm.status, abort_flag, 18);
        tc_fence_after();
        const uint32_t vbase = smem_u32(sm.kv[vslot][0]);
#pragma unroll
        for (int k = 0; k < kTile / 16; ++k) {
          const uint64_t a = umma_desc_sw128(vbase + (uint32_t)k * 16 * 128, kHalfBytes, 1024);
          const uint64_t b =
              umma_desc_sw128(smem_u32(sm.pt[k >> 2]) + (uint32_t)(k & 3) * 32, 16, 1024);
          umma_bf16(tmem + 2 * kN, a, b, idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&sm.o_done);
        umma_commit(&sm.empty[vslot]);
      }
      // Drain: every MMA has completed before TMEM is released.
      mbar_wait(&sm.o_done, (n_tiles - 1) & 1, prm.status, 19);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad+32)
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;

    if constexpr (kFused) fused_rows<G>(sm, prm, seq, kvh, ctx, store_here, lane);

    // Q^T operand: row g = bf16(q_g * scale*log2e), row G+g = the bf16
    // remainder, rows >= 2G zero; thread r fills column (dim) r.  P^T rows
    // >= 2G are zeroed once and never written again.
    {
      const float* qp = prm.q + ((long long)seq * prm.Hq + (long long)kvh * G) * kD + r;
      uint8_t* qt = reinterpret_cast<uint8_t*>(sm.qt[r >> 6]);
      uint8_t* pt = reinterpret_cast<uint8_t*>(sm.pt[r >> 6]);
      const int c = r & 63;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float x = (kFused ? sm.qf[g][r] : qp[g * kD]) * prm.scale_log2;
        const uint16_t hi = bf16_rn(x);
        const uint16_t lo = bf16_rn(x - __uint_as_float((uint32_t)hi << 16));
        *reinterpret_cast<uint16_t*>(qt + sw128_offset(g, c)) = hi;
        *reinterpret_cast<uint16_t*>(qt + sw128_offset(G + g, c)) = lo;
      }
#pragma unroll
      for (int n = 2 * G; n < kN; ++n) {
        *reinterpret_cast<uint16_t*>(qt + sw128_offset(n, c)) = 0;
        *reinterpret_cast<uint16_t*>(pt + sw128_offset(n, c)) = 0;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.q_ready);
    }

    float m_used[G], l_part[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_used[g] = -INFINITY;
      l_part[g] = 0.0f;
    }

    for (int j = 0; j < n_tiles; ++j) {
      mbar_wait(&sm.s_full[j & 1], (j >> 1) & 1, prm.status, abort_flag, 20);
      tc_fence_after();
      uint32_t sv[16];
      tmem_ld16(tmem + lane_off + (j & 1) * kN, sv);
      tmem_wait_ld();
      const int tile0 = t_begin + j * kTile;
      const bool valid = tile0 + r < t_end;
      float sg[G];
#pragma unroll
      for (int g = 0; g < G; ++g)
        sg[g] = valid ? __uint_as_float(sv[g]) + __uint_as_float(sv[G + g]) : -INFINITY;

      // per-head maximum over the tile's 128 tokens
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float v = sg[g];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) sm.red[j & 1][quad][g] = v;
      }
      named_barrier_sync(1, 128);
      float alpha[G];
      bool rescale = false;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float tmax = fmaxf(fmaxf(sm.red[j & 1][0][g], sm.red[j & 1][1][g]),
                                 fmaxf(sm.red[j & 1][2][g], sm.red[j & 1][3][g]));
        const float m_new = fmaxf(m_used[g], tmax);
        alpha[g] = 1.0f;
        if (m_new > m_used[g] + kRescaleThreshold) {
          alpha[g] = fast_exp2(m_used[g] - m_new);
          rescale = rescale || j > 0;
          m_used[g] = m_new;
        }
      }
      float p[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        p[g] = valid ? fast_exp2(sg[g] - m_used[g]) : 0.0f;
        l_part[g] = fmaf(l_part[g], alpha[g], p[g]);
      }

      if (j > 0) {
        // PV(j-1) has finished: O is stable and the P^T buffer is free.
        mbar_wait(&sm.o_done, (j - 1) & 1, prm.status, abort_flag, 21);
        tc_fence_after();
      }
      if (rescale) {  // the same for every thread (shared tile maxima)
        uint32_t ov[16];
        tmem_ld16(tmem + lane_off + 2 * kN, ov);
        tmem_wait_ld();
#pragma unroll
        for (int n = 0; n < 2 * G; ++n)
          ov[n] = __float_as_uint(__uint_as_float(ov[n]) * alpha[n < G ? n : n - G]);
        tmem_st16(tmem + lane_off + 2 * kN, ov);
        tmem_wait_st();
      }
      if (tile0 + kTile > t_end) {
        // Keys at or past the context end hold whatever the cache slot
        // contains; zero their V rows so that P = 0 never meets a NaN.
        const int vidx = 2 * j + 1;
        mbar_wait(&sm.full[ring_slot(vidx)], ring_parity(vidx), prm.status, abort_flag, 22);
        if (!valid) {
          const uint4 z = make_uint4(0, 0, 0, 0);
          uint4* v0 = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sm.kv[ring_slot(vidx)][0]) + r * 128);
          uint4* v1 = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sm.kv[ring_slot(vidx)][1]) + r * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            v0[c] = z;
            v1[c] = z;
          }
        }
      }
      // P^T column r (token): row g = bf16(p_g), row G+g = remainder.
      uint8_t* pt = reinterpret_cast<uint8_t*>(sm.pt[r >> 6]);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const uint16_t hi = bf16_rn(p[g]);
        const uint16_t lo = bf16_rn(p[g] - __uint_as_float((uint32_t)hi << 16));
        *reinterpret_cast<uint16_t*>(pt + sw128_offset(g, r & 63)) = hi;
        *reinterpret_cast<uint16_t*>(pt + sw128_offset(G + g, r & 63)) = lo;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full);
    }

    // ---- epilogue: thread r = head dim r ----
    float l_tot[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float v = l_part[g];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) sm.red_sum[quad][g] = v;
    }
    named_barrier_sync(1, 128);
#pragma unroll
    for (int g = 0; g < G; ++g)
      l_tot[g] = (sm.red_sum[0][g] + sm.red_sum[1][g]) + (sm.red_sum[2][g] + sm.red_sum[3][g]);
    uint32_t ov[16];
    if (n_tiles > 0) {
      mbar_wait(&sm.o_done, (n_tiles - 1) & 1, prm.status, abort_flag, 23);
      tc_fence_after();
      tmem_ld16(tmem + lane_off + 2 * kN, ov);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int n = 0; n < 16; ++n) ov[n] = 0u;
    }
    if (n_splits == 1) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float o = __uint_as_float(ov[g]) + __uint_as_float(ov[G + g]);
        const long long oi = ((long long)seq * prm.Hq + kvh * G + g) * kD + r;
        const float y = l_tot[g] > 0.0f ? o / l_tot[g] : 0.0f;
        prm.out[oi] = y;
        for (int p = 0; p < prm.g_n; ++p) prm.g_dst[p][oi] = y;
      }
    } else {
      const long long base = (long long)(seq * prm.Hkv + kvh) * prm.max_splits;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const long long pidx = (base + split) * G + g;
        prm.ws_o[pidx * kD + r] = __uint_as_float(ov[g]) + __uint_as_float(ov[G + g]);
        if (r == 0) {
          prm.ws_ml[pidx * 2 + 0] = m_used[g];
          prm.ws_ml[pidx * 2 + 1] = l_tot[g];
        }
      }
      // Publish the partial, then take a ticket: the CTA that takes the
      // last one sees every other split's partial (fence, atomic, fence).
      __threadfence();
      named_barrier_sync(1, 128);
      if (r == 0) {
        int* tk = prm.tickets + (long long)seq * prm.Hkv + kvh;
        const int last = atomicAdd(tk, 1) == n_splits - 1;
        if (last) atomicExch(tk, 0);  // re-armed for the next launch
        sm.last_split = last;
      }
      named_barrier_sync(1, 128);
      if (sm.last_split) {
        __threadfence();
        // merge: thread r = head dim r, every split in order
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float M = -INFINITY;
          for (int i = 0; i < n_splits; ++i)
            M = fmaxf(M, __ldcg(prm.ws_ml + ((base + i) * G + g) * 2));
          float L = 0.0f, O = 0.0f;
          for (int i = 0; i < n_splits; ++i) {
            const long long pidx = (base + i) * G + g;
            const float w = fast_exp2(__ldcg(prm.ws_ml + pidx * 2) - M);
            L = fmaf(__ldcg(prm.ws_ml + pidx * 2 + 1), w, L);
            O = fmaf(__ldcg(prm.ws_o + pidx * kD + r), w, O);
          }
          const long long oi = ((long long)seq * prm.Hq + kvh * G + g) * kD + r;
          const float y = L > 0.0f ? O / L : 0.0f;
          prm.out[oi] = y;
          for (int p = 0; p < prm.g_n; ++p) prm.g_dst[p][oi] = y;
        }
      }
    }
    // rows stored to peers are visible system-wide before the CTA ends; only
    // the CTAs that wrote final rows (the one split, or the merging one) pay
    // for the system-scope fence -- the other splits stored nothing off-GPU.
    // With the release in the launch, each such CTA then counts itself, and
    // the last one releases the step's rows to every rank and waits for
    // theirs: every other CTA of the grid has finished its work by then.
    if (prm.g_n > 0 && (n_splits == 1 || sm.last_split)) {
      __threadfence_system();
      if (prm.g_done != nullptr) {
        named_barrier_sync(1, 128);
        if (r == 0 && atomicAdd(prm.g_done, 1u) == prm.g_done_target - 1u)
          gather_release_wait(prm.g_flag, prm.g_n, prm.g_own_flag, prm.g_flag_target,
                              prm.status);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int G, bool kFused = false>
nvattn_status launch_g(const CUtensorMap* tk, const CUtensorMap* tv, const DecodeParams& prm,
                       int n_seqs, int max_context_len, cudaStream_t stream) {
  const size_t smem = sizeof(DecodeSmem<G>) + 1024;
  // The attribute is per device; remember which devices have it.
  // (atomic: handles on different threads may launch at the same time)
  static std::atomic<unsigned long long> attr_set_mask{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVATTN_ERR_CUDA;
  if (dev >= 64 || !(attr_set_mask.load(std::memory_order_relaxed) & (1ull << dev))) {
    if (cudaFuncSetAttribute(paged_decode_kernel<G, kFused>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return NVATTN_ERR_CUDA;
    if (dev < 64) attr_set_mask.fetch_or(1ull << dev, std::memory_order_relaxed);
  }
  const int n_splits_max = max_context_len > 0
                               ? (max_context_len + prm.split_tokens - 1) / prm.split_tokens
                               : 1;
  dim3 grid(n_splits_max, prm.Hkv, n_seqs);
  paged_decode_kernel<G, kFused><<<grid, kThreads, smem, stream>>>(*tk, *tv, prm);
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace

// Tokens per split: whole 256-token blocks, small enough that the grid fills
// the GPU several times over when sequences are short, and at most 2048 so
// that log-uniform context lengths still balance across SMs.
static int split_tokens_for(int sm_count, int block_size, int n_kv_heads, int max_splits,
                            int n_seqs, int max_context_len) {
  const long long target_ctas = 4LL * 2 * sm_count;
  const long long units = (long long)n_seqs * n_kv_heads;
  int split = 2048;
  while (split > block_size && units * ((max_context_len + split - 1) / split) < target_ctas)
    split /= 2;
  if (split < block_size) split = block_size;
  // never more splits per sequence than the workspace holds
  while ((max_context_len + split - 1) / split > max_splits) split *= 2;
  return split;
}

// Splits per (sequence, kv head) that the workspace of a handle created with
// this max_context holds (the same rule nvattn_create applies).
static int workspace_max_splits(const nvattn_config& c) {
  const long long splits = (c.max_context + c.block_size - 1) / c.block_size;
  return (int)(splits < 64 ? splits : 64);
}

int decode_split_tokens(const nvattn_handle* h, int n_seqs, int max_context_len) {
  return split_tokens_for(h->sm_count, h->cfg.block_size, h->cfg.n_kv_heads, h->max_splits,
                          n_seqs, max_context_len);
}

// Handle-path launch of the plain decode (fused == nullptr) or of the fused
// step (fused: the raw k/v rows, norm weights, positions and slots).
struct FusedStepInputs {
  const float* k_new;
  const float* v_new;
  const uint16_t* qw;
  const uint16_t* kw;
  const int32_t* positions;
  const int32_t* slots;
  uint16_t* k_cache;  // the caches the new rows are written to
  uint16_t* v_cache;
};

// `step_check`: the plain decode of a step run as two launches (only the
// positions and slots of `fused` are used, for the slot check).
static nvattn_status launch_decode_common(nvattn_handle* h, int layer, int n_seqs, const float* q,
                                          const uint16_t* k_cache, const uint16_t* v_cache,
                                          const int32_t* block_tables, int max_blocks,
                                          const int32_t* context_lens, int max_context_len,
                                          float* out, const FusedStepInputs* fused,
                                          bool step_check, const DecodeParams* gather,
                                          cudaStream_t stream) {
  if (n_seqs == 0) return NVATTN_OK;
  CUtensorMap tk, tv;
  nvattn_status st = get_cache_tensor_map(h, k_cache, 64, kTile, CU_TENSOR_MAP_SWIZZLE_128B, &tk);
  if (st != NVATTN_OK) return st;
  st = get_cache_tensor_map(h, v_cache, 64, kTile, CU_TENSOR_MAP_SWIZZLE_128B, &tv);
  if (st != NVATTN_OK) return st;

  DecodeParams prm = {};
  prm.Hq = h->cfg.n_q_heads;
  prm.Hkv = h->cfg.n_kv_heads;
  prm.layer = layer;
  prm.block_size = h->cfg.block_size;
  prm.max_blocks = max_blocks;
  prm.max_context = max_context_len;
  prm.split_tokens = decode_split_tokens(h, n_seqs, max_context_len);
  prm.max_splits = h->max_splits;
  prm.n_slots = h->n_slots;
  prm.num_blocks = h->cfg.num_blocks;
  prm.scale_log2 = h->cfg.scale * kLog2e;
  prm.q = q;
  prm.block_tables = block_tables;
  prm.context_lens = context_lens;
  prm.out = out;
  prm.ws_o = h->ws_o;
  prm.ws_ml = h->ws_ml;
  prm.tickets = h->decode_tickets;
  prm.status = h->status_dev;
  if (gather != nullptr) {
    for (int p = 0; p < gather->g_n; ++p) {
      prm.g_dst[p] = gather->g_dst[p];
      prm.g_flag[p] = gather->g_flag[p];
    }
    prm.g_n = gather->g_n;
    prm.g_own_flag = gather->g_own_flag;
    prm.g_done = gather->g_done;
    prm.g_done_target = gather->g_done_target;
    prm.g_flag_target = gather->g_flag_target;
  }
  if (fused != nullptr && step_check) {
    prm.positions = fused->positions;
    prm.slots = fused->slots;
    prm.max_position = h->cfg.max_position;
  } else if (fused != nullptr) {
    prm.k_new = fused->k_new;
    prm.v_new = fused->v_new;
    prm.qw = fused->qw;
    prm.kw = fused->kw;
    prm.positions = fused->positions;
    prm.slots = fused->slots;
    prm.rope = h->rope_table_dev;
    prm.max_position = h->cfg.max_position;
    prm.eps = h->cfg.rms_eps;
    prm.k_cache = fused->k_cache;
    prm.v_cache = fused->v_cache;
    switch (prm.Hq / prm.Hkv) {
      case 1: return launch_g<1, true>(&tk, &tv, prm, n_seqs, max_context_len, stream);
      case 2: return launch_g<2, true>(&tk, &tv, prm, n_seqs, max_context_len, stream);
      case 4: return launch_g<4, true>(&tk, &tv, prm, n_seqs, max_context_len, stream);
      case 8: return launch_g<8, true>(&tk, &tv, prm, n_seqs, max_context_len, stream);
      default: return NVATTN_ERR_UNSUPPORTED;
    }
  }
  switch (prm.Hq / prm.Hkv) {
    case 1: return launch_g<1>(&tk, &tv, prm, n_seqs, max_context_len, stream);
    case 2: return launch_g<2>(&tk, &tv, prm, n_seqs, max_context_len, stream);
    case 4: return launch_g<4>(&tk, &tv, prm, n_seqs, max_context_len, stream);
    case 8: return launch_g<8>(&tk, &tv, prm, n_seqs, max_context_len, stream);
    default: return NVATTN_ERR_UNSUPPORTED;
  }
}

nvattn_status launch_paged_decode(nvattn_handle* h, int layer, int n_seqs, const float* q,
                                  const uint16_t* k_cache, const uint16_t* v_cache,
                                  const int32_t* block_tables, int max_blocks,
                                  const int32_t* context_lens, int max_context_len,
                                  float* out, cudaStream_t stream) {
  return launch_decode_common(h, layer, n_seqs, q, k_cache, v_cache, block_tables, max_blocks,
                              context_lens, max_context_len, out, nullptr, false, nullptr, stream);
}

// The step as one launch or two.  Each CTA of the fused kernel norms and
// rotates its own G query rows -- the position, then the RoPE row, then the
// norm, 0.7-1 us on its critical path -- where the separate KV store does
// that once per head.  Measured on the 256-sequence, 8-kv-head,
// 1k-32k-token workload (interleaved runs on one GPU) against the store and
// decode launches: its full grid (32,768 CTAs) ran the fused step ~1 %
// slower, its 4-way shard (8,192 CTAs, 55 per SM) 0.6 % slower, its 8-way
// shard (4,096, 28 per SM) ~1 % faster, and small batches gain the whole
// store launch.  Grids above 32 CTAs per SM take the two launches.
constexpr long long kStepFusedMaxGridPerSm = 32;

int decode_step_launches(const nvattn_handle* h, int n_seqs, int max_context_len) {
  const int split = decode_split_tokens(h, n_seqs, max_context_len);
  const long long splits = max_context_len > 0 ? (max_context_len + split - 1) / split : 1;
  const long long grid = (long long)n_seqs * h->cfg.n_kv_heads * splits;
  return grid <= kStepFusedMaxGridPerSm * h->sm_count ? 1 : 2;
}

static nvattn_status decode_step_impl(nvattn_handle* h, int layer, int n_seqs, const float* q,
                                      const float* k_new, const float* v_new,
                                      const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                      const int32_t* positions, const int32_t* slots,
                                      uint16_t* k_cache, uint16_t* v_cache,
                                      const int32_t* block_tables, int max_blocks,
                                      const int32_t* context_lens, int max_context_len, float* out,
                                      const DecodeParams* gather, cudaStream_t stream) {
  const FusedStepInputs f{k_new, v_new, q_norm_w, k_norm_w, positions, slots, k_cache, v_cache};
  if (decode_step_launches(h, n_seqs, max_context_len) == 2) {
    const nvattn_status st =
        launch_kv_store(h, layer, n_seqs, q, k_new, v_new, q_norm_w, k_norm_w, positions, slots,
                        h->q_step, NVATTN_DTYPE_F32, k_cache, v_cache, nullptr, nullptr, stream);
    if (st != NVATTN_OK) return st;
    return launch_decode_common(h, layer, n_seqs, h->q_step, k_cache, v_cache, block_tables,
                                max_blocks, context_lens, max_context_len, out, &f, true, gather,
                                stream);
  }
  return launch_decode_common(h, layer, n_seqs, q, k_cache, v_cache, block_tables, max_blocks,
                              context_lens, max_context_len, out, &f, false, gather, stream);
}

nvattn_status launch_paged_decode_step(nvattn_handle* h, int layer, int n_seqs, const float* q,
                                       const float* k_new, const float* v_new,
                                       const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                       const int32_t* positions, const int32_t* slots,
                                       uint16_t* k_cache, uint16_t* v_cache,
                                       const int32_t* block_tables, int max_blocks,
                                       const int32_t* context_lens, int max_context_len,
                                       float* out, cudaStream_t stream) {
  return decode_step_impl(h, layer, n_seqs, q, k_new, v_new, q_norm_w, k_norm_w, positions, slots,
                          k_cache, v_cache, block_tables, max_blocks, context_lens,
                          max_context_len, out, nullptr, stream);
}

namespace {
struct GatherSync {
  uint32_t* flag[nvattn_handle::kMaxGatherRanks];  // every rank's counter, mapped here
  uint32_t* own;
  int n;
  uint32_t target;
  DeviceStatus* status;
};

// A step with no sequences has no decode launch to release from: one thread
// releases and waits instead (gather_release_wait).
__global__ void gather_sync_kernel(GatherSync g) {
  if (threadIdx.x == 0) gather_release_wait(g.flag, g.n, g.own, g.target, g.status);
}
}  // namespace

nvattn_status launch_paged_decode_step_gather(nvattn_handle* h, int layer, int n_seqs,
                                              const float* q, const float* k_new,
                                              const float* v_new, const uint16_t* q_norm_w,
                                              const uint16_t* k_norm_w, const int32_t* positions,
                                              const int32_t* slots, uint16_t* k_cache,
                                              uint16_t* v_cache, const int32_t* block_tables,
                                              int max_blocks, const int32_t* context_lens,
                                              int max_context_len, float* out,
                                              cudaStream_t stream) {
  if (!h->g_connected) return NVATTN_ERR_INVALID_ARG;
  const long long parity_off = (long long)(h->g_steps & 1u) * h->g_ranks * h->g_slice;
  const uint32_t flag_target = (uint32_t)h->g_ranks * (h->g_steps + 1u);
  uint32_t* own_flag = reinterpret_cast<uint32_t*>(h->g_own + h->g_flag_off);
  if (n_seqs == 0) {
    GatherSync gs = {};
    for (int p = 0; p < h->g_ranks; ++p)
      gs.flag[p] = reinterpret_cast<uint32_t*>(h->g_peer[p] + h->g_flag_off);
    gs.own = own_flag;
    gs.n = h->g_ranks;
    gs.target = flag_target;
    gs.status = h->status_dev;
    gather_sync_kernel<<<1, 32, 0, stream>>>(gs);
    if (cudaGetLastError() != cudaSuccess) return NVATTN_ERR_CUDA;
    ++h->g_steps;
    return NVATTN_OK;
  }
  // One CTA per (sequence, kv head) writes that pair's final rows; the
  // count runs on across steps (compared modulo 2^32), so nothing re-arms it.
  const unsigned done_target = h->g_done_total + (unsigned)n_seqs * (unsigned)h->cfg.n_kv_heads;
  DecodeParams gd = {};
  gd.g_n = h->g_ranks;
  for (int p = 0; p < h->g_ranks; ++p) {
    gd.g_dst[p] = reinterpret_cast<float*>(h->g_peer[p]) + parity_off +
                  (long long)h->g_rank * h->g_slice;
    gd.g_flag[p] = reinterpret_cast<uint32_t*>(h->g_peer[p] + h->g_flag_off);
  }
  gd.g_own_flag = own_flag;
  gd.g_done =
      reinterpret_cast<unsigned*>(h->g_own + h->g_flag_off + nvattn_handle::kGatherDoneOffset);
  gd.g_done_target = done_target;
  gd.g_flag_target = flag_target;
  nvattn_status st = decode_step_impl(h, layer, n_seqs, q, k_new, v_new, q_norm_w, k_norm_w,
                                      positions, slots, k_cache, v_cache, block_tables,
                                      max_blocks, context_lens, max_context_len, out, &gd, stream);
  if (st != NVATTN_OK) return st;
  h->g_done_total = done_target;
  ++h->g_steps;
  return NVATTN_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free decode (nvattn_paged_decode_noalloc).
//
// The split-KV partials live in this file-scope device array instead of a
// handle's cudaMalloc'd workspace.  Every GPU that loads the library holds
// these 32 MiB until the process exits.  The array's name is only a host-side
// stand-in for the device symbol, so the host fetches its real device address
// with cudaGetSymbolAddress, once per device, and passes that to the kernel.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
static_assert(sizeof(DeviceStatus) == sizeof(nvattn_device_status), "status layout");
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
// Per-device set-up, done once under std::call_once: the scratch's device
// address and the SM count.  call_once publishes both to every thread that
// later passes the same flag, so no caller can see the address without the
// SM count that chooses its splits.
struct NoAllocDevice {
  std::once_flag once;
  cudaError_t err = cudaSuccess;
  void* scratch = nullptr;
  int sm_count = 0;
};
NoAllocDevice g_noalloc_dev[kMaxDevices];

// Runs on the current device `dev` (the caller made it current).
void noalloc_setup(NoAllocDevice& d, int dev) {
  void* addr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
  int sms = 0;
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess && (addr == nullptr || sms <= 0)) e = cudaErrorInvalidValue;
  d.err = e;
  if (e == cudaSuccess) {
    d.scratch = addr;
    d.sm_count = sms;
  }
}
}  // namespace

}  // namespace nvattn

extern "C" NVATTN_API nvattn_status nvattn_paged_decode_noalloc(
    const nvattn_config* cfg, int layer, int n_seqs, const float* q_dev,
    const uint16_t* k_cache_dev, const uint16_t* v_cache_dev, const int32_t* block_tables_dev,
    int max_blocks, const int32_t* context_lens_dev, int max_context_len, float* out_dev,
    nvattn_device_status* status_dev, nvattn_stream_t stream) {
  using namespace nvattn;
  if (cfg == nullptr) return NVATTN_ERR_INVALID_ARG;
  const nvattn_config& c = *cfg;
  if (c.n_layer <= 0 || c.n_q_heads <= 0 || c.n_kv_heads <= 0 || c.num_blocks <= 0 ||
      c.block_size <= 0 || c.max_context <= 0 || c.n_q_heads % c.n_kv_heads != 0 ||
      !(c.scale > 0.0f))
    return NVATTN_ERR_INVALID_ARG;
  const int G = c.n_q_heads / c.n_kv_heads;
  if (c.head_dim != kD || c.block_size % 128 != 0 || c.block_size > 1024 ||
      !(G == 1 || G == 2 || G == 4 || G == 8))
    return NVATTN_ERR_UNSUPPORTED;
  const long long n_slots = c.num_blocks * (long long)c.block_size;
  if ((long long)c.n_layer * n_slots >= (1LL << 31)) return NVATTN_ERR_UNSUPPORTED;
  if (layer < 0 || layer >= c.n_layer || n_seqs < 0 || n_seqs > kMaxDecodeSeqs ||
      max_blocks <= 0 || max_context_len < 0 ||
      max_context_len > c.max_context ||
      (long long)max_context_len > (long long)max_blocks * c.block_size)
    return NVATTN_ERR_INVALID_ARG;
  if (n_seqs == 0) return NVATTN_OK;
  const void* ptrs[] = {q_dev, k_cache_dev, v_cache_dev, out_dev};
  for (const void* p : ptrs)
    if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) != 0) return NVATTN_ERR_INVALID_ARG;
  if (block_tables_dev == nullptr || context_lens_dev == nullptr) return NVATTN_ERR_INVALID_ARG;

  // Runs on the caller's current device, which must be cfg->device.
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVATTN_ERR_CUDA;
  if (dev != c.device || dev < 0 || dev >= kMaxDevices) return NVATTN_ERR_INVALID_ARG;
  // One-time set-up on this device (allocates nothing).  A failure is kept
  // and returned by every later call on the device.
  NoAllocDevice& nd = g_noalloc_dev[dev];
  std::call_once(nd.once, noalloc_setup, std::ref(nd), dev);
  if (nd.err != cudaSuccess) return NVATTN_ERR_CUDA;

  // Same split rule as a handle created from this config, so the result
  // equals nvattn_paged_decode's.
  const int split = split_tokens_for(nd.sm_count, c.block_size, c.n_kv_heads,
                                     workspace_max_splits(c), n_seqs, max_context_len);
  const int n_splits = max_context_len > 0 ? (max_context_len + split - 1) / split : 1;
  const size_t rows = n_splits > 1 ? (size_t)n_seqs * c.n_q_heads * n_splits : 0;
  // scratch layout: split tickets (n_seqs x n_kv_heads ints, padded to 256 B),
  // then the partial rows' O (rows x 128 f32) and (m, l) (rows x 2 f32)
  const size_t ticket_bytes =
      n_splits > 1 ? ((size_t)n_seqs * c.n_kv_heads * sizeof(int) + 255) / 256 * 256 : 0;
  if (ticket_bytes + rows * (kD + 2) * sizeof(float) > kNoAllocScratchBytes)
    return NVATTN_ERR_SCRATCH_LIMIT;

  CUtensorMap tk, tv;
  nvattn_status st = encode_tensor_map_3d(&tk, k_cache_dev, kD, (uint64_t)c.n_kv_heads,
                                          (uint64_t)c.n_layer * (uint64_t)n_slots, kD * 2,
                                          (uint64_t)c.n_kv_heads * kD * 2, 64, 1, kTile,
                                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVATTN_OK) return st;
  st = encode_tensor_map_3d(&tv, v_cache_dev, kD, (uint64_t)c.n_kv_heads,
                            (uint64_t)c.n_layer * (uint64_t)n_slots, kD * 2,
                            (uint64_t)c.n_kv_heads * kD * 2, 64, 1, kTile,
                            CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVATTN_OK) return st;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* tickets = static_cast<int*>(nd.scratch);
  float* scratch = reinterpret_cast<float*>(static_cast<char*>(nd.scratch) + ticket_bytes);
  // The tickets must start at zero: the array keeps whatever the last call
  // (possibly one cut short by a timeout) left there.
  if (ticket_bytes > 0 && cudaMemsetAsync(tickets, 0, ticket_bytes, s) != cudaSuccess)
    return NVATTN_ERR_CUDA;
  DecodeParams prm = {};  // fused-step, slot-check and gather fields stay null
  prm.Hq = c.n_q_heads;
  prm.Hkv = c.n_kv_heads;
  prm.layer = layer;
  prm.block_size = c.block_size;
  prm.max_blocks = max_blocks;
  prm.max_context = max_context_len;
  prm.split_tokens = split;
  prm.max_splits = n_splits;  // partial-row stride
  prm.n_slots = n_slots;
  prm.num_blocks = c.num_blocks;
  prm.scale_log2 = c.scale * kLog2e;
  prm.q = q_dev;
  prm.block_tables = block_tables_dev;
  prm.context_lens = context_lens_dev;
  prm.out = out_dev;
  prm.ws_o = scratch;
  prm.ws_ml = scratch + rows * kD;
  prm.tickets = tickets;
  prm.status = reinterpret_cast<DeviceStatus*>(status_dev);
  switch (G) {
    case 1: return launch_g<1>(&tk, &tv, prm, n_seqs, max_context_len, s);
    case 2: return launch_g<2>(&tk, &tv, prm, n_seqs, max_context_len, s);
    case 4: return launch_g<4>(&tk, &tv, prm, n_seqs, max_context_len, s);
    default: return launch_g<8>(&tk, &tv, prm, n_seqs, max_context_len, s);
  }
}
