// prefill.cu -- causal paged prefill / prefix-hit / chunked-prefill attention
// on the 5th-generation tensor cores (tcgen05 + TMEM, CTA pairs), sm_100a.
//
// Replaces the reference's prefill attention: FillCausalMask
// (src/engine/model_runner.cpp:188-217), the prefill pad/permute
// (src/models/qwen3.cpp:524-531) and BuildAttention's ggml_flash_attn_ext
// (qwen3.cpp:377-405).  The reference attends only over the batch's new
// tokens and ignores a cached prefix (qwen3.cpp:445-446); here a row at
// position P attends keys [0, P] of its sequence through the block table,
// which covers prefix-cache hits and chunked prefill alike.
//
// Precision: the reference's flash attention runs on F16 Q, K and V
// (ggml_cast of K/V, qwen3.cpp:388-393, and the F16 conversion of Q inside
// ggml_flash_attn_ext).  Here Q arrives as f16 (the fused store's f16 q
// output), each K and V tile is converted bf16 -> f16 in shared memory (exact
// in f16's range; overflow above 65504 as in ggml_cast), S = Q K^T multiplies
// f16 operands, P is rounded to f16 for P.V, and accumulation is f32.  (A bf16
// Q, 8 significant bits, put the output ~1.4e-3 mean-rel from exact math on
// f32 queries; f16 Q, 11 bits, ~2e-4.)
//
// CTA pairs (clusters of two, tcgen05 cta_group::2).  A work item is four
// 128-row query tiles that read the same keys, two per CTA: four GQA heads
// of the same rows, or -- when a kv head serves fewer than four q heads --
// consecutive row tiles.  Keys come in 128-key tiles, and each CTA stages
// half of every tile: K for keys [64r, 64r+64) of the tile (all 128 dims)
// and V for dims [64r, 64r+64) (all 128 keys), r = the CTA's rank in the
// pair.  The pair MMAs (M = 256) read A rows from each CTA's own shared
// memory or TMEM and B columns from both CTAs' halves, and each CTA's TMEM
// receives its own 128 rows:
//   S_t  = Q_t K^T  (M=256 rows of the pair, N=128 keys, K=128 dims)
//   O_t += P_t V    (A = P from each CTA's TMEM, N=128 dims, K=128 keys)
// so each SM stages, converts and feeds the tensor core half of each K/V
// tile, and one thread issues the MMAs of both SMs.  The kernel is
// persistent (one CTA per SM): the leader (rank 0) takes items in the order a
// (query tile, kv head, sequence) grid would launch them -- the query tiles
// of one sequence and kv head together, longest first, which keeps their K/V
// shared in L2 -- from a counter in the handle's workspace (the last CTA to
// finish zeroes it) and hands each item to both CTAs' roles through a 2-slot
// work ring in shared memory; the next item's Q, first K tile and first S
// MMAs overlap the current item's last softmax and epilogue.
//   warp 0       leader: work items from the counter into both CTAs' work
//                rings; both CTAs: TMA producer of the CTA's own Q tiles and
//                K/V halves through a ring of 16 KiB slots (128-byte swizzle)
//                that runs on across items.
//   warp 1       TMEM allocation for the pair; in the leader the warp runs
//                the MMA loop converged and one elected lane issues the pair
//                MMAs, interleaving the two tiles so the tensor cores work on
//                one tile while the other tile's softmax runs:
//                  PV0(j), S0(j+1), PV1(j), S1(j+1), ...
//                (strictly in this order from one thread: MMAs execute in
//                issue order, and two issuing threads would interleave the
//                tiles' P.V -> S bursts and lengthen each tile's chain).
//   warps 12-15  K/V converters (one per SM sub-partition): bf16 -> f16 in
//                place, K one key tile ahead of V, V rows past the context
//                zeroed (a cache slot past a sequence's end may hold NaN
//                bits; masked K columns never reach P).
// With the step's own K/V rows given in f16 (nvattn_paged_prefill_rows),
// keys at or past a sequence's cached prefix are the reference's F16 casts of
// the graph rows instead of the BF16 cache's: a key tile that starts there is
// loaded from those rows (no conversion), and the one tile that straddles
// the prefix end takes its later keys from the rows while converting the
// rest.
//   warps 2-3    idle.
//   warps 4-7    softmax of tile 0; warps 8-11 softmax of tile 1: thread =
//                query row = TMEM lane.  Causal mask, online softmax in the
//                log2 domain, P written as f16 into the TMEM columns of its
//                own S (S was read to registers), lazy O rescaling (only when
//                a row max grows by more than 2^8), epilogue O / l.
// Barriers the leader's MMA lane waits on (K/V converted, P written, work
// slot free) live in the leader and count both CTAs' arrivals (the leader's
// warps arrive locally, the follower's remotely: CTA-scope release for the
// per-tile barriers, whose payload only the MMAs read, cluster scope for the
// work ring, which carries data); MMA completions arrive on the barrier at
// the same offset in both CTAs.
// MMAs issued by one thread execute in order, so S(j+1) may overwrite the
// columns of P(j) right after PV(j) is issued, and the completion of S(j+1)
// implies PV(j) is done (its O may then be rescaled).
// TMEM columns (each CTA): tile t uses [256t, 256t+128) for S/P and
// [256t+128, 256t+256) for O.
#include <algorithm>
#include <atomic>
#include <climits>

#include "common.cuh"
#include "internal.h"

namespace nvattn {
namespace {

constexpr int kD = 128;
constexpr int kBM = 128;  // query rows per tile
constexpr int kBN = 128;  // keys per tile
constexpr int kSlots = 10;
constexpr int kThreads = 16 * 32;
constexpr int kConvThreads = 128;          // warps 12-15
constexpr int kConvAhead = 4;              // converter lead, in key tiles (barrier sets)
constexpr int kSlotBytes = 16 * 1024;      // one CTA's half of a K or V tile
constexpr int kQBoxBytes = 128 * 64 * 2;   // one 128-row x 64-column f16 box
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct PrefillParams {
  int Hq, Hkv, G, layer, block_size, max_blocks, n_mtiles, mode;
  int gx, n_items;  // pair items per (sequence, kv head); items in all
  int n_tokens;     // rows of q and out
  long long n_slots, num_blocks;
  float scale_log2;
  const int32_t* cu_q;
  const int32_t* q_starts;
  const int32_t* context_lens;
  const int32_t* block_tables;
  const uint16_t* k_rows;  // nullable: the step's rows in f16, [n_tokens][Hkv][128]
  const uint16_t* v_rows;
  float* out;
  DeviceStatus* status;
  int* sched;  // [0] next work item, [1] CTAs finished; the last CTA zeroes both
};

// Item modes: how a pair item's four query tiles are chosen.
constexpr int kModeHeads = 0;  // four heads of one row tile (G >= 4)
constexpr int kModePair = 1;   // two heads x two row tiles (G == 2)
constexpr int kModeRows = 2;   // one head x four row tiles (G == 1)

// One CTA's view of a work item (written by the leader's producer into both
// CTAs' rings, read by every role).  valid == 0 ends the CTA's loop.
struct Work {
  int valid, seq, kvh, q0, q_start, ctx, n_kv, p_last0, n_q;
  int head[2], row0[2], rows[2];
};
constexpr int kWorkWords = sizeof(Work) / 4;

struct __align__(1024) PrefillSmem {
  uint16_t q[2][2][kBM * 64];     // [tile][d half][row][64]
  uint16_t kv[kSlots][kBN * 64];  // K half: [d half][64 keys][64]; V half: [128 keys][64]
  uint64_t q_full;                // leader: both CTAs' Q bytes
  uint64_t full[kSlots], empty[kSlots];
  uint64_t s_full[2], p_full[2];
  // per key tile gj, indexed gj % kConvAhead: converted K / V ready for the
  // MMAs (leader; v_ready(gj) also covers K(gj+1))
  uint64_t k_ready[4], v_ready[4];
  uint64_t o_final;
  uint64_t q_empty;                      // the item's last S MMAs have read Q
  uint64_t work_full[2], work_empty[2];  // the work ring (work_empty: leader)
  Work work[2];
  uint32_t tmem_base;
  int abort_flag;  // raised by the first wait that times out
};

// Dynamic shared memory (+1 KiB for the 1024-byte alignment) within the
// 227 KiB a CTA may use.
static_assert(sizeof(PrefillSmem) + 1024 <= 227 * 1024, "prefill shared memory");

// Arrivals that release a work-ring slot: per CTA the 4 converter warps and
// the 8 softmax warps, plus the leader's MMA lane and the follower's
// producer.
constexpr int kWorkReaders = 2 * (1 + 4 + 8);
// Arrivals on the leader's per-tile barriers: one per warp of both CTAs.
constexpr int kPairWarps4 = 2 * 4;

__device__ __forceinline__ int ring_slot(int idx) { return idx % kSlots; }
__device__ __forceinline__ uint32_t ring_parity(int idx) { return (uint32_t)(idx / kSlots) & 1u; }

// ---------------------------------------------------------------- work items
// Pair item `item` in launch order: x fastest, then kv head, then sequence,
// as a gx x Hkv x n_seqs grid.  Fills both CTAs' views.  Returns false for an
// item without query rows or with invalid metadata (the latter recorded in
// the status word).  The items without rows of a (sequence, kv head) are its
// first x values (longest tiles first); for one of them `skip_to` is the
// group's first item with rows (or the next group), so the caller can move
// the counter past the rest.
__device__ __forceinline__ bool decode_item(const PrefillParams& prm, int item, Work (&w)[2],
                                            int& skip_to) {
  const int x = item % prm.gx;
  const int yz = item / prm.gx;
  const int kvh = yz % prm.Hkv;
  const int seq = yz / prm.Hkv;
  for (int r = 0; r < 2; ++r) {
    w[r].kvh = kvh;
    w[r].seq = seq;
    if (prm.mode == kModeHeads) {
      const int per_tile = prm.G / 4;  // pair items per row tile
      const int mt = prm.n_mtiles - 1 - x / per_tile;
      const int h0 = kvh * prm.G + 4 * (x % per_tile) + 2 * r;
      w[r].head[0] = h0;
      w[r].head[1] = h0 + 1;
      w[r].row0[0] = w[r].row0[1] = mt * kBM;
    } else if (prm.mode == kModePair) {
      const int m = (prm.n_mtiles + 1) / 2 - 1 - x;
      w[r].head[0] = kvh * 2;
      w[r].head[1] = kvh * 2 + 1;
      w[r].row0[0] = w[r].row0[1] = (2 * m + r) * kBM;
    } else {
      const int m = (prm.n_mtiles + 3) / 4 - 1 - x;
      w[r].head[0] = w[r].head[1] = kvh;
      w[r].row0[0] = (4 * m + 2 * r) * kBM;
      w[r].row0[1] = w[r].row0[0] + kBM;
    }
  }
  const int q0 = prm.cu_q[seq];
  const int q1 = prm.cu_q[seq + 1];
  if (q0 < 0 || q1 < q0 || q1 > prm.n_tokens) {
    // rows outside q / out: the sequence is skipped (all its items)
    record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 25, q1);
    skip_to = item - x + prm.gx;
    return false;
  }
  const int n_q = q1 - q0;
  if (n_q > prm.n_mtiles * kBM && x == 0 && kvh == 0)
    record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 21, n_q);
  skip_to = item + 1;
  if (w[0].row0[0] >= n_q) {  // the item's first (smallest-row) tile has no rows
    int x_first = prm.gx;
    if (n_q > 0) {
      const int last = (n_q - 1) / kBM;  // last row tile with rows
      x_first = prm.mode == kModeHeads  ? (prm.n_mtiles - 1 - last) * (prm.G / 4)
                : prm.mode == kModePair ? (prm.n_mtiles + 1) / 2 - 1 - last / 2
                                        : (prm.n_mtiles + 3) / 4 - 1 - last / 4;
    }
    skip_to = item - x + max(x_first, x + 1);
    return false;
  }
  const int q_start = prm.q_starts[seq];
  int p_last = 0;
  for (int r = 0; r < 2; ++r)
    for (int t = 0; t < 2; ++t) {
      w[r].rows[t] = max(0, min(kBM, n_q - w[r].row0[t]));
      if (w[r].rows[t] > 0) p_last = max(p_last, q_start + w[r].row0[t] + w[r].rows[t] - 1);
    }
  if (q_start < 0 || (long long)p_last >= (long long)prm.max_blocks * prm.block_size) {
    record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 22, p_last);
    return false;
  }
  int ctx = prm.context_lens[seq];
  if (ctx <= p_last) {
    record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 23, ctx);
    ctx = p_last + 1;
  }
  // Rows past a tile's end (or a tile without rows) mimic the item's first
  // tile's last row, which always exists.
  const int p_last0 = q_start + w[0].row0[0] + w[0].rows[0] - 1;
  for (int r = 0; r < 2; ++r) {
    w[r].q0 = q0;
    w[r].n_q = n_q;
    w[r].q_start = q_start;
    w[r].ctx = ctx;
    w[r].n_kv = p_last / kBN + 1;
    w[r].p_last0 = p_last0;
    w[r].valid = 1;
  }
  return true;
}

// Every role runs the same sequence of items, so each keeps the CTA-wide
// count of key tiles before the current item (`tb`): key tile j of the item
// is tile gj = tb + j, its K and V halves are ring loads 2*gj and 2*gj + 1,
// and the per-tile barriers are in phase gj.

// ---------------------------------------------------------------- producer
__device__ __forceinline__ void producer_role(PrefillSmem& sm, const CUtensorMap* tm_q,
                                              const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                                              const CUtensorMap* tm_kr, const CUtensorMap* tm_vr,
                                              const PrefillParams& prm, uint32_t rank) {
  volatile int* abort_flag = &sm.abort_flag;
  tma_prefetch_desc(tm_q);
  tma_prefetch_desc(tm_k);
  tma_prefetch_desc(tm_v);
  const bool staged = prm.k_rows != nullptr;
  if (staged) {
    tma_prefetch_desc(tm_kr);
    tma_prefetch_desc(tm_vr);
  }
  const uint32_t q_full_leader = smem_peer(&sm.q_full, 0);
  int g = 0;  // ring loads issued so far
  for (int k = 0;; ++k) {
    const int ws = k & 1;
    Work w;
    if (rank == 0) {
      // Take the next item for the pair and publish both CTAs' views (after
      // every reader of the slot, in both CTAs, has released it; a wait that
      // ran out has raised the abort flag, which ends the work below).
      if (k >= 2)
        mbar_wait_cluster(&sm.work_empty[ws], ((k >> 1) - 1) & 1, prm.status, abort_flag, 45);
      Work pw[2];
      pw[0].valid = pw[1].valid = 0;
      // An earlier launch that timed out leaves its status: take no work then.
      while (!*abort_flag && !timeout_recorded(prm.status)) {
        const int item = atomicAdd(prm.sched, 1);
        int skip_to;
        if (item >= prm.n_items) break;
        if (decode_item(prm, item, pw, skip_to)) break;
        pw[0].valid = pw[1].valid = 0;
        // Items in (item, skip_to) are empty: nobody needs to take them.
        if (skip_to > item + 1) atomicMax(prm.sched, skip_to);
      }
      sm.work[ws] = pw[0];
      const uint32_t peer = smem_peer(&sm.work[ws], 1);
      const uint32_t* src = reinterpret_cast<const uint32_t*>(&pw[1]);
#pragma unroll
      for (int i = 0; i < kWorkWords; ++i) st_cluster_u32(peer + 4 * i, src[i]);
      mbar_arrive(&sm.work_full[ws]);
      mbar_arrive_cluster(smem_peer(&sm.work_full[ws], 1));
      w = pw[0];
    } else {
      if (!mbar_wait_cluster(&sm.work_full[ws], (k >> 1) & 1, prm.status, abort_flag, 45)) break;
      w = sm.work[ws];
      mbar_arrive_cluster(smem_peer(&sm.work_empty[ws], 0));
    }
    if (!w.valid) break;
    // Q of the previous item is free once its last S MMAs have completed.
    if (k >= 1) mbar_wait(&sm.q_empty, (k - 1) & 1, prm.status, abort_flag, 46);
    if (rank == 0) mbar_arrive_expect_tx(&sm.q_full, 2 * 4 * kQBoxBytes);
    for (int t = 0; t < 2; ++t) {
      tma_load_3d_pair(sm.q[t][0], tm_q, q_full_leader, 0, w.head[t], w.q0 + w.row0[t]);
      tma_load_3d_pair(sm.q[t][1], tm_q, q_full_leader, 64, w.head[t], w.q0 + w.row0[t]);
    }
    const int n_loads = 2 * w.n_kv;
    long long bid = 0;
    for (int i = 0; i < n_loads; ++i) {
      const int idx = g + i;
      const int slot = ring_slot(idx);
      if (idx >= kSlots)
        mbar_wait(&sm.empty[slot], ring_parity(idx) ^ 1u, prm.status, abort_flag, 30);
      const int key0 = (i >> 1) * kBN;
      if ((i & 1) == 0) {
        bid = prm.block_tables[(long long)w.seq * prm.max_blocks + key0 / prm.block_size];
        if (bid < 0 || bid >= prm.num_blocks) {
          record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 24, bid);
          bid = 0;
        }
      }
      // A tile at or past the cached prefix comes from the step's f16 rows
      // (row q0 + key - q_start); every other tile from the cache.
      const bool from_rows = staged && key0 >= w.q_start;
      const int row = from_rows ? w.q0 + key0 - w.q_start
                                : (int)((long long)prm.layer * prm.n_slots +
                                        bid * prm.block_size + key0 % prm.block_size);
      const CUtensorMap* map_k = from_rows ? tm_kr : tm_k;
      const CUtensorMap* map_v = from_rows ? tm_vr : tm_v;
      mbar_arrive_expect_tx(&sm.full[slot], kSlotBytes);
      if ((i & 1) == 0) {
        // K: keys [64r, 64r+64) of the tile, both 64-dim halves
        uint16_t* dst = sm.kv[slot];
        tma_load_3d(dst, map_k, &sm.full[slot], 0, w.kvh, row + 64 * (int)rank);
        tma_load_3d(dst + 64 * 64, map_k, &sm.full[slot], 64, w.kvh, row + 64 * (int)rank);
      } else {
        // V: dims [64r, 64r+64) of all 128 keys
        tma_load_3d(sm.kv[slot], map_v, &sm.full[slot], 64 * (int)rank, w.kvh, row);
      }
    }
    g += n_loads;
  }
  // Drain: the last load of every slot has landed before the CTA can exit
  // (immediate in normal operation; bounded after an abort).
  for (int idx = max(0, g - kSlots); idx < g; ++idx)
    mbar_wait(&sm.full[ring_slot(idx)], ring_parity(idx), prm.status, 40);
}

// Takes the next item from the work ring (every lane of a warp calls it; lane
// 0 releases the slot at the leader).  Returns false when the CTA's work is
// over.
__device__ __forceinline__ bool next_work(PrefillSmem& sm, const PrefillParams& prm, int k,
                                          int lane, Work& w, int site) {
  const int ws = k & 1;
  if (!mbar_wait_cluster(&sm.work_full[ws], (k >> 1) & 1, prm.status, &sm.abort_flag, site))
    return false;
  w = sm.work[ws];
  __syncwarp();
  if (lane == 0) mbar_arrive_cluster(smem_peer(&sm.work_empty[ws], 0));
  return w.valid != 0;
}

// Arrives on the pair leader's copy of a per-tile barrier `bar`: a local
// arrive in the leader, a remote one in the follower, both with the default
// (CTA-scope) release.  What these barriers publish -- converted K/V halves
// behind fence.proxy.async, P in TMEM behind tcgen05.wait::st and
// tcgen05.fence -- is read only by the pair MMAs that the leader's MMA lane
// issues after its wait; a cluster-scope release would add a cluster-wide
// memory fence (about a thousand cycles) to every follower arrival on the
// S -> softmax -> P.V chain.
__device__ __forceinline__ void arrive_leader(uint64_t* bar, bool leader) {
  if (leader)
    mbar_arrive(bar);
  else
    mbar_arrive_remote(smem_peer(bar, 0));
}

// ---------------------------------------------------------------- K/V converters
// One CTA's half of a key tile, 16 KiB = 1024 16-byte chunks, 128-byte rows
// with 16-byte chunks swizzled by row % 8.  K half: [d half][64 keys][64
// dims] (keys 64r + row of the tile); V half: [128 keys][64 dims] (dims 64r
// + ...).  Each chunk of a key past the context is zeroed (V only), of a key
// at or past the cached prefix taken from the step's f16 rows (a tile that
// straddles the prefix end), and otherwise converted bf16 -> f16 in place.
// Consecutive threads touch consecutive chunks (no bank conflicts).
struct HalfTile {
  uint16_t* smem;
  bool is_v;
  int key_base;       // key of the half tile's first row
  int zero_from;      // keys at or past this are zeroed (V), INT_MAX for none
  int rows_from;      // keys in [rows_from, rows_end) come from the rows
  int rows_end;       //   (the sequence's own rows: never past the buffer)
  const uint16_t* rows;  // row of key rows_from, at this CTA's dims / head
  int row_stride;        // elements between consecutive keys' rows
};

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 v) {
  v.x = cvt_f16x2(bf16lo_to_f32(v.x), bf16hi_to_f32(v.x));
  v.y = cvt_f16x2(bf16lo_to_f32(v.y), bf16hi_to_f32(v.y));
  v.z = cvt_f16x2(bf16lo_to_f32(v.z), bf16hi_to_f32(v.z));
  v.w = cvt_f16x2(bf16lo_to_f32(v.w), bf16hi_to_f32(v.w));
  return v;
}

__device__ __forceinline__ void convert_half(const HalfTile& t, int c, uint32_t rank) {
  const int n_keys = t.is_v ? kBN : kBN / 2;
  if (t.key_base + n_keys <= t.zero_from &&
      (t.rows_from >= t.key_base + n_keys || t.rows_end <= t.key_base)) {
    // Every chunk converts in place: shared-memory loads of four chunks are
    // issued before any is converted and stored.
    const uint32_t base = smem_u32(t.smem) + (uint32_t)c * 16;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint4 v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = lds128(base + (uint32_t)(4 * h + i) * kConvThreads * 16);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        sts128(base + (uint32_t)(4 * h + i) * kConvThreads * 16, bf16x8_to_f16x8(v[i]));
    }
    fence_proxy_async_smem();
    __syncwarp();
    return;
  }
  uint8_t* base = reinterpret_cast<uint8_t*>(t.smem);
#pragma unroll 4
  for (int f = c; f < kSlotBytes / 16; f += kConvThreads) {
    uint4* p = reinterpret_cast<uint4*>(base + f * 16);
    const int row = t.is_v ? (f >> 3) : ((f >> 3) & 63);
    const int key = t.key_base + row;
    uint4 v;
    if (key >= t.zero_from) {
      v = make_uint4(0, 0, 0, 0);
    } else if (key >= t.rows_from && key < t.rows_end) {
      // logical 8-dim chunk of this physical chunk, and (K) its d half
      const int chunk = (f & 7) ^ (row & 7);
      const int dim = t.is_v ? chunk * 8 : (f >> 9) * 64 + chunk * 8;
      v = *reinterpret_cast<const uint4*>(t.rows + (long long)(key - t.rows_from) * t.row_stride +
                                          dim);
    } else {
      v = bf16x8_to_f16x8(*p);
    }
    *p = v;
  }
  fence_proxy_async_smem();
  __syncwarp();
}

// Zeroes the V half's keys at or past zero_from (a tile loaded from the
// step's f16 rows needs no conversion).
__device__ __forceinline__ void zero_v_tail(uint16_t* smem, int c, int first_zero_row) {
  uint8_t* base = reinterpret_cast<uint8_t*>(smem);
  for (int f = c; f < kSlotBytes / 16; f += kConvThreads)
    if ((f >> 3) >= first_zero_row) *reinterpret_cast<uint4*>(base + f * 16) = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  __syncwarp();
}

// The converters run ahead of the MMAs as far as the TMA ring and their lead
// limit let them, so the conversion stays off the S -> softmax -> P.V chain,
// and keep K one key tile ahead of V: an item's first K, then per key tile
// the next tile's K and this tile's V.  v_ready(gj) therefore also publishes
// K(gj+1), and the MMA lane waits once per key tile (on k_ready only for an
// item's first tile; the converters arrive on it for every tile, so its
// phases stay in step).  Their barriers come in sets of kConvAhead, one per
// key tile mod kConvAhead; converting K(g) first waits for P.V of tile
// g - kConvAhead (the completion of that tile's V ring slot), which has
// waited for its v_ready and k_ready phases, so no barrier runs more than one
// phase ahead of its waiter.
__device__ __forceinline__ void converter_role(PrefillSmem& sm, const PrefillParams& prm, int c,
                                               bool leader) {
  volatile int* abort_flag = &sm.abort_flag;
  const int lane = c & 31;
  const bool staged = prm.k_rows != nullptr;
  const uint32_t rank = leader ? 0u : 1u;
  int tb = 0;
  Work w;
  // key tile j of the current item (global tile g = tb + j)
  auto convert_k = [&](int j) {
    const int g = tb + j;
    if (g >= kConvAhead) {
      const int lead_idx = 2 * (g - kConvAhead) + 1;  // V of tile g - kConvAhead
      mbar_wait(&sm.empty[ring_slot(lead_idx)], ring_parity(lead_idx), prm.status, abort_flag,
                43);
    }
    const int key0 = j * kBN, kidx = 2 * g;
    mbar_wait(&sm.full[ring_slot(kidx)], ring_parity(kidx), prm.status, abort_flag, 50);
    // from the rows entirely (TMA), partly (the prefix end inside), or not
    if (!(staged && key0 >= w.q_start)) {
      const long long row0 = (long long)w.q0 * prm.Hkv + w.kvh;  // key q_start's row
      HalfTile t{sm.kv[ring_slot(kidx)], false, key0 + 64 * (int)rank, INT_MAX,
                 staged && w.q_start < key0 + kBN ? w.q_start : INT_MAX, w.q_start + w.n_q,
                 staged ? prm.k_rows + row0 * kD : nullptr, prm.Hkv * kD};
      convert_half(t, c, rank);
    }
    if (lane == 0) arrive_leader(&sm.k_ready[g % kConvAhead], leader);
  };
  auto convert_v = [&](int j) {
    const int g = tb + j;
    const int key0 = j * kBN, vidx = 2 * g + 1;
    mbar_wait(&sm.full[ring_slot(vidx)], ring_parity(vidx), prm.status, abort_flag, 44);
    const int zero_from = w.ctx - key0 < kBN ? w.ctx : INT_MAX;
    if (!(staged && key0 >= w.q_start)) {
      const long long row0 = (long long)w.q0 * prm.Hkv + w.kvh;
      HalfTile t{sm.kv[ring_slot(vidx)], true, key0, zero_from,
                 staged && w.q_start < key0 + kBN ? w.q_start : INT_MAX, w.q_start + w.n_q,
                 staged ? prm.v_rows + row0 * kD + 64 * (int)rank : nullptr, prm.Hkv * kD};
      convert_half(t, c, rank);
    } else if (zero_from != INT_MAX) {
      zero_v_tail(sm.kv[ring_slot(vidx)], c, max(zero_from - key0, 0));
    }
    if (lane == 0) arrive_leader(&sm.v_ready[g % kConvAhead], leader);
  };
  for (int k = 0; next_work(sm, prm, k, lane, w, 49); ++k) {
    convert_k(0);
    for (int j = 0; j < w.n_kv; ++j) {
      if (j + 1 < w.n_kv) convert_k(j + 1);
      convert_v(j);
    }
    tb += w.n_kv;
  }
}

// ---------------------------------------------------------------- MMA issuer
// Leader only, the whole warp: the loop, its waits and the descriptor
// arithmetic run converged (warp-uniform values), and one elected lane
// issues each tcgen05.mma and commit.
__device__ __forceinline__ void mma_role(PrefillSmem& sm, uint32_t tmem, const PrefillParams& prm,
                                         int lane) {
  volatile int* abort_flag = &sm.abort_flag;
  constexpr uint32_t idesc_s = umma_idesc_f16_f32(2 * kBM, kBN, 0, 0);
  constexpr uint32_t idesc_o = umma_idesc_f16_f32(2 * kBM, kD, 0, 1);
  // Shared-memory descriptors are built once; an MMA adds its operand's
  // offset to the start-address field (16-byte units; no field overflows: a
  // shared address is below 2^18 bytes).  A single thread issues at most one
  // tcgen05.mma per ~53 cycles against 64 cycles of tensor work per MMA, so
  // per-MMA descriptor arithmetic would leave the tensor pipe idle.
  const uint64_t q_desc[2][2] = {
      {umma_desc_sw128(smem_u32(sm.q[0][0]), 16, 1024),
       umma_desc_sw128(smem_u32(sm.q[0][1]), 16, 1024)},
      {umma_desc_sw128(smem_u32(sm.q[1][0]), 16, 1024),
       umma_desc_sw128(smem_u32(sm.q[1][1]), 16, 1024)}};
  const uint64_t k_desc0 = umma_desc_sw128(smem_u32(sm.kv[0]), 16, 1024);
  const uint64_t v_desc0 = umma_desc_sw128(smem_u32(sm.kv[0]), kSlotBytes, 1024);
  constexpr uint64_t kSlotUnits = kSlotBytes / 16;
  auto issue_s = [&](int t, int gj) {
    const uint64_t kd = k_desc0 + (uint64_t)ring_slot(2 * gj) * kSlotUnits;
    const uint64_t qd0 = q_desc[t][0], qd1 = q_desc[t][1];
#pragma unroll
    for (int k = 0; k < kD / 16; ++k) {
      // +32 bytes per 16 dims inside a 64-dim half; K's second half starts
      // 64 x 128 bytes further
      const uint64_t a = (k < 4 ? qd0 : qd1) + (uint64_t)((k & 3) * 2);
      const uint64_t b = kd + (uint64_t)((k >> 2) * (64 * 128 / 16) + (k & 3) * 2);
      if (elect_one()) umma_pair_ss(tmem + t * 256, a, b, idesc_s, k > 0 ? 1u : 0u);
    }
  };
  auto issue_pv = [&](int t, int gj, bool accumulate) {
    const uint64_t vd = v_desc0 + (uint64_t)ring_slot(2 * gj + 1) * kSlotUnits;
#pragma unroll
    for (int k = 0; k < kBN / 16; ++k)
      if (elect_one())
        umma_pair_ts(tmem + t * 256 + 128, tmem + t * 256 + k * 8,
                     vd + (uint64_t)(k * 16 * 128 / 16), idesc_o, (accumulate || k > 0) ? 1u : 0u);
  };
  auto commit = [&](uint64_t* bar) {
    if (elect_one()) umma_commit_pair(bar);
  };
  int tb = 0, k = 0;
  for (;; ++k) {
    const int ws = k & 1;
    if (!mbar_wait_cluster(&sm.work_full[ws], (k >> 1) & 1, prm.status, abort_flag, 48)) break;
    const int valid = sm.work[ws].valid, n_kv = sm.work[ws].n_kv;
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(smem_peer(&sm.work_empty[ws], 0));
    if (!valid) break;
    mbar_wait(&sm.q_full, k & 1, prm.status, abort_flag, 31);
    mbar_wait(&sm.k_ready[tb % kConvAhead], (uint32_t)(tb / kConvAhead) & 1u, prm.status,
              abort_flag, 32);
    tc_fence_after();
    // S_t(0) overwrites the S/P columns of the previous item: its P.V MMAs
    // were issued before and execute first.  Its O columns are rewritten by
    // the first P.V below, which waits for P_t(0), i.e. for the softmax warps
    // to have read the previous O out in their epilogue.
    issue_s(0, tb);
    commit(&sm.s_full[0]);
    issue_s(1, tb);
    commit(&sm.s_full[1]);
    commit(&sm.empty[ring_slot(2 * tb)]);
    if (n_kv == 1) commit(&sm.q_empty);
    for (int j = 0; j < n_kv; ++j) {
      const int gj = tb + j;
      const int vidx = 2 * gj + 1, kidx = 2 * gj + 2;
      // V(gj) converted, and K(gj+1) with it
      mbar_wait(&sm.v_ready[gj % kConvAhead], (uint32_t)(gj / kConvAhead) & 1u, prm.status,
                abort_flag, 33);
      mbar_wait(&sm.p_full[0], gj & 1, prm.status, abort_flag, 34);
      tc_fence_after();
      issue_pv(0, gj, j > 0);
      if (j + 1 < n_kv) {
        issue_s(0, gj + 1);
        commit(&sm.s_full[0]);
      }
      mbar_wait(&sm.p_full[1], gj & 1, prm.status, abort_flag, 36);
      tc_fence_after();
      issue_pv(1, gj, j > 0);
      commit(&sm.empty[ring_slot(vidx)]);
      if (j + 1 < n_kv) {
        issue_s(1, gj + 1);
        commit(&sm.s_full[1]);
        commit(&sm.empty[ring_slot(kidx)]);
        if (j + 2 == n_kv) commit(&sm.q_empty);
      }
    }
    commit(&sm.o_final);
    tb += n_kv;
  }
  // Drain: every MMA has completed before TMEM is released.
  if (k > 0) mbar_wait(&sm.o_final, (k - 1) & 1, prm.status, 42);
}

// ---------------------------------------------------------------- softmax
__device__ __forceinline__ void softmax_role(PrefillSmem& sm, uint32_t tmem,
                                             const PrefillParams& prm, int warp, int lane,
                                             bool leader) {
  volatile int* abort_flag = &sm.abort_flag;
  const int t = (warp - 4) >> 2;  // query tile
  const int quad = warp & 3;      // TMEM lanes [32*quad, 32*quad+32)
  const int row = quad * 32 + lane;
  const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
  const uint32_t s_col = tmem + lane_off + t * 256;
  const uint32_t o_col = s_col + 128;
  const float sc = prm.scale_log2;
  const uint64_t sc2 = pack2(sc, sc);
  int tb = 0;
  Work w;
  for (int k = 0; next_work(sm, prm, k, lane, w, 47); ++k) {
    const int my_rows = t ? w.rows[1] : w.rows[0];
    const int my_row0 = t ? w.row0[1] : w.row0[0];
    const int my_head = t ? w.head[1] : w.head[0];
    // Rows past the end of the sequence mimic a real row (never stored).
    const int pos_row = my_rows > 0 ? w.q_start + my_row0 + min(row, my_rows - 1) : w.p_last0;
    const int vis_last = min(pos_row, w.ctx - 1);  // last visible key
    float* dst = prm.out + ((long long)(w.q0 + my_row0 + row) * prm.Hq + my_head) * kD;
    const int n_kv = w.n_kv, tb0 = tb;
    tb += n_kv;
    float m_used = -INFINITY;
    float l = 0.0f;

    for (int j = 0; j < n_kv; ++j) {
      const int gj = tb0 + j;
      mbar_wait(&sm.s_full[t], gj & 1, prm.status, abort_flag, 37);
      tc_fence_after();
      uint32_t sr[kBN];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld32(s_col + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_wait_ld();

      const int lim = vis_last - j * kBN;  // keys c <= lim are visible
      // Warp-uniform: the paths below end in tcgen05.st, a warp-collective
      // instruction that every lane of the warp must execute together.
      const bool masked = __any_sync(0xffffffffu, lim < kBN - 1);
      if (masked) {
#pragma unroll
        for (int c = 0; c < kBN; ++c)
          if (c > lim) sr[c] = __float_as_uint(-INFINITY);
      }
      float mx[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) mx[a] = __uint_as_float(sr[a]);
#pragma unroll
      for (int c = 4; c < kBN; c += 2)
        mx[(c >> 1) & 3] =
            fmax3(mx[(c >> 1) & 3], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
      const float tile_max = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sc;
      const float m_new = fmaxf(m_used, tile_max);
      float alpha = 1.0f;
      bool rescale = false;
      if (m_new > m_used + kRescaleThreshold) {
        alpha = fast_exp2(m_used - m_new);
        rescale = j > 0;
        m_used = m_new;
      }
      // p = 2^(s*sc - m) in f32 pairs (ex2.approx on the XU port), stored as
      // f16.  The exponentials set this loop's length (~1,800 cycles per
      // tile with them, ~700 without); an FMA-pipe polynomial for a share of
      // the pairs and ex2.approx.f16x2 were both measured slower.
      const uint64_t nm2 = pack2(-m_used, -m_used);
      // Pairs of the next 32-key chunk are exponentiated interleaved with
      // the conversion, sum and store of the current chunk, and the row sum
      // runs in four accumulators, so the sums do not serialise behind each
      // pair's ex2 results.
      uint64_t sum4[4] = {pack2(0.0f, 0.0f), pack2(0.0f, 0.0f), pack2(0.0f, 0.0f),
                          pack2(0.0f, 0.0f)};
      auto expo = [&](int i) {  // pair i: 2^(s*sc - m) in place
        const uint64_t x2 = ffma2(pack2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])),
                                  sc2, nm2);
        float x0, x1;
        unpack2(x2, x0, x1);
        sr[2 * i] = __float_as_uint(fast_exp2(x0));
        sr[2 * i + 1] = __float_as_uint(fast_exp2(x1));
      };
#pragma unroll
      for (int i = 0; i < 16; ++i) expo(i);
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 32 keys -> 16 packed columns
        uint32_t ph[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (c < 3) expo((c + 1) * 16 + i);  // the next chunk's pair, interleaved
          const float p0 = __uint_as_float(sr[c * 32 + 2 * i]);
          const float p1 = __uint_as_float(sr[c * 32 + 2 * i + 1]);
          sum4[i & 3] = fadd2(sum4[i & 3], pack2(p0, p1));
          ph[i] = cvt_f16x2(p0, p1);
        }
        tmem_st16(s_col + c * 16, ph);
      }
      const uint64_t sum2 = fadd2(fadd2(sum4[0], sum4[1]), fadd2(sum4[2], sum4[3]));
      float s0, s1;
      unpack2(sum2, s0, s1);
      l = l * alpha + (s0 + s1);

      // O_t: the completion of S_t(j) implies PV_t(j-1) has completed.
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(o_col + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(o_col + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive_leader(&sm.p_full[t], leader);
    }

    // ---- epilogue: O_t / l.  The next item's first P.V (which rewrites O_t)
    // is issued only after this warp's next P_t arrival, i.e. after these
    // loads have completed.
    mbar_wait(&sm.o_final, k & 1, prm.status, abort_flag, 39);
    tc_fence_after();
    const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      tmem_ld32(o_col + c * 32, o);
      tmem_wait_ld();
      if (row < my_rows) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + c * 32 + i) =
              make_float4(__uint_as_float(o[i]) * inv_l, __uint_as_float(o[i + 1]) * inv_l,
                          __uint_as_float(o[i + 2]) * inv_l, __uint_as_float(o[i + 3]) * inv_l);
      }
    }
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v,
                         const __grid_constant__ CUtensorMap tm_kr,
                         const __grid_constant__ CUtensorMap tm_vr, PrefillParams prm) {
  extern __shared__ uint8_t smem_raw[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < kConvAhead; ++i) {
      mbar_init(&sm.k_ready[i], kPairWarps4);
      mbar_init(&sm.v_ready[i], kPairWarps4);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_full[t], kPairWarps4);
      mbar_init(&sm.work_full[t], 1);
      mbar_init(&sm.work_empty[t], kWorkReaders);
    }
    mbar_init(&sm.o_final, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&sm.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Both CTAs' barriers exist before either CTA arrives on the other's.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  // 512 threads x 128 registers at launch: warpgroup 0 (TMA, MMA) gives back
  // down to 96, warpgroup 3 (converters) to 48 (at 40 their loop spilled),
  // the two softmax warpgroups take 184 each
  // (128*96 + 128*48 + 256*184 = 65536 = 512*128).
  if (warp < 4) {
    regs_dec<96>();
    if (warp == 0 && lane == 0) producer_role(sm, &tm_q, &tm_k, &tm_v, &tm_kr, &tm_vr, prm, rank);
    if (warp == 1 && rank == 0) mma_role(sm, tmem, prm, lane);
  } else if (warp >= 12) {
    regs_dec<48>();
    converter_role(sm, prm, threadIdx.x - 384, rank == 0);
  } else {
    regs_inc<184>();
    softmax_role(sm, tmem, prm, warp, lane, rank == 0);
  }

  tc_fence_before();
  __syncthreads();
  // Neither CTA leaves (or frees TMEM) while the other may still arrive on
  // its barriers or run pair MMAs on its memory.
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
  // The last CTA to finish zeroes the work counter for the next launch
  // (every CTA has taken its last item before it counts itself finished).
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&prm.sched[1], 1) == (int)gridDim.x - 1) {
      atomicExch(&prm.sched[0], 0);
      atomicExch(&prm.sched[1], 0);
    }
  }
}

}  // namespace

nvattn_status launch_paged_prefill(nvattn_handle* h, int layer, int n_seqs, int n_tokens,
                                   const uint16_t* q, const int32_t* cu_q,
                                   const int32_t* q_starts, const int32_t* context_lens,
                                   const int32_t* block_tables, int max_blocks, int max_q_len,
                                   const uint16_t* k_cache, const uint16_t* v_cache,
                                   const uint16_t* k_rows, const uint16_t* v_rows, float* out,
                                   cudaStream_t stream) {
  if (max_q_len <= 0) return NVATTN_OK;
  const int Hq = h->cfg.n_q_heads, Hkv = h->cfg.n_kv_heads;
  CUtensorMap tm_q;
  nvattn_status st =
      encode_tensor_map_3d(&tm_q, q, kD, (uint64_t)Hq, (uint64_t)n_tokens, kD * 2,
                           (uint64_t)Hq * kD * 2, 64, 1, kBM, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  if (st != NVATTN_OK) return st;
  // K halves: boxes of 64 keys x 64 dims; V halves: 128 keys x 64 dims.
  CUtensorMap tk, tv;
  st = get_cache_tensor_map(h, k_cache, 64, kBN / 2, CU_TENSOR_MAP_SWIZZLE_128B, &tk);
  if (st != NVATTN_OK) return st;
  st = get_cache_tensor_map(h, v_cache, 64, kBN, CU_TENSOR_MAP_SWIZZLE_128B, &tv);
  if (st != NVATTN_OK) return st;
  // The step's f16 rows [n_tokens][Hkv][128], boxed like the cache.
  CUtensorMap tkr = tk, tvr = tv;
  if (k_rows != nullptr) {
    st = encode_tensor_map_3d(&tkr, k_rows, kD, (uint64_t)Hkv, (uint64_t)n_tokens, kD * 2,
                              (uint64_t)Hkv * kD * 2, 64, 1, kBN / 2, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    if (st != NVATTN_OK) return st;
    st = encode_tensor_map_3d(&tvr, v_rows, kD, (uint64_t)Hkv, (uint64_t)n_tokens, kD * 2,
                              (uint64_t)Hkv * kD * 2, 64, 1, kBN, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
    if (st != NVATTN_OK) return st;
  }

  PrefillParams prm = {};
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.G = Hq / Hkv;
  prm.layer = layer;
  prm.block_size = h->cfg.block_size;
  prm.max_blocks = max_blocks;
  prm.n_mtiles = (max_q_len + kBM - 1) / kBM;
  prm.mode = prm.G >= 4 ? kModeHeads : prm.G == 2 ? kModePair : kModeRows;
  prm.n_slots = h->n_slots;
  prm.num_blocks = h->cfg.num_blocks;
  prm.scale_log2 = h->cfg.scale * kLog2e;
  prm.cu_q = cu_q;
  prm.q_starts = q_starts;
  prm.context_lens = context_lens;
  prm.block_tables = block_tables;
  prm.k_rows = k_rows;
  prm.v_rows = v_rows;
  prm.out = out;
  prm.status = h->status_dev;
  prm.sched = h->prefill_sched_dev;

  const long long gx = prm.mode == kModeHeads  ? (long long)prm.n_mtiles * (prm.G / 4)
                       : prm.mode == kModePair ? (long long)(prm.n_mtiles + 1) / 2
                                               : (long long)(prm.n_mtiles + 3) / 4;
  const long long n_items = gx * Hkv * (long long)n_seqs;
  if (n_items <= 0) return NVATTN_OK;
  // The counter overshoots n_items by at most one step per pair.
  if (n_items > 0x7fffffffLL - h->sm_count) return NVATTN_ERR_UNSUPPORTED;
  prm.gx = (int)gx;
  prm.n_items = (int)n_items;
  prm.n_tokens = n_tokens;
  // Persistent: one CTA per SM (the shared-memory footprint allows no more),
  // in pairs.
  const int pairs = (int)std::min<long long>(n_items, std::max(1, h->sm_count / 2));
  const size_t smem = sizeof(PrefillSmem) + 1024;
  // The attribute is per device; remember which devices have it.
  // (atomic: handles on different threads may launch at the same time)
  static std::atomic<unsigned long long> attr_set_mask{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVATTN_ERR_CUDA;
  if (dev >= 64 || !(attr_set_mask.load(std::memory_order_relaxed) & (1ull << dev))) {
    if (cudaFuncSetAttribute(paged_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return NVATTN_ERR_CUDA;
    if (dev < 64) attr_set_mask.fetch_or(1ull << dev, std::memory_order_relaxed);
  }
  paged_prefill_kernel<<<2 * pairs, kThreads, smem, stream>>>(tm_q, tk, tv, tkr, tvr, prm);
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace nvattn
