// sample.cu -- next-token sampling over a batch of logits rows on the device:
// ModelRunner::Sample (src/engine/model_runner.cpp:417-489) -- repetition
// penalty, greedy argmax (temperature < 1e-6) or temperature sampling by
// inverse CDF with a caller-supplied uniform draw.
//
// Three launches:
//  1. count  -- one 512-thread CTA per penalised sequence and 49,152-id
//     segment of the vocabulary (two per SM) builds the segment's histogram
//     of the history in shared memory (16-bit counters, plain atomic adds)
//     and writes it out densely as 4-bit counts
//     min(c, 15) per id, plus the exact count of every id seen 15 or more
//     times into a [n_seqs][vocab] u32 table (sparse writes, read only
//     where the 4-bit count is 15).  No state survives between calls: every
//     penalised row is rewritten.
//  2. pass   -- persistent CTAs (three per SM) stream (sequence, 4096-element
//     chunk) items: a producer warp bulk-copies each chunk's logits (16 KB)
//     and 4-bit counts (2 KB) into a 3-stage shared-memory ring; each of 8
//     consumer warps takes one 512-element piece of the chunk, applies the
//     penalty in shared memory (the reference's v = v < 0 ? v*p : v/p once
//     per occurrence, bit for bit; the piece's history ids are listed and
//     spread over the lanes) and writes the piece's maximum, first arg-max,
//     NaN flags and -- for sampling rows -- the sum of exp((x - piece max)/t)
//     in a fixed order, with warp shuffles only (no block barrier).
//  3. finish -- one CTA per sequence combines the pieces: greedy rows take
//     the first arg-max; sampling rows scale each piece's sum by
//     exp((piece max - row max)/t), draw r = u*S, find the piece whose running
//     total reaches r, and one warp recomputes that piece exactly as pass 2
//     did and walks slab -> lane -> element.
// Traffic: one pass over the logits plus 1/8 of their size in 4-bit counts
// (the HBM floor; the passes are issue/latency-bound above it).
//
// Greedy tokens are bit-exact with the reference (same penalised values,
// same first-index rule, same NaN outcomes).  Sampled tokens follow the same
// inverse-CDF rule on the same draw; the probabilities differ from the
// reference's float chain by a few ulp (exp by ex2.approx on
// (x - m)*log2(e)/t, piece sums combined in double), so a draw within that
// rounding of a CDF step can land on the neighbouring token -- as the
// reference's own sequential float sum, ~sqrt(n)*eps*S off the exact CDF,
// does against exact math.
#include <math.h>

#include <algorithm>
#include <climits>

#include "common.cuh"
#include "internal.h"

namespace nvattn {
namespace {

constexpr int kThreads = 256;            // consumer threads; finish kernel threads
constexpr int kPassThreads = kThreads + 32;
constexpr int kChunk = 4096;             // logits per work item (8 pieces of 512)
constexpr int kMaxChunks = 512;          // n_vocab <= 2,097,152
constexpr int kStages = 3;
constexpr int kNibBytes = kChunk / 2;    // 4-bit counts of one chunk
constexpr int kCountThreads = 512;
constexpr int kSegment = 12 * kChunk;    // ids one CTA counts (16-bit counts in shared memory)
constexpr int kOvSlots = 1024;           // ids seen more than 65535 times, per segment
constexpr int kPassSmem = kStages * (kChunk * 4 + kNibBytes);
constexpr int kPassCtasPerSm = 3;
constexpr int kCountSmem = 2 * kSegment + kOvSlots * 8;

struct PiecePartial {
  float max;   // maximum of the piece's non-NaN penalised values (-inf if none)
  int argmax;  // first index holding it, INT_MAX if the piece has no non-NaN value
  float sum;   // sampling rows: sum of exp((x - max)/t) in the fixed scan order
  int flags;   // bit 0: a NaN in the piece; bit 1: element 0 of the row is NaN
};
static_assert(sizeof(PiecePartial) == 16, "partial layout");

struct SampleArgs {
  int n_seqs, n_vocab, n_chunks;
  const float* logits;
  long long row_stride;
  const float* temps;
  const float* pens;
  const int32_t* hist;
  const int64_t* hist_off;
  const float* uniforms;
  int32_t* tokens;
  uint8_t* nib;          // [max_seqs][cap/2] 4-bit counts
  uint32_t* cnt_exact;   // [max_seqs][cap] exact counts of ids with a 4-bit count of 15
  long long cap;         // vocabulary capacity, a multiple of kChunk
  PiecePartial* part;    // [max_seqs][kMaxChunks * 8] piece summaries
  DeviceStatus* status;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// mbar_wait with a sleep between polls: a warp that waits here (the producer
// on a full ring, consumers ahead of the copies) then leaves the issue slots
// to the warps that compute.  Same bound and abort protocol as mbar_wait.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, DeviceStatus* st,
                                                int site, volatile int* abort_flag,
                                                unsigned sleep_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  uint32_t it = 0;
  while (true) {
    __nanosleep(sleep_ns);
    if (mbar_try_wait(bar, parity)) return true;
    if ((++it & 15u) == 0) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        record_error(st, NVATTN_ERR_TIMEOUT, site, 0);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// History bounds of sequence s, or false if the offsets are unusable (a
// history of 2^30 ids or more per sequence included).
__device__ __forceinline__ bool hist_range(const SampleArgs& a, int s, long long& b,
                                           long long& e) {
  b = a.hist_off[s];
  e = a.hist_off[s + 1];
  return b >= 0 && e >= b && e - b < (1LL << 30);
}

// Rows whose penalty the count kernel prepared.
__device__ __forceinline__ bool pen_row(const SampleArgs& a, int s) {
  if (a.hist == nullptr || !(a.pens[s] > 1.0f)) return false;
  long long b, e;
  return hist_range(a, s, b, e);
}

// The reference's penalty, applied once per occurrence.  Zero, infinities and
// NaN are fixed points of the step, so the loop stops early on them.
__device__ __forceinline__ float apply_penalty(float v, float p, uint32_t c) {
  if (c <= 14u) {  // every 4-bit count; no early exit needed
    for (uint32_t k = 0; k < c; ++k) v = v < 0.0f ? __fmul_rn(v, p) : __fdiv_rn(v, p);
    return v;
  }
  for (uint32_t k = 0; k < c; ++k) {
    if (v == 0.0f || isinf(v) || isnan(v)) break;
    v = v < 0.0f ? __fmul_rn(v, p) : __fdiv_rn(v, p);
  }
  return v;
}

// ---------------------------------------------------------------------------
// 1. history histogram
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t ov_hash(int key) {
  return ((uint32_t)key * 2654435761u) >> 22;  // multiplicative hashing, 10 bits
}

__device__ void ov_add(int* keys, uint32_t* vals, int key, uint32_t n, int* full) {
  const uint32_t h = ov_hash(key);
  for (int i = 0; i < kOvSlots; ++i) {
    const int slot = (int)((h + i) & (kOvSlots - 1));
    const int prev = atomicCAS(&keys[slot], -1, key);
    if (prev == -1 || prev == key) {
      atomicAdd(&vals[slot], n);
      return;
    }
  }
  *full = 1;
}

__device__ uint32_t ov_get(const int* keys, const uint32_t* vals, int key) {
  const uint32_t h = ov_hash(key);
  for (int i = 0; i < kOvSlots; ++i) {
    const int slot = (int)((h + i) & (kOvSlots - 1));
    if (keys[slot] == key) return vals[slot];
    if (keys[slot] == -1) return 0;
  }
  return 0;
}

// min(c, 15) of both 16-bit halves of w, left in bits 0-3 and 16-19.
__device__ __forceinline__ uint32_t sat15x2(uint32_t w) {
  // bit 15 of a half is set iff that half >= 16: adding 0x7FF0 to its low 15
  // bits carries into bit 15 exactly then (no carry leaves the half), and a
  // half >= 0x8000 has it set already
  const uint32_t ge16 = (((w & 0x7FFF7FFFu) + 0x7FF07FF0u) | w) & 0x80008000u;
  return (w & 0x000F000Fu) | ((ge16 >> 15) * 0xFu);
}

// Ids 2k, 2k+1 of a 16-bit-count word as bytes 0, 1 of the result.
__device__ __forceinline__ uint32_t sat_pair_bytes(uint32_t w) {
  const uint32_t t = sat15x2(w);
  return (t | (t >> 8)) & 0x0F0Fu;
}

__global__ void __launch_bounds__(kCountThreads, 2) sample_count_kernel(SampleArgs a) {
  extern __shared__ __align__(16) uint8_t csm[];
  __shared__ int ov_full;
  const int s = blockIdx.x;
  if (a.hist == nullptr || !(a.pens[s] > 1.0f)) return;
  long long hb, he;
  if (!hist_range(a, s, hb, he)) {
    if (threadIdx.x == 0) record_error(a.status, NVATTN_ERR_INVALID_ARG, 70, s);
    return;
  }
  uint32_t* c16 = reinterpret_cast<uint32_t*>(csm);  // 16-bit counts, 2 per word
  int* ov_key = reinterpret_cast<int*>(csm + 2 * kSegment);
  uint32_t* ov_val = reinterpret_cast<uint32_t*>(ov_key + kOvSlots);
  uint8_t* nib_row = a.nib + (long long)s * (a.cap / 2);
  uint32_t* exact_row = a.cnt_exact + (long long)s * a.cap;
  // A history of at most 65535 ids cannot overflow a 16-bit count: plain
  // atomic adds.  Longer ones saturate at 65535 and keep the excess in a
  // small hash table.
  const bool short_hist = he - hb <= 65535;
  {
    const long long v0 = (long long)blockIdx.y * kSegment;
    if (v0 >= a.cap) return;
    const int seg = (int)min((long long)kSegment, a.cap - v0);
    for (int i = threadIdx.x; i < seg / 8; i += kCountThreads)
      reinterpret_cast<uint4*>(c16)[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = threadIdx.x; i < kOvSlots; i += kCountThreads) {
      ov_key[i] = -1;
      ov_val[i] = 0u;
    }
    if (threadIdx.x == 0) ov_full = 0;
    __syncthreads();
    constexpr int kBatch = 8;  // independent id loads in flight per thread
    // ids outside [0, n_vocab) are skipped, as the reference does: one
    // unsigned test covers them and the ids of other segments
    const uint32_t seg_ids = (uint32_t)min((long long)seg, (long long)a.n_vocab - v0);
    const int32_t* hs = a.hist + hb;
    const int n_hist = (int)(he - hb);
    for (int j0 = 0; j0 < n_hist; j0 += kBatch * kCountThreads) {
      int keys[kBatch];
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        const int j = j0 + q * kCountThreads + (int)threadIdx.x;
        const uint32_t key = j < n_hist ? (uint32_t)(__ldcs(hs + j) - (int)v0) : 0xFFFFFFFFu;
        keys[q] = key < seg_ids ? (int)key : -1;
      }
#pragma unroll
      for (int q = 0; q < kBatch; ++q) {
        const int key = keys[q];
        if (key < 0) continue;
        uint32_t* w = c16 + (key >> 1);
        const int sh = (key & 1) * 16;
        if (short_hist) {
          atomicAdd(w, 1u << sh);
        } else {
          uint32_t old = *reinterpret_cast<volatile uint32_t*>(w), assumed;
          bool sat = false;
          do {
            assumed = old;
            if (((assumed >> sh) & 0xFFFFu) == 0xFFFFu) {
              sat = true;
              break;
            }
            old = atomicCAS(w, assumed, assumed + (1u << sh));
          } while (old != assumed);
          if (sat) ov_add(ov_key, ov_val, key, 1u, &ov_full);
        }
      }
    }
    __syncthreads();
    if (ov_full && threadIdx.x == 0) record_error(a.status, NVATTN_ERR_UNSUPPORTED, 72, s);
    // 16 bytes of 4-bit counts per thread and step: ids [32g, 32g + 32).
    // Each 32-bit word holds ids 8q..8q+7: id 8q+j in bits 8j..8j+3 and
    // id 8q+4+j in bits 8j+4..8j+7.
    for (int g = threadIdx.x; g < seg / 32; g += kCountThreads) {
      const uint4* src = reinterpret_cast<const uint4*>(c16) + 4 * g;
      uint32_t out[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = src[q];  // ids 32g + 8q .. +7, two per word
        // The usual group: every count below 15 (the or of the counts below
        // 16 with a low nibble short of 15): the counts are the low bytes of
        // the halves.  Otherwise saturate and record exact counts.
        const uint32_t any = w.x | w.y | w.z | w.w;
        if (!(any & 0xFFF0FFF0u) && !(((any & 0x000F000Fu) + 0x00010001u) & 0x00100010u)) {
          out[q] = __byte_perm(w.x, w.y, 0x6420) | (__byte_perm(w.z, w.w, 0x6420) << 4);
          continue;
        }
        const uint32_t lo = sat_pair_bytes(w.x) | (sat_pair_bytes(w.y) << 16);
        const uint32_t hi = sat_pair_bytes(w.z) | (sat_pair_bytes(w.w) << 16);
        out[q] = lo | (hi << 4);
        // ids whose 4-bit count saturated: exact counts for the rare lookup
        if (((lo + 0x01010101u) | (hi + 0x01010101u)) & 0x10101010u) {
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            const uint32_t c = (ws[b >> 1] >> (16 * (b & 1))) & 0xFFFFu;
            if (c >= 15u) {
              const int key = g * 32 + q * 8 + b;
              exact_row[v0 + key] = c == 0xFFFFu ? 0xFFFFu + ov_get(ov_key, ov_val, key) : c;
            }
          }
        }
      }
      reinterpret_cast<uint4*>(nib_row + v0 / 2)[g] = make_uint4(out[0], out[1], out[2], out[3]);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// 2./3. piece pass and finish
// ---------------------------------------------------------------------------
// A piece is 512 consecutive logits of a row, handled by one warp: lane l
// holds, for slab v = 0..3, the 4 elements at piece offset 128 v + 4 l + j.
// Every piece summary below is computed in one fixed order that the finish
// kernel repeats for the selected piece.

__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// (max, first arg-max) pair order: a larger value wins, then the smaller index.
__device__ __forceinline__ void max_combine(float& m, int& am, float m2, int am2) {
  if (am2 == INT_MAX) return;
  if (am == INT_MAX || m2 > m || (m2 == m && am2 < am)) {
    m = m2;
    am = am2;
  }
}

constexpr int kPiece = 512;
constexpr int kPiecesPerChunk = kChunk / kPiece;  // one per consumer warp
constexpr int kPieceSlabs = 4;
constexpr int kMaxPieces = kMaxChunks * kPiecesPerChunk;

// 4-bit counts of 4 consecutive ids starting at a multiple of 4: ids 8q+j
// (j < 4) sit in bits 8j..8j+3 of word q and ids 8q+4+j in bits 8j+4..8j+7,
// so the 4 counts come back as the 4 bytes of the result.
__device__ __forceinline__ uint32_t nibbles4(uint32_t word, int id) {
  return (word >> (4 * ((id >> 2) & 1))) & 0x0F0F0F0Fu;
}

// Applies the penalty to 4 consecutive elements given their counts (byte j
// of n4 is element j's 4-bit count; 15 means "look up the exact count").
// Out of line: it runs only where a history id falls, and one copy keeps the
// pass kernel's code small.
__device__ __noinline__ float4 penalise4_call(const uint32_t* exact, float pen, uint32_t n4,
                                              float4 q) {
  float x[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t n = (n4 >> (8 * j)) & 15u;
    if (n == 0u) continue;
    x[j] = apply_penalty(x[j], pen, n < 15u ? n : __ldcg(exact + j));
  }
  return make_float4(x[0], x[1], x[2], x[3]);
}

__device__ __forceinline__ void penalise4(const SampleArgs& a, int s, int idx, float pen,
                                          uint32_t n4, float (&x)[4]) {
  if (n4 == 0u) return;
  const float4 r = penalise4_call(a.cnt_exact + (long long)s * a.cap + idx, pen, n4,
                                  make_float4(x[0], x[1], x[2], x[3]));
  x[0] = r.x;
  x[1] = r.y;
  x[2] = r.z;
  x[3] = r.w;
}

// Piece `p` of row s straight from global memory (unaligned rows, and the
// finish kernel's re-read), penalty applied.
__device__ __forceinline__ void load_piece_global(const SampleArgs& a, int s, int p, bool pn,
                                                  float pen, bool vec, int lane,
                                                  float (&x)[kPieceSlabs][4],
                                                  unsigned (&valid)[kPieceSlabs]) {
  const float* row = a.logits + (long long)s * a.row_stride;
  const uint32_t* nib_row = reinterpret_cast<const uint32_t*>(a.nib + (long long)s * (a.cap / 2));
#pragma unroll
  for (int v = 0; v < kPieceSlabs; ++v) {
    const int idx = p * kPiece + v * 128 + 4 * lane;
    if (vec && idx + 3 < a.n_vocab) {
      const float4 q = __ldg(reinterpret_cast<const float4*>(row + idx));
      x[v][0] = q.x;
      x[v][1] = q.y;
      x[v][2] = q.z;
      x[v][3] = q.w;
      valid[v] = 0xFu;
    } else {
      valid[v] = 0u;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        x[v][j] = 0.0f;
        if (idx + j < a.n_vocab) {
          x[v][j] = __ldg(row + idx + j);
          valid[v] |= 1u << j;
        }
      }
    }
    if (pn && valid[v]) penalise4(a, s, idx, pen, nibbles4(__ldcg(nib_row + idx / 8), idx), x[v]);
  }
}

// Warp-wide (max, first arg-max, flags) of a piece.  Ties go to the smaller
// index; NaN values only set flag bit 0 (bit 1 when at row index 0).  The
// arg-max is only looked for when `want_arg` (greedy rows); otherwise it is
// `base` (or INT_MAX when the piece holds no non-NaN value).  kFull: every
// element lies inside the row.
template <bool kFull>
__device__ __forceinline__ void piece_max(const float (&x)[kPieceSlabs][4],
                                          const unsigned (&valid)[kPieceSlabs], int base,
                                          int lane, bool want_arg, float& m, int& am,
                                          int& flags) {
  m = -INFINITY;
  bool nan = false, num = false;
  if (kFull) {
    // 3-input max that propagates NaN: without a NaN (the usual case) it is
    // the maximum; a NaN anywhere falls back to the NaN-skipping loop below
    float mn = max3_nan(max3_nan(x[0][0], x[0][1], x[0][2]), x[0][3], x[1][0]);
    mn = max3_nan(mn, x[1][1], x[1][2]);
    mn = max3_nan(mn, x[1][3], x[2][0]);
    mn = max3_nan(mn, x[2][1], x[2][2]);
    mn = max3_nan(mn, x[2][3], x[3][0]);
    mn = max3_nan(mn, x[3][1], x[3][2]);
    mn = max3_nan(mn, x[3][3], x[3][3]);
    nan = isnan(mn);
    m = mn;
    num = true;
  }
  if (!kFull || __any_sync(0xffffffffu, nan)) {
    m = -INFINITY;
    nan = num = false;
#pragma unroll
    for (int v = 0; v < kPieceSlabs; ++v)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (!kFull && !(valid[v] >> j & 1u)) continue;
        const bool isn = x[v][j] != x[v][j];
        nan |= isn;
        num |= !isn;
        m = fmaxf(m, x[v][j]);  // fmaxf skips NaN
      }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  flags = __any_sync(0xffffffffu, nan) ? 1 : 0;
  if (flags && base == 0 && __shfl_sync(0xffffffffu, x[0][0] != x[0][0], 0)) flags |= 2;
  am = __any_sync(0xffffffffu, num) ? base : INT_MAX;
  if (!want_arg || am == INT_MAX) return;
  // first index holding m: the first slab with a hit, its first lane, that
  // lane's first element
  bool done = false;
#pragma unroll
  for (int v = 0; v < kPieceSlabs; ++v) {
    int jf = 4;
#pragma unroll
    for (int j = 3; j >= 0; --j)
      if ((kFull || (valid[v] >> j & 1u)) && x[v][j] == m) jf = j;
    const unsigned ball = __ballot_sync(0xffffffffu, jf < 4);
    if (!done && ball) {  // warp-uniform
      const int l = __ffs(ball) - 1;
      am = base + v * 128 + 4 * l + __shfl_sync(0xffffffffu, jf, l);
      done = true;
    }
  }
}

// p = exp((x - m)/t) as 2^((x - m)*k2), k2 = log2(e)/t; 0 outside the row.
template <bool kFull>
__device__ __forceinline__ void piece_probs(float (&x)[kPieceSlabs][4],
                                            const unsigned (&valid)[kPieceSlabs], float m,
                                            float k2) {
#pragma unroll
  for (int v = 0; v < kPieceSlabs; ++v)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float p = ex2_approx(__fmul_rn(__fsub_rn(x[v][j], m), k2));
      x[v][j] = kFull || (valid[v] >> j & 1u) ? p : 0.0f;
    }
}

// Inclusive prefix over lanes of each lane's ((p0+p1)+p2)+p3, per slab
// (Hillis-Steele shuffles); S[v] = lane 31's value, the slab total.
__device__ __forceinline__ void piece_scan(const float (&p)[kPieceSlabs][4], int lane,
                                           float (&P)[kPieceSlabs], float (&S)[kPieceSlabs]) {
#pragma unroll
  for (int v = 0; v < kPieceSlabs; ++v)
    P[v] = __fadd_rn(__fadd_rn(__fadd_rn(p[v][0], p[v][1]), p[v][2]), p[v][3]);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int v = 0; v < kPieceSlabs; ++v) {
      const float y = __shfl_up_sync(0xffffffffu, P[v], o);
      if (lane >= o) P[v] = __fadd_rn(P[v], y);
    }
  }
#pragma unroll
  for (int v = 0; v < kPieceSlabs; ++v) S[v] = __shfl_sync(0xffffffffu, P[v], 31);
}

__device__ __forceinline__ float k2_of(float temp) { return __fdiv_rn(1.4426950408889634f, temp); }

// Summary of one piece (every lane returns the same value).
template <bool kFull>
__device__ __forceinline__ PiecePartial summarise(float (&x)[kPieceSlabs][4],
                                                  const unsigned (&valid)[kPieceSlabs], int base,
                                                  int lane, bool greedy, float temp) {
  PiecePartial cp;
  piece_max<kFull>(x, valid, base, lane, greedy, cp.max, cp.argmax, cp.flags);
  cp.sum = 0.0f;
  if (!greedy && !(cp.flags & 1) && cp.argmax != INT_MAX && isfinite(cp.max)) {
    piece_probs<kFull>(x, valid, cp.max, k2_of(temp));
    float P[kPieceSlabs], S[kPieceSlabs];
    piece_scan(x, lane, P, S);
    cp.sum = __fadd_rn(__fadd_rn(__fadd_rn(S[0], S[1]), S[2]), S[3]);
  }
  return cp;
}

// Applies the penalty in shared memory to the history ids of this warp's
// piece of a ring stage: the ids with a nonzero 4-bit count are listed (lane
// l scans ids 16l..16l+15) and then spread over the lanes, one id per lane
// per round, so a handful of hits costs a round instead of a divergent loop
// in every lane that holds one.  Ids at or past `bulk_el` (not in the
// stage) are left to the caller.
__device__ __forceinline__ void penalise_piece_smem(const SampleArgs& a, int s, int c, int warp,
                                                    int lane, float pen, float* sx,
                                                    const uint32_t* sn, uint16_t* list,
                                                    int bulk_el) {
  const int pbase = warp * kPiece;  // the piece's offset in the chunk
  const uint32_t* pw = sn + pbase / 8;
  auto nonzero = [](uint32_t w) {  // bit 4k set iff nibble k != 0
    uint32_t t = w | (w >> 1);
    t |= t >> 2;
    return t & 0x11111111u;
  };
  uint32_t h0 = nonzero(pw[2 * lane]), h1 = nonzero(pw[2 * lane + 1]);
  const int cnt = __popc(h0) + __popc(h1);
  int inc = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  const int total = __shfl_sync(0xffffffffu, inc, 31);
  if (total == 0) return;
  // nibble k of word q holds id 8q + k/2 (k even) or 8q + 4 + k/2 (k odd)
  int pos = inc - cnt;
  while (h0) {
    const int k = (__ffs(h0) - 1) >> 2;
    h0 &= h0 - 1;
    list[pos++] = (uint16_t)(16 * lane + (k & 1 ? 4 : 0) + (k >> 1));
  }
  while (h1) {
    const int k = (__ffs(h1) - 1) >> 2;
    h1 &= h1 - 1;
    list[pos++] = (uint16_t)(16 * lane + 8 + (k & 1 ? 4 : 0) + (k >> 1));
  }
  __syncwarp();
  const uint32_t* exact = a.cnt_exact + (long long)s * a.cap + (long long)c * kChunk + pbase;
  for (int k = lane; k < total; k += 32) {
    const int il = list[k];
    if (pbase + il >= bulk_el) continue;
    const int ii = il & 7;
    const uint32_t n = (pw[il >> 3] >> (ii < 4 ? 8 * ii : 8 * (ii - 4) + 4)) & 15u;
    float* xp = sx + pbase + il;
    *xp = apply_penalty(*xp, pen, n < 15u ? n : __ldcg(exact + il));
  }
  __syncwarp();
}

// Row parameters of a ring stage's item, written by the producer before it
// arms the stage.
struct StageMeta {
  int s, c;
  float temp, pen;
  int pn;
};

// The summary of a piece that crosses the end of the row (one per row), out
// of line so that only the full-piece version is inlined into the pass.
__device__ __noinline__ PiecePartial summarise_partial(float4 q0, float4 q1, float4 q2, float4 q3,
                                                       uint32_t valid16, int base, int lane,
                                                       bool greedy, float temp) {
  float x[kPieceSlabs][4] = {{q0.x, q0.y, q0.z, q0.w},
                             {q1.x, q1.y, q1.z, q1.w},
                             {q2.x, q2.y, q2.z, q2.w},
                             {q3.x, q3.y, q3.z, q3.w}};
  const unsigned valid[kPieceSlabs] = {valid16 & 15u, (valid16 >> 4) & 15u, (valid16 >> 8) & 15u,
                                       (valid16 >> 12) & 15u};
  return summarise<false>(x, valid, base, lane, greedy, temp);
}

template <bool kBulk>
__global__ void __launch_bounds__(kPassThreads, kPassCtasPerSm) sample_pass_kernel(SampleArgs a) {
  extern __shared__ __align__(128) uint8_t psm[];
  __shared__ __align__(8) uint64_t full[kStages];
  __shared__ __align__(8) uint64_t empty[kStages];
  __shared__ int abort_flag;
  __shared__ StageMeta meta[kStages];
  __shared__ uint16_t hit_list[kThreads / 32][kPiece];
  float* st_x = reinterpret_cast<float*>(psm);           // [kStages][kChunk]
  uint8_t* st_nib = psm + (size_t)kStages * kChunk * 4;  // [kStages][kNibBytes]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = a.n_seqs * a.n_chunks;
  if (threadIdx.x == 0) {
    for (int b = 0; b < kStages; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], kThreads / 32);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kThreads / 32) {
    // ---- producer warp: lane k looks up the row parameters of the k-th
    // next item (32 items per batch, loads in parallel); lane 0 publishes
    // them in the stage's meta slot and issues the bulk copies ----
    if (!kBulk) return;
    const uint64_t pol = l2_policy_evict_first();
    int it = 0;
    bool ok = true;
    for (int i0 = blockIdx.x; i0 < n_items && ok; i0 += 32 * gridDim.x) {
      const int mi = i0 + lane * gridDim.x;
      StageMeta mm = {};
      if (mi < n_items) {
        mm.s = mi / a.n_chunks;
        mm.c = mi - mm.s * a.n_chunks;
        mm.temp = a.temps[mm.s];
        mm.pen = a.pens[mm.s];
        mm.pn = pen_row(a, mm.s) ? 1 : 0;
      }
      for (int k = 0; k < 32; ++k) {
        if (i0 + k * gridDim.x >= n_items) break;
        StageMeta m;
        m.s = __shfl_sync(0xffffffffu, mm.s, k);
        m.c = __shfl_sync(0xffffffffu, mm.c, k);
        m.temp = __shfl_sync(0xffffffffu, mm.temp, k);
        m.pen = __shfl_sync(0xffffffffu, mm.pen, k);
        m.pn = __shfl_sync(0xffffffffu, mm.pn, k);
        const int b = it % kStages, use = it / kStages;
        if (lane == 0) {
          if (use > 0 &&
              !mbar_wait_sleep(&empty[b], (use - 1) & 1, a.status, 73, &abort_flag, 128)) {
            ok = false;
          } else {
            meta[b] = m;
            const int n_el = min(kChunk, a.n_vocab - m.c * kChunk);
            const uint32_t bytes = (uint32_t)(n_el * 4) & ~15u;
            mbar_arrive_expect_tx(&full[b], bytes + (m.pn ? (uint32_t)kNibBytes : 0u));
            if (bytes)
              bulk_load(st_x + (size_t)b * kChunk,
                        a.logits + (long long)m.s * a.row_stride + (long long)m.c * kChunk, bytes,
                        &full[b], pol);
            if (m.pn)
              bulk_load(st_nib + (size_t)b * kNibBytes,
                        a.nib + (long long)m.s * (a.cap / 2) + (long long)m.c * kNibBytes,
                        kNibBytes, &full[b], pol);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        ++it;
      }
    }
    // the CTA must not exit with copies in flight
    if (lane == 0)
      for (int b = 0; b < kStages && b < it; ++b) {
        const int last = b + ((it - 1 - b) / kStages) * kStages;
        mbar_wait(&full[b], (last / kStages) & 1, a.status, 74);
      }
    return;
  }

  // ---- consumer warp `warp`: piece `warp` of every chunk this CTA takes ----
  const bool vec = (reinterpret_cast<uintptr_t>(a.logits) & 15u) == 0 && a.row_stride % 4 == 0;
  int it = 0;
  for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++it) {
    int s, c;
    float temp, pen;
    bool pn, full_piece;
    float x[kPieceSlabs][4];
    unsigned valid[kPieceSlabs];
    if (kBulk) {
      const int b = it % kStages;
      const bool got = mbar_wait_sleep(&full[b], (it / kStages) & 1, a.status, 75, &abort_flag, 32);
      if (!__all_sync(0xffffffffu, got)) break;
      s = meta[b].s;
      c = meta[b].c;
      temp = meta[b].temp;
      pen = meta[b].pen;
      pn = meta[b].pn != 0;
      float* sx = st_x + (size_t)b * kChunk;
      const uint32_t* sn = reinterpret_cast<const uint32_t*>(st_nib + (size_t)b * kNibBytes);
      const int bulk_el = ((min(kChunk, a.n_vocab - c * kChunk) * 4) & ~15) / 4;
      full_piece = (warp + 1) * kPiece <= bulk_el;
      if (pn) penalise_piece_smem(a, s, c, warp, lane, pen, sx, sn, hit_list[warp], bulk_el);
#pragma unroll
      for (int v = 0; v < kPieceSlabs; ++v) {
        const int off = warp * kPiece + v * 128 + 4 * lane;  // offset in the chunk
        const int idx = c * kChunk + off;
        valid[v] = 0u;
        if (full_piece || off + 3 < bulk_el) {
          const float4 q = *reinterpret_cast<const float4*>(sx + off);
          x[v][0] = q.x;
          x[v][1] = q.y;
          x[v][2] = q.z;
          x[v][3] = q.w;
          valid[v] = 0xFu;
        } else {
          uint32_t from_global = 0u;  // the row's last 1-3 logits when n_vocab % 4 != 0
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            x[v][j] = 0.0f;
            if (idx + j < a.n_vocab) {
              if (off + j < bulk_el) {
                x[v][j] = sx[off + j];
              } else {
                x[v][j] = __ldg(a.logits + (long long)s * a.row_stride + idx + j);
                from_global |= 0xFFu << (8 * j);
              }
              valid[v] |= 1u << j;
            }
          }
          if (pn && from_global)
            penalise4(a, s, idx, pen, nibbles4(sn[off / 8], off) & from_global, x[v]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[b]);  // this warp's piece is in registers
    } else {
      s = i / a.n_chunks;
      c = i - s * a.n_chunks;
      temp = a.temps[s];
      pen = a.pens[s];
      pn = pen_row(a, s);
      load_piece_global(a, s, c * kPiecesPerChunk + warp, pn, pen, vec, lane, x, valid);
      full_piece = (c * kPiecesPerChunk + warp + 1) * kPiece <= a.n_vocab;
    }
    const int p = c * kPiecesPerChunk + warp;
    const bool greedy = temp < 1e-6f;
    PiecePartial cp;
    if (full_piece)
      cp = summarise<true>(x, valid, p * kPiece, lane, greedy, temp);
    else
      cp = summarise_partial(make_float4(x[0][0], x[0][1], x[0][2], x[0][3]),
                             make_float4(x[1][0], x[1][1], x[1][2], x[1][3]),
                             make_float4(x[2][0], x[2][1], x[2][2], x[2][3]),
                             make_float4(x[3][0], x[3][1], x[3][2], x[3][3]),
                             valid[0] | (valid[1] << 4) | (valid[2] << 8) | (valid[3] << 12),
                             p * kPiece, lane, greedy, temp);
    if (lane == 0) a.part[(long long)s * kMaxPieces + p] = cp;
  }
}

__device__ __forceinline__ double piece_scale(const PiecePartial& cp, float gm, float temp) {
  return cp.argmax == INT_MAX || !isfinite(cp.max) ? 0.0 : exp(((double)cp.max - gm) / temp);
}

__device__ __forceinline__ bool reaches(double base, double scale, float local, double r) {
  return base + scale * (double)local >= r;
}

__global__ void __launch_bounds__(kThreads) sample_finish_kernel(SampleArgs a) {
  __shared__ float red_m[kThreads / 32];
  __shared__ int red_am[kThreads / 32], red_fl[kThreads / 32], red_sel[kThreads / 32];
  __shared__ double red_sum[kThreads / 32];
  __shared__ int sel_piece;
  __shared__ float sel_max;
  __shared__ double sel_base, sel_scale;
  const int s = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float temp = a.temps[s], pen = a.pens[s];
  const bool greedy = temp < 1e-6f;
  const int n_p = a.n_chunks * kPiecesPerChunk;
  const int per = (n_p + kThreads - 1) / kThreads;
  const int p0 = min(n_p, tid * per), p1 = min(n_p, p0 + per);
  const PiecePartial* parts = a.part + (long long)s * kMaxPieces;

  // (max, arg-max, flags) over the row
  float m = -INFINITY;
  int am = INT_MAX, fl = 0;
  for (int k = p0; k < p1; ++k) {
    const PiecePartial cp = parts[k];
    max_combine(m, am, cp.max, cp.argmax);
    fl |= cp.flags;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const int a2 = __shfl_xor_sync(0xffffffffu, am, o);
    fl |= __shfl_xor_sync(0xffffffffu, fl, o);
    max_combine(m, am, m2, a2);
  }
  if (lane == 0) {
    red_m[warp] = m;
    red_am[warp] = am;
    red_fl[warp] = fl;
  }
  __syncthreads();
  float gm = red_m[0];
  int gam = red_am[0], gfl = red_fl[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) {
    max_combine(gm, gam, red_m[w], red_am[w]);
    gfl |= red_fl[w];
  }
  if (greedy) {
    if (tid == 0) a.tokens[s] = (gfl & 2) || gam == INT_MAX ? 0 : gam;
    return;
  }
  const float u = a.uniforms[s];
  if (!(u >= 0.0f && u < 1.0f)) {
    if (tid == 0) {
      record_error(a.status, NVATTN_ERR_INVALID_ARG, 71, s);
      a.tokens[s] = a.n_vocab - 1;
    }
    return;
  }
  if ((gfl & 1) || gam == INT_MAX || !isfinite(gm) || isnan(temp)) {
    if (tid == 0) a.tokens[s] = a.n_vocab - 1;  // the reference's NaN sum never reaches r
    return;
  }

  // inclusive prefix of scale_k * sum_k over pieces, in double: serial over
  // this thread's run, Hillis-Steele over the warp, warp totals in order
  double acc = 0.0;
  for (int k = p0; k < p1; ++k) acc += piece_scale(parts[k], gm, temp) * (double)parts[k].sum;
  double inc = acc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) red_sum[warp] = inc;
  __syncthreads();
  double wbase = 0.0, S = 0.0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    if (w < warp) wbase += red_sum[w];
    S += red_sum[w];
  }
  const double tbase = wbase + (inc - acc);  // exclusive prefix of this thread's run
  if (!(S > 0.0) || !isfinite(S)) {
    if (tid == 0) a.tokens[s] = a.n_vocab - 1;
    return;
  }
  const double r = (double)u * S;
  // first piece whose inclusive prefix reaches r (the run re-summed in the
  // same order as above)
  int first = INT_MAX;
  double run = 0.0, before = 0.0;
  for (int k = p0; k < p1; ++k) {
    const double term = piece_scale(parts[k], gm, temp) * (double)parts[k].sum;
    const double next = run + term;
    if (first == INT_MAX && term > 0.0 && tbase + next >= r) {
      first = k;
      before = run;
    }
    run = next;
  }
  const int mine = first;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
  if (lane == 0) red_sel[warp] = first;
  __syncthreads();
  int ksel = INT_MAX;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) ksel = min(ksel, red_sel[w]);
  if (ksel == INT_MAX) {  // rounding: the walk ends past the last piece
    if (tid == 0) a.tokens[s] = a.n_vocab - 1;
    return;
  }
  if (mine == ksel) {
    sel_piece = ksel;
    sel_max = parts[ksel].max;
    sel_scale = piece_scale(parts[ksel], gm, temp);
    sel_base = tbase + before;
  }
  __syncthreads();
  if (warp != 0) return;

  // warp 0 recomputes the selected piece as the pass kernel did and walks
  // slab -> lane -> element
  const int kp = sel_piece;
  const bool vec = (reinterpret_cast<uintptr_t>(a.logits) & 15u) == 0 && a.row_stride % 4 == 0;
  float x[kPieceSlabs][4];
  unsigned valid[kPieceSlabs];
  load_piece_global(a, s, kp, pen_row(a, s), pen, vec, lane, x, valid);
  piece_probs<false>(x, valid, sel_max, k2_of(temp));
  float P[kPieceSlabs], Sv[kPieceSlabs];
  piece_scan(x, lane, P, Sv);
  const double base = sel_base, scale = sel_scale;
  int v = kPieceSlabs - 1;
  float sb = 0.0f;
#pragma unroll
  for (int w = 0; w < kPieceSlabs; ++w) {
    if (reaches(base, scale, __fadd_rn(sb, Sv[w]), r)) {
      v = w;
      break;
    }
    if (w < kPieceSlabs - 1) sb = __fadd_rn(sb, Sv[w]);
  }
  float Pv = P[0], pv[4];
  unsigned vv = valid[0];
#pragma unroll
  for (int j = 0; j < 4; ++j) pv[j] = x[0][j];
#pragma unroll
  for (int w = 1; w < kPieceSlabs; ++w)
    if (w == v) {
      Pv = P[w];
      vv = valid[w];
#pragma unroll
      for (int j = 0; j < 4; ++j) pv[j] = x[w][j];
    }
  const unsigned ball = __ballot_sync(0xffffffffu, reaches(base, scale, __fadd_rn(sb, Pv), r));
  const int l_sel = ball ? __ffs(ball) - 1 : 31;  // lane 31's prefix is the slab total
  const float prev = __shfl_up_sync(0xffffffffu, Pv, 1);
  if (lane == l_sel) {
    float run = lane == 0 ? 0.0f : prev;
    int jsel = -1, jlast_pos = -1, jlast_valid = -1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (!(vv >> j & 1u)) continue;
      jlast_valid = j;
      if (pv[j] > 0.0f) jlast_pos = j;
      run = __fadd_rn(run, pv[j]);
      if (jsel < 0 && pv[j] > 0.0f && reaches(base, scale, __fadd_rn(sb, run), r)) jsel = j;
    }
    if (jsel < 0) jsel = jlast_pos >= 0 ? jlast_pos : (jlast_valid >= 0 ? jlast_valid : 0);
    a.tokens[s] = kp * kPiece + v * 128 + 4 * lane + jsel;
  }
}

}  // namespace

int sample_max_vocab() { return kMaxChunks * kChunk; }
int sample_vocab_granule() { return kChunk; }
size_t sample_partial_bytes() { return sizeof(PiecePartial) * kMaxPieces; }

nvattn_status sample_prepare_device() {
  // large dynamic shared memory: set before the first launch, outside captures
  if (cudaFuncSetAttribute(sample_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kCountSmem) != cudaSuccess ||
      cudaFuncSetAttribute(sample_pass_kernel<true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, kPassSmem) != cudaSuccess ||
      cudaFuncSetAttribute(sample_pass_kernel<false>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, kPassSmem) != cudaSuccess)
    return NVATTN_ERR_CUDA;
  return NVATTN_OK;
}

nvattn_status launch_sample(nvattn_handle* h, int n_seqs, int n_vocab, const float* logits,
                            long long row_stride, const float* temps, const float* pens,
                            const int32_t* hist, const int64_t* hist_off, const float* uniforms,
                            int32_t* tokens, cudaStream_t stream) {
  SampleArgs a = {};
  a.n_seqs = n_seqs;
  a.n_vocab = n_vocab;
  a.n_chunks = (n_vocab + kChunk - 1) / kChunk;
  a.logits = logits;
  a.row_stride = row_stride;
  a.temps = temps;
  a.pens = pens;
  a.hist = hist;
  a.hist_off = hist_off;
  a.uniforms = uniforms;
  a.tokens = tokens;
  a.nib = h->samp_nib;
  a.cnt_exact = h->samp_exact;
  a.cap = h->samp_cap;
  a.part = reinterpret_cast<PiecePartial*>(h->samp_part);
  a.status = h->status_dev;
  if (hist != nullptr)
    sample_count_kernel<<<dim3((unsigned)n_seqs, (unsigned)((a.cap + kSegment - 1) / kSegment)),
                          kCountThreads, kCountSmem, stream>>>(a);
  const bool bulk = (reinterpret_cast<uintptr_t>(logits) & 15u) == 0 && row_stride % 4 == 0;
  const long long items = (long long)n_seqs * a.n_chunks;
  const int grid = (int)std::min<long long>(items, (long long)kPassCtasPerSm * h->sm_count);
  if (bulk)
    sample_pass_kernel<true><<<grid, kPassThreads, kPassSmem, stream>>>(a);
  else
    sample_pass_kernel<false><<<grid, kPassThreads, kPassSmem, stream>>>(a);
  sample_finish_kernel<<<n_seqs, kThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace nvattn
