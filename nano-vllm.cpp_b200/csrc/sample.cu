// sample.cu -- next-token sampling over a batch of logits rows on the device:
// ModelRunner::Sample (src/engine/model_runner.cpp:417-489) -- repetition
// penalty, greedy argmax (temperature < 1e-6) or temperature sampling by
// inverse CDF with a caller-supplied uniform draw.
//
// Two launches.  The first counts, per sequence with penalty > 1, how often
// each token id occurs in its history (an atomic histogram over a
// [n_seqs][n_vocab] u32 array that is all zero between calls) and marks the
// ids in a per-sequence bitmap, so the row pass reads one bit per logit and
// touches a count only for history ids.  The second splits every row into
// 4096-element chunks, one 256-thread CTA per (chunk, sequence): it loads the
// chunk (four 1024-element slabs, one float4 per thread each), applies the
// penalty (the reference's v = v < 0 ? v*p : v/p once per occurrence, so bit
// for bit), and writes the chunk's maximum, first arg-max, NaN flags and --
// for sampling rows -- sum of exp((x - chunk max)/t).  The last CTA of a
// sequence to finish (an atomic ticket) combines the chunk results: greedy
// rows take the first arg-max; sampling rows scale each chunk's sum by
// exp((chunk max - row max)/t), draw r = u*S, pick the chunk whose running
// total reaches r, re-read that one chunk and find the element.  The same
// CTA then zeroes the counts and bitmap words its history set, and the
// ticket.  One pass over the logits: HBM-bound.
//
// Greedy tokens are bit-exact with the reference (same penalised values,
// same first-index rule, same NaN outcomes).  Sampled tokens follow the same
// inverse-CDF rule on the same draw; the probabilities differ from the
// reference's float chain by a few ulp (exp by ex2.approx on
// (x - m)*log2(e)/t, chunk-wise sums in double), so a draw within that
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

constexpr int kThreads = 256;
constexpr int kSlabs = 4;
constexpr int kSlab = kThreads * 4;     // elements per slab
constexpr int kChunk = kSlab * kSlabs;  // elements per CTA
constexpr int kMaxChunks = 512;         // n_vocab <= 2,097,152

struct ChunkPartial {
  float max;   // maximum of the chunk's non-NaN penalised values (-inf if none)
  int argmax;  // first index holding it, INT_MAX if the chunk has no non-NaN value
  float sum;   // sampling rows: sum of exp((x - max)/t) in the fixed scan order
  int flags;   // bit 0: a NaN in the chunk; bit 1: element 0 of the row is NaN
};
static_assert(sizeof(ChunkPartial) == 16, "partial layout");

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
  uint32_t* cnt;  // [max_seqs][cap]
  uint32_t* bits;  // [max_seqs][cap/32]
  long long cap;
  ChunkPartial* part;  // [max_seqs][kMaxChunks]
  unsigned* ticket;    // [max_seqs]
  DeviceStatus* status;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool penalised(const SampleArgs& a, int s) {
  return a.hist != nullptr && a.pens[s] > 1.0f;
}

// History bounds of sequence s, or false if the offsets are unusable.
__device__ __forceinline__ bool hist_range(const SampleArgs& a, int s, long long& b,
                                           long long& e) {
  b = a.hist_off[s];
  e = a.hist_off[s + 1];
  return b >= 0 && e >= b;
}

// The reference's penalty, applied once per occurrence.  Zero, infinities and
// NaN are fixed points of the step, so the loop stops early on them.
__device__ __forceinline__ float apply_penalty(float v, float p, uint32_t c) {
  for (uint32_t k = 0; k < c; ++k) {
    if (v == 0.0f || isinf(v) || isnan(v)) break;
    v = v < 0.0f ? __fmul_rn(v, p) : __fdiv_rn(v, p);
  }
  return v;
}

__global__ void __launch_bounds__(kThreads) sample_count_kernel(SampleArgs a) {
  const int s = blockIdx.y;
  if (!penalised(a, s)) return;
  long long b, e;
  if (!hist_range(a, s, b, e)) {
    if (blockIdx.x == 0 && threadIdx.x == 0) record_error(a.status, NVATTN_ERR_INVALID_ARG, 70, s);
    return;
  }
  uint32_t* cnt = a.cnt + (long long)s * a.cap;
  uint32_t* bits = a.bits + (long long)s * (a.cap / 32);
  for (long long j = b + (long long)blockIdx.x * kThreads + threadIdx.x; j < e;
       j += (long long)gridDim.x * kThreads) {
    const int32_t tok = a.hist[j];
    if (tok < 0 || tok >= a.n_vocab) continue;  // the reference skips ids >= n_vocab
    if (atomicAdd(&cnt[tok], 1u) == 0u) atomicOr(&bits[tok >> 5], 1u << (tok & 31));
  }
}

// Loads chunk `c` of row s into x[slab][j] (element c*kChunk + slab*kSlab +
// 4*tid + j) with the penalty applied; valid[slab] has bit j set for elements
// inside the row.
template <bool kVec>
__device__ __forceinline__ void load_chunk(const SampleArgs& a, int s, int c, bool pen_on,
                                           float pen, float (&x)[kSlabs][4],
                                           unsigned (&valid)[kSlabs]) {
  const float* row = a.logits + (long long)s * a.row_stride;
#pragma unroll
  for (int v = 0; v < kSlabs; ++v) {
    const int idx = c * kChunk + v * kSlab + threadIdx.x * 4;
    if (kVec && idx + 3 < a.n_vocab) {
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
  }
  if (!pen_on) return;
  const uint32_t* bits = a.bits + (long long)s * (a.cap / 32);
  const uint32_t* cnt = a.cnt + (long long)s * a.cap;
#pragma unroll
  for (int v = 0; v < kSlabs; ++v) {
    const int idx = c * kChunk + v * kSlab + threadIdx.x * 4;
    if (valid[v] == 0u) continue;
    unsigned hit = (__ldcg(bits + (idx >> 5)) >> (idx & 31)) & valid[v];
    while (hit) {
      const int j = __ffs(hit) - 1;
      hit &= hit - 1;
      float val = x[v][0];
#pragma unroll
      for (int jj = 1; jj < 4; ++jj)
        if (jj == j) val = x[v][jj];
      val = apply_penalty(val, pen, __ldcg(cnt + idx + j));
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        if (jj == j) x[v][jj] = val;
    }
  }
}

// (max, first arg-max) pair order: a larger value wins, then the smaller index.
__device__ __forceinline__ void max_combine(float& m, int& am, float m2, int am2) {
  if (am2 == INT_MAX) return;
  if (am == INT_MAX || m2 > m || (m2 == m && am2 < am)) {
    m = m2;
    am = am2;
  }
}

struct BlockScratch {
  float wm[kThreads / 32];
  int wam[kThreads / 32];
  int wflags[kThreads / 32];
  float wsum[kSlabs][kThreads / 32];
  float pref[kThreads];  // inclusive thread prefixes of one slab (final phase)
  ChunkPartial parts[kMaxChunks];
  int sel_chunk, is_last, token;
  float sel_max;
  double base, scale, r;
};

// Block-wide (max, arg-max, flags) of the chunk, broadcast to every thread.
__device__ __forceinline__ void chunk_max(const float (&x)[kSlabs][4],
                                          const unsigned (&valid)[kSlabs], int c,
                                          BlockScratch& sh, float& m, int& am, int& flags) {
  m = -INFINITY;
  am = INT_MAX;
  flags = 0;
#pragma unroll
  for (int v = 0; v < kSlabs; ++v) {
    const int idx = c * kChunk + v * kSlab + threadIdx.x * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (!(valid[v] >> j & 1u)) continue;
      if (isnan(x[v][j])) {
        flags |= 1 | (idx + j == 0 ? 2 : 0);
      } else if (am == INT_MAX || x[v][j] > m) {
        m = x[v][j];
        am = idx + j;
      }
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const int a2 = __shfl_xor_sync(0xffffffffu, am, o);
    flags |= __shfl_xor_sync(0xffffffffu, flags, o);
    max_combine(m, am, m2, a2);
  }
  if (lane == 0) {
    sh.wm[warp] = m;
    sh.wam[warp] = am;
    sh.wflags[warp] = flags;
  }
  __syncthreads();
  m = sh.wm[0];
  am = sh.wam[0];
  flags = sh.wflags[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) {
    max_combine(m, am, sh.wm[w], sh.wam[w]);
    flags |= sh.wflags[w];
  }
  __syncthreads();
}

// p = exp((x - m)/t) as 2^((x - m)*k2), k2 = log2(e)/t; 0 outside the row.
__device__ __forceinline__ void chunk_probs(float (&x)[kSlabs][4], const unsigned (&valid)[kSlabs],
                                            float m, float k2) {
#pragma unroll
  for (int v = 0; v < kSlabs; ++v)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      x[v][j] = (valid[v] >> j & 1u) ? ex2_approx(__fmul_rn(__fsub_rn(x[v][j], m), k2)) : 0.0f;
}

// Inclusive prefix of each thread's 4-element sum, per slab, in one fixed
// order: ((p0+p1)+p2)+p3 per thread, Hillis-Steele shuffles across the warp,
// then the warp totals summed in warp order.  P[v] is this thread's inclusive
// prefix; S[v] the slab total, equal bit for bit to thread 255's P[v].
__device__ __forceinline__ void slab_scan(const float (&p)[kSlabs][4], BlockScratch& sh,
                                          float (&P)[kSlabs], float (&S)[kSlabs]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float inc[kSlabs];
#pragma unroll
  for (int v = 0; v < kSlabs; ++v)
    inc[v] = __fadd_rn(__fadd_rn(__fadd_rn(p[v][0], p[v][1]), p[v][2]), p[v][3]);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
    for (int v = 0; v < kSlabs; ++v) {
      const float y = __shfl_up_sync(0xffffffffu, inc[v], o);
      if (lane >= o) inc[v] = __fadd_rn(inc[v], y);
    }
  }
  if (lane == 31)
#pragma unroll
    for (int v = 0; v < kSlabs; ++v) sh.wsum[v][warp] = inc[v];
  __syncthreads();
#pragma unroll
  for (int v = 0; v < kSlabs; ++v) {
    float base = 0.0f, tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) {
      if (w < warp) base = __fadd_rn(base, sh.wsum[v][w]);
      tot = __fadd_rn(tot, sh.wsum[v][w]);
    }
    P[v] = warp == 0 ? inc[v] : __fadd_rn(base, inc[v]);
    S[v] = tot;
  }
  __syncthreads();
}

__device__ __forceinline__ bool reaches(double base, double scale, float local, double r) {
  return base + scale * (double)local >= r;
}

template <bool kVec>
__global__ void __launch_bounds__(kThreads) sample_chunk_kernel(SampleArgs a) {
  __shared__ BlockScratch sh;
  const int s = blockIdx.y, c = blockIdx.x, tid = threadIdx.x;
  const float temp = a.temps[s];
  const bool greedy = temp < 1e-6f;
  const bool pen_on = penalised(a, s);
  const float pen = a.pens[s];
  long long hb = 0, he = 0;
  const bool hist_ok = pen_on && hist_range(a, s, hb, he);

  float x[kSlabs][4];
  unsigned valid[kSlabs];
  load_chunk<kVec>(a, s, c, hist_ok, pen, x, valid);
  float m;
  int am, flags;
  chunk_max(x, valid, c, sh, m, am, flags);
  float sum = 0.0f;
  const float k2 = __fdiv_rn(1.4426950408889634f, temp);
  if (!greedy && !(flags & 1) && am != INT_MAX && isfinite(m)) {
    chunk_probs(x, valid, m, k2);
    float P[kSlabs], S[kSlabs];
    slab_scan(x, sh, P, S);
    sum = __fadd_rn(__fadd_rn(__fadd_rn(S[0], S[1]), S[2]), S[3]);
  }
  if (tid == 0) {
    ChunkPartial cp;
    cp.max = m;
    cp.argmax = am;
    cp.sum = sum;
    cp.flags = flags;
    a.part[(long long)s * kMaxChunks + c] = cp;
    __threadfence();
    sh.is_last = atomicAdd(&a.ticket[s], 1u) == (unsigned)(a.n_chunks - 1);
  }
  __syncthreads();
  if (!sh.is_last) return;
  __threadfence();

  // ---- last CTA of sequence s: combine the chunks ----
  for (int i = tid; i < a.n_chunks; i += kThreads) {
    const float4 q = __ldcg(reinterpret_cast<const float4*>(a.part + (long long)s * kMaxChunks + i));
    ChunkPartial cp;
    cp.max = q.x;
    cp.argmax = __float_as_int(q.y);
    cp.sum = q.z;
    cp.flags = __float_as_int(q.w);
    sh.parts[i] = cp;
  }
  __syncthreads();
  if (tid == 0) {
    float gm = -INFINITY;
    int gam = INT_MAX, gflags = 0;
    for (int i = 0; i < a.n_chunks; ++i) {
      max_combine(gm, gam, sh.parts[i].max, sh.parts[i].argmax);
      gflags |= sh.parts[i].flags;
    }
    int token = -1;
    if (greedy) {
      token = (gflags & 2) || gam == INT_MAX ? 0 : gam;
    } else {
      const float u = a.uniforms[s];
      if (!(u >= 0.0f && u < 1.0f)) {
        record_error(a.status, NVATTN_ERR_INVALID_ARG, 71, s);
        token = a.n_vocab - 1;
      } else if ((gflags & 1) || gam == INT_MAX || !isfinite(gm) || isnan(temp)) {
        token = a.n_vocab - 1;  // the reference's NaN sum never reaches r
      } else {
        double S = 0.0;
        for (int i = 0; i < a.n_chunks; ++i) {
          const ChunkPartial& cp = sh.parts[i];
          const double sc =
              cp.argmax == INT_MAX || !isfinite(cp.max) ? 0.0 : exp(((double)cp.max - gm) / temp);
          S += sc * (double)cp.sum;
        }
        if (!(S > 0.0) || !isfinite(S)) {
          token = a.n_vocab - 1;
        } else {
          const double r = (double)u * S;
          double base = 0.0;
          int k = a.n_chunks - 1;
          double ksc = 0.0, kbase = 0.0;
          for (int i = 0; i < a.n_chunks; ++i) {
            const ChunkPartial& cp = sh.parts[i];
            const double sc = cp.argmax == INT_MAX || !isfinite(cp.max)
                                  ? 0.0
                                  : exp(((double)cp.max - gm) / temp);
            const double next = base + sc * (double)cp.sum;
            k = i;
            ksc = sc;
            kbase = base;
            if (next >= r && sc > 0.0) break;
            base = next;
          }
          sh.sel_chunk = k;
          sh.sel_max = sh.parts[k].max;
          sh.base = kbase;
          sh.scale = ksc;
          sh.r = r;
        }
      }
    }
    sh.token = token;
  }
  __syncthreads();
  if (sh.token < 0) {
    // re-read the selected chunk and walk slab -> thread -> element
    const int kc = sh.sel_chunk;
    load_chunk<kVec>(a, s, kc, hist_ok, pen, x, valid);
    chunk_probs(x, valid, sh.sel_max, k2);
    float P[kSlabs], S[kSlabs];
    slab_scan(x, sh, P, S);
    const double base = sh.base, scale = sh.scale, r = sh.r;
    int v = kSlabs - 1;
    float sb = 0.0f;
#pragma unroll
    for (int w = 0; w < kSlabs; ++w) {
      if (reaches(base, scale, __fadd_rn(sb, S[w]), r)) {
        v = w;
        break;
      }
      if (w < kSlabs - 1) sb = __fadd_rn(sb, S[w]);
    }
    // v and sb are the same in every thread (computed from block-uniform values)
    float Pv = P[0];
#pragma unroll
    for (int w = 1; w < kSlabs; ++w)
      if (w == v) Pv = P[w];
    sh.pref[tid] = Pv;
    const bool hit = reaches(base, scale, __fadd_rn(sb, Pv), r);
    const unsigned ball = __ballot_sync(0xffffffffu, hit);
    if ((tid & 31) == 0) sh.wam[tid >> 5] = ball ? (tid & ~31) + __ffs(ball) - 1 : INT_MAX;
    __syncthreads();
    int t_sel = INT_MAX;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) t_sel = min(t_sel, sh.wam[w]);
    if (t_sel == INT_MAX) t_sel = kThreads - 1;  // P of thread 255 is the slab total
    if (tid == t_sel) {
      float acc = tid == 0 ? 0.0f : sh.pref[tid - 1];
      int jsel = -1, jlast_pos = -1, jlast_valid = -1;
      float pv[4];
#pragma unroll
      for (int w = 0; w < kSlabs; ++w)
        if (w == v)
#pragma unroll
          for (int j = 0; j < 4; ++j) pv[j] = x[w][j];
      unsigned vv = 0;
#pragma unroll
      for (int w = 0; w < kSlabs; ++w)
        if (w == v) vv = valid[w];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (!(vv >> j & 1u)) continue;
        jlast_valid = j;
        if (pv[j] > 0.0f) jlast_pos = j;
        acc = __fadd_rn(acc, pv[j]);
        if (jsel < 0 && pv[j] > 0.0f && reaches(base, scale, __fadd_rn(sb, acc), r)) jsel = j;
      }
      if (jsel < 0) jsel = jlast_pos >= 0 ? jlast_pos : (jlast_valid >= 0 ? jlast_valid : 0);
      sh.token = kc * kChunk + v * kSlab + tid * 4 + jsel;
    }
    __syncthreads();
  }
  if (tid == 0) a.tokens[s] = sh.token;

  // ---- leave the histogram and bitmap zero for the next call ----
  if (hist_ok) {
    uint32_t* cnt = a.cnt + (long long)s * a.cap;
    uint32_t* bits = a.bits + (long long)s * (a.cap / 32);
    for (long long j = hb + tid; j < he; j += kThreads) {
      const int32_t tok = a.hist[j];
      if (tok < 0 || tok >= a.n_vocab) continue;
      cnt[tok] = 0u;
      bits[tok >> 5] = 0u;
    }
  }
  if (tid == 0) a.ticket[s] = 0u;
}

}  // namespace

int sample_max_vocab() { return kMaxChunks * kChunk; }

nvattn_status launch_sample(nvattn_handle* h, int n_seqs, int n_vocab, const float* logits,
                            long long row_stride, const float* temps, const float* pens,
                            const int32_t* hist, const int64_t* hist_off, const float* uniforms,
                            int32_t* tokens, cudaStream_t stream) {
  SampleArgs a;
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
  a.cnt = h->samp_cnt;
  a.bits = h->samp_bits;
  a.cap = h->samp_cap;
  a.part = reinterpret_cast<ChunkPartial*>(h->samp_part);
  a.ticket = h->samp_ticket;
  a.status = h->status_dev;
  if (hist != nullptr) {
    // enough CTAs per sequence to spread a long history over the SMs
    const int per_seq = std::max(1, std::min(64, 4 * h->sm_count / std::max(1, n_seqs)));
    sample_count_kernel<<<dim3(per_seq, n_seqs), kThreads, 0, stream>>>(a);
  }
  const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15u) == 0 && row_stride % 4 == 0;
  const dim3 grid(a.n_chunks, n_seqs);
  if (vec)
    sample_chunk_kernel<true><<<grid, kThreads, 0, stream>>>(a);
  else
    sample_chunk_kernel<false><<<grid, kThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

size_t sample_partial_bytes() { return sizeof(ChunkPartial) * kMaxChunks; }

}  // namespace nvattn
