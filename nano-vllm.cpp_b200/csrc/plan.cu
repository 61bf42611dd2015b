// plan.cu -- device-side planners: positions, slot mapping, cu_q_lens,
// q_starts and context lengths from device-resident sequence lengths, cached
// prefix lengths and block tables.  The same derivation as the host planners
// in api.cu (nvattn_plan_prefill / nvattn_plan_decode), i.e. the reference's
// PrepareInputs (src/engine/model_runner.cpp:138-186) over BlockManager's
// tables (src/engine/block_manager.cpp:96-184), bit for bit.
//
// Prefill is two launches: one CTA scans the per-sequence token counts into
// cu_q_lens (1024 threads, each owning a contiguous run of sequences), then a
// grid over the max_tokens bound fills positions and slots, each thread
// finding its sequence by binary search in cu_q_lens.  Decode is one thread
// per sequence.
#include "common.cuh"
#include "internal.h"

namespace nvattn {
namespace {

constexpr int kScanThreads = 1024;

// Per-sequence query count and start, with the host planner's checks.
// Returns false (and the count 0) for an invalid sequence.
__device__ __forceinline__ bool seq_plan(long long len, long long start, int block_size,
                                         int max_blocks, long long& count, long long& first) {
  count = 0;
  first = 0;
  if (len <= 0 || start < 0 || start > len || len > 0x7fffffffLL) return false;
  // A prompt whose every block hit the prefix cache still computes its last
  // token (the reference would feed zero tokens and sample from index -1,
  // model_runner.cpp:158-160,182).
  if (start == len) start = len - 1;
  if ((len + block_size - 1) / block_size > max_blocks) return false;
  count = len - start;
  first = start;
  return true;
}

__global__ void __launch_bounds__(kScanThreads)
    plan_prefill_scan_kernel(int n_seqs, const int64_t* seq_lens, const int64_t* num_cached,
                             int max_blocks, int block_size, int max_tokens, int32_t* cu_q,
                             int32_t* q_starts, int32_t* context_lens, DeviceStatus* status) {
  __shared__ long long warp_tot[kScanThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n_seqs + kScanThreads - 1) / kScanThreads;
  const int s0 = min(n_seqs, tid * per), s1 = min(n_seqs, s0 + per);
  long long local = 0;
  for (int s = s0; s < s1; ++s) {
    long long c, f;
    if (!seq_plan(seq_lens[s], num_cached[s], block_size, max_blocks, c, f))
      record_error(status, NVATTN_ERR_INVALID_ARG, 60, s);
    local += c;
  }
  // exclusive scan of `local` over the block
  long long incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    long long t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long v = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += v;
    }
    warp_tot[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  long long off = incl - local + (warp > 0 ? warp_tot[warp - 1] : 0);
  if (tid == 0) cu_q[0] = 0;
  for (int s = s0; s < s1; ++s) {
    long long c, f;
    seq_plan(seq_lens[s], num_cached[s], block_size, max_blocks, c, f);
    off += c;
    if (off > max_tokens) record_error(status, NVATTN_ERR_INVALID_ARG, 61, s);
    q_starts[s] = (int32_t)f;
    context_lens[s] = (int32_t)seq_lens[s];
    cu_q[s + 1] = (int32_t)min(off, (long long)0x7fffffff);
  }
}

__global__ void plan_prefill_fill_kernel(int n_seqs, const int32_t* cu_q, const int32_t* q_starts,
                                         const int32_t* block_tables, int max_blocks,
                                         int block_size, int max_tokens, int32_t* positions,
                                         int32_t* slot_mapping, DeviceStatus* status) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int total = min(cu_q[n_seqs], max_tokens);
  if (t >= total) return;
  // largest s with cu_q[s] <= t
  int lo = 0, hi = n_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu_q[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int s = lo;
  const long long pos = q_starts[s] + (t - cu_q[s]);
  const long long bi = pos / block_size;
  const int32_t bid = bi < max_blocks ? block_tables[(long long)s * max_blocks + bi] : -1;
  if (bid < 0) record_error(status, NVATTN_ERR_OUT_OF_RANGE, 62, s);
  positions[t] = (int32_t)pos;
  slot_mapping[t] = bid < 0 ? -1 : (int32_t)((long long)bid * block_size + pos % block_size);
}

__global__ void plan_decode_kernel(int n_seqs, const int64_t* seq_lens,
                                   const int32_t* block_tables, int max_blocks, int block_size,
                                   int32_t* context_lens, int32_t* positions,
                                   int32_t* slot_mapping, DeviceStatus* status) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n_seqs) return;
  const long long len = seq_lens[s];
  if (len <= 0 || len > 0x7fffffffLL || (len - 1) / block_size >= max_blocks) {
    record_error(status, NVATTN_ERR_INVALID_ARG, 63, s);
    return;
  }
  const long long pos = len - 1;
  const int32_t bid = block_tables[(long long)s * max_blocks + pos / block_size];
  if (bid < 0) record_error(status, NVATTN_ERR_OUT_OF_RANGE, 64, s);
  context_lens[s] = (int32_t)len;
  positions[s] = (int32_t)pos;
  slot_mapping[s] = bid < 0 ? -1 : (int32_t)((long long)bid * block_size + pos % block_size);
}

}  // namespace

nvattn_status launch_plan_prefill(nvattn_handle* h, int n_seqs, const int64_t* seq_lens,
                                  const int64_t* num_cached, const int32_t* block_tables,
                                  int max_blocks, int max_tokens, int32_t* cu_q,
                                  int32_t* q_starts, int32_t* context_lens, int32_t* positions,
                                  int32_t* slot_mapping, cudaStream_t stream) {
  const int bs = h->cfg.block_size;
  plan_prefill_scan_kernel<<<1, kScanThreads, 0, stream>>>(n_seqs, seq_lens, num_cached,
                                                          max_blocks, bs, max_tokens, cu_q,
                                                          q_starts, context_lens, h->status_dev);
  if (max_tokens > 0) {
    const int threads = 256;
    const long long blocks = ((long long)max_tokens + threads - 1) / threads;
    plan_prefill_fill_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
        n_seqs, cu_q, q_starts, block_tables, max_blocks, bs, max_tokens, positions,
        slot_mapping, h->status_dev);
  }
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

nvattn_status launch_plan_decode(nvattn_handle* h, int n_seqs, const int64_t* seq_lens,
                                 const int32_t* block_tables, int max_blocks,
                                 int32_t* context_lens, int32_t* positions,
                                 int32_t* slot_mapping, cudaStream_t stream) {
  const int threads = 256;
  plan_decode_kernel<<<(n_seqs + threads - 1) / threads, threads, 0, stream>>>(
      n_seqs, seq_lens, block_tables, max_blocks, h->cfg.block_size, context_lens, positions,
      slot_mapping, h->status_dev);
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace nvattn
