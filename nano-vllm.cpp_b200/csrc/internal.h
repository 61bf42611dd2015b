// internal.h -- host-side state shared by the libnvattn translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "nvattn.h"
#ifdef __CUDACC__
#include "common.cuh"
#else
namespace nvattn {
struct DeviceStatus;
}
#endif

// One cached TMA descriptor for a cache buffer (keyed by its base pointer and
// the box it was encoded with).
struct NvattnTensorMapEntry {
  const void* base;
  int box_d;     // inner box extent (elements)
  int box_rows;  // tokens per box
  int swizzle;   // CUtensorMapSwizzle value
  CUtensorMap map;
};

struct nvattn_handle {
  nvattn_config cfg;
  int64_t n_slots;  // num_blocks * block_size (slots per layer)
  int sm_count;

  float* rope_table_dev = nullptr;  // [max_position][cos x head_dim/2 | sin x head_dim/2]
  nvattn::DeviceStatus* status_dev = nullptr;
  // prefill work counter: [0] next item, [1] CTAs finished (zero between
  // launches; the last CTA of each launch zeroes both)
  int* prefill_sched_dev = nullptr;

  // split-KV workspace for decode
  float* ws_o = nullptr;   // [max_seqs][n_kv_heads][max_splits][G][head_dim]
  float* ws_ml = nullptr;  // [max_seqs][n_kv_heads][max_splits][G][2]
  int* decode_tickets = nullptr;  // [max_seqs][n_kv_heads], zero between launches
  int max_splits = 0;
  // the normed, rotated q of a decode step run as two launches (the KV store
  // writes it, the decode reads it): [max_seqs][n_q_heads][head_dim] f32
  float* q_step = nullptr;

  // all-gather of decode outputs over peer memory (nvattn_gather_*): this
  // rank's allocation holds [2 step parities][g_ranks][g_slice] f32 and, at
  // g_flag_off, the completion counter; g_peer[p] is rank p's allocation
  // mapped on this device (g_peer[g_rank] == g_own)
  static constexpr int kMaxGatherRanks = 8;
  // byte offset, from the completion counter, of this rank's count of the
  // decode CTAs that have written final rows (zeroed with the counter)
  static constexpr size_t kGatherDoneOffset = 64;
  int g_ranks = 0, g_rank = 0;
  long long g_slice = 0;  // floats per rank: max_seqs * n_q_heads * head_dim
  size_t g_flag_off = 0;
  char* g_own = nullptr;
  char* g_peer[kMaxGatherRanks] = {};
  bool g_connected = false;
  unsigned g_steps = 0;   // gather steps issued on this handle
  // final-row CTAs counted so far at g_flag_off + kGatherDoneOffset (the
  // decode launch's last one releases the step's rows)
  unsigned g_done_total = 0;

  // TMA descriptor cache: fixed storage, replaced round-robin once full, so
  // an entry never moves while the handle lives.
  static constexpr int kMapCacheSize = 16;
  NvattnTensorMapEntry maps[kMapCacheSize] = {};
  int n_maps = 0;
  int next_map = 0;  // slot the next new descriptor replaces once full

  // sampler workspace (sample.cu), allocated by the first nvattn_sample call
  // for a vocabulary size; no contents survive between calls
  uint8_t* samp_nib = nullptr;     // [max_seqs][samp_cap/2] 4-bit history id counts
  uint32_t* samp_exact = nullptr;  // [max_seqs][samp_cap] exact counts where 4 bits saturate
  void* samp_part = nullptr;       // [max_seqs][512] chunk partials
  long long samp_cap = 0;          // vocabulary capacity (multiple of 4096)
};

namespace nvattn {

// Largest n_seqs of one decode launch (the grid's z extent).
constexpr int kMaxDecodeSeqs = 65535;

// Copies into *out a TMA descriptor over a whole K or V cache (all layers):
// dims {head_dim, n_kv_heads, n_layer*n_slots}, bf16, box {box_d, 1, box_rows}.
// Encoded descriptors are cached per handle; the copy keeps the caller's
// descriptor valid whatever later lookups do to the cache.
nvattn_status get_cache_tensor_map(nvattn_handle* h, const void* base, int box_d,
                                   int box_rows, int swizzle, CUtensorMap* out);

// Generic 3-D tensor map of 16-bit elements (bf16 caches; f16 Q in prefill).
nvattn_status encode_tensor_map_3d(CUtensorMap* map, const void* base, uint64_t d0,
                                   uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                                   uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                                   uint32_t box2, int swizzle,
                                   CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);

nvattn_status launch_kv_store(nvattn_handle* h, int layer, int n_tokens, const float* q,
                              const float* k, const float* v, const uint16_t* qw,
                              const uint16_t* kw, const int32_t* positions,
                              const int32_t* slots, void* q_out, nvattn_dtype q_out_dtype,
                              uint16_t* k_cache, uint16_t* v_cache, uint16_t* k_rows,
                              uint16_t* v_rows, cudaStream_t stream);

nvattn_status launch_paged_decode(nvattn_handle* h, int layer, int n_seqs, const float* q,
                                  const uint16_t* k_cache, const uint16_t* v_cache,
                                  const int32_t* block_tables, int max_blocks,
                                  const int32_t* context_lens, int max_context_len,
                                  float* out, cudaStream_t stream);
// The fused decode step: q/k RMSNorm + RoPE of the raw rows, the store of the
// new K/V row and the decode in one launch (nvattn_paged_decode_step).
// Launches nvattn_paged_decode_step makes for this batch shape: 1 (the fused
// kernel) or 2 (the KV store into q_step, then the plain decode).
int decode_step_launches(const nvattn_handle* h, int n_seqs, int max_context_len);
// The decode step with every output row also stored into every rank's
// gathered buffer, then the release/wait launch (nvattn_paged_decode_step_gather).
nvattn_status launch_paged_decode_step_gather(nvattn_handle* h, int layer, int n_seqs,
                                              const float* q, const float* k_new,
                                              const float* v_new, const uint16_t* q_norm_w,
                                              const uint16_t* k_norm_w, const int32_t* positions,
                                              const int32_t* slots, uint16_t* k_cache,
                                              uint16_t* v_cache, const int32_t* block_tables,
                                              int max_blocks, const int32_t* context_lens,
                                              int max_context_len, float* out,
                                              cudaStream_t stream);
nvattn_status launch_paged_decode_step(nvattn_handle* h, int layer, int n_seqs, const float* q,
                                       const float* k_new, const float* v_new,
                                       const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                       const int32_t* positions, const int32_t* slots,
                                       uint16_t* k_cache, uint16_t* v_cache,
                                       const int32_t* block_tables, int max_blocks,
                                       const int32_t* context_lens, int max_context_len,
                                       float* out, cudaStream_t stream);

nvattn_status launch_paged_prefill(nvattn_handle* h, int layer, int n_seqs, int n_tokens,
                                   const uint16_t* q, const int32_t* cu_q,
                                   const int32_t* q_starts, const int32_t* context_lens,
                                   const int32_t* block_tables, int max_blocks,
                                   int max_q_len, const uint16_t* k_cache,
                                   const uint16_t* v_cache, const uint16_t* k_rows,
                                   const uint16_t* v_rows, float* out, cudaStream_t stream);

// Device-side planners (plan.cu): the host planners' outputs from
// device-resident sequence lengths and block tables, errors to status_dev.
nvattn_status launch_plan_prefill(nvattn_handle* h, int n_seqs, const int64_t* seq_lens,
                                  const int64_t* num_cached, const int32_t* block_tables,
                                  int max_blocks, int max_tokens, int32_t* cu_q,
                                  int32_t* q_starts, int32_t* context_lens, int32_t* positions,
                                  int32_t* slot_mapping, cudaStream_t stream);

nvattn_status launch_plan_decode(nvattn_handle* h, int n_seqs, const int64_t* seq_lens,
                                 const int32_t* block_tables, int max_blocks,
                                 int32_t* context_lens, int32_t* positions,
                                 int32_t* slot_mapping, cudaStream_t stream);

// Token sampler (sample.cu).
int sample_max_vocab();
int sample_vocab_granule();      // samp_cap is a multiple of this
size_t sample_partial_bytes();   // per sequence
nvattn_status sample_prepare_device();  // kernel attributes, outside captures
nvattn_status launch_sample(nvattn_handle* h, int n_seqs, int n_vocab, const float* logits,
                            long long row_stride, const float* temps, const float* pens,
                            const int32_t* hist, const int64_t* hist_off, const float* uniforms,
                            int32_t* tokens, cudaStream_t stream);

// Host RoPE table: ggml's rope cache recurrence for positions [0, n_pos).
void build_rope_table(const nvattn_config& cfg, int n_pos, float* table);

}  // namespace nvattn
