// attention_runner.h -- C++ host layer above the libnvattn C ABI, shaped like
// the part of nano-vllm.cpp's engine::ModelRunner that the attention hot path
// replaces (src/include/engine/model_runner.h:14-72).
//
// The reference's ModelRunner::Run (model_runner.cpp:25-136) builds inputs,
// runs the ggml graph, and moves K/V between the graph and the BF16 cache on
// the host (StorePrefillKV / LoadHistoryKV / AppendDecodeKV).  With the graph
// cut around the attention node, the runner instead:
//   1. PrepareInputs: derives positions, slot mapping, block tables and
//      context lengths from the scheduled sequences (model_runner.cpp:138-186)
//      and uploads them once per step;
//   2. per layer, RunAttentionLayer: fused q/k norm + RoPE + KV store, then
//      paged decode or prefill attention, all on the device.
// Error behaviour follows the reference: the constructor throws
// std::runtime_error (as Qwen3Model's does, qwen3.cpp:33-35, 106-108);
// per-step calls return false where ModelRunner::Run returns {}
// (model_runner.cpp:46-49, 67).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <random>
#include <string>
#include <vector>

#include "nvattn.h"

namespace nvattn_host {

// The fields of engine::Sequence the attention path reads
// (src/include/engine/sequence.h:19-88).
struct SequenceView {
  std::vector<size_t> block_table;  // Sequence::GetBlockTable()
  size_t seq_len = 0;               // Sequence::SequenceLen()
  size_t num_cached_tokens = 0;     // Sequence::GetNumCachedTokens()
};

class AttentionRunner {
 public:
  // sample_seed seeds the runner's std::mt19937 for temperature sampling
  // (the reference seeds its own from std::random_device).
  explicit AttentionRunner(const nvattn_config& cfg,
                           uint32_t sample_seed = std::mt19937::default_seed);
  ~AttentionRunner();
  AttentionRunner(const AttentionRunner&) = delete;
  AttentionRunner& operator=(const AttentionRunner&) = delete;

  // Builds and uploads this step's attention metadata.  Returns false on
  // invalid input (no block for a position, too many tokens) or CUDA failure.
  bool PrepareInputs(const std::vector<SequenceView*>& seqs, bool is_prefill,
                     cudaStream_t stream);

  // One layer of the cut graph: q [n_tokens][Hq][d] f32 (read only: a
  // prefill step writes the normed, rotated q as f16 to the runner's own
  // buffer; a decode step is one nvattn_paged_decode_step call), k/v
  // [n_tokens][Hkv][d] f32 (graph projections), the layer's q/k norm weights
  // (bf16 [d]), and the BF16 caches (all layers).  Writes attention output
  // [n_tokens][Hq][d] f32.
  bool RunAttentionLayer(int layer, const float* q, const float* k, const float* v,
                         const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                         uint16_t* k_cache, uint16_t* v_cache, float* out,
                         cudaStream_t stream);

  // ModelRunner::Sample (model_runner.cpp:417-489) on the device.
  // logits_dev: [n_seqs][n_vocab] f32 (the graph's output rows);
  // temperatures, penalties and histories (prompt ids, then completion ids)
  // per sequence.  Each row with temperature >= 1e-6 takes one draw, in row
  // order, from the runner's mt19937 as the reference's
  // uniform_real_distribution<float> does.  Returns the tokens after
  // synchronising the stream, or {} on invalid input, a failed call or an
  // error in the handle's status word (read and cleared here).
  std::vector<int> Sample(const float* logits_dev, int n_vocab,
                          const std::vector<float>& temperatures,
                          const std::vector<float>& penalties,
                          const std::vector<std::vector<int32_t>>& histories,
                          cudaStream_t stream);
  // The draws the last Sample call used (0 for greedy rows).
  const std::vector<float>& LastUniforms() const { return uniforms_; }

  int NumTokens() const { return n_tokens_; }
  int NumSeqs() const { return n_seqs_; }
  bool IsPrefill() const { return is_prefill_; }
  nvattn_handle* Handle() const { return handle_; }
  // Host copies of the last plan (for inspection and tests).
  const std::vector<int32_t>& Positions() const { return positions_; }
  const std::vector<int32_t>& SlotMapping() const { return slots_; }

 private:
  bool Reserve(size_t n_tokens, size_t n_seqs, size_t max_blocks);

  nvattn_config cfg_;
  nvattn_handle* handle_ = nullptr;
  bool is_prefill_ = false;
  int n_tokens_ = 0, n_seqs_ = 0, max_blocks_ = 0, max_q_len_ = 0, max_context_ = 0;

  std::vector<int32_t> positions_, slots_, block_tables_, context_lens_, cu_q_, q_starts_;

  // device buffers (owned)
  size_t cap_tokens_ = 0, cap_seqs_ = 0, cap_blocks_ = 0;
  int32_t* d_positions_ = nullptr;
  int32_t* d_slots_ = nullptr;
  int32_t* d_block_tables_ = nullptr;
  int32_t* d_context_lens_ = nullptr;
  int32_t* d_cu_q_ = nullptr;
  int32_t* d_q_starts_ = nullptr;
  uint16_t* d_q_f16_ = nullptr;

  // sampling
  std::mt19937 rng_;
  std::vector<float> uniforms_;
  size_t cap_sample_rows_ = 0, cap_history_ = 0;
  float* d_temps_ = nullptr;
  float* d_pens_ = nullptr;
  float* d_uniforms_ = nullptr;
  int32_t* d_tokens_ = nullptr;
  int64_t* d_hist_offsets_ = nullptr;
  int32_t* d_history_ = nullptr;
};

}  // namespace nvattn_host
