// attention_runner.cpp -- see attention_runner.h.
#include "attention_runner.h"

#include <algorithm>
#include <stdexcept>

namespace nvattn_host {

namespace {
template <typename T>
bool grow(T** ptr, size_t n) {
  if (*ptr) cudaFree(*ptr);
  *ptr = nullptr;
  return cudaMalloc(reinterpret_cast<void**>(ptr), std::max<size_t>(n, 1) * sizeof(T)) ==
         cudaSuccess;
}
}  // namespace

AttentionRunner::AttentionRunner(const nvattn_config& cfg) : cfg_(cfg) {
  const nvattn_status st = nvattn_create(&cfg_, &handle_);
  if (st != NVATTN_OK)
    throw std::runtime_error(std::string("nvattn_create failed: ") + nvattn_status_string(st));
}

AttentionRunner::~AttentionRunner() {
  int32_t* bufs[] = {d_positions_, d_slots_, d_block_tables_, d_context_lens_, d_cu_q_,
                     d_q_starts_};
  for (int32_t* b : bufs)
    if (b) cudaFree(b);
  if (d_q_bf16_) cudaFree(d_q_bf16_);
  nvattn_destroy(handle_);
}

bool AttentionRunner::Reserve(size_t n_tokens, size_t n_seqs, size_t max_blocks) {
  bool ok = true;
  if (n_tokens > cap_tokens_) {
    const size_t cap = std::max(n_tokens, cap_tokens_ * 2);
    ok = ok && grow(&d_positions_, cap) && grow(&d_slots_, cap) &&
         grow(&d_q_bf16_, cap * (size_t)cfg_.n_q_heads * cfg_.head_dim);
    cap_tokens_ = ok ? cap : 0;
  }
  if (n_seqs > cap_seqs_ || max_blocks > cap_blocks_) {
    const size_t cs = std::max(n_seqs, cap_seqs_), cb = std::max(max_blocks, cap_blocks_);
    ok = ok && grow(&d_context_lens_, cs) && grow(&d_cu_q_, cs + 1) && grow(&d_q_starts_, cs) &&
         grow(&d_block_tables_, cs * cb);
    cap_seqs_ = ok ? cs : 0;
    cap_blocks_ = ok ? cb : 0;
  }
  return ok;
}

bool AttentionRunner::PrepareInputs(const std::vector<SequenceView*>& seqs, bool is_prefill,
                                    cudaStream_t stream) {
  is_prefill_ = is_prefill;
  n_seqs_ = static_cast<int>(seqs.size());
  if (n_seqs_ == 0 || n_seqs_ > cfg_.max_seqs) return false;
  size_t max_blocks = 1;
  for (const SequenceView* s : seqs) max_blocks = std::max(max_blocks, s->block_table.size());
  max_blocks_ = static_cast<int>(max_blocks);

  // Block tables as int32 [n_seqs][max_blocks] (Sequence::block_table_ is a
  // std::vector<size_t>, sequence.h:85); unused entries are -1.
  block_tables_.assign(static_cast<size_t>(n_seqs_) * max_blocks, -1);
  std::vector<int64_t> lens(n_seqs_), cached(n_seqs_);
  max_context_ = 0;
  for (int s = 0; s < n_seqs_; ++s) {
    const SequenceView* sv = seqs[s];
    for (size_t b = 0; b < sv->block_table.size(); ++b) {
      if (sv->block_table[b] >= static_cast<size_t>(cfg_.num_blocks)) return false;
      block_tables_[static_cast<size_t>(s) * max_blocks + b] =
          static_cast<int32_t>(sv->block_table[b]);
    }
    lens[s] = static_cast<int64_t>(sv->seq_len);
    cached[s] = static_cast<int64_t>(sv->num_cached_tokens);
    max_context_ = std::max<int>(max_context_, static_cast<int>(sv->seq_len));
  }
  context_lens_.assign(n_seqs_, 0);
  q_starts_.assign(n_seqs_, 0);
  cu_q_.assign(n_seqs_ + 1, 0);
  if (is_prefill) {
    int64_t total = 0;
    for (int s = 0; s < n_seqs_; ++s) total += std::max<int64_t>(1, lens[s] - cached[s]);
    positions_.assign(total, 0);
    slots_.assign(total, 0);
    if (nvattn_plan_prefill(n_seqs_, lens.data(), cached.data(), block_tables_.data(),
                            max_blocks_, cfg_.block_size, static_cast<int>(total), cu_q_.data(),
                            q_starts_.data(), context_lens_.data(), positions_.data(),
                            slots_.data()) != NVATTN_OK)
      return false;
    n_tokens_ = cu_q_[n_seqs_];
    max_q_len_ = 0;
    for (int s = 0; s < n_seqs_; ++s) max_q_len_ = std::max(max_q_len_, cu_q_[s + 1] - cu_q_[s]);
  } else {
    positions_.assign(n_seqs_, 0);
    slots_.assign(n_seqs_, 0);
    if (nvattn_plan_decode(n_seqs_, lens.data(), block_tables_.data(), max_blocks_,
                           cfg_.block_size, context_lens_.data(), positions_.data(),
                           slots_.data()) != NVATTN_OK)
      return false;
    n_tokens_ = n_seqs_;
    max_q_len_ = 1;
    for (int s = 0; s <= n_seqs_; ++s) cu_q_[s] = s;
    for (int s = 0; s < n_seqs_; ++s) q_starts_[s] = static_cast<int32_t>(lens[s] - 1);
  }
  if (max_context_ > cfg_.max_context) return false;
  if (!Reserve(n_tokens_, n_seqs_, max_blocks)) return false;
  auto up = [&](int32_t* dst, const std::vector<int32_t>& src) {
    return cudaMemcpyAsync(dst, src.data(), src.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                           stream) == cudaSuccess;
  };
  return up(d_positions_, positions_) && up(d_slots_, slots_) &&
         up(d_block_tables_, block_tables_) && up(d_context_lens_, context_lens_) &&
         up(d_cu_q_, cu_q_) && up(d_q_starts_, q_starts_);
}

bool AttentionRunner::RunAttentionLayer(int layer, float* q, const float* k, const float* v,
                                        const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                        uint16_t* k_cache, uint16_t* v_cache, float* out,
                                        cudaStream_t stream) {
  auto* s = reinterpret_cast<nvattn_stream_t>(stream);
  if (is_prefill_) {
    if (nvattn_kv_store_qk_norm_rope(handle_, layer, n_tokens_, q, k, v, q_norm_w, k_norm_w,
                                     d_positions_, d_slots_, d_q_bf16_, NVATTN_DTYPE_BF16,
                                     k_cache, v_cache, s) != NVATTN_OK)
      return false;
    return nvattn_paged_prefill(handle_, layer, n_seqs_, n_tokens_, d_q_bf16_, d_cu_q_,
                                d_q_starts_, d_context_lens_, d_block_tables_, max_blocks_,
                                max_q_len_, k_cache, v_cache, out, s) == NVATTN_OK;
  }
  if (nvattn_kv_store_qk_norm_rope(handle_, layer, n_tokens_, q, k, v, q_norm_w, k_norm_w,
                                   d_positions_, d_slots_, q, NVATTN_DTYPE_F32, k_cache, v_cache,
                                   s) != NVATTN_OK)
    return false;
  return nvattn_paged_decode(handle_, layer, n_seqs_, q, k_cache, v_cache, d_block_tables_,
                             max_blocks_, d_context_lens_, max_context_, out, s) == NVATTN_OK;
}

}  // namespace nvattn_host
