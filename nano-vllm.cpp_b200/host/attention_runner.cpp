// attention_runner.cpp -- see attention_runner.h.
#include "attention_runner.h"

#include <algorithm>
#include <limits>
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

AttentionRunner::AttentionRunner(const nvattn_config& cfg, uint32_t sample_seed)
    : cfg_(cfg), rng_(sample_seed) {
  const nvattn_status st = nvattn_create(&cfg_, &handle_);
  if (st != NVATTN_OK)
    throw std::runtime_error(std::string("nvattn_create failed: ") + nvattn_status_string(st));
}

AttentionRunner::~AttentionRunner() {
  int32_t* bufs[] = {d_positions_, d_slots_, d_block_tables_, d_context_lens_, d_cu_q_,
                     d_q_starts_};
  for (int32_t* b : bufs)
    if (b) cudaFree(b);
  if (d_q_f16_) cudaFree(d_q_f16_);
  void* sbufs[] = {d_temps_, d_pens_, d_uniforms_, d_tokens_, d_hist_offsets_, d_history_};
  for (void* b : sbufs)
    if (b) cudaFree(b);
  nvattn_destroy(handle_);
}

std::vector<int> AttentionRunner::Sample(const float* logits_dev, int n_vocab,
                                         const std::vector<float>& temperatures,
                                         const std::vector<float>& penalties,
                                         const std::vector<std::vector<int32_t>>& histories,
                                         cudaStream_t stream) {
  const size_t n = temperatures.size();
  if (n == 0 || n > (size_t)cfg_.max_seqs || penalties.size() != n || histories.size() != n ||
      n_vocab <= 0)
    return {};
  // the draws, as the reference's loop takes them: one per sampled row
  uniforms_.assign(n, 0.0f);
  for (size_t s = 0; s < n; ++s)
    if (!(temperatures[s] < 1e-6f))
      uniforms_[s] = std::generate_canonical<float, std::numeric_limits<float>::digits>(rng_);
  std::vector<int64_t> offsets(n + 1, 0);
  for (size_t s = 0; s < n; ++s) offsets[s + 1] = offsets[s] + (int64_t)histories[s].size();
  std::vector<int32_t> ids;
  ids.reserve((size_t)offsets[n]);
  for (const auto& h : histories) ids.insert(ids.end(), h.begin(), h.end());

  bool ok = true;
  if (n > cap_sample_rows_) {
    ok = grow(&d_temps_, n) && grow(&d_pens_, n) && grow(&d_uniforms_, n) &&
         grow(&d_tokens_, n) && grow(&d_hist_offsets_, n + 1);
    cap_sample_rows_ = ok ? n : 0;
  }
  if (ok && ids.size() > cap_history_) {
    ok = grow(&d_history_, ids.size());
    cap_history_ = ok ? ids.size() : 0;
  }
  if (!ok) return {};
  auto up = [&](void* dst, const void* src, size_t bytes) {
    return bytes == 0 ||
           cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream) == cudaSuccess;
  };
  if (!up(d_temps_, temperatures.data(), n * sizeof(float)) ||
      !up(d_pens_, penalties.data(), n * sizeof(float)) ||
      !up(d_uniforms_, uniforms_.data(), n * sizeof(float)) ||
      !up(d_hist_offsets_, offsets.data(), (n + 1) * sizeof(int64_t)) ||
      !up(d_history_, ids.data(), ids.size() * sizeof(int32_t)))
    return {};
  if (nvattn_sample(handle_, (int)n, n_vocab, logits_dev, n_vocab, d_temps_, d_pens_,
                    ids.empty() ? nullptr : d_history_, ids.empty() ? nullptr : d_hist_offsets_,
                    d_uniforms_, d_tokens_, stream) != NVATTN_OK)
    return {};
  std::vector<int32_t> tok(n);
  if (cudaMemcpyAsync(tok.data(), d_tokens_, n * sizeof(int32_t), cudaMemcpyDeviceToHost,
                      stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return {};
  int64_t detail = 0;
  if (nvattn_get_error(handle_, &detail) != NVATTN_OK) return {};
  return std::vector<int>(tok.begin(), tok.end());
}

bool AttentionRunner::Reserve(size_t n_tokens, size_t n_seqs, size_t max_blocks) {
  bool ok = true;
  if (n_tokens > cap_tokens_) {
    const size_t cap = std::max(n_tokens, cap_tokens_ * 2);
    ok = ok && grow(&d_positions_, cap) && grow(&d_slots_, cap) &&
         grow(&d_q_f16_, cap * (size_t)cfg_.n_q_heads * cfg_.head_dim);
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

bool AttentionRunner::RunAttentionLayer(int layer, const float* q, const float* k, const float* v,
                                        const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                        uint16_t* k_cache, uint16_t* v_cache, float* out,
                                        cudaStream_t stream) {
  auto* s = reinterpret_cast<nvattn_stream_t>(stream);
  if (is_prefill_) {
    if (nvattn_kv_store_qk_norm_rope(handle_, layer, n_tokens_, q, k, v, q_norm_w, k_norm_w,
                                     d_positions_, d_slots_, d_q_f16_, NVATTN_DTYPE_F16,
                                     k_cache, v_cache, s) != NVATTN_OK)
      return false;
    return nvattn_paged_prefill(handle_, layer, n_seqs_, n_tokens_, d_q_f16_, d_cu_q_,
                                d_q_starts_, d_context_lens_, d_block_tables_, max_blocks_,
                                max_q_len_, k_cache, v_cache, out, s) == NVATTN_OK;
  }
  // one token per sequence: the store of the new token and the decode in one
  // call (one fused launch, or the two launches for large grids)
  return nvattn_paged_decode_step(handle_, layer, n_seqs_, q, k, v, q_norm_w, k_norm_w,
                                  d_positions_, d_slots_, k_cache, v_cache, d_block_tables_,
                                  max_blocks_, d_context_lens_, max_context_, out,
                                  s) == NVATTN_OK;
}

}  // namespace nvattn_host
