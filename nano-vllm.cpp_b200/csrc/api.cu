// api.cu -- the extern "C" surface of libnvattn (include/nvattn.h): handle
// lifetime, argument validation, device selection, TMA descriptor cache and
// the host-side planning functions that mirror ModelRunner::PrepareInputs.
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "internal.h"

namespace {

// Makes the handle's device current for the duration of a call and restores
// the caller's device afterwards.
class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    ok_ = cudaGetDevice(&prev_) == cudaSuccess;
    if (ok_ && prev_ != dev) ok_ = cudaSetDevice(dev) == cudaSuccess;
    switched_ = ok_ && prev_ != dev;
  }
  ~DeviceGuard() {
    if (switched_) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }

 private:
  int prev_ = 0;
  bool ok_ = false;
  bool switched_ = false;
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

namespace nvattn {

nvattn_status encode_tensor_map_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1,
                                   uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                                   uint32_t box0, uint32_t box1, uint32_t box2, int swizzle,
                                   CUtensorMapDataType dtype) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return NVATTN_ERR_CUDA;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {box0, box1, box2};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, (CUtensorMapSwizzle)swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NVATTN_OK : NVATTN_ERR_CUDA;
}

nvattn_status get_cache_tensor_map(nvattn_handle* h, const void* base, int box_d, int box_rows,
                                   int swizzle, CUtensorMap* out) {
  for (int i = 0; i < h->n_maps; ++i) {
    const NvattnTensorMapEntry& e = h->maps[i];
    if (e.base == base && e.box_d == box_d && e.box_rows == box_rows && e.swizzle == swizzle) {
      *out = e.map;
      return NVATTN_OK;
    }
  }
  NvattnTensorMapEntry e;
  e.base = base;
  e.box_d = box_d;
  e.box_rows = box_rows;
  e.swizzle = swizzle;
  const uint64_t D = (uint64_t)h->cfg.head_dim, Hkv = (uint64_t)h->cfg.n_kv_heads;
  nvattn_status st = encode_tensor_map_3d(&e.map, base, D, Hkv,
                                          (uint64_t)h->cfg.n_layer * (uint64_t)h->n_slots, D * 2,
                                          Hkv * D * 2, (uint32_t)box_d, 1, (uint32_t)box_rows,
                                          swizzle);
  if (st != NVATTN_OK) return st;
  int slot;
  if (h->n_maps < nvattn_handle::kMapCacheSize) {
    slot = h->n_maps++;
  } else {
    slot = h->next_map;
    h->next_map = (h->next_map + 1) % nvattn_handle::kMapCacheSize;
  }
  h->maps[slot] = e;
  *out = e.map;
  return NVATTN_OK;
}

}  // namespace nvattn

extern "C" {

void nvattn_version(int* major, int* minor) {
  if (major) *major = NVATTN_VERSION_MAJOR;
  if (minor) *minor = NVATTN_VERSION_MINOR;
}

const char* nvattn_status_string(nvattn_status s) {
  switch (s) {
    case NVATTN_OK: return "ok";
    case NVATTN_ERR_INVALID_ARG: return "invalid argument";
    case NVATTN_ERR_OUT_OF_RANGE: return "block id, slot or position out of range";
    case NVATTN_ERR_CUDA: return "CUDA error";
    case NVATTN_ERR_TIMEOUT: return "bounded device wait timed out";
    case NVATTN_ERR_UNSUPPORTED: return "unsupported shape";
    case NVATTN_ERR_NO_MEMORY: return "out of device memory";
    case NVATTN_ERR_SCRATCH_LIMIT:
      return "split-KV partials exceed the 32 MiB static scratch of nvattn_paged_decode_noalloc";
  }
  return "unknown status";
}

void nvattn_config_init_qwen3(nvattn_config* c) {
  if (c == nullptr) return;
  std::memset(c, 0, sizeof(*c));
  c->n_layer = 28;
  c->n_q_heads = 16;
  c->n_kv_heads = 8;
  c->head_dim = 128;
  c->block_size = 256;
  c->num_blocks = 160;  // ceil(40960 / 256), llm_engine.cpp:45-49
  c->rms_eps = 1e-6f;
  c->rope_theta = 1000000.0f;
  c->rope_freq_scale = 1.0f;
  c->rope_ext_factor = 1.0f;
  c->rope_attn_factor = 1.0f;
  c->rope_beta_fast = 32.0f;
  c->rope_beta_slow = 1.0f;
  c->rope_n_ctx_orig = 40960;
  c->scale = 1.0f / sqrtf(128.0f);
  c->max_position = 40960;
  c->max_seqs = 512;       // Config::max_num_seqs
  c->max_context = 40960;  // Qwen3Hparams::n_ctx
  c->device = 0;
}

nvattn_status nvattn_create(const nvattn_config* cfg, nvattn_handle** out) {
  if (cfg == nullptr || out == nullptr) return NVATTN_ERR_INVALID_ARG;
  *out = nullptr;
  const nvattn_config& c = *cfg;
  if (c.n_layer <= 0 || c.n_q_heads <= 0 || c.n_kv_heads <= 0 || c.num_blocks <= 0 ||
      c.max_position <= 0 || c.max_seqs <= 0 || c.max_context <= 0 || c.block_size <= 0 ||
      c.n_q_heads % c.n_kv_heads != 0 || !(c.scale > 0.0f) || !(c.rope_theta > 0.0f))
    return NVATTN_ERR_INVALID_ARG;
  const int G = c.n_q_heads / c.n_kv_heads;
  if (c.head_dim != 128 || c.block_size % 128 != 0 || c.block_size > 1024 ||
      !(G == 1 || G == 2 || G == 4 || G == 8))
    return NVATTN_ERR_UNSUPPORTED;
  const long long n_slots = c.num_blocks * (long long)c.block_size;
  if ((long long)c.n_layer * n_slots >= (1LL << 31)) return NVATTN_ERR_UNSUPPORTED;

  DeviceGuard guard(c.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;

  nvattn_handle* h = new (std::nothrow) nvattn_handle();
  if (h == nullptr) return NVATTN_ERR_NO_MEMORY;
  h->cfg = c;
  h->n_slots = n_slots;
  if (cudaDeviceGetAttribute(&h->sm_count, cudaDevAttrMultiProcessorCount, c.device) !=
      cudaSuccess) {
    delete h;
    return NVATTN_ERR_CUDA;
  }

  nvattn_status st = NVATTN_OK;
  {
    std::vector<float> table((size_t)c.max_position * c.head_dim);
    nvattn::build_rope_table(c, c.max_position, table.data());
    if (cudaMalloc(&h->rope_table_dev, table.size() * sizeof(float)) != cudaSuccess)
      st = NVATTN_ERR_NO_MEMORY;
    else if (cudaMemcpy(h->rope_table_dev, table.data(), table.size() * sizeof(float),
                        cudaMemcpyHostToDevice) != cudaSuccess)
      st = NVATTN_ERR_CUDA;
  }
  if (st == NVATTN_OK) {
    if (cudaMalloc(&h->status_dev, sizeof(nvattn::DeviceStatus)) != cudaSuccess)
      st = NVATTN_ERR_NO_MEMORY;
    else if (cudaMemset(h->status_dev, 0, sizeof(nvattn::DeviceStatus)) != cudaSuccess)
      st = NVATTN_ERR_CUDA;
  }
  if (st == NVATTN_OK) {
    if (cudaMalloc(&h->prefill_sched_dev, 2 * sizeof(int)) != cudaSuccess)
      st = NVATTN_ERR_NO_MEMORY;
    else if (cudaMemset(h->prefill_sched_dev, 0, 2 * sizeof(int)) != cudaSuccess)
      st = NVATTN_ERR_CUDA;
  }
  if (st == NVATTN_OK) {
    // Split-KV workspace: at most 64 splits per (sequence, kv head).
    long long splits = (c.max_context + c.block_size - 1) / c.block_size;
    h->max_splits = (int)(splits < 64 ? splits : 64);
    const size_t rows = (size_t)c.max_seqs * c.n_q_heads * h->max_splits;
    const size_t tickets = (size_t)c.max_seqs * c.n_kv_heads * sizeof(int);
    const size_t q_rows = (size_t)c.max_seqs * c.n_q_heads;
    if (cudaMalloc(&h->ws_o, rows * c.head_dim * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&h->ws_ml, rows * 2 * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&h->decode_tickets, tickets) != cudaSuccess ||
        cudaMalloc(&h->q_step, q_rows * c.head_dim * sizeof(float)) != cudaSuccess)
      st = NVATTN_ERR_NO_MEMORY;
    else if (cudaMemset(h->decode_tickets, 0, tickets) != cudaSuccess)
      st = NVATTN_ERR_CUDA;
  }
  if (st != NVATTN_OK) {
    cudaGetLastError();  // clear a sticky allocation error
    nvattn_destroy(h);
    return st;
  }
  *out = h;
  return NVATTN_OK;
}

nvattn_status nvattn_destroy(nvattn_handle* h) {
  if (h == nullptr) return NVATTN_OK;
  DeviceGuard guard(h->cfg.device);
  if (h->rope_table_dev) cudaFree(h->rope_table_dev);
  if (h->status_dev) cudaFree(h->status_dev);
  if (h->prefill_sched_dev) cudaFree(h->prefill_sched_dev);
  if (h->ws_o) cudaFree(h->ws_o);
  if (h->ws_ml) cudaFree(h->ws_ml);
  if (h->decode_tickets) cudaFree(h->decode_tickets);
  if (h->q_step) cudaFree(h->q_step);
  for (int p = 0; p < h->g_ranks; ++p)
    if (p != h->g_rank && h->g_peer[p] != nullptr) cudaIpcCloseMemHandle(h->g_peer[p]);
  if (h->g_own) cudaFree(h->g_own);
  if (h->samp_nib) cudaFree(h->samp_nib);
  if (h->samp_exact) cudaFree(h->samp_exact);
  if (h->samp_part) cudaFree(h->samp_part);
  delete h;
  return NVATTN_OK;
}

nvattn_status nvattn_get_error(nvattn_handle* h, int64_t* detail) {
  if (detail) *detail = 0;
  if (h == nullptr) return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return NVATTN_ERR_CUDA;
  nvattn::DeviceStatus st;
  if (cudaMemcpy(&st, h->status_dev, sizeof(st), cudaMemcpyDeviceToHost) != cudaSuccess)
    return NVATTN_ERR_CUDA;
  if (st.code != 0 && cudaMemset(h->status_dev, 0, sizeof(st)) != cudaSuccess)
    return NVATTN_ERR_CUDA;
  // A launch cut short by a timeout may leave split tickets taken (and, in
  // the worst case, a work counter short of its reset).
  if (st.code == NVATTN_ERR_TIMEOUT &&
      (cudaMemset(h->decode_tickets, 0,
                  (size_t)h->cfg.max_seqs * h->cfg.n_kv_heads * sizeof(int)) != cudaSuccess ||
       cudaMemset(h->prefill_sched_dev, 0, 2 * sizeof(int)) != cudaSuccess))
    return NVATTN_ERR_CUDA;
  // ...and ends the peer-memory gather: the ranks' step counters and this
  // rank's count of final-row CTAs no longer agree, so a later step could
  // not tell when every rank's rows have arrived.
  if (st.code == NVATTN_ERR_TIMEOUT) h->g_connected = false;
  if (detail) *detail = st.detail;
  return (nvattn_status)st.code;
}

nvattn_status nvattn_plan_prefill(int n_seqs, const int64_t* seq_lens, const int64_t* num_cached,
                                  const int32_t* block_tables, int max_blocks, int block_size,
                                  int max_tokens, int32_t* cu_q_lens, int32_t* q_starts,
                                  int32_t* context_lens, int32_t* positions,
                                  int32_t* slot_mapping) {
  if (n_seqs < 0 || max_blocks <= 0 || block_size <= 0 || max_tokens < 0) return NVATTN_ERR_INVALID_ARG;
  if (n_seqs > 0 && (!seq_lens || !num_cached || !block_tables || !cu_q_lens || !q_starts ||
                     !context_lens || !positions || !slot_mapping))
    return NVATTN_ERR_INVALID_ARG;
  if (cu_q_lens) cu_q_lens[0] = 0;
  long long off = 0;
  for (int s = 0; s < n_seqs; ++s) {
    const long long len = seq_lens[s];
    long long start = num_cached[s];
    if (len <= 0 || start < 0 || start > len || len > 0x7fffffffLL) return NVATTN_ERR_INVALID_ARG;
    // A prompt whose every block hit the prefix cache still needs its last
    // token computed (the reference would feed zero tokens and sample from
    // index -1, model_runner.cpp:158-160,182).
    if (start == len) start = len - 1;
    if ((len + block_size - 1) / block_size > max_blocks) return NVATTN_ERR_INVALID_ARG;
    if (off + (len - start) > max_tokens) return NVATTN_ERR_INVALID_ARG;
    q_starts[s] = (int32_t)start;
    context_lens[s] = (int32_t)len;
    for (long long pos = start; pos < len; ++pos, ++off) {
      const int32_t bid = block_tables[(long long)s * max_blocks + pos / block_size];
      if (bid < 0) return NVATTN_ERR_OUT_OF_RANGE;
      positions[off] = (int32_t)pos;
      slot_mapping[off] = (int32_t)((long long)bid * block_size + pos % block_size);
    }
    cu_q_lens[s + 1] = (int32_t)off;
  }
  return NVATTN_OK;
}

nvattn_status nvattn_plan_decode(int n_seqs, const int64_t* seq_lens, const int32_t* block_tables,
                                 int max_blocks, int block_size, int32_t* context_lens,
                                 int32_t* positions, int32_t* slot_mapping) {
  if (n_seqs < 0 || max_blocks <= 0 || block_size <= 0) return NVATTN_ERR_INVALID_ARG;
  if (n_seqs > 0 && (!seq_lens || !block_tables || !context_lens || !positions || !slot_mapping))
    return NVATTN_ERR_INVALID_ARG;
  for (int s = 0; s < n_seqs; ++s) {
    const long long len = seq_lens[s];
    if (len <= 0 || len > 0x7fffffffLL) return NVATTN_ERR_INVALID_ARG;
    const long long pos = len - 1;
    if (pos / block_size >= max_blocks) return NVATTN_ERR_INVALID_ARG;
    const int32_t bid = block_tables[(long long)s * max_blocks + pos / block_size];
    if (bid < 0) return NVATTN_ERR_OUT_OF_RANGE;
    context_lens[s] = (int32_t)len;
    positions[s] = (int32_t)pos;
    slot_mapping[s] = (int32_t)((long long)bid * block_size + pos % block_size);
  }
  return NVATTN_OK;
}

nvattn_status nvattn_plan_prefill_device(nvattn_handle* h, int n_seqs,
                                         const int64_t* seq_lens_dev,
                                         const int64_t* num_cached_dev,
                                         const int32_t* block_tables_dev, int max_blocks,
                                         int max_tokens, int32_t* cu_q_lens_dev,
                                         int32_t* q_starts_dev, int32_t* context_lens_dev,
                                         int32_t* positions_dev, int32_t* slot_mapping_dev,
                                         nvattn_stream_t stream) {
  if (h == nullptr || n_seqs < 0 || max_blocks <= 0 || max_tokens < 0)
    return NVATTN_ERR_INVALID_ARG;
  if (cu_q_lens_dev == nullptr) return NVATTN_ERR_INVALID_ARG;
  if (n_seqs > 0 && (!seq_lens_dev || !num_cached_dev || !block_tables_dev || !q_starts_dev ||
                     !context_lens_dev || !positions_dev || !slot_mapping_dev))
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  return nvattn::launch_plan_prefill(h, n_seqs, seq_lens_dev, num_cached_dev, block_tables_dev,
                                     max_blocks, max_tokens, cu_q_lens_dev, q_starts_dev,
                                     context_lens_dev, positions_dev, slot_mapping_dev,
                                     reinterpret_cast<cudaStream_t>(stream));
}

nvattn_status nvattn_plan_decode_device(nvattn_handle* h, int n_seqs,
                                        const int64_t* seq_lens_dev,
                                        const int32_t* block_tables_dev, int max_blocks,
                                        int32_t* context_lens_dev, int32_t* positions_dev,
                                        int32_t* slot_mapping_dev, nvattn_stream_t stream) {
  if (h == nullptr || n_seqs < 0 || max_blocks <= 0) return NVATTN_ERR_INVALID_ARG;
  if (n_seqs == 0) return NVATTN_OK;
  if (!seq_lens_dev || !block_tables_dev || !context_lens_dev || !positions_dev ||
      !slot_mapping_dev)
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  return nvattn::launch_plan_decode(h, n_seqs, seq_lens_dev, block_tables_dev, max_blocks,
                                    context_lens_dev, positions_dev, slot_mapping_dev,
                                    reinterpret_cast<cudaStream_t>(stream));
}

nvattn_status nvattn_sample(nvattn_handle* h, int n_seqs, int n_vocab, const float* logits_dev,
                            int64_t row_stride, const float* temperatures_dev,
                            const float* penalties_dev, const int32_t* history_dev,
                            const int64_t* history_offsets_dev, const float* uniforms_dev,
                            int32_t* tokens_dev, nvattn_stream_t stream) {
  if (h == nullptr || n_seqs < 0 || n_seqs > h->cfg.max_seqs || n_vocab <= 0 ||
      row_stride < n_vocab)
    return NVATTN_ERR_INVALID_ARG;
  if (n_vocab > nvattn::sample_max_vocab()) return NVATTN_ERR_UNSUPPORTED;
  if (n_seqs == 0) return NVATTN_OK;
  if (!logits_dev || !temperatures_dev || !penalties_dev || !uniforms_dev || !tokens_dev ||
      (history_dev == nullptr) != (history_offsets_dev == nullptr))
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (n_vocab > h->samp_cap) {
    // Workspace for this vocabulary: allocation cannot happen inside a graph
    // capture, so the first call per vocabulary size must run eagerly.
    cudaStreamCaptureStatus cap_status = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap_status) != cudaSuccess) return NVATTN_ERR_CUDA;
    if (cap_status != cudaStreamCaptureStatusNone) return NVATTN_ERR_UNSUPPORTED;
    if (cudaStreamSynchronize(st) != cudaSuccess) return NVATTN_ERR_CUDA;
    if (h->samp_nib) cudaFree(h->samp_nib);
    if (h->samp_exact) cudaFree(h->samp_exact);
    if (h->samp_part) cudaFree(h->samp_part);
    h->samp_nib = nullptr;
    h->samp_exact = nullptr;
    h->samp_part = nullptr;
    h->samp_cap = 0;
    const long long g = nvattn::sample_vocab_granule();
    const long long cap = ((long long)n_vocab + g - 1) / g * g;
    const size_t seqs = (size_t)h->cfg.max_seqs;
    if (nvattn::sample_prepare_device() != NVATTN_OK) return NVATTN_ERR_CUDA;
    if (cudaMalloc(&h->samp_nib, seqs * cap / 2) != cudaSuccess ||
        cudaMalloc(&h->samp_exact, seqs * cap * 4) != cudaSuccess ||
        cudaMalloc(&h->samp_part, seqs * nvattn::sample_partial_bytes()) != cudaSuccess) {
      cudaGetLastError();
      return NVATTN_ERR_NO_MEMORY;
    }
    h->samp_cap = cap;
  }
  return nvattn::launch_sample(h, n_seqs, n_vocab, logits_dev, row_stride, temperatures_dev,
                               penalties_dev, history_dev, history_offsets_dev, uniforms_dev,
                               tokens_dev, st);
}

}  // extern "C"

namespace {

nvattn_status kv_store_common(nvattn_handle* h, int layer, int n_tokens, const float* q_dev,
                              const float* k_dev, const float* v_dev,
                              const uint16_t* q_norm_w_dev, const uint16_t* k_norm_w_dev,
                              const int32_t* positions_dev, const int32_t* slot_mapping_dev,
                              void* q_out_dev, nvattn_dtype q_out_dtype, uint16_t* k_cache_dev,
                              uint16_t* v_cache_dev, uint16_t* k_rows_dev, uint16_t* v_rows_dev,
                              nvattn_stream_t stream) {
  if (h == nullptr || layer < 0 || layer >= h->cfg.n_layer || n_tokens < 0)
    return NVATTN_ERR_INVALID_ARG;
  if (q_out_dtype != NVATTN_DTYPE_F32 && q_out_dtype != NVATTN_DTYPE_BF16 &&
      q_out_dtype != NVATTN_DTYPE_F16)
    return NVATTN_ERR_INVALID_ARG;
  if (n_tokens == 0) return NVATTN_OK;
  const void* ptrs[] = {q_dev, k_dev, v_dev, q_norm_w_dev, k_norm_w_dev, q_out_dev,
                        k_cache_dev, v_cache_dev};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return NVATTN_ERR_INVALID_ARG;
  if (positions_dev == nullptr || slot_mapping_dev == nullptr) return NVATTN_ERR_INVALID_ARG;
  if ((k_rows_dev != nullptr && !aligned16(k_rows_dev)) ||
      (v_rows_dev != nullptr && !aligned16(v_rows_dev)))
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  return nvattn::launch_kv_store(h, layer, n_tokens, q_dev, k_dev, v_dev, q_norm_w_dev,
                                 k_norm_w_dev, positions_dev, slot_mapping_dev, q_out_dev,
                                 q_out_dtype, k_cache_dev, v_cache_dev, k_rows_dev, v_rows_dev,
                                 reinterpret_cast<cudaStream_t>(stream));
}

nvattn_status prefill_common(nvattn_handle* h, int layer, int n_seqs, int n_tokens,
                             const uint16_t* q_dev, const int32_t* cu_q_lens_dev,
                             const int32_t* q_starts_dev, const int32_t* context_lens_dev,
                             const int32_t* block_tables_dev, int max_blocks, int max_q_len,
                             const uint16_t* k_cache_dev, const uint16_t* v_cache_dev,
                             const uint16_t* k_rows_dev, const uint16_t* v_rows_dev,
                             float* out_dev, nvattn_stream_t stream) {
  if (h == nullptr || layer < 0 || layer >= h->cfg.n_layer || n_seqs < 0 ||
      n_seqs > h->cfg.max_seqs || n_tokens < 0 || max_blocks <= 0 || max_q_len < 0)
    return NVATTN_ERR_INVALID_ARG;
  if (n_seqs == 0 || n_tokens == 0) return NVATTN_OK;
  if (!q_dev || !cu_q_lens_dev || !q_starts_dev || !context_lens_dev || !block_tables_dev ||
      !k_cache_dev || !v_cache_dev || !out_dev || !aligned16(q_dev) || !aligned16(out_dev) ||
      !aligned16(k_cache_dev) || !aligned16(v_cache_dev))
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  return nvattn::launch_paged_prefill(h, layer, n_seqs, n_tokens, q_dev, cu_q_lens_dev,
                                      q_starts_dev, context_lens_dev, block_tables_dev,
                                      max_blocks, max_q_len, k_cache_dev, v_cache_dev,
                                      k_rows_dev, v_rows_dev, out_dev,
                                      reinterpret_cast<cudaStream_t>(stream));
}

}  // namespace

extern "C" {

nvattn_status nvattn_kv_store_qk_norm_rope(nvattn_handle* h, int layer, int n_tokens,
                                           const float* q_dev, const float* k_dev,
                                           const float* v_dev, const uint16_t* q_norm_w_dev,
                                           const uint16_t* k_norm_w_dev,
                                           const int32_t* positions_dev,
                                           const int32_t* slot_mapping_dev, void* q_out_dev,
                                           nvattn_dtype q_out_dtype, uint16_t* k_cache_dev,
                                           uint16_t* v_cache_dev, nvattn_stream_t stream) {
  return kv_store_common(h, layer, n_tokens, q_dev, k_dev, v_dev, q_norm_w_dev, k_norm_w_dev,
                         positions_dev, slot_mapping_dev, q_out_dev, q_out_dtype, k_cache_dev,
                         v_cache_dev, nullptr, nullptr, stream);
}

nvattn_status nvattn_kv_store_qk_norm_rope_rows(
    nvattn_handle* h, int layer, int n_tokens, const float* q_dev, const float* k_dev,
    const float* v_dev, const uint16_t* q_norm_w_dev, const uint16_t* k_norm_w_dev,
    const int32_t* positions_dev, const int32_t* slot_mapping_dev, void* q_out_dev,
    nvattn_dtype q_out_dtype, uint16_t* k_cache_dev, uint16_t* v_cache_dev,
    uint16_t* k_rows_f16_dev, uint16_t* v_rows_f16_dev, nvattn_stream_t stream) {
  if (k_rows_f16_dev == nullptr || v_rows_f16_dev == nullptr) return NVATTN_ERR_INVALID_ARG;
  return kv_store_common(h, layer, n_tokens, q_dev, k_dev, v_dev, q_norm_w_dev, k_norm_w_dev,
                         positions_dev, slot_mapping_dev, q_out_dev, q_out_dtype, k_cache_dev,
                         v_cache_dev, k_rows_f16_dev, v_rows_f16_dev, stream);
}

nvattn_status nvattn_paged_decode(nvattn_handle* h, int layer, int n_seqs, const float* q_dev,
                                  const uint16_t* k_cache_dev, const uint16_t* v_cache_dev,
                                  const int32_t* block_tables_dev, int max_blocks,
                                  const int32_t* context_lens_dev, int max_context_len,
                                  float* out_dev, nvattn_stream_t stream) {
  if (h == nullptr || layer < 0 || layer >= h->cfg.n_layer || n_seqs < 0 ||
      n_seqs > h->cfg.max_seqs || n_seqs > nvattn::kMaxDecodeSeqs || max_blocks <= 0 ||
      max_context_len < 0 || max_context_len > h->cfg.max_context ||
      (long long)max_context_len > (long long)max_blocks * h->cfg.block_size)
    return NVATTN_ERR_INVALID_ARG;
  if (n_seqs == 0) return NVATTN_OK;
  if (!q_dev || !k_cache_dev || !v_cache_dev || !block_tables_dev || !context_lens_dev ||
      !out_dev || !aligned16(q_dev) || !aligned16(out_dev) || !aligned16(k_cache_dev) ||
      !aligned16(v_cache_dev))
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  return nvattn::launch_paged_decode(h, layer, n_seqs, q_dev, k_cache_dev, v_cache_dev,
                                     block_tables_dev, max_blocks, context_lens_dev,
                                     max_context_len, out_dev,
                                     reinterpret_cast<cudaStream_t>(stream));
}

nvattn_status nvattn_paged_decode_step(nvattn_handle* h, int layer, int n_seqs, const float* q_dev,
                                       const float* k_dev, const float* v_dev,
                                       const uint16_t* q_norm_w_dev,
                                       const uint16_t* k_norm_w_dev,
                                       const int32_t* positions_dev,
                                       const int32_t* slot_mapping_dev, uint16_t* k_cache_dev,
                                       uint16_t* v_cache_dev, const int32_t* block_tables_dev,
                                       int max_blocks, const int32_t* context_lens_dev,
                                       int max_context_len, float* out_dev,
                                       nvattn_stream_t stream) {
  if (h == nullptr || layer < 0 || layer >= h->cfg.n_layer || n_seqs < 0 ||
      n_seqs > h->cfg.max_seqs || n_seqs > nvattn::kMaxDecodeSeqs || max_blocks <= 0 ||
      max_context_len < 0 || max_context_len > h->cfg.max_context ||
      (long long)max_context_len > (long long)max_blocks * h->cfg.block_size)
    return NVATTN_ERR_INVALID_ARG;
  if (n_seqs == 0) return NVATTN_OK;
  const void* ptrs[] = {q_dev, k_dev, v_dev, q_norm_w_dev, k_norm_w_dev, k_cache_dev,
                        v_cache_dev, out_dev};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return NVATTN_ERR_INVALID_ARG;
  if (positions_dev == nullptr || slot_mapping_dev == nullptr || block_tables_dev == nullptr ||
      context_lens_dev == nullptr)
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  return nvattn::launch_paged_decode_step(
      h, layer, n_seqs, q_dev, k_dev, v_dev, q_norm_w_dev, k_norm_w_dev, positions_dev,
      slot_mapping_dev, k_cache_dev, v_cache_dev, block_tables_dev, max_blocks,
      context_lens_dev, max_context_len, out_dev, reinterpret_cast<cudaStream_t>(stream));
}

nvattn_status nvattn_paged_decode_step_launches(const nvattn_handle* h, int n_seqs,
                                                int max_context_len, int* launches) {
  if (h == nullptr || launches == nullptr || n_seqs < 0 || n_seqs > h->cfg.max_seqs ||
      max_context_len < 0 || max_context_len > h->cfg.max_context)
    return NVATTN_ERR_INVALID_ARG;
  *launches = n_seqs == 0 ? 0 : nvattn::decode_step_launches(h, n_seqs, max_context_len);
  return NVATTN_OK;
}

namespace {
// What a rank's exported handle carries after the CUDA IPC handle: the shape
// every rank's buffer must share (peer stores land at offsets computed from
// this rank's own shape).
struct GatherMeta {
  long long slice;
  long long flag_off;
  int n_ranks;
  int rank;
};
static_assert(sizeof(cudaIpcMemHandle_t) + sizeof(GatherMeta) <= NVATTN_IPC_HANDLE_BYTES,
              "IPC handle size");
}  // namespace

nvattn_status nvattn_gather_init(nvattn_handle* h, int n_ranks, int rank, void* ipc_handle_out) {
  if (h == nullptr || ipc_handle_out == nullptr || n_ranks < 1 ||
      n_ranks > nvattn_handle::kMaxGatherRanks || rank < 0 || rank >= n_ranks ||
      h->g_own != nullptr)
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  const long long slice = (long long)h->cfg.max_seqs * h->cfg.n_q_heads * h->cfg.head_dim;
  const size_t flag_off = ((size_t)2 * n_ranks * slice * sizeof(float) + 255) / 256 * 256;
  char* own = nullptr;
  if (cudaMalloc(&own, flag_off + 256) != cudaSuccess) {
    cudaGetLastError();
    return NVATTN_ERR_NO_MEMORY;
  }
  cudaIpcMemHandle_t ipc;
  if (cudaMemset(own + flag_off, 0, 256) != cudaSuccess ||
      cudaIpcGetMemHandle(&ipc, own) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(own);
    return NVATTN_ERR_CUDA;
  }
  std::memset(ipc_handle_out, 0, NVATTN_IPC_HANDLE_BYTES);
  std::memcpy(ipc_handle_out, &ipc, sizeof(ipc));
  const GatherMeta meta{slice, (long long)flag_off, n_ranks, rank};
  std::memcpy(static_cast<char*>(ipc_handle_out) + sizeof(ipc), &meta, sizeof(meta));
  h->g_own = own;
  h->g_ranks = n_ranks;
  h->g_rank = rank;
  h->g_slice = slice;
  h->g_flag_off = flag_off;
  h->g_peer[rank] = own;
  h->g_steps = 0;
  h->g_done_total = 0;
  return NVATTN_OK;
}

nvattn_status nvattn_gather_connect(nvattn_handle* h, const void* ipc_handles) {
  if (h == nullptr || ipc_handles == nullptr || h->g_own == nullptr || h->g_connected)
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  const char* all = static_cast<const char*>(ipc_handles);
  for (int p = 0; p < h->g_ranks; ++p) {
    GatherMeta meta;
    std::memcpy(&meta, all + (size_t)p * NVATTN_IPC_HANDLE_BYTES + sizeof(cudaIpcMemHandle_t),
                sizeof(meta));
    if (meta.slice != h->g_slice || meta.flag_off != (long long)h->g_flag_off ||
        meta.n_ranks != h->g_ranks || meta.rank != p)
      return NVATTN_ERR_INVALID_ARG;
  }
  for (int p = 0; p < h->g_ranks; ++p) {
    if (p == h->g_rank) continue;
    cudaIpcMemHandle_t ipc;
    std::memcpy(&ipc, all + (size_t)p * NVATTN_IPC_HANDLE_BYTES, sizeof(ipc));
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, ipc, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      for (int q = 0; q < p; ++q)
        if (q != h->g_rank && h->g_peer[q] != nullptr) {
          cudaIpcCloseMemHandle(h->g_peer[q]);
          h->g_peer[q] = nullptr;
        }
      return NVATTN_ERR_CUDA;
    }
    h->g_peer[p] = static_cast<char*>(ptr);
  }
  h->g_connected = true;
  return NVATTN_OK;
}

nvattn_status nvattn_paged_decode_step_gather(
    nvattn_handle* h, int layer, int n_seqs, const float* q_dev, const float* k_dev,
    const float* v_dev, const uint16_t* q_norm_w_dev, const uint16_t* k_norm_w_dev,
    const int32_t* positions_dev, const int32_t* slot_mapping_dev, uint16_t* k_cache_dev,
    uint16_t* v_cache_dev, const int32_t* block_tables_dev, int max_blocks,
    const int32_t* context_lens_dev, int max_context_len, float* out_dev,
    nvattn_stream_t stream) {
  if (h == nullptr || !h->g_connected || layer < 0 || layer >= h->cfg.n_layer || n_seqs < 0 ||
      n_seqs > h->cfg.max_seqs || n_seqs > nvattn::kMaxDecodeSeqs || max_blocks <= 0 ||
      max_context_len < 0 || max_context_len > h->cfg.max_context ||
      (long long)max_context_len > (long long)max_blocks * h->cfg.block_size)
    return NVATTN_ERR_INVALID_ARG;
  const void* ptrs[] = {q_dev, k_dev, v_dev, q_norm_w_dev, k_norm_w_dev, k_cache_dev,
                        v_cache_dev, out_dev};
  for (const void* p : ptrs)
    if (p == nullptr || !aligned16(p)) return NVATTN_ERR_INVALID_ARG;
  if (positions_dev == nullptr || slot_mapping_dev == nullptr || block_tables_dev == nullptr ||
      context_lens_dev == nullptr)
    return NVATTN_ERR_INVALID_ARG;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  return nvattn::launch_paged_decode_step_gather(
      h, layer, n_seqs, q_dev, k_dev, v_dev, q_norm_w_dev, k_norm_w_dev, positions_dev,
      slot_mapping_dev, k_cache_dev, v_cache_dev, block_tables_dev, max_blocks, context_lens_dev,
      max_context_len, out_dev, reinterpret_cast<cudaStream_t>(stream));
}

nvattn_status nvattn_gather_read(nvattn_handle* h, unsigned step, int n_seqs, float* out_dev,
                                 nvattn_stream_t stream) {
  if (h == nullptr || !h->g_connected || out_dev == nullptr || n_seqs < 0 ||
      n_seqs > h->cfg.max_seqs || h->g_steps == 0u || step != h->g_steps - 1u)
    return NVATTN_ERR_INVALID_ARG;
  if (n_seqs == 0) return NVATTN_OK;
  DeviceGuard guard(h->cfg.device);
  if (!guard.ok()) return NVATTN_ERR_CUDA;
  const size_t row_bytes = (size_t)n_seqs * h->cfg.n_q_heads * h->cfg.head_dim * sizeof(float);
  const float* src = reinterpret_cast<const float*>(h->g_own) +
                     (long long)(step & 1u) * h->g_ranks * h->g_slice;
  return cudaMemcpy2DAsync(out_dev, row_bytes, src, (size_t)h->g_slice * sizeof(float), row_bytes,
                           (size_t)h->g_ranks, cudaMemcpyDeviceToDevice,
                           reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
             ? NVATTN_OK
             : NVATTN_ERR_CUDA;
}

nvattn_status nvattn_paged_prefill(nvattn_handle* h, int layer, int n_seqs, int n_tokens,
                                   const uint16_t* q_dev, const int32_t* cu_q_lens_dev,
                                   const int32_t* q_starts_dev, const int32_t* context_lens_dev,
                                   const int32_t* block_tables_dev, int max_blocks, int max_q_len,
                                   const uint16_t* k_cache_dev, const uint16_t* v_cache_dev,
                                   float* out_dev, nvattn_stream_t stream) {
  return prefill_common(h, layer, n_seqs, n_tokens, q_dev, cu_q_lens_dev, q_starts_dev,
                        context_lens_dev, block_tables_dev, max_blocks, max_q_len, k_cache_dev,
                        v_cache_dev, nullptr, nullptr, out_dev, stream);
}

nvattn_status nvattn_paged_prefill_rows(nvattn_handle* h, int layer, int n_seqs, int n_tokens,
                                        const uint16_t* q_dev, const int32_t* cu_q_lens_dev,
                                        const int32_t* q_starts_dev,
                                        const int32_t* context_lens_dev,
                                        const int32_t* block_tables_dev, int max_blocks,
                                        int max_q_len, const uint16_t* k_cache_dev,
                                        const uint16_t* v_cache_dev,
                                        const uint16_t* k_rows_f16_dev,
                                        const uint16_t* v_rows_f16_dev, float* out_dev,
                                        nvattn_stream_t stream) {
  if (k_rows_f16_dev == nullptr || v_rows_f16_dev == nullptr || !aligned16(k_rows_f16_dev) ||
      !aligned16(v_rows_f16_dev))
    return NVATTN_ERR_INVALID_ARG;
  return prefill_common(h, layer, n_seqs, n_tokens, q_dev, cu_q_lens_dev, q_starts_dev,
                        context_lens_dev, block_tables_dev, max_blocks, max_q_len, k_cache_dev,
                        v_cache_dev, k_rows_f16_dev, v_rows_f16_dev, out_dev, stream);
}

}  // extern "C"
