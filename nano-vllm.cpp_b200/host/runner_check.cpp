// runner_check.cpp -- drives the C++ host layer (AttentionRunner) through one
// prefill step and one decode step on the GPU, the way
// engine::ModelRunner::Run drives a layer (model_runner.cpp:25-136), and
// writes every input and output to a directory so a test can recompute them.
//
// Scenario (layer 1 of a 2-layer cache, Qwen3-0.6B attention heads 16/8):
//   prefill: sequence A, 300 new tokens; sequence B, 600 tokens of which the
//            first 512 (two blocks) are a prefix-cache hit; sequence C, 37.
//   decode:  each sequence appends one token.
//   sample:  two Sample calls on the same 3 x 5003 logits (unaligned rows):
//            greedy rows with and without a repetition penalty (histories
//            include ids past the vocabulary) and a temperature row with one
//            dominant logit, so every token is determined.
// Usage: runner_check <out_dir> [seed]
// Output: <out_dir>/manifest.txt lines "name dtype d0 d1 ..." and one raw
// little-endian <name>.bin per array.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <string>
#include <vector>

#include "attention_runner.h"

namespace {

struct Rng {  // xorshift64*, then Box-Muller for normals
  uint64_t s;
  explicit Rng(uint64_t seed) : s(seed * 0x9E3779B97F4A7C15ull + 1) {}
  uint64_t next() {
    s ^= s >> 12;
    s ^= s << 25;
    s ^= s >> 27;
    return s * 0x2545F4914F6CDD1Dull;
  }
  double uniform() { return ((next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
  float normal() {
    const double u = uniform(), v = uniform();
    return static_cast<float>(std::sqrt(-2.0 * std::log(u)) * std::cos(6.283185307179586 * v));
  }
};

uint16_t to_bf16(float f) {  // round to nearest even (finite inputs only here)
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return static_cast<uint16_t>((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

struct Dump {
  std::string dir;
  FILE* manifest = nullptr;
  explicit Dump(const std::string& d) : dir(d) {
    manifest = std::fopen((dir + "/manifest.txt").c_str(), "w");
  }
  ~Dump() {
    if (manifest) std::fclose(manifest);
  }
  template <typename T>
  bool put(const char* name, const char* dtype, const std::vector<T>& v,
           std::initializer_list<size_t> shape) {
    FILE* f = std::fopen((dir + "/" + name + ".bin").c_str(), "wb");
    if (!f) return false;
    const bool ok = std::fwrite(v.data(), sizeof(T), v.size(), f) == v.size();
    std::fclose(f);
    std::fprintf(manifest, "%s %s", name, dtype);
    for (size_t d : shape) std::fprintf(manifest, " %zu", d);
    std::fprintf(manifest, "\n");
    return ok;
  }
};

#define CK(x)                                                                     \
  do {                                                                            \
    if ((x) != cudaSuccess) {                                                     \
      std::fprintf(stderr, "CUDA error at %s:%d: %s\n", __FILE__, __LINE__, #x); \
      return 1;                                                                   \
    }                                                                             \
  } while (0)

template <typename T>
T* upload(const std::vector<T>& h) {
  T* d = nullptr;
  if (cudaMalloc(&d, h.size() * sizeof(T)) != cudaSuccess) return nullptr;
  if (cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess)
    return nullptr;
  return d;
}

template <typename T>
std::vector<T> download(const T* d, size_t n) {
  std::vector<T> h(n);
  cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost);
  return h;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: %s <out_dir> [seed]\n", argv[0]);
    return 2;
  }
  const uint64_t seed = argc > 2 ? std::strtoull(argv[2], nullptr, 10) : 1;
  Rng rng(seed);

  nvattn_config cfg;
  nvattn_config_init_qwen3(&cfg);
  cfg.n_layer = 2;
  cfg.n_q_heads = 16;
  cfg.n_kv_heads = 8;
  cfg.num_blocks = 12;
  cfg.max_seqs = 4;
  cfg.max_context = 1024;
  cfg.max_position = 4096;
  const int layer = 1, Hq = cfg.n_q_heads, Hkv = cfg.n_kv_heads, D = cfg.head_dim;
  const size_t n_slots = static_cast<size_t>(cfg.num_blocks) * cfg.block_size;
  const size_t cache_elems = static_cast<size_t>(cfg.n_layer) * n_slots * Hkv * D;

  Dump out(argv[1]);
  if (!out.manifest) {
    std::fprintf(stderr, "cannot write to %s\n", argv[1]);
    return 2;
  }

  // cache contents: random bf16 everywhere (a prefix hit reads real values)
  std::vector<uint16_t> kc(cache_elems), vc(cache_elems);
  for (size_t i = 0; i < cache_elems; ++i) kc[i] = to_bf16(rng.normal());
  for (size_t i = 0; i < cache_elems; ++i) vc[i] = to_bf16(rng.normal());
  out.put("k_cache0", "u16", kc, {(size_t)cfg.n_layer, n_slots, (size_t)Hkv, (size_t)D});
  out.put("v_cache0", "u16", vc, {(size_t)cfg.n_layer, n_slots, (size_t)Hkv, (size_t)D});
  uint16_t* d_kc = upload(kc);
  uint16_t* d_vc = upload(vc);
  std::vector<uint16_t> qw(D), kw(D);
  for (int i = 0; i < D; ++i) qw[i] = to_bf16(1.0f + 0.02f * rng.normal());
  for (int i = 0; i < D; ++i) kw[i] = to_bf16(1.0f + 0.02f * rng.normal());
  out.put("q_norm_w", "u16", qw, {(size_t)D});
  out.put("k_norm_w", "u16", kw, {(size_t)D});
  uint16_t* d_qw = upload(qw);
  uint16_t* d_kw = upload(kw);
  if (!d_kc || !d_vc || !d_qw || !d_kw) {
    std::fprintf(stderr, "upload failed\n");
    return 1;
  }

  try {
    nvattn_host::AttentionRunner runner(cfg);
    nvattn_host::SequenceView a, b, c;
    a.block_table = {3, 7};
    a.seq_len = 300;
    b.block_table = {1, 5, 9};
    b.seq_len = 600;
    b.num_cached_tokens = 512;
    c.block_table = {10};
    c.seq_len = 37;
    std::vector<nvattn_host::SequenceView*> seqs = {&a, &b, &c};

    for (int step = 0; step < 2; ++step) {
      const bool prefill = step == 0;
      if (!prefill) {
        for (auto* s : seqs) {
          s->num_cached_tokens = s->seq_len;
          s->seq_len += 1;
        }
      }
      if (!runner.PrepareInputs(seqs, prefill, nullptr)) {
        std::fprintf(stderr, "PrepareInputs failed (step %d)\n", step);
        return 1;
      }
      const int T = runner.NumTokens();
      std::vector<float> q((size_t)T * Hq * D), k((size_t)T * Hkv * D), v((size_t)T * Hkv * D);
      for (auto& x : q) x = rng.normal();
      for (auto& x : k) x = rng.normal();
      for (auto& x : v) x = rng.normal();
      float* d_q = upload(q);
      float* d_k = upload(k);
      float* d_v = upload(v);
      float* d_out = nullptr;
      CK(cudaMalloc(&d_out, (size_t)T * Hq * D * sizeof(float)));
      if (!d_q || !d_k || !d_v) return 1;
      if (!runner.RunAttentionLayer(layer, d_q, d_k, d_v, d_qw, d_kw, d_kc, d_vc, d_out,
                                    nullptr)) {
        std::fprintf(stderr, "RunAttentionLayer failed (step %d)\n", step);
        return 1;
      }
      CK(cudaDeviceSynchronize());
      int64_t detail = 0;
      const nvattn_status st = nvattn_get_error(runner.Handle(), &detail);
      if (st != NVATTN_OK) {
        std::fprintf(stderr, "device error %s (detail %lld)\n", nvattn_status_string(st),
                     (long long)detail);
        return 1;
      }
      const std::string p = prefill ? "prefill_" : "decode_";
      std::vector<int32_t> lens, cached, bt(seqs.size() * 3, -1);
      for (size_t s = 0; s < seqs.size(); ++s) {
        lens.push_back((int32_t)seqs[s]->seq_len);
        cached.push_back((int32_t)seqs[s]->num_cached_tokens);
        for (size_t j = 0; j < seqs[s]->block_table.size(); ++j)
          bt[s * 3 + j] = (int32_t)seqs[s]->block_table[j];
      }
      out.put((p + "seq_lens").c_str(), "i32", lens, {seqs.size()});
      out.put((p + "num_cached").c_str(), "i32", cached, {seqs.size()});
      out.put((p + "block_tables").c_str(), "i32", bt, {seqs.size(), (size_t)3});
      out.put((p + "positions").c_str(), "i32", runner.Positions(), {(size_t)T});
      out.put((p + "slots").c_str(), "i32", runner.SlotMapping(), {(size_t)T});
      out.put((p + "q").c_str(), "f32", q, {(size_t)T, (size_t)Hq, (size_t)D});
      out.put((p + "k").c_str(), "f32", k, {(size_t)T, (size_t)Hkv, (size_t)D});
      out.put((p + "v").c_str(), "f32", v, {(size_t)T, (size_t)Hkv, (size_t)D});
      out.put((p + "q_after").c_str(), "f32", download(d_q, q.size()),
              {(size_t)T, (size_t)Hq, (size_t)D});
      out.put((p + "out").c_str(), "f32", download(d_out, (size_t)T * Hq * D),
              {(size_t)T, (size_t)Hq, (size_t)D});
      out.put((p + "k_cache").c_str(), "u16", download(d_kc, cache_elems),
              {(size_t)cfg.n_layer, n_slots, (size_t)Hkv, (size_t)D});
      out.put((p + "v_cache").c_str(), "u16", download(d_vc, cache_elems),
              {(size_t)cfg.n_layer, n_slots, (size_t)Hkv, (size_t)D});
      cudaFree(d_q);
      cudaFree(d_k);
      cudaFree(d_v);
      cudaFree(d_out);
    }

    // ---- sampling: the next token of each sequence ----
    const int V = 5003;
    std::vector<float> logits((size_t)3 * V);
    for (auto& x : logits) x = 2.0f * rng.normal();
    logits[(size_t)1 * V + 4321] = 40.0f;  // row 1 samples this id whatever the draw
    const std::vector<float> temps = {0.0f, 0.7f, 0.0f}, pens = {1.3f, 1.2f, 1.0f};
    std::vector<std::vector<int32_t>> hist(3);
    for (int i = 0; i < 200; ++i) hist[0].push_back((int32_t)(rng.next() % (V + 50)));
    for (int i = 0; i < 50; ++i) hist[1].push_back((int32_t)(rng.next() % V));
    float* d_logits = upload(logits);
    if (!d_logits) return 1;
    std::vector<int32_t> tokens, offsets = {0}, flat;
    std::vector<float> draws;
    for (int call = 0; call < 2; ++call) {
      const std::vector<int> t = runner.Sample(d_logits, V, temps, pens, hist, nullptr);
      if (t.size() != 3) {
        std::fprintf(stderr, "Sample failed (call %d)\n", call);
        return 1;
      }
      tokens.insert(tokens.end(), t.begin(), t.end());
      draws.insert(draws.end(), runner.LastUniforms().begin(), runner.LastUniforms().end());
    }
    for (const auto& h : hist) {
      flat.insert(flat.end(), h.begin(), h.end());
      offsets.push_back((int32_t)flat.size());
    }
    out.put("sample_logits", "f32", logits, {(size_t)3, (size_t)V});
    out.put("sample_temperatures", "f32", temps, {(size_t)3});
    out.put("sample_penalties", "f32", pens, {(size_t)3});
    out.put("sample_history", "i32", flat, {flat.size()});
    out.put("sample_history_offsets", "i32", offsets, {(size_t)4});
    out.put("sample_uniforms", "f32", draws, {(size_t)2, (size_t)3});
    out.put("sample_tokens", "i32", tokens, {(size_t)2, (size_t)3});
    cudaFree(d_logits);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }
  cudaFree(d_kc);
  cudaFree(d_vc);
  cudaFree(d_qw);
  cudaFree(d_kw);
  std::printf("ok\n");
  return 0;
}
