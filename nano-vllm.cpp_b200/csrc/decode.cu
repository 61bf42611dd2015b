// decode.cu -- paged GQA split-KV decode attention over the BF16 block cache.
//
// Replaces the reference's decode attention path: LoadHistoryKV's per-token
// gather through block_table + bf16->f32 + reorder (src/engine/
// model_runner.cpp:300-376), FillVarlenMask (:219-243), the graph concat /
// pad / permute (src/models/qwen3.cpp:648-661) and BuildAttention's
// ggml_flash_attn_ext (qwen3.cpp:377-405).  The reference attends every query
// row over all sequences' concatenated history (O(B * sum L)); here each
// (sequence, kv head) reads only its own blocks, once, for all its GQA heads.
//
// Grid (split, kv_head, seq).  A split is a run of split_tokens tokens of one
// sequence.  Warp 4 is the producer: one lane streams 64-token K and V tiles
// (16 KiB each, TMA boxes {128, 1, 64} over the cache viewed as
// [layer*slot][kv_head][128]) into a 3-stage shared-memory ring guarded by
// mbarriers.  Warps 0-3 are consumers: each owns 16 tokens of a tile; a lane
// owns 4 head dims.  Scores use a transposed butterfly reduction, softmax is
// online in the log2 domain, and P.V accumulates in fp32 registers.  A split
// writes either the final row (single split) or its (m, l, O) partial, which
// paged_decode_combine_kernel merges.
#include "common.cuh"
#include "internal.h"

namespace nvattn {
namespace {

constexpr int kD = 128;
constexpr int kTile = 64;
constexpr int kStages = 3;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kTokPerWarp = kTile / kConsumerWarps;  // 16
constexpr int kTileBytes = kTile * kD * 2;           // 16 KiB
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  int Hq, Hkv, layer, block_size, max_blocks, split_tokens, max_splits;
  int max_context;  // host bound on context_lens (<= max_blocks * block_size)
  long long n_slots, num_blocks;
  float scale_log2;  // softmax scale * log2(e)
  const float* q;
  const int32_t* block_tables;
  const int32_t* context_lens;
  float* out;
  float* ws_o;
  float* ws_ml;
  DeviceStatus* status;
};

template <int G>
struct __align__(1024) DecodeSmem {
  uint16_t k[kStages][kTile * kD];
  uint16_t v[kStages][kTile * kD];
  float s[G][kTile];  // scores, log2 domain
  float p[kTile][G];  // probabilities
  float alpha[G];
  float m_run[G];
  float l_run[G];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int abort_flag;  // raised by the first wait that times out
};

// Butterfly transpose-reduction of V per-lane partial sums across the warp.
// Afterwards, for V >= 32 lane l holds the totals of indices l*(V/32) + j in
// v[j]; for V < 32 every lane holds the total of index l >> (5 - log2 V).
template <int V>
__device__ __forceinline__ void transpose_reduce(float (&v)[V], int lane) {
  int n = V;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    if (n > 1) {
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < n / 2) {
          const float send = upper ? v[i] : v[i + n / 2];
          const float keep = upper ? v[i + n / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      n >>= 1;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
}

template <int G>
__device__ __forceinline__ void load_p(const float* row, float (&pg)[G]) {
  if constexpr (G == 1) {
    pg[0] = row[0];
  } else if constexpr (G == 2) {
    const float2 a = *reinterpret_cast<const float2*>(row);
    pg[0] = a.x; pg[1] = a.y;
  } else {
#pragma unroll
    for (int i = 0; i < G / 4; ++i) {
      const float4 a = reinterpret_cast<const float4*>(row)[i];
      pg[4 * i] = a.x; pg[4 * i + 1] = a.y; pg[4 * i + 2] = a.z; pg[4 * i + 3] = a.w;
    }
  }
}

template <int G>
__global__ void __launch_bounds__(kThreads, 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, DecodeParams prm) {
  extern __shared__ uint8_t smem_raw[];
  DecodeSmem<G>& sm = *reinterpret_cast<DecodeSmem<G>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int ctx = prm.context_lens[seq];
  const int t_begin = split * prm.split_tokens;
  if (ctx < 0 || ctx > prm.max_context) {
    // A length outside [0, max_context_len] would index past the block table
    // row or the grid; flag it and attend over the clamped range.
    if (threadIdx.x == 0 && split == 0) record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 10, ctx);
    ctx = ctx < 0 ? 0 : prm.max_context;
  }
  if (t_begin >= ctx && split > 0) return;  // nothing for this split
  if (timeout_recorded(prm.status)) return;
  const int t_end = min(ctx, t_begin + prm.split_tokens);
  const int n_tiles = t_end > t_begin ? (t_end - t_begin + kTile - 1) / kTile : 0;
  const int n_splits = ctx > 0 ? (ctx + prm.split_tokens - 1) / prm.split_tokens : 1;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kConsumerWarps);
    }
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < G) {
    sm.m_run[threadIdx.x] = -INFINITY;
    sm.l_run[threadIdx.x] = 0.0f;
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const uint64_t policy = l2_policy_evict_first();
      for (int i = 0; i < n_tiles; ++i) {
        const int stage = i % kStages;
        if (i >= kStages) mbar_wait(&sm.empty[stage], ((i / kStages) & 1) ^ 1, prm.status, &sm.abort_flag, 11);
        const int tok = t_begin + i * kTile;
        const int bi = tok / prm.block_size;
        long long bid = prm.block_tables[(long long)seq * prm.max_blocks + bi];
        if (bid < 0 || bid >= prm.num_blocks) {
          record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 12, bid);
          bid = 0;  // keep the pipeline flowing; the result is flagged invalid
        }
        const int row = (int)((long long)prm.layer * prm.n_slots + bid * prm.block_size +
                              tok % prm.block_size);
        mbar_arrive_expect_tx(&sm.full[stage], 2 * kTileBytes);
        tma_load_3d_hint(sm.k[stage], &tm_k, &sm.full[stage], 0, kvh, row, policy);
        tma_load_3d_hint(sm.v[stage], &tm_v, &sm.full[stage], 0, kvh, row, policy);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  float qr[G][4];
  {
    const float* qp = prm.q + ((long long)seq * prm.Hq + (long long)kvh * G) * kD + 4 * lane;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float4 a = *reinterpret_cast<const float4*>(qp + g * kD);
      qr[g][0] = a.x * prm.scale_log2;
      qr[g][1] = a.y * prm.scale_log2;
      qr[g][2] = a.z * prm.scale_log2;
      qr[g][3] = a.w * prm.scale_log2;
    }
  }
  float acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[g][j] = 0.0f;

  constexpr int TB = (G >= 8) ? 8 : 16;  // tokens per reduction batch
  constexpr int V = G * TB;              // values reduced per batch

  for (int i = 0; i < n_tiles; ++i) {
    const int stage = i % kStages;
    mbar_wait(&sm.full[stage], (i / kStages) & 1, prm.status, &sm.abort_flag, 13);
    const uint16_t* kt = sm.k[stage];
    const uint16_t* vt = sm.v[stage];
    const int tok0 = t_begin + i * kTile;
    const int n_valid = min(kTile, t_end - tok0);

    // ---- scores for this warp's 16 tokens ----
#pragma unroll
    for (int b = 0; b < kTokPerWarp / TB; ++b) {
      float vals[V];
#pragma unroll
      for (int tt = 0; tt < TB; ++tt) {
        const int tl = warp * kTokPerWarp + b * TB + tt;
        const uint2 kr = *reinterpret_cast<const uint2*>(kt + tl * kD + 4 * lane);
        const float k0 = bf16lo_to_f32(kr.x), k1 = bf16hi_to_f32(kr.x);
        const float k2 = bf16lo_to_f32(kr.y), k3 = bf16hi_to_f32(kr.y);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float a = qr[g][0] * k0;
          a = fmaf(qr[g][1], k1, a);
          a = fmaf(qr[g][2], k2, a);
          a = fmaf(qr[g][3], k3, a);
          vals[tt * G + g] = a;
        }
      }
      transpose_reduce<V>(vals, lane);
      if constexpr (V >= 32) {
#pragma unroll
        for (int j = 0; j < V / 32; ++j) {
          const int idx = lane * (V / 32) + j;
          const int tl = warp * kTokPerWarp + b * TB + idx / G;
          sm.s[idx % G][tl] = tl < n_valid ? vals[j] : -INFINITY;
        }
      } else {
        if ((lane & 1) == 0) {
          const int tl = warp * kTokPerWarp + b * TB + (lane >> 1);
          sm.s[0][tl] = tl < n_valid ? vals[0] : -INFINITY;
        }
      }
    }
    named_barrier_sync(1, kConsumerWarps * 32);

    // ---- online softmax statistics: warp w owns heads w, w+4, ... ----
    for (int g = warp; g < G; g += kConsumerWarps) {
      const float s0 = sm.s[g][lane], s1 = sm.s[g][lane + 32];
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = sm.m_run[g];
      const float m_new = fmaxf(m_old, mx);
      float p0 = 0.0f, p1 = 0.0f, alpha = 1.0f;
      if (m_new != -INFINITY) {
        p0 = fast_exp2(s0 - m_new);
        p1 = fast_exp2(s1 - m_new);
        alpha = fast_exp2(m_old - m_new);
      }
      sm.p[lane][g] = p0;
      sm.p[lane + 32][g] = p1;
      float sum = p0 + p1;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      __syncwarp();
      if (lane == 0) {
        sm.l_run[g] = sm.l_run[g] * alpha + sum;
        sm.m_run[g] = m_new;
        sm.alpha[g] = alpha;
      }
    }
    named_barrier_sync(1, kConsumerWarps * 32);

    // ---- P.V for this warp's 16 tokens ----
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float a = sm.alpha[g];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[g][j] *= a;
    }
    const int tl0 = warp * kTokPerWarp;
    const int n_mine = min(kTokPerWarp, n_valid - tl0);
#pragma unroll 4
    for (int tt = 0; tt < n_mine; ++tt) {
      const int tl = tl0 + tt;
      const uint2 vr = *reinterpret_cast<const uint2*>(vt + tl * kD + 4 * lane);
      const float v0 = bf16lo_to_f32(vr.x), v1 = bf16hi_to_f32(vr.x);
      const float v2 = bf16lo_to_f32(vr.y), v3 = bf16hi_to_f32(vr.y);
      float pg[G];
      load_p<G>(&sm.p[tl][0], pg);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        acc[g][0] = fmaf(pg[g], v0, acc[g][0]);
        acc[g][1] = fmaf(pg[g], v1, acc[g][1]);
        acc[g][2] = fmaf(pg[g], v2, acc[g][2]);
        acc[g][3] = fmaf(pg[g], v3, acc[g][3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[stage]);
  }

  // ---- cross-warp reduction of the 4 partial accumulators ----
  named_barrier_sync(1, kConsumerWarps * 32);  // every stage consumed
  float* red = reinterpret_cast<float*>(&sm.k[0][0]);  // [4][G][128] fp32 <= 16 KiB
  static_assert(kConsumerWarps * G * kD * 4 <= kTileBytes * kStages * 2, "reduction buffer");
#pragma unroll
  for (int g = 0; g < G; ++g)
    *reinterpret_cast<float4*>(red + (warp * G + g) * kD + 4 * lane) =
        make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
  named_barrier_sync(1, kConsumerWarps * 32);
  const int d = threadIdx.x;  // 0..127
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) o += red[(w * G + g) * kD + d];
    const int h = kvh * G + g;
    if (n_splits == 1) {
      const float l = sm.l_run[g];
      prm.out[((long long)seq * prm.Hq + h) * kD + d] = l > 0.0f ? o / l : 0.0f;
    } else {
      const long long pidx = ((long long)(seq * prm.Hkv + kvh) * prm.max_splits + split) * G + g;
      prm.ws_o[pidx * kD + d] = o;
      if (d == 0) {
        prm.ws_ml[pidx * 2 + 0] = sm.m_run[g];
        prm.ws_ml[pidx * 2 + 1] = sm.l_run[g];
      }
    }
  }
}

// Merges the split partials of one (sequence, q head); one thread per dim.
__global__ void __launch_bounds__(kD) paged_decode_combine_kernel(DecodeParams prm, int G) {
  const int h = blockIdx.x, seq = blockIdx.y, d = threadIdx.x;
  const int ctx = min(prm.context_lens[seq], prm.max_context);
  if (ctx <= 0) return;
  const int n = (ctx + prm.split_tokens - 1) / prm.split_tokens;
  if (n <= 1) return;
  const int kvh = h / G, g = h % G;
  const long long base = (long long)(seq * prm.Hkv + kvh) * prm.max_splits;
  float M = -INFINITY;
  for (int i = 0; i < n; ++i) M = fmaxf(M, prm.ws_ml[((base + i) * G + g) * 2]);
  float L = 0.0f, O = 0.0f;
  for (int i = 0; i < n; ++i) {
    const long long pidx = (base + i) * G + g;
    const float w = fast_exp2(prm.ws_ml[pidx * 2] - M);
    L = fmaf(prm.ws_ml[pidx * 2 + 1], w, L);
    O = fmaf(prm.ws_o[pidx * kD + d], w, O);
  }
  prm.out[((long long)seq * prm.Hq + h) * kD + d] = L > 0.0f ? O / L : 0.0f;
}

template <int G>
nvattn_status launch_g(const CUtensorMap* tk, const CUtensorMap* tv, const DecodeParams& prm,
                       int n_seqs, int max_context_len, cudaStream_t stream) {
  const size_t smem = sizeof(DecodeSmem<G>) + 1024;
  // The attribute is per device; remember which devices have it.
  static unsigned long long attr_set_mask = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVATTN_ERR_CUDA;
  if (dev >= 64 || !(attr_set_mask & (1ull << dev))) {
    if (cudaFuncSetAttribute(paged_decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return NVATTN_ERR_CUDA;
    if (dev < 64) attr_set_mask |= 1ull << dev;
  }
  const int n_splits_max = max_context_len > 0
                               ? (max_context_len + prm.split_tokens - 1) / prm.split_tokens
                               : 1;
  dim3 grid(n_splits_max, prm.Hkv, n_seqs);
  paged_decode_kernel<G><<<grid, kThreads, smem, stream>>>(*tk, *tv, prm);
  if (n_splits_max > 1) {
    dim3 cgrid(prm.Hq, n_seqs);
    paged_decode_combine_kernel<<<cgrid, kD, 0, stream>>>(prm, G);
  }
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace

// Tokens per split: whole 256-token blocks, small enough that the grid fills
// the GPU several times over when sequences are short, and at most 2048 so
// that log-uniform context lengths still balance across SMs.
static int split_tokens_for(int sm_count, int block_size, int n_kv_heads, int max_splits,
                            int n_seqs, int max_context_len) {
  const long long target_ctas = 4LL * 2 * sm_count;
  const long long units = (long long)n_seqs * n_kv_heads;
  int split = 2048;
  while (split > block_size && units * ((max_context_len + split - 1) / split) < target_ctas)
    split /= 2;
  if (split < block_size) split = block_size;
  // never more splits per sequence than the workspace holds
  while ((max_context_len + split - 1) / split > max_splits) split *= 2;
  return split;
}

// Splits per (sequence, kv head) that the workspace of a handle created with
// this max_context holds (the same rule nvattn_create applies).
static int workspace_max_splits(const nvattn_config& c) {
  const long long splits = (c.max_context + c.block_size - 1) / c.block_size;
  return (int)(splits < 64 ? splits : 64);
}

int decode_split_tokens(const nvattn_handle* h, int n_seqs, int max_context_len) {
  return split_tokens_for(h->sm_count, h->cfg.block_size, h->cfg.n_kv_heads, h->max_splits,
                          n_seqs, max_context_len);
}

nvattn_status launch_paged_decode(nvattn_handle* h, int layer, int n_seqs, const float* q,
                                  const uint16_t* k_cache, const uint16_t* v_cache,
                                  const int32_t* block_tables, int max_blocks,
                                  const int32_t* context_lens, int max_context_len,
                                  float* out, cudaStream_t stream) {
  if (n_seqs == 0) return NVATTN_OK;
  const CUtensorMap* tk = nullptr;
  const CUtensorMap* tv = nullptr;
  nvattn_status st = get_cache_tensor_map(h, k_cache, kD, kTile, 0, &tk);
  if (st != NVATTN_OK) return st;
  st = get_cache_tensor_map(h, v_cache, kD, kTile, 0, &tv);
  if (st != NVATTN_OK) return st;

  DecodeParams prm;
  prm.Hq = h->cfg.n_q_heads;
  prm.Hkv = h->cfg.n_kv_heads;
  prm.layer = layer;
  prm.block_size = h->cfg.block_size;
  prm.max_blocks = max_blocks;
  prm.max_context = max_context_len;
  prm.split_tokens = decode_split_tokens(h, n_seqs, max_context_len);
  prm.max_splits = h->max_splits;
  prm.n_slots = h->n_slots;
  prm.num_blocks = h->cfg.num_blocks;
  prm.scale_log2 = h->cfg.scale * kLog2e;
  prm.q = q;
  prm.block_tables = block_tables;
  prm.context_lens = context_lens;
  prm.out = out;
  prm.ws_o = h->ws_o;
  prm.ws_ml = h->ws_ml;
  prm.status = h->status_dev;
  switch (prm.Hq / prm.Hkv) {
    case 1: return launch_g<1>(tk, tv, prm, n_seqs, max_context_len, stream);
    case 2: return launch_g<2>(tk, tv, prm, n_seqs, max_context_len, stream);
    case 4: return launch_g<4>(tk, tv, prm, n_seqs, max_context_len, stream);
    case 8: return launch_g<8>(tk, tv, prm, n_seqs, max_context_len, stream);
    default: return NVATTN_ERR_UNSUPPORTED;
  }
}

// ---------------------------------------------------------------------------
// Allocation-free decode (nvattn_paged_decode_noalloc).
//
// The split-KV partials live in this file-scope device array instead of a
// handle's cudaMalloc'd workspace.  Every GPU that loads the library holds
// these 32 MiB until the process exits.  The array's name is only a host-side
// stand-in for the device symbol, so the host fetches its real device address
// with cudaGetSymbolAddress, once per device, and passes that to the kernel.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
static_assert(sizeof(DeviceStatus) == sizeof(nvattn_device_status), "status layout");
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
void* g_noalloc_scratch_addr[kMaxDevices];  // device address per device (set once)
int g_noalloc_sm_count[kMaxDevices];
}  // namespace

}  // namespace nvattn

extern "C" NVATTN_API nvattn_status nvattn_paged_decode_noalloc(
    const nvattn_config* cfg, int layer, int n_seqs, const float* q_dev,
    const uint16_t* k_cache_dev, const uint16_t* v_cache_dev, const int32_t* block_tables_dev,
    int max_blocks, const int32_t* context_lens_dev, int max_context_len, float* out_dev,
    nvattn_device_status* status_dev, nvattn_stream_t stream) {
  using namespace nvattn;
  if (cfg == nullptr) return NVATTN_ERR_INVALID_ARG;
  const nvattn_config& c = *cfg;
  if (c.n_layer <= 0 || c.n_q_heads <= 0 || c.n_kv_heads <= 0 || c.num_blocks <= 0 ||
      c.block_size <= 0 || c.max_context <= 0 || c.n_q_heads % c.n_kv_heads != 0 ||
      !(c.scale > 0.0f))
    return NVATTN_ERR_INVALID_ARG;
  const int G = c.n_q_heads / c.n_kv_heads;
  if (c.head_dim != kD || c.block_size % 128 != 0 || c.block_size > 1024 ||
      !(G == 1 || G == 2 || G == 4 || G == 8))
    return NVATTN_ERR_UNSUPPORTED;
  const long long n_slots = c.num_blocks * (long long)c.block_size;
  if ((long long)c.n_layer * n_slots >= (1LL << 31)) return NVATTN_ERR_UNSUPPORTED;
  if (layer < 0 || layer >= c.n_layer || n_seqs < 0 || max_blocks <= 0 || max_context_len < 0 ||
      max_context_len > c.max_context ||
      (long long)max_context_len > (long long)max_blocks * c.block_size)
    return NVATTN_ERR_INVALID_ARG;
  if (n_seqs == 0) return NVATTN_OK;
  const void* ptrs[] = {q_dev, k_cache_dev, v_cache_dev, out_dev};
  for (const void* p : ptrs)
    if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) != 0) return NVATTN_ERR_INVALID_ARG;
  if (block_tables_dev == nullptr || context_lens_dev == nullptr) return NVATTN_ERR_INVALID_ARG;

  // Runs on the caller's current device, which must be cfg->device.
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVATTN_ERR_CUDA;
  if (dev != c.device || dev < 0 || dev >= kMaxDevices) return NVATTN_ERR_INVALID_ARG;
  // One-time set-up on this device: the scratch's device address and the SM
  // count (neither allocates).
  if (g_noalloc_scratch_addr[dev] == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_noalloc_scratch) != cudaSuccess || addr == nullptr)
      return NVATTN_ERR_CUDA;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return NVATTN_ERR_CUDA;
    g_noalloc_sm_count[dev] = sms;
    g_noalloc_scratch_addr[dev] = addr;
  }

  // Same split rule as a handle created from this config, so the result
  // equals nvattn_paged_decode's.
  const int split = split_tokens_for(g_noalloc_sm_count[dev], c.block_size, c.n_kv_heads,
                                     workspace_max_splits(c), n_seqs, max_context_len);
  const int n_splits = max_context_len > 0 ? (max_context_len + split - 1) / split : 1;
  const size_t rows = n_splits > 1 ? (size_t)n_seqs * c.n_q_heads * n_splits : 0;
  if (rows * (kD + 2) * sizeof(float) > kNoAllocScratchBytes) return NVATTN_ERR_SCRATCH_LIMIT;

  CUtensorMap tk, tv;
  nvattn_status st = encode_tensor_map_3d(&tk, k_cache_dev, kD, (uint64_t)c.n_kv_heads,
                                          (uint64_t)c.n_layer * (uint64_t)n_slots, kD * 2,
                                          (uint64_t)c.n_kv_heads * kD * 2, kD, 1, kTile, 0);
  if (st != NVATTN_OK) return st;
  st = encode_tensor_map_3d(&tv, v_cache_dev, kD, (uint64_t)c.n_kv_heads,
                            (uint64_t)c.n_layer * (uint64_t)n_slots, kD * 2,
                            (uint64_t)c.n_kv_heads * kD * 2, kD, 1, kTile, 0);
  if (st != NVATTN_OK) return st;

  float* scratch = static_cast<float*>(g_noalloc_scratch_addr[dev]);
  DecodeParams prm;
  prm.Hq = c.n_q_heads;
  prm.Hkv = c.n_kv_heads;
  prm.layer = layer;
  prm.block_size = c.block_size;
  prm.max_blocks = max_blocks;
  prm.max_context = max_context_len;
  prm.split_tokens = split;
  prm.max_splits = n_splits;  // partial-row stride
  prm.n_slots = n_slots;
  prm.num_blocks = c.num_blocks;
  prm.scale_log2 = c.scale * kLog2e;
  prm.q = q_dev;
  prm.block_tables = block_tables_dev;
  prm.context_lens = context_lens_dev;
  prm.out = out_dev;
  prm.ws_o = scratch;
  prm.ws_ml = scratch + rows * kD;
  prm.status = reinterpret_cast<DeviceStatus*>(status_dev);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (G) {
    case 1: return launch_g<1>(&tk, &tv, prm, n_seqs, max_context_len, s);
    case 2: return launch_g<2>(&tk, &tv, prm, n_seqs, max_context_len, s);
    case 4: return launch_g<4>(&tk, &tv, prm, n_seqs, max_context_len, s);
    default: return launch_g<8>(&tk, &tv, prm, n_seqs, max_context_len, s);
  }
}
