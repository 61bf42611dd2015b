// prefill.cu -- causal paged prefill / prefix-hit / chunked-prefill attention
// on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Replaces the reference's prefill attention: FillCausalMask
// (src/engine/model_runner.cpp:188-217), the prefill pad/permute
// (src/models/qwen3.cpp:524-531) and BuildAttention's ggml_flash_attn_ext
// (qwen3.cpp:377-405).  The reference attends only over the batch's new
// tokens and ignores a cached prefix (qwen3.cpp:445-446); here a row at
// position P attends keys [0, P] of its sequence through the block table,
// which covers prefix-cache hits and chunked prefill alike.
//
// One CTA = (sequence, q head, tile of 128 query rows); 128-key KV tiles.
//   warp 0      TMA producer: Q once, then K and V tiles (two 64-column
//               boxes each, 128-byte swizzle) into a 2-stage ring.
//   warp 1      TMEM allocation; one lane issues the MMAs:
//                 S[b] = Q K^T   (M=128, N=128, K=128; A, B K-major)
//                 O   += P V     (M=128, N=128, K=128; P K-major, V MN-major)
//               S is double-buffered in TMEM so S(j+1) runs while the
//               softmax warps work on S(j).
//   warps 2-5   softmax: thread = query row = TMEM lane.  Causal mask,
//               online softmax in the log2 domain, P written to shared
//               memory as bf16 in the UMMA operand layout, lazy O rescaling
//               (only when a row max grows by more than 2^8), epilogue
//               O / l -> f32 output.
// TMEM: columns [0,256) two S buffers, [256,384) O.
#include "common.cuh"
#include "internal.h"

namespace nvattn {
namespace {

constexpr int kD = 128;
constexpr int kBM = 128;  // query rows per CTA
constexpr int kBN = 128;  // keys per KV tile
constexpr int kThreads = 192;
constexpr int kHalfBytes = 128 * 64 * 2;  // one 128-row x 64-column bf16 box: 16 KiB
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct PrefillParams {
  int Hq, Hkv, G, layer, block_size, max_blocks, n_mtiles;
  long long n_slots, num_blocks;
  float scale_log2;
  const int32_t* cu_q;
  const int32_t* q_starts;
  const int32_t* context_lens;
  const int32_t* block_tables;
  float* out;
  DeviceStatus* status;
};

template <bool kSplitP>
struct __align__(1024) PrefillSmem {
  uint16_t q[2][kBM * 64];     // [d half][row][64]
  uint16_t k[2][2][kBN * 64];  // [stage][d half][key][64]
  uint16_t v[2][2][kBN * 64];  // [stage][d half][key][64]
  uint16_t p[2][kBM * 64];     // [key half][row][64]
  uint16_t p_lo[kSplitP ? 2 : 1][kSplitP ? kBM * 64 : 512];  // bf16 remainder of P
  uint64_t q_full;
  uint64_t k_full[2], v_full[2], kv_empty[2];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full, o_done;
  uint32_t tmem_base;
  int abort_flag;  // raised by the first wait that times out
};

template <bool kSplitP>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, PrefillParams prm) {
  extern __shared__ uint8_t smem_raw[];
  PrefillSmem<kSplitP>& sm = *reinterpret_cast<PrefillSmem<kSplitP>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int G = prm.G;
  const int g = blockIdx.x % G;
  const int mt = prm.n_mtiles - 1 - (int)(blockIdx.x / G);  // longest tiles launch first
  const int kvh = blockIdx.y, seq = blockIdx.z;
  const int h = kvh * G + g;
  const int q0 = prm.cu_q[seq];
  const int n_q = prm.cu_q[seq + 1] - q0;
  if (n_q > prm.n_mtiles * kBM) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && kvh == 0)
      record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 21, n_q);
  }
  if (mt * kBM >= n_q) return;  // whole CTA: nothing to do
  if (timeout_recorded(prm.status)) return;
  const int rows = min(kBM, n_q - mt * kBM);
  const int p_first = prm.q_starts[seq] + mt * kBM;  // position of tile row 0
  const int p_last = p_first + rows - 1;
  int ctx = prm.context_lens[seq];
  if (p_first < 0 || (long long)p_last >= (long long)prm.max_blocks * prm.block_size) {
    if (threadIdx.x == 0) record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 22, p_last);
    return;
  }
  if (ctx <= p_last) {
    if (threadIdx.x == 0) record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 23, ctx);
    ctx = p_last + 1;
  }
  const int n_kv = p_last / kBN + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.k_full[i], 1);
      mbar_init(&sm.v_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], 4);
    }
    mbar_init(&sm.p_full, 4);
    mbar_init(&sm.o_done, 1);
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t tmem_o = tmem + 256;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&sm.q_full, 2 * kHalfBytes);
      tma_load_3d(sm.q[0], &tm_q, &sm.q_full, 0, h, q0 + mt * kBM);
      tma_load_3d(sm.q[1], &tm_q, &sm.q_full, 64, h, q0 + mt * kBM);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        if (j >= 2) mbar_wait(&sm.kv_empty[st], ((j >> 1) - 1) & 1, prm.status, &sm.abort_flag, 30);
        const int key0 = j * kBN;
        long long bid = prm.block_tables[(long long)seq * prm.max_blocks + key0 / prm.block_size];
        if (bid < 0 || bid >= prm.num_blocks) {
          record_error(prm.status, NVATTN_ERR_OUT_OF_RANGE, 24, bid);
          bid = 0;
        }
        const int row = (int)((long long)prm.layer * prm.n_slots + bid * prm.block_size +
                              key0 % prm.block_size);
        mbar_arrive_expect_tx(&sm.k_full[st], 2 * kHalfBytes);
        tma_load_3d(sm.k[st][0], &tm_k, &sm.k_full[st], 0, kvh, row);
        tma_load_3d(sm.k[st][1], &tm_k, &sm.k_full[st], 64, kvh, row);
        mbar_arrive_expect_tx(&sm.v_full[st], 2 * kHalfBytes);
        tma_load_3d(sm.v[st][0], &tm_v, &sm.v_full[st], 0, kvh, row);
        tma_load_3d(sm.v[st][1], &tm_v, &sm.v_full[st], 64, kvh, row);
      }
      // Drain: the last loads of each stage have landed before the CTA
      // can exit (immediate in normal operation; bounded after an abort).
      for (int j = n_kv - 2 < 0 ? 0 : n_kv - 2; j < n_kv; ++j) {
        mbar_wait(&sm.k_full[j & 1], (j >> 1) & 1, prm.status, 40);
        mbar_wait(&sm.v_full[j & 1], (j >> 1) & 1, prm.status, 41);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16_f32(kBM, kBN, 0, 0);
      constexpr uint32_t idesc_o = umma_idesc_bf16_f32(kBM, kD, 0, 1);
      mbar_wait(&sm.q_full, 0, prm.status, &sm.abort_flag, 31);
      auto issue_s = [&](int j) {
        const int st = j & 1;
        mbar_wait(&sm.k_full[st], (j >> 1) & 1, prm.status, &sm.abort_flag, 32);
        if (j >= 2) mbar_wait(&sm.s_free[st], ((j >> 1) - 1) & 1, prm.status, &sm.abort_flag, 33);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const uint32_t koff = (uint32_t)(k & 3) * 32;
          const uint64_t a = umma_desc_sw128(smem_u32(sm.q[k >> 2]) + koff, 16, 1024);
          const uint64_t b = umma_desc_sw128(smem_u32(sm.k[st][k >> 2]) + koff, 16, 1024);
          umma_bf16(tmem + st * 128, a, b, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&sm.s_full[st]);
      };
      issue_s(0);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        if (j + 1 < n_kv) issue_s(j + 1);
        mbar_wait(&sm.p_full, j & 1, prm.status, &sm.abort_flag, 34);
        mbar_wait(&sm.v_full[st], (j >> 1) & 1, prm.status, &sm.abort_flag, 35);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          const uint64_t a =
              umma_desc_sw128(smem_u32(sm.p[k >> 2]) + (uint32_t)(k & 3) * 32, 16, 1024);
          const uint64_t b =
              umma_desc_sw128(smem_u32(sm.v[st][0]) + (uint32_t)k * 16 * 128, kHalfBytes, 1024);
          umma_bf16(tmem_o, a, b, idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        }
        if constexpr (kSplitP) {
#pragma unroll
          for (int k = 0; k < kBN / 16; ++k) {
            const uint64_t a =
                umma_desc_sw128(smem_u32(sm.p_lo[k >> 2]) + (uint32_t)(k & 3) * 32, 16, 1024);
            const uint64_t b = umma_desc_sw128(smem_u32(sm.v[st][0]) + (uint32_t)k * 16 * 128,
                                               kHalfBytes, 1024);
            umma_bf16(tmem_o, a, b, idesc_o, 1u);
          }
        }
        umma_commit(&sm.o_done);
        umma_commit(&sm.kv_empty[st]);
      }
      // Drain: every MMA has completed before TMEM is released.
      mbar_wait(&sm.o_done, (n_kv - 1) & 1, prm.status, 42);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad+32)
    const int row = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    // Rows past the end of the sequence mimic its last row (never stored).
    const int pos_row = p_first + min(row, rows - 1);
    const float sc = prm.scale_log2;
    float m_used = -INFINITY;
    float l = 0.0f;

    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      mbar_wait(&sm.s_full[st], (j >> 1) & 1, prm.status, &sm.abort_flag, 36);
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_off + st * 128 + c * 32, sr[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.s_free[st]);

      const int key0 = j * kBN;
      const int lim = pos_row - key0;  // keys c <= lim are visible (causal)
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = __uint_as_float(sr[c][i]) * sc;
          x = (c * 32 + i <= lim) ? x : -INFINITY;
          sr[c][i] = __float_as_uint(x);
          mt = fmaxf(mt, x);
        }
      }
      const float m_new = fmaxf(m_used, mt);
      float alpha = 1.0f;
      bool rescale = false;
      if (m_new > m_used + kRescaleThreshold) {
        alpha = fast_exp2(m_used - m_new);
        rescale = j > 0;
        m_used = m_new;
      }
      // P as bf16 pairs; with kSplitP also the bf16 remainder P - bf16(P),
      // so that the two P.V passes together carry ~16 significant bits.
      uint32_t pk[64];
      uint32_t pl[kSplitP ? 64 : 1];
      float rs = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = fast_exp2(__uint_as_float(sr[c][i]) - m_used);
          const float p1 = fast_exp2(__uint_as_float(sr[c][i + 1]) - m_used);
          const uint32_t w = pack_bf16x2(p0, p1);
          pk[c * 16 + i / 2] = w;
          if constexpr (kSplitP) {
            pl[c * 16 + i / 2] = pack_bf16x2(p0 - bf16lo_to_f32(w), p1 - bf16hi_to_f32(w));
            rs += p0 + p1;
          } else {
            rs += bf16lo_to_f32(w) + bf16hi_to_f32(w);
          }
        }
      }
      l = l * alpha + rs;

      if (j > 0) {
        // PV(j-1) has finished: O is stable and the P buffer is free.
        mbar_wait(&sm.o_done, (j - 1) & 1, prm.status, &sm.abort_flag, 37);
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tmem_o + lane_off + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tmem_o + lane_off + c * 32, o);
          }
          tmem_wait_st();
        }
      }
      if (key0 + kBN > ctx) {
        // Keys at or past the context end hold whatever the cache slot
        // contains; zero their V rows so that P=0 never meets a NaN.
        mbar_wait(&sm.v_full[st], (j >> 1) & 1, prm.status, &sm.abort_flag, 38);
        if (key0 + row >= ctx) {
          uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sm.v[st][0]) + row * 128)[c] = z;
            reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sm.v[st][1]) + row * 128)[c] = z;
          }
        }
      }
      // P row -> shared memory, UMMA K-major layout with 128-byte swizzle.
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const int half = c >> 3, cc = c & 7;
        const int off = row * 128 + ((cc ^ (row & 7)) * 16);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sm.p[half]) + off) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        if constexpr (kSplitP)
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sm.p_lo[half]) + off) =
              make_uint4(pl[4 * c], pl[4 * c + 1], pl[4 * c + 2], pl[4 * c + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full);
    }

    // ------------------------------------------------------------ epilogue
    mbar_wait(&sm.o_done, (n_kv - 1) & 1, prm.status, &sm.abort_flag, 39);
    tc_fence_after();
    const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;
    float* dst = prm.out + ((long long)(q0 + mt * kBM + row) * prm.Hq + h) * kD;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      tmem_ld32(tmem_o + lane_off + c * 32, o);
      tmem_wait_ld();
      if (row < rows) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + c * 32 + i) =
              make_float4(__uint_as_float(o[i]) * inv_l, __uint_as_float(o[i + 1]) * inv_l,
                          __uint_as_float(o[i + 2]) * inv_l, __uint_as_float(o[i + 3]) * inv_l);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <bool kSplitP>
nvattn_status launch_variant(dim3 grid, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                             const CUtensorMap& tm_v, const PrefillParams& prm,
                             cudaStream_t stream) {
  const size_t smem = sizeof(PrefillSmem<kSplitP>) + 1024;
  // The attribute is per device; remember which devices have it.
  static unsigned long long attr_set_mask = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NVATTN_ERR_CUDA;
  if (dev >= 64 || !(attr_set_mask & (1ull << dev))) {
    if (cudaFuncSetAttribute(paged_prefill_kernel<kSplitP>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return NVATTN_ERR_CUDA;
    if (dev < 64) attr_set_mask |= 1ull << dev;
  }
  paged_prefill_kernel<kSplitP><<<grid, kThreads, smem, stream>>>(tm_q, tm_k, tm_v, prm);
  return cudaGetLastError() == cudaSuccess ? NVATTN_OK : NVATTN_ERR_CUDA;
}

}  // namespace

nvattn_status launch_paged_prefill(nvattn_handle* h, int layer, int n_seqs, int n_tokens,
                                   const uint16_t* q, const int32_t* cu_q,
                                   const int32_t* q_starts, const int32_t* context_lens,
                                   const int32_t* block_tables, int max_blocks, int max_q_len,
                                   const uint16_t* k_cache, const uint16_t* v_cache, float* out,
                                   cudaStream_t stream) {
  if (max_q_len <= 0) return NVATTN_OK;
  const int Hq = h->cfg.n_q_heads, Hkv = h->cfg.n_kv_heads;
  CUtensorMap tm_q;
  nvattn_status st =
      encode_tensor_map_3d(&tm_q, q, kD, (uint64_t)Hq, (uint64_t)n_tokens, kD * 2,
                           (uint64_t)Hq * kD * 2, 64, 1, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != NVATTN_OK) return st;
  const CUtensorMap* tk = nullptr;
  const CUtensorMap* tv = nullptr;
  st = get_cache_tensor_map(h, k_cache, 64, kBN, CU_TENSOR_MAP_SWIZZLE_128B, &tk);
  if (st != NVATTN_OK) return st;
  st = get_cache_tensor_map(h, v_cache, 64, kBN, CU_TENSOR_MAP_SWIZZLE_128B, &tv);
  if (st != NVATTN_OK) return st;

  PrefillParams prm;
  prm.Hq = Hq;
  prm.Hkv = Hkv;
  prm.G = Hq / Hkv;
  prm.layer = layer;
  prm.block_size = h->cfg.block_size;
  prm.max_blocks = max_blocks;
  prm.n_mtiles = (max_q_len + kBM - 1) / kBM;
  prm.n_slots = h->n_slots;
  prm.num_blocks = h->cfg.num_blocks;
  prm.scale_log2 = h->cfg.scale * kLog2e;
  prm.cu_q = cu_q;
  prm.q_starts = q_starts;
  prm.context_lens = context_lens;
  prm.block_tables = block_tables;
  prm.out = out;
  prm.status = h->status_dev;

  const long long gx = (long long)prm.n_mtiles * prm.G;
  if (gx > 0x7fffffffLL || Hkv > 65535 || n_seqs > 65535) return NVATTN_ERR_UNSUPPORTED;
  dim3 grid((unsigned)gx, Hkv, n_seqs);
  if (h->cfg.prefill_split_p)
    return launch_variant<true>(grid, tm_q, *tk, *tv, prm, stream);
  return launch_variant<false>(grid, tm_q, *tk, *tv, prm, stream);
}

}  // namespace nvattn
