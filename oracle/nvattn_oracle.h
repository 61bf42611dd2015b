/*
 * nvattn_oracle.h -- CPU oracle for the paged-attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code; only the test-suite, the smoke check and the CPU-baseline
 * leg of the benchmark use it, as the checker.
 *
 * It restates, in plain C, what nano-vllm.cpp computes on this path:
 *   - src/models/qwen3.cpp:326-353   BuildNorm (ggml_rms_norm + ggml_mul)
 *   - src/models/qwen3.cpp:497-514   q/k norm + NEOX RoPE (ggml_rope_ext)
 *   - src/models/qwen3.cpp:377-405   BuildAttention (ggml_flash_attn_ext,
 *                                    K/V cast F32->F16, scale 1/sqrt(128))
 *   - src/models/qwen3.cpp:407-435   KV cache layout / slot addressing
 *   - src/engine/model_runner.cpp:248-415  StorePrefillKV / LoadHistoryKV /
 *                                    AppendDecodeKV (fp32<->bf16 rows)
 *   - src/engine/model_runner.cpp:219-243  FillVarlenMask (decode concat)
 * The arithmetic itself lives in ggml (github.com/ggml-org/ggml), a git
 * submodule that the reference does not vendor; its pinned commit is not
 * recoverable.  The ggml CPU algorithms used here (rms_norm, rope cache with
 * the YaRN ramp, flash_attn_ext with an F16 V accumulator, fp32<->bf16/f16
 * conversions) are restated from ggml's published source, scalar paths.
 *
 * PARITY AGAINST THE REFERENCE IS UNPINNED: the reference ships no tests,
 * fixtures or golden vectors and cannot be built here (ggml absent).  The
 * oracle is pinned instead by known-answer tests (IEEE conversion edge cases,
 * single-key / constant-key attention, RoPE at position 0) and by the
 * bit-identity of the reference's own concat-all decode algorithm
 * (orc_concat_decode_ggml) with the paged restatement.
 *
 * Two attention modes:
 *   ORC_MODE_TRUTH  fp64 scores/softmax/accumulation on the exact inputs.
 *   ORC_MODE_GGML   the reference's dtype chain: Q f32->f16, K/V bf16->f32->f16,
 *                   f32 scores, f32 online softmax, f16 V accumulator.
 *
 * Build with -ffp-contract=off: every product and sum is rounded separately,
 * as in ggml's scalar code.
 */
#ifndef NVATTN_ORACLE_H
#define NVATTN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_MODE_TRUTH = 0, ORC_MODE_GGML = 1 };

typedef struct orc_params {
  int n_q_heads;      /* Hq */
  int n_kv_heads;     /* Hkv */
  int head_dim;       /* d (128 for Qwen3) */
  int block_size;     /* tokens per KV block (256) */
  int64_t n_slots;    /* num_blocks * block_size, slots per layer */
  float rms_eps;      /* 1e-6 */
  float rope_theta;   /* 1e6 */
  float rope_freq_scale;
  float rope_ext_factor;
  float rope_attn_factor;
  float rope_beta_fast;
  float rope_beta_slow;
  int rope_n_ctx_orig; /* Qwen3Hparams::n_ctx, passed as n_ctx_orig */
  float scale;         /* softmax scale, 1/sqrt(d) */
  int n_threads;       /* 0 = all online cores */
} orc_params;

/* ---- scalar conversions (ggml semantics) ---- */
uint16_t orc_f32_to_bf16(float f);
float orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
void orc_f32_to_bf16_row(const float* x, uint16_t* y, int64_t n);
void orc_bf16_to_f32_row(const uint16_t* x, float* y, int64_t n);

/* ---- RoPE ---- */
void orc_rope_corr_dims(int n_dims, int n_ctx_orig, float freq_base,
                        float beta_fast, float beta_slow, float dims[2]);
/* cos/sin for one position: cache[2*i] = cos(theta_i), cache[2*i+1] = sin. */
void orc_rope_cache(int pos, const orc_params* p, float* cache);
/* Whole table [n_pos][d/2][2] (the library builds the same table itself). */
void orc_rope_table(int n_pos, const orc_params* p, float* table);

/* ---- fused q/k RMSNorm + NEOX RoPE + paged KV store ---- */
/* q [T][Hq][d], k/v [T][Hkv][d] f32; weights bf16 [d]; positions/slots [T].
 * q_out [T][Hq][d] f32 (post norm+rope); k_out nullable [T][Hkv][d] f32.
 * Rows with slot < 0 are not stored. */
void orc_qk_norm_rope_store(const orc_params* p, int layer, int n_tokens,
                            const float* q, const float* k, const float* v,
                            const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                            const int32_t* positions, const int32_t* slots,
                            float* q_out, float* k_out,
                            uint16_t* k_cache, uint16_t* v_cache);

/* ---- paged decode: one query token per sequence, keys [0, context_len) ----
 * q [B][Hq][d] f32, out [B][Hq][d] f32.  block_tables [B][max_blocks].
 * new_k/new_v (nullable, [B][Hkv][d] f32): the newest key (index
 * context_len-1) is taken from these f32 rows instead of the bf16 cache, as
 * in the reference's decode graph concat (model_runner.cpp:116-124,
 * qwen3.cpp:648-661); GGML mode casts them to f16, TRUTH uses them as they
 * are (exact math on the reference's graph values). */
void orc_paged_decode(const orc_params* p, int mode, int layer, int n_seqs,
                      const float* q, const uint16_t* k_cache,
                      const uint16_t* v_cache, const int32_t* block_tables,
                      int max_blocks, const int32_t* context_lens,
                      const float* new_k, const float* new_v, float* out);

/* ---- paged prefill: causal, prefix aware ----
 * Sequence s owns query rows [cu_q[s], cu_q[s+1]) at positions
 * q_start[s] + i; a row at position P attends keys [0, P].  Keys come from the
 * cache through the block table.  new_k/new_v (nullable, [T][Hkv][d] f32):
 * keys at positions >= q_start[s] use these f32 rows (the reference's graph
 * rows; GGML mode casts them to f16, TRUTH uses them as they are). */
void orc_paged_prefill(const orc_params* p, int mode, int layer, int n_seqs,
                       const float* q, const int32_t* cu_q,
                       const int32_t* q_start, const int32_t* context_lens,
                       const int32_t* block_tables, int max_blocks,
                       const uint16_t* k_cache, const uint16_t* v_cache,
                       const float* new_k, const float* new_v, float* out);

/* ---- the reference's own decode algorithm (GGML mode only) ----
 * Gathers every sequence's history (context_len-1 rows) into one
 * concatenated K/V, appends the new rows after all histories, pads to 256 and
 * runs masked attention over the whole buffer for each query row
 * (model_runner.cpp:85-124,219-243,298-376; qwen3.cpp:573-662).
 * O(B * sum(L)); small cases only. */
void orc_concat_decode_ggml(const orc_params* p, int layer, int n_seqs,
                            const float* q, const uint16_t* k_cache,
                            const uint16_t* v_cache,
                            const int32_t* block_tables, int max_blocks,
                            const int32_t* context_lens, const float* new_k,
                            const float* new_v, float* out);

/* ---- the reference's own prefill attention (GGML mode only) ----
 * The batch's new tokens concatenated (sequence s owns rows [cu_q[s],
 * cu_q[s+1])), their f32 K/V zero-padded to a multiple of 256 and cast to
 * F16, and masked attention over the whole buffer with FillCausalMask's
 * block-diagonal causal mask (model_runner.cpp:188-217; qwen3.cpp:461-531,
 * 377-405).  A cached prefix is not attended: the reference's prefill sees
 * only the batch's tokens.  O(T * PAD(T, 256)) mask work per kv head. */
void orc_concat_prefill_ggml(const orc_params* p, int n_seqs, const int32_t* cu_q,
                             const float* q, const float* new_k, const float* new_v,
                             float* out);

/* ---- token sampling (ModelRunner::Sample, model_runner.cpp:417-489) ----
 * Row s of logits (n_vocab f32 at logits + s*row_stride):
 *  - penalty[s] > 1: every occurrence of a history id t in [0, n_vocab)
 *    (sequence s's ids at [history_offsets[s], history_offsets[s+1]), prompt
 *    then completion) applies v = v < 0 ? v*penalty : v/penalty once more to
 *    a copy of the row (:428-446);
 *  - temperature < 1e-6: the first index of the maximum by a strict '>' scan
 *    from index 0 (:448-456);
 *  - otherwise: m = the same scan's maximum, p_i = expf((x_i - m)/t), S the
 *    sequential float sum, r = u*S (std::uniform_real_distribution<float>(0, S)
 *    = S * generate_canonical<float>), and the first i whose sequential float
 *    prefix sum is >= r, else n_vocab-1 (:457-481).  u = uniforms[s]. */
void orc_penalize_rows(int n_seqs, int n_vocab, const float* logits, int64_t row_stride,
                       const float* penalties, const int32_t* history,
                       const int64_t* history_offsets, float* out);
void orc_sample(int n_seqs, int n_vocab, const float* logits, int64_t row_stride,
                const float* temperatures, const float* penalties, const int32_t* history,
                const int64_t* history_offsets, const float* uniforms, int32_t* tokens);

/* libstdc++'s generate_canonical<float, 24> over one 32-bit mt19937 output:
 * float(x) / 2^32, and the largest float below 1 when that rounds to 1. */
float orc_canonical_float(uint32_t x);

#ifdef __cplusplus
}
#endif
#endif /* NVATTN_ORACLE_H */
