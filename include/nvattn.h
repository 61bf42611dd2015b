/*
 * nvattn.h -- C ABI of libnvattn, the B200 (sm_100a) paged-attention hot path
 * for nano-vllm.cpp.
 *
 * The library replaces, inside ModelRunner::Run (src/engine/model_runner.cpp:25),
 * the host-side KV gather / store loops and the ggml attention node:
 *
 *   reference (nano-vllm.cpp)                              -> libnvattn
 *   ---------------------------------------------------------------------------
 *   Qwen3Model::Qwen3Model KV alloc (qwen3.cpp:186-213)   -> caller allocates the
 *       [n_layer][num_blocks*block_size][n_kv_heads][head_dim] BF16 K and V
 *       buffers (same layout); nvattn_create sizes only the workspace.
 *   BuildNorm + ggml_rope_ext on q/k (qwen3.cpp:497-514, 627-641) and
 *   StorePrefillKV / AppendDecodeKV + WriteKVToCache
 *       (model_runner.cpp:248-296, 380-415; qwen3.cpp:411-422)
 *                                                          -> nvattn_kv_store_qk_norm_rope
 *   LoadHistoryKV + ReadKVFromCache + FillVarlenMask + decode concat +
 *   BuildAttention (model_runner.cpp:219-243, 300-376; qwen3.cpp:424-435,
 *   648-662, 377-405)                                      -> nvattn_paged_decode
 *   FillCausalMask + prefill pad/permute + BuildAttention
 *       (model_runner.cpp:188-217; qwen3.cpp:515-533, 377-405)
 *                                                          -> nvattn_paged_prefill
 *   PrepareInputs position/slot derivation (model_runner.cpp:138-186,
 *   286-288, 332-333, 402-405)                              -> nvattn_plan_prefill /
 *                                                             nvattn_plan_decode
 *
 * Conventions:
 *   - Every pointer argument named *_dev is device memory on the handle's
 *     device; every other pointer is host memory.  No pointer is retained
 *     after a call returns.
 *   - All device work is ordered on the stream argument (NULL = legacy
 *     default stream).  Calls return after launching; they do not
 *     synchronise.  Errors detected by the kernels (a block id or slot out of
 *     range, a bounded wait that ran out) are recorded in a device status word
 *     and reported by nvattn_get_error.
 *   - No C++ exception crosses this interface.  A handle is not thread-safe;
 *     distinct handles are independent.
 *   - bf16 values are passed as uint16_t bit patterns.
 */
#ifndef NVATTN_H
#define NVATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NVATTN_API __attribute__((visibility("default")))
#else
#define NVATTN_API
#endif

#define NVATTN_VERSION_MAJOR 0
#define NVATTN_VERSION_MINOR 5

typedef enum nvattn_status {
  NVATTN_OK = 0,
  NVATTN_ERR_INVALID_ARG = 1,  /* bad pointer, size or shape */
  NVATTN_ERR_OUT_OF_RANGE = 2, /* a block id / slot outside the cache */
  NVATTN_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed */
  NVATTN_ERR_TIMEOUT = 4,      /* a bounded device wait ran out */
  NVATTN_ERR_UNSUPPORTED = 5,  /* shape not built (head_dim != 128, ...) */
  NVATTN_ERR_NO_MEMORY = 6,    /* workspace allocation failed */
  NVATTN_ERR_SCRATCH_LIMIT = 7 /* nvattn_paged_decode_noalloc: the call needs
                                  more split-KV scratch than its fixed array */
} nvattn_status;

typedef enum nvattn_dtype {
  NVATTN_DTYPE_F32 = 0,
  NVATTN_DTYPE_BF16 = 1,
  NVATTN_DTYPE_F16 = 2
} nvattn_dtype;

/* Same type as cudaStream_t, without pulling in CUDA headers. */
typedef struct CUstream_st* nvattn_stream_t;

typedef struct nvattn_config {
  int n_layer;          /* Qwen3Hparams::n_layer (qwen3.h:32) */
  int n_q_heads;        /* query heads served by this handle */
  int n_kv_heads;       /* KV heads held in this handle's cache */
  int head_dim;         /* 128 (only value built) */
  int block_size;       /* Config::kvcache_block_size, 256 (only value built) */
  int64_t num_blocks;   /* physical blocks per layer */
  float rms_eps;        /* 1e-6 */
  float rope_theta;     /* rope_freq_base, 1e6 */
  float rope_freq_scale;  /* 1 */
  float rope_ext_factor;  /* 1 */
  float rope_attn_factor; /* 1 */
  float rope_beta_fast;   /* 32 */
  float rope_beta_slow;   /* 1 */
  int rope_n_ctx_orig;  /* n_ctx passed to ggml_rope_ext (40960 for Qwen3) */
  float scale;          /* softmax scale, 1/sqrt(head_dim) */
  int max_position;     /* RoPE table covers positions [0, max_position) */
  int max_seqs;         /* largest n_seqs of any call */
  int max_context;      /* largest context length of any call */
  int device;           /* CUDA device ordinal */
} nvattn_config;

typedef struct nvattn_handle nvattn_handle;

/* ---- lifetime --------------------------------------------------------- */

/* Qwen3-0.6B defaults (Qwen3Hparams, qwen3.h:30-56; Config, config.h:5-15). */
NVATTN_API void nvattn_config_init_qwen3(nvattn_config* cfg);

/* Validates cfg, builds the RoPE cos/sin table (ggml's float recurrence,
 * computed on the host once and copied to the device) and allocates the
 * split-KV workspace and status word.  Replaces the KV/backend set-up of
 * Qwen3Model::Qwen3Model (qwen3.cpp:99-108, 186-213), whose failures throw;
 * here they return a status. */
NVATTN_API nvattn_status nvattn_create(const nvattn_config* cfg, nvattn_handle** out);
NVATTN_API nvattn_status nvattn_destroy(nvattn_handle* h);

NVATTN_API const char* nvattn_status_string(nvattn_status s);
NVATTN_API void nvattn_version(int* major, int* minor);

/* Synchronises the handle's device, returns the first error recorded by a
 * kernel since the last call (NVATTN_OK if none) and clears it.  *detail
 * (nullable) receives the offending value (block id, slot or wait site).
 * Reporting NVATTN_ERR_TIMEOUT also re-arms the handle's split tickets and
 * prefill work counter, and ends its peer-memory gather (later
 * nvattn_paged_decode_step_gather / nvattn_gather_read calls return
 * NVATTN_ERR_INVALID_ARG; every rank destroys its handle and starts over). */
NVATTN_API nvattn_status nvattn_get_error(nvattn_handle* h, int64_t* detail);

/* ---- host-side planning (no device work) ------------------------------- */

/* ModelRunner::PrepareInputs for a prefill batch (model_runner.cpp:138-186)
 * plus the slot derivation of StorePrefillKV (:286-288).
 * Inputs per sequence s: seq_lens[s] (Sequence::SequenceLen),
 * num_cached[s] (Sequence::GetNumCachedTokens), block_tables [n_seqs][max_blocks]
 * (Sequence::block_table_).  Outputs: cu_q_lens[n_seqs+1], q_starts[n_seqs],
 * context_lens[n_seqs], and for each of the cu_q_lens[n_seqs] new tokens
 * positions[] and slot_mapping[] (capacity max_tokens).
 * Returns INVALID_ARG if a sequence has no new token or too few blocks. */
NVATTN_API nvattn_status nvattn_plan_prefill(int n_seqs, const int64_t* seq_lens,
                                  const int64_t* num_cached,
                                  const int32_t* block_tables, int max_blocks,
                                  int block_size, int max_tokens,
                                  int32_t* cu_q_lens, int32_t* q_starts,
                                  int32_t* context_lens, int32_t* positions,
                                  int32_t* slot_mapping);

/* Decode batch: one new token per sequence at position seq_lens[s]-1
 * (model_runner.cpp:161-165, 402-405). */
NVATTN_API nvattn_status nvattn_plan_decode(int n_seqs, const int64_t* seq_lens,
                                 const int32_t* block_tables, int max_blocks,
                                 int block_size, int32_t* context_lens,
                                 int32_t* positions, int32_t* slot_mapping);

/* Device-side planners: the same outputs as nvattn_plan_prefill /
 * nvattn_plan_decode (bit for bit), computed by kernels on `stream` from
 * device-resident sequence lengths and block tables, for an engine that keeps
 * its block tables on the GPU (the per-step H2D copy of positions, slots and
 * tables then disappears).  Replaces the same PrepareInputs derivation
 * (model_runner.cpp:138-186) over BlockManager's tables
 * (block_manager.cpp:96-184; Sequence, sequence.h:63-88); block_size comes
 * from the handle.  Invalid input (seq_lens[s] <= 0, num_cached[s] outside
 * [0, seq_lens[s]], more tokens than max_tokens, a position beyond
 * max_blocks) is recorded as NVATTN_ERR_INVALID_ARG, a negative block id for
 * a position as NVATTN_ERR_OUT_OF_RANGE, each with detail = the sequence
 * index, and read with nvattn_get_error; the outputs are then unspecified.
 * The caller knows the token count on the host (the scheduler's sum of
 * seq_lens - num_cached, with 1 for a fully cached prompt), as the attention
 * calls need it; max_tokens bounds the positions/slot_mapping arrays. */
NVATTN_API nvattn_status nvattn_plan_prefill_device(
    nvattn_handle* h, int n_seqs, const int64_t* seq_lens_dev, const int64_t* num_cached_dev,
    const int32_t* block_tables_dev, int max_blocks, int max_tokens, int32_t* cu_q_lens_dev,
    int32_t* q_starts_dev, int32_t* context_lens_dev, int32_t* positions_dev,
    int32_t* slot_mapping_dev, nvattn_stream_t stream);

NVATTN_API nvattn_status nvattn_plan_decode_device(
    nvattn_handle* h, int n_seqs, const int64_t* seq_lens_dev, const int32_t* block_tables_dev,
    int max_blocks, int32_t* context_lens_dev, int32_t* positions_dev,
    int32_t* slot_mapping_dev, nvattn_stream_t stream);

/* ---- chunked-prefill admission (host only) -------------------------------- */

/* One step's prefill admission with chunking: the reference's
 * Scheduler::Schedule prefill loop (scheduler.cpp:27-44) admitting parts of
 * prompts.  Waiting sequences s = 0..n_waiting-1 in FIFO order, each with
 * prompt_lens[s] tokens of which done[s] (0 <= done < len; a fully cached
 * prompt passes len - 1) are already in the KV cache and held_blocks[s] KV
 * blocks already allocated.  Each admitted sequence gets the chunk
 * [done[s], chunk_end[k]) -- as many of its remaining tokens as the step's
 * remaining token budget (max_num_batched_tokens, charged with computed
 * tokens) and the free blocks (free_blocks, charged with new_blocks[k] =
 * blocks the chunk adds) allow -- at most max_num_seqs sequences; admission
 * stops at the first sequence that gets no token.  selected[k] = the
 * sequence index of the k-th admitted sequence, *n_selected = k's count.
 * Run each chunk as a prefill with num_cached = done[s] and seq_len =
 * chunk_end[k]; the chunked outputs equal the one-shot prefill's bit for bit.
 * Host only: no device, no handle. */
NVATTN_API nvattn_status nvattn_schedule_prefill_chunks(
    int n_waiting, const int64_t* prompt_lens, const int64_t* done, const int64_t* held_blocks,
    int block_size, int64_t free_blocks, int max_num_seqs, int64_t max_num_batched_tokens,
    int32_t* selected, int64_t* chunk_end, int64_t* new_blocks, int* n_selected);

/* ---- token sampling ------------------------------------------------------ */

/* Next-token sampling for a batch: ModelRunner::Sample
 * (model_runner.cpp:417-489) on the device.  Row s of the logits is n_vocab
 * f32 values at logits_dev + s*row_stride (elements).  Per row:
 *  - penalties_dev[s] > 1: each occurrence of an id t in [0, n_vocab) among
 *    the row's history ids -- history_dev[history_offsets_dev[s] ..
 *    history_offsets_dev[s+1]), the prompt then the completion, int32 ids,
 *    int64 offsets -- applies v = v < 0 ? v*p : v/p to logit t once more,
 *    bit for bit as the reference does; other ids are skipped.  Both
 *    history pointers may be NULL: no penalty.
 *  - temperatures_dev[s] < 1e-6: the first index of the maximum (bit-exact);
 *  - otherwise: inverse-CDF sampling of softmax(x/t) with the draw
 *    uniforms_dev[s] in [0,1) -- the generate_canonical<float> value that
 *    the reference's std::uniform_real_distribution<float>(0, sum) scales by
 *    the sum.  The token is the first whose running probability sum reaches
 *    u * sum, n_vocab-1 if none does (a NaN or infinite logit, as in the
 *    reference).  Probabilities are within a few ulp of the reference's.
 * tokens_dev[s] receives the token.  A draw outside [0,1) or unusable
 * history offsets (decreasing, negative, or 2^30 ids or more for one
 * sequence) are recorded as NVATTN_ERR_INVALID_ARG (detail = s).
 * n_vocab <= 2,097,152.  The first call for a vocabulary size allocates the
 * handle's sampler workspace (history count tables of about 4.5 bytes per id
 * for each of max_seqs rows, plus 64 KiB of piece summaries per row; nothing
 * in it carries over between calls) and cannot be captured
 * (NVATTN_ERR_UNSUPPORTED while the stream captures); later calls are
 * capturable. */
NVATTN_API nvattn_status nvattn_sample(
    nvattn_handle* h, int n_seqs, int n_vocab, const float* logits_dev, int64_t row_stride,
    const float* temperatures_dev, const float* penalties_dev, const int32_t* history_dev,
    const int64_t* history_offsets_dev, const float* uniforms_dev, int32_t* tokens_dev,
    nvattn_stream_t stream);

/* ---- device kernels ----------------------------------------------------- */

/* Fused per-head q/k RMSNorm (weight = q_norm / k_norm), NEOX RoPE at
 * positions[t], and the BF16 store of K (normed, rotated) and V (raw) into
 * layer `layer` of the paged cache at slot_mapping[t] (slot < 0: not stored).
 *   q_dev   [n_tokens][n_q_heads][head_dim]  f32
 *   k_dev, v_dev [n_tokens][n_kv_heads][head_dim] f32
 *   q_norm_w_dev, k_norm_w_dev [head_dim] bf16
 *   q_out_dev [n_tokens][n_q_heads][head_dim] in q_out_dtype (may alias q_dev
 *            when f32); f16 is the query type nvattn_paged_prefill takes
 *            (round to nearest even, as ggml_fp32_to_fp16, which the
 *            reference's flash attention applies to Q)
 *   k_cache_dev, v_cache_dev: cache base (all layers).
 * The stored K/V bytes equal ggml_fp32_to_bf16_row of the reference's f32
 * graph outputs (round to nearest even). */
NVATTN_API nvattn_status nvattn_kv_store_qk_norm_rope(
    nvattn_handle* h, int layer, int n_tokens, const float* q_dev,
    const float* k_dev, const float* v_dev, const uint16_t* q_norm_w_dev,
    const uint16_t* k_norm_w_dev, const int32_t* positions_dev,
    const int32_t* slot_mapping_dev, void* q_out_dev, nvattn_dtype q_out_dtype,
    uint16_t* k_cache_dev, uint16_t* v_cache_dev, nvattn_stream_t stream);

/* nvattn_kv_store_qk_norm_rope that also writes the step's own K rows
 * (normed, rotated) and V rows as f16 -- the reference's F16 cast of its
 * graph's f32 rows (ggml_cast in BuildAttention, qwen3.cpp:388-393; round to
 * nearest even) -- for nvattn_paged_prefill_rows:
 *   k_rows_f16_dev, v_rows_f16_dev [n_tokens][n_kv_heads][head_dim] f16
 * (also for rows whose slot is < 0).  Everything else as
 * nvattn_kv_store_qk_norm_rope. */
NVATTN_API nvattn_status nvattn_kv_store_qk_norm_rope_rows(
    nvattn_handle* h, int layer, int n_tokens, const float* q_dev,
    const float* k_dev, const float* v_dev, const uint16_t* q_norm_w_dev,
    const uint16_t* k_norm_w_dev, const int32_t* positions_dev,
    const int32_t* slot_mapping_dev, void* q_out_dev, nvattn_dtype q_out_dtype,
    uint16_t* k_cache_dev, uint16_t* v_cache_dev, uint16_t* k_rows_f16_dev,
    uint16_t* v_rows_f16_dev, nvattn_stream_t stream);

/* Paged GQA decode: for each sequence s, one query row per q head attends
 * keys [0, context_lens[s]) of layer `layer`, read through
 * block_tables[s][t / block_size].  The new token's K/V must already be in
 * the cache (nvattn_kv_store_qk_norm_rope first).
 *   q_dev   [n_seqs][n_q_heads][head_dim] f32
 *   out_dev [n_seqs][n_q_heads][head_dim] f32
 * max_context_len: host-side upper bound of context_lens (sizes the grid).
 * n_seqs <= 65535 (INVALID_ARG above).
 * Split-KV partial results go to the handle's workspace. */
NVATTN_API nvattn_status nvattn_paged_decode(
    nvattn_handle* h, int layer, int n_seqs, const float* q_dev,
    const uint16_t* k_cache_dev, const uint16_t* v_cache_dev,
    const int32_t* block_tables_dev, int max_blocks,
    const int32_t* context_lens_dev, int max_context_len, float* out_dev,
    nvattn_stream_t stream);

/* One decode step: nvattn_kv_store_qk_norm_rope of the step's
 * new token (one per sequence) followed by nvattn_paged_decode -- the
 * reference's q/k RMSNorm + NEOX RoPE of the decode graph (qwen3.cpp:619-641),
 * AppendDecodeKV (model_runner.cpp:380-415) and the decode attention -- with
 * the same results bit for bit (the stored K/V rows and the output rows):
 *   q_dev        [n_seqs][n_q_heads][head_dim] f32, the raw q projection
 *                (read only; the normed, rotated q stays on chip)
 *   k_dev, v_dev [n_seqs][n_kv_heads][head_dim] f32, the new token's rows
 *   q_norm_w_dev, k_norm_w_dev, positions_dev: as nvattn_kv_store_qk_norm_rope
 *   slot_mapping_dev[s]: the cache slot of position context_lens[s] - 1
 *                (what nvattn_plan_decode produces; -1 stores nothing); any
 *                other slot is still written but reported as
 *                NVATTN_ERR_INVALID_ARG, since the attention reads position
 *                context_lens[s] - 1 through the block table
 *   the rest as nvattn_paged_decode.
 * Batches whose decode grid (n_seqs x n_kv_heads x the splits of
 * max_context_len) stays within 32 CTAs per SM run as ONE launch: every CTA
 * norms and rotates its own query rows, and the CTA whose key range holds the
 * new token stores its K/V row and reads the tile that holds it only
 * afterwards (no other CTA reads that position).  Larger grids run as two
 * launches -- the KV store writing the normed q once per head into the
 * handle's workspace, then the decode -- because there the CTAs' own query
 * paths cost more than the store launch; the results are the same bits and
 * the same errors are reported either way (the decode launch checks the
 * slot).  nvattn_paged_decode_step_launches tells which form a batch takes. */
NVATTN_API nvattn_status nvattn_paged_decode_step(
    nvattn_handle* h, int layer, int n_seqs, const float* q_dev,
    const float* k_dev, const float* v_dev, const uint16_t* q_norm_w_dev,
    const uint16_t* k_norm_w_dev, const int32_t* positions_dev,
    const int32_t* slot_mapping_dev, uint16_t* k_cache_dev, uint16_t* v_cache_dev,
    const int32_t* block_tables_dev, int max_blocks, const int32_t* context_lens_dev,
    int max_context_len, float* out_dev, nvattn_stream_t stream);

/* The number of kernel launches nvattn_paged_decode_step makes for a batch
 * of n_seqs sequences and this max_context_len: 1 (the fused kernel), 2 (the
 * KV store, then the decode) or 0 (n_seqs == 0).  Host-only; launches
 * nothing.  NVATTN_ERR_INVALID_ARG for the arguments nvattn_paged_decode_step
 * would reject (n_seqs above the handle's max_seqs, max_context_len outside
 * [0, max_context]). */
NVATTN_API nvattn_status nvattn_paged_decode_step_launches(const nvattn_handle* h, int n_seqs,
                                                           int max_context_len, int* launches);

/* ---- The decode step with the all-gather of head outputs over peer memory ----
 * KV-head sharding across n_ranks GPUs of one node (one process and one
 * handle per GPU, every handle created with the same max_seqs; the ranks'
 * launches wait on one another, so no two ranks share a GPU): rank r's
 * output rows [n_seqs][n_q_heads][head_dim] are the heads of its kv-head
 * share, and o_proj needs every rank's rows.  Instead of a separate
 * all-gather, the decode launch stores each output row into every rank's
 * gathered buffer directly (plain peer-to-peer stores over NVLink, as each
 * row is finished); the last CTA of that launch to write final rows then
 * releases this rank's rows to all ranks and waits -- bounded,
 * NVATTN_ERR_TIMEOUT after ~2 s -- until every rank's rows of the step have
 * arrived, so the launch ends with the whole step gathered.  After a
 * recorded timeout the handle's later launches skip their work and release
 * nothing, so the other ranks time out as well.
 *   nvattn_gather_init: allocates this rank's gathered buffer
 *     [2][n_ranks][max_seqs][n_q_heads][head_dim] f32 (two step parities)
 *     and a completion counter, and writes their CUDA IPC handle
 *     (NVATTN_IPC_HANDLE_BYTES bytes) to ipc_handle_out.
 *   nvattn_gather_connect: ipc_handles = every rank's handle, rank order
 *     (n_ranks x NVATTN_IPC_HANDLE_BYTES bytes, exchanged by the caller);
 *     maps every peer's buffer on this device.  NVATTN_ERR_INVALID_ARG if a
 *     handle's rank count, rank or buffer shape differs from this rank's.
 *     All ranks connect before any rank takes a gather step, and no rank
 *     destroys its handle while another may still store to it.
 *   nvattn_paged_decode_step_gather: nvattn_paged_decode_step (same
 *     arguments and results) plus the gather of its output rows; a
 *     collective -- every rank calls it the same number of times, with the
 *     same n_seqs.  Step s (counted per handle from 0) fills parity s & 1.
 *     A step with n_seqs = 0 has no decode launch; a one-thread launch
 *     releases and waits in its place.
 *   nvattn_gather_read: copies step `step`'s gathered rows into out_dev
 *     [n_ranks][n_seqs][n_q_heads][head_dim] on the stream -- rank-major, as
 *     an all-gather of the ranks' outputs.  Only the latest step this handle
 *     took can be read, and only before its next gather step: once every
 *     rank has released step s, a peer may already run step s + 1 and store
 *     into the other parity, so step s - 1's rows are no longer stable;
 *     step s's parity is not written again until this rank has released
 *     step s + 1, which stream order puts after the read.  Consumers that
 *     read the gathered buffer directly follow the same rule.
 *     NVATTN_ERR_INVALID_ARG for any other step. */
#define NVATTN_IPC_HANDLE_BYTES 128
NVATTN_API nvattn_status nvattn_gather_init(nvattn_handle* h, int n_ranks, int rank,
                                            void* ipc_handle_out);
NVATTN_API nvattn_status nvattn_gather_connect(nvattn_handle* h, const void* ipc_handles);
NVATTN_API nvattn_status nvattn_paged_decode_step_gather(
    nvattn_handle* h, int layer, int n_seqs, const float* q_dev,
    const float* k_dev, const float* v_dev, const uint16_t* q_norm_w_dev,
    const uint16_t* k_norm_w_dev, const int32_t* positions_dev,
    const int32_t* slot_mapping_dev, uint16_t* k_cache_dev, uint16_t* v_cache_dev,
    const int32_t* block_tables_dev, int max_blocks, const int32_t* context_lens_dev,
    int max_context_len, float* out_dev, nvattn_stream_t stream);
NVATTN_API nvattn_status nvattn_gather_read(nvattn_handle* h, unsigned step, int n_seqs,
                                            float* out_dev, nvattn_stream_t stream);

/* Causal paged prefill, prefix aware (also serves chunked prefill): sequence
 * s owns query rows [cu_q_lens[s], cu_q_lens[s+1]) at positions
 * q_starts[s] + i; a row at position P attends keys [0, P] of layer `layer`
 * through the block table.  The rows' own K/V must already be stored.
 *   q_dev   [n_tokens][n_q_heads][head_dim] f16 (q_out of
 *           nvattn_kv_store_qk_norm_rope with NVATTN_DTYPE_F16)
 * Scores multiply f16 Q with the cache's K converted to f16 and P.V uses f16
 * probabilities and V -- the F16 Q/K/V of the reference's
 * ggml_flash_attn_ext -- with f32 accumulation.
 *   out_dev [n_tokens][n_q_heads][head_dim] f32
 * max_q_len: host-side upper bound of the per-sequence query count.
 * A sequence whose rows [cu_q_lens[s], cu_q_lens[s+1]) do not lie inside
 * [0, n_tokens) is skipped and reported as NVATTN_ERR_OUT_OF_RANGE (detail =
 * cu_q_lens[s+1]); nothing is read or written for it.
 * The CTAs take their work from a counter in the handle's workspace, so two
 * prefill launches on one handle must not run concurrently (issue them on
 * one stream, as the split-KV workspace of nvattn_paged_decode also needs). */
NVATTN_API nvattn_status nvattn_paged_prefill(
    nvattn_handle* h, int layer, int n_seqs, int n_tokens,
    const uint16_t* q_dev, const int32_t* cu_q_lens_dev,
    const int32_t* q_starts_dev, const int32_t* context_lens_dev,
    const int32_t* block_tables_dev, int max_blocks, int max_q_len,
    const uint16_t* k_cache_dev, const uint16_t* v_cache_dev, float* out_dev,
    nvattn_stream_t stream);

/* nvattn_paged_prefill where the keys and values at or past each sequence's
 * cached prefix (positions q_starts[s] .. q_starts[s] + its row count - 1)
 * are the step's own rows as nvattn_kv_store_qk_norm_rope_rows wrote them in
 * f16 (row cu_q_lens[s] + position - q_starts[s]), while the prefix comes
 * from the BF16 cache.  This is the reference's prefill attention
 * (qwen3.cpp:461-533, model_runner.cpp:188-217), which attends the batch's
 * own graph rows cast to F16, extended to a cached prefix; the plain
 * nvattn_paged_prefill attends the step's rows as the BF16 cache holds them
 * (what every later step reads), which moves a prompt's outputs by the
 * cache's rounding (~2e-3 mean-rel on a prompt without prefix). */
NVATTN_API nvattn_status nvattn_paged_prefill_rows(
    nvattn_handle* h, int layer, int n_seqs, int n_tokens,
    const uint16_t* q_dev, const int32_t* cu_q_lens_dev,
    const int32_t* q_starts_dev, const int32_t* context_lens_dev,
    const int32_t* block_tables_dev, int max_blocks, int max_q_len,
    const uint16_t* k_cache_dev, const uint16_t* v_cache_dev,
    const uint16_t* k_rows_f16_dev, const uint16_t* v_rows_f16_dev, float* out_dev,
    nvattn_stream_t stream);

/* ---- decode without any allocation -------------------------------------- */

/* Where a kernel records the first error it meets (device memory owned by
 * the caller; zero it before use).  Same meaning as nvattn_get_error's
 * status and detail. */
typedef struct nvattn_device_status {
  int32_t code;   /* nvattn_status */
  int32_t site;   /* which check fired */
  int64_t detail; /* the offending value */
} nvattn_device_status;

/* No counterpart in the reference: an extra entry point of this library.
 *
 * nvattn_paged_decode for callers that cannot allocate device memory: an
 * engine that has already handed nearly all of the GPU to its KV cache (the
 * reference sizes the cache from gpu_memory_utilization = 0.9), or a host
 * that may not call cudaMalloc while serving a step, where an allocation
 * could fail or synchronise the device.  It needs no handle and allocates
 * nothing: cfg supplies the shapes (as for nvattn_create), the caller passes
 * every input and output, and the split-KV partial results go to a fixed
 * 32 MiB device array inside the library (held by every GPU that loads the
 * library until the process exits).  A call whose partials do not fit
 * (n_seqs * n_q_heads * splits * 520 bytes plus n_seqs * n_kv_heads * 4
 * bytes of split counters > 32 MiB, splits chosen as for a handle created
 * from cfg) returns NVATTN_ERR_SCRATCH_LIMIT; a call that splits clears the
 * counters first (cudaMemsetAsync on the stream, no allocation).
 * n_seqs <= 65535 (INVALID_ARG above).
 * It runs on the caller's current device, which must be cfg->device.  The
 * first call on a device looks up the array's device address and the SM
 * count (once per device, safe when several threads make that first call
 * together); make that first call before any stream capture.  All calls share the one array and
 * it keeps the last call's contents: calls whose kernels overlap on the GPU
 * (other streams, other threads) race on it, so serialise them.
 * status_dev (nullable) receives errors the kernels detect; results equal
 * nvattn_paged_decode's for the same cfg. */
NVATTN_API nvattn_status nvattn_paged_decode_noalloc(
    const nvattn_config* cfg, int layer, int n_seqs, const float* q_dev,
    const uint16_t* k_cache_dev, const uint16_t* v_cache_dev,
    const int32_t* block_tables_dev, int max_blocks,
    const int32_t* context_lens_dev, int max_context_len, float* out_dev,
    nvattn_device_status* status_dev, nvattn_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* NVATTN_H */
