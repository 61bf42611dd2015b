// chunk_scheduler.cpp -- chunked-prefill admission (host only).
//
// The reference's Scheduler::Schedule (src/engine/scheduler.cpp:27-44) admits
// waiting sequences in FIFO order while the step's token budget
// (max_num_bathced_tokens), the sequence cap (max_num_seqs) and the free KV
// blocks (BlockManager::CanAllocate, block_manager.cpp:96-98) allow, but only
// whole prompts: a prompt longer than the budget is never admitted, and one
// long prompt holds every later one back for a whole step.  This admits part
// of a prompt: each selected sequence gets the next chunk of its remaining
// prompt tokens, as many as the budget and the free blocks allow, and the
// caller runs the chunk as a prefill with num_cached = the tokens already in
// the cache (nvattn_plan_prefill / nvattn_paged_prefill handle unaligned
// chunk starts).  Differences from the reference, on purpose:
//   * the budget is charged with the tokens actually computed (the reference
//     tests the whole SequenceLen against it but adds only the uncached
//     tokens, scheduler.cpp:30-37);
//   * the block check counts only the blocks the chunk adds to those the
//     sequence already holds (the reference asks for all of the sequence's
//     blocks to be free, block_manager.cpp:96-98).
// As in the reference, admission stops at the first sequence that cannot get
// any token (FIFO: no later sequence overtakes it).
#include <stdint.h>

#include <algorithm>

#include "nvattn.h"

extern "C" {

nvattn_status nvattn_schedule_prefill_chunks(int n_waiting, const int64_t* prompt_lens,
                                             const int64_t* done, const int64_t* held_blocks,
                                             int block_size, int64_t free_blocks,
                                             int max_num_seqs, int64_t max_num_batched_tokens,
                                             int32_t* selected, int64_t* chunk_end,
                                             int64_t* new_blocks, int* n_selected) {
  if (n_selected == nullptr) return NVATTN_ERR_INVALID_ARG;
  *n_selected = 0;
  if (n_waiting < 0 || block_size <= 0 || free_blocks < 0 || max_num_seqs < 0 ||
      max_num_batched_tokens < 0)
    return NVATTN_ERR_INVALID_ARG;
  if (n_waiting > 0 && (!prompt_lens || !done || !held_blocks || !selected || !chunk_end ||
                        !new_blocks))
    return NVATTN_ERR_INVALID_ARG;
  for (int s = 0; s < n_waiting; ++s) {
    // a waiting sequence has at least one prompt token left to compute (a
    // fully cached prompt recomputes its last token: done = len - 1)
    if (prompt_lens[s] <= 0 || done[s] < 0 || done[s] >= prompt_lens[s] || held_blocks[s] < 0)
      return NVATTN_ERR_INVALID_ARG;
  }
  int n = 0;
  int64_t used = 0, free_left = free_blocks;
  for (int s = 0; s < n_waiting && n < max_num_seqs; ++s) {
    const int64_t budget_left = max_num_batched_tokens - used;
    if (budget_left <= 0) break;
    int64_t want = std::min(prompt_lens[s] - done[s], budget_left);
    // blocks covering positions [0, done + want) beyond those already held
    const int64_t can_hold = (held_blocks[s] + free_left) * block_size;  // positions
    want = std::min(want, can_hold - done[s]);
    if (want <= 0) break;  // this sequence cannot get a token: FIFO stops here
    const int64_t end = done[s] + want;
    const int64_t need = (end + block_size - 1) / block_size;
    const int64_t add = std::max<int64_t>(0, need - held_blocks[s]);
    selected[n] = s;
    chunk_end[n] = end;
    new_blocks[n] = add;
    ++n;
    used += want;
    free_left -= add;
  }
  *n_selected = n;
  return NVATTN_OK;
}

}  // extern "C"
