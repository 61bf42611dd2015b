"""CPU tests of nvattn_schedule_prefill_chunks: chunked-prefill admission, the
reference's Scheduler::Schedule prefill loop (src/engine/scheduler.cpp:27-44)
admitting parts of prompts under the step's token budget, the sequence cap
and the free KV blocks (BlockManager::CanAllocate,
src/engine/block_manager.cpp:96-98)."""
import numpy as np
import pytest

import nvattn

BS = 256


def restated(lens, done, held, free_blocks, max_seqs, budget, bs=BS):
    """The admission rule in plain Python (FIFO; stop at the first sequence
    that gets no token)."""
    sel, ends, adds = [], [], []
    used, free_left = 0, free_blocks
    for s in range(len(lens)):
        if len(sel) >= max_seqs or budget - used <= 0:
            break
        want = min(lens[s] - done[s], budget - used, (held[s] + free_left) * bs - done[s])
        if want <= 0:
            break
        end = done[s] + want
        add = max(0, -(-end // bs) - held[s])
        sel.append(s)
        ends.append(end)
        adds.append(add)
        used += want
        free_left -= add
    return sel, ends, adds


def random_state(rng, n):
    lens = rng.integers(1, 20000, n)
    done = np.minimum(rng.integers(0, 20000, n) * (rng.random(n) < 0.4), lens - 1)
    held = -(-done // BS) + rng.integers(0, 2, n) * (done > 0)
    return lens, done, held


@pytest.mark.parametrize("seed", range(40))
def test_matches_restatement(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(0, 40))
    lens, done, held = random_state(rng, n)
    free_blocks = int(rng.integers(0, 400))
    max_seqs = int(rng.integers(1, 64))
    budget = int(rng.integers(0, 20000))
    sel, ends, adds = nvattn.schedule_prefill_chunks(lens, done, held, free_blocks, max_seqs,
                                                     budget)
    want = restated(lens.tolist(), done.tolist(), held.tolist(), free_blocks, max_seqs, budget)
    assert sel.tolist() == want[0]
    assert ends.tolist() == want[1]
    assert adds.tolist() == want[2]
    # invariants: FIFO prefix, budgets, block accounting
    assert sel.tolist() == list(range(len(sel)))
    assert len(sel) <= max_seqs
    assert int((ends - done[sel]).sum()) <= budget
    assert int(adds.sum()) <= free_blocks
    assert ((ends > done[sel]) & (ends <= lens[sel])).all()


def test_whole_prompts_when_everything_fits():
    """With room for every prompt the schedule is the reference's: whole
    prompts, FIFO, one step."""
    lens = np.array([3561, 2795, 2344, 1479, 1615, 658, 781, 571])
    done = np.array([1024, 1024, 1024, 1024, 1024, 512, 512, 512])
    held = -(-done // BS)
    sel, ends, adds = nvattn.schedule_prefill_chunks(lens, done, held, 10**6, 256, 10**6)
    assert sel.tolist() == list(range(8))
    assert ends.tolist() == lens.tolist()
    assert adds.tolist() == (-(-lens // BS) - held).tolist()


def test_long_prompt_is_chunked_and_later_ones_wait():
    # the reference never admits a 10k prompt under a 2048-token budget
    sel, ends, _ = nvattn.schedule_prefill_chunks([10000, 100], [0, 0], [0, 0], 1000, 8, 2048)
    assert sel.tolist() == [0] and ends.tolist() == [2048]
    sel, ends, _ = nvattn.schedule_prefill_chunks([10000, 100], [9000, 0], [36, 0], 1000, 8, 2048)
    assert sel.tolist() == [0, 1] and ends.tolist() == [10000, 100]


def test_blocks_limit_the_chunk_and_stop_admission():
    # 3 free blocks: sequence 0 (holding 2) may grow to 5 blocks = 1280 positions
    sel, ends, adds = nvattn.schedule_prefill_chunks([5000, 10], [500, 0], [2, 0], 3, 8, 4096)
    assert sel.tolist() == [0] and ends.tolist() == [1280] and adds.tolist() == [3]
    # no free block and a block boundary at done: nothing is admitted
    sel, _, _ = nvattn.schedule_prefill_chunks([5000], [512], [2], 0, 8, 4096)
    assert sel.size == 0
    # a partly filled last block still takes tokens without a new block
    sel, ends, adds = nvattn.schedule_prefill_chunks([5000], [500], [2], 0, 8, 4096)
    assert ends.tolist() == [512] and adds.tolist() == [0]


def test_fully_cached_prompt_recomputes_its_last_token():
    sel, ends, adds = nvattn.schedule_prefill_chunks([512], [511], [2], 0, 8, 16)
    assert sel.tolist() == [0] and ends.tolist() == [512] and adds.tolist() == [0]


def test_schedule_runs_every_prompt_token_once():
    """Steps until every prompt is computed: each step's chunks continue
    where the last ended, and every token is computed exactly once."""
    rng = np.random.default_rng(7)
    lens = rng.integers(1, 9000, 30)
    done = np.zeros(30, np.int64)
    held = np.zeros(30, np.int64)
    free = 10**6
    seen = np.zeros(int(lens.sum()), np.int32)
    offs = np.concatenate([[0], np.cumsum(lens)])
    waiting = list(range(30))
    steps = 0
    while waiting:
        idx = np.array(waiting)
        sel, ends, adds = nvattn.schedule_prefill_chunks(lens[idx], done[idx], held[idx], free,
                                                         16, 4096)
        assert sel.size > 0
        for k, e, a in zip(sel, ends, adds):
            s = idx[k]
            seen[offs[s] + done[s]:offs[s] + e] += 1
            done[s] = e
            held[s] += a
            free -= a
        waiting = [s for s in waiting if done[s] < lens[s]]
        steps += 1
    assert (seen == 1).all()
    assert steps == -(-int(lens.sum()) // 4096)  # every step but the last is full


@pytest.mark.parametrize("lens,done,held", [([0], [0], [0]), ([5], [5], [1]), ([5], [-1], [0]),
                                            ([5], [0], [-1])])
def test_invalid_state_is_rejected(lens, done, held):
    with pytest.raises(nvattn.NvattnError) as e:
        nvattn.schedule_prefill_chunks(lens, done, held, 10, 8, 100)
    assert e.value.status == nvattn.ERR_INVALID_ARG
