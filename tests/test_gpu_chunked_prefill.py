"""Chunked prefill driven by nvattn_schedule_prefill_chunks equals one-shot
prefill bit for bit: each chunk runs as a prefill with num_cached = the tokens
already in the cache, and a row attends the same keys in the same key-tile
order whichever step computes it (rows are independent in the kernel:
per-row max, sum and lazy rescale)."""
import numpy as np
import pytest

import cases
import nvattn
import oracle as O
from gpu_util import dev, handle, prefill_q

pytestmark = pytest.mark.gpu


def prefill_rows(h, c, seqs, starts, ends):
    """Prefill of tokens [starts[i], ends[i]) of sequences seqs[i] of case c;
    returns {sequence: output rows}."""
    import torch
    q_rows, cu = [], [0]
    for s, a, b in zip(seqs, starts, ends):
        base = int(c.cu_q[s]) + (a - int(c.q_starts[s]))
        q_rows.append(c.q[base:base + (b - a)])
        cu.append(cu[-1] + (b - a))
    q = np.concatenate(q_rows)
    out = torch.full((q.shape[0], c.Hq, 128), float("nan"), device="cuda")
    bt = np.ascontiguousarray(c.block_tables[np.asarray(seqs)])
    h.prefill(c.layer, prefill_q(q), dev(np.asarray(cu, np.int32)),
              dev(np.asarray(starts, np.int32)), dev(np.asarray(ends, np.int32)), dev(bt),
              int(max(b - a for a, b in zip(starts, ends))), dev(c.cache.k), dev(c.cache.v), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    return {s: got[cu[i]:cu[i + 1]] for i, s in enumerate(seqs)}


@pytest.mark.parametrize("Hq,Hkv,budget", [(16, 8, 700), (64, 8, 1500), (8, 8, 300)])
def test_chunked_equals_one_shot(cuda, Hq, Hkv, budget):
    lens = [3000, 129, 2600, 1, 900, 1537]
    cached = [0, 0, 512, 0, 256, 1536]  # prefix hits, a one-token prompt, a fully cached tail
    c = cases.prefill_case(Hq * 5 + budget, Hq, Hkv, lens, cached)
    n = len(lens)
    h = handle(Hq, Hkv, c.cache.num_blocks, n_layer=c.cache.n_layer, max_seqs=n)
    try:
        one = prefill_rows(h, c, list(range(n)), cached, lens)
        got = {s: [] for s in range(n)}
        done = np.array(cached, np.int64)
        held = -(-done // cases.BS)
        free = 10**6
        steps = 0
        while (done < np.array(lens)).any():
            waiting = [s for s in range(n) if done[s] < lens[s]]
            idx = np.array(waiting)
            sel, ends, adds = nvattn.schedule_prefill_chunks(
                np.array(lens)[idx], done[idx], held[idx], free, 4, budget)
            assert sel.size > 0
            seqs = [int(idx[k]) for k in sel]
            rows = prefill_rows(h, c, seqs, [int(done[s]) for s in seqs], ends.tolist())
            for s, e, a in zip(seqs, ends.tolist(), adds.tolist()):
                got[s].append(rows[s])
                done[s] = e
                held[s] += a
                free -= a
            steps += 1
        h.check_device()
    finally:
        h.close()
    assert steps > 2
    for s in range(n):
        chunked = np.concatenate(got[s])
        assert chunked.shape == one[s].shape
        np.testing.assert_array_equal(chunked.view(np.uint32), one[s].view(np.uint32))
