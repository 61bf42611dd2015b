"""The prefill kernel's persistent work scheduling: CTAs take (query-tile
pair, kv head, sequence) items from a counter in the handle's workspace,
skip runs of items that have no query rows, and the last CTA of a launch
zeroes the counter.  These tests target that machinery: batches where most
items are empty (one long prompt among one-token ones, a max_q_len bound far
above the longest prompt), CUDA-graph replays (the counter must be back at
zero before every replay, with no host-side reset), and launches of
different shapes back to back on one handle; and query rows named outside
q and out, which are reported and skipped.  Outputs are checked against
the oracle's fp64 attention (max-abs 2e-2, mean-rel 1e-3) and, across
launches, bit for bit against each other."""
import numpy as np
import pytest

import cases
import nvattn
import oracle as O
from gpu_util import dev, handle, prefill_q

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-3


def truth(c):
    p = cases.oracle_params(c.Hq, c.Hkv, c.cache)
    return O.paged_prefill(p, O.MODE_TRUTH, c.layer, c.q, c.cu_q, c.q_starts, c.seq_lens,
                           c.block_tables, c.cache.k, c.cache.v)


class Inputs:
    """A case's inputs resident on the device, and an output buffer."""

    def __init__(self, c, max_q=None):
        import torch
        self.c = c
        self.q = prefill_q(c.q)
        self.cu = dev(c.cu_q)
        self.qs = dev(c.q_starts)
        self.cl = dev(c.seq_lens)
        self.bt = dev(c.block_tables)
        self.k = dev(c.cache.k)
        self.v = dev(c.cache.v)
        self.max_q = int((c.seq_lens - c.q_starts).max()) if max_q is None else max_q
        self.out = torch.full((c.q.shape[0], c.Hq, 128), float("nan"), device="cuda")

    def launch(self, h, stream=None):
        h.prefill(self.c.layer, self.q, self.cu, self.qs, self.cl, self.bt, self.max_q, self.k,
                  self.v, self.out, stream=stream)

    def result(self):
        import torch
        torch.cuda.synchronize()
        return self.out.cpu().numpy()


def check(got, ref):
    assert np.isfinite(got).all()
    mx, mr = O.err_stats(got, ref)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)


@pytest.mark.parametrize("Hq,Hkv,inflate", [(16, 8, 1), (16, 8, 4), (2, 1, 3)])
def test_mostly_empty_items(cuda, Hq, Hkv, inflate):
    """One 1,500-token prompt (with a 256-token cached prefix) among 40
    one-token prompts and three short ones: every short sequence's work
    group is all but its last items empty; `inflate` multiplies the
    max_q_len bound, adding whole runs of empty items to every group."""
    lens = [1500] + [1] * 20 + [300, 129, 700] + [1] * 20
    starts = [256] + [0] * 20 + [0, 128, 699] + [0] * 20
    c = cases.prefill_case(900 + Hq + inflate, Hq, Hkv, lens, starts)
    x = Inputs(c)
    x.max_q *= inflate
    h = handle(Hq, Hkv, c.cache.num_blocks, max_seqs=len(lens))
    try:
        x.launch(h)
        got = x.result()
        h.check_device()
    finally:
        h.close()
    check(got, truth(c))


def test_graph_replays_and_eager_launches_agree(cuda):
    """A prefill captured in a CUDA graph and replayed three times gives the
    eager launch's output bit for bit each time, and so does an eager launch
    after the replays: the counter is zero again after every launch."""
    import torch
    c = cases.prefill_case(910, 16, 8, [900, 1, 400, 1300], [0, 0, 300, 1024])
    x = Inputs(c)
    h = handle(16, 8, c.cache.num_blocks, max_seqs=4)
    try:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            x.launch(h, stream=s)
        eager = x.result()
        check(eager, truth(c))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            x.launch(h, stream=s)
        for _ in range(3):
            x.out.fill_(float("nan"))
            g.replay()
            np.testing.assert_array_equal(x.result().view(np.uint32), eager.view(np.uint32))
        del g
        x.out.fill_(float("nan"))
        x.launch(h)
        np.testing.assert_array_equal(x.result().view(np.uint32), eager.view(np.uint32))
        h.check_device()
    finally:
        h.close()


def test_back_to_back_launches_of_different_shapes(cuda):
    """Two batches of different sizes (so different persistent grids)
    alternate on one handle without a synchronisation between launches;
    every launch matches the first launch of its batch bit for bit."""
    a = cases.prefill_case(920, 16, 8, [2000, 1, 1, 513], [1024, 0, 0, 0], num_blocks=64)
    b = cases.prefill_case(921, 16, 8, [129], [0], num_blocks=64)
    xa, xb = Inputs(a), Inputs(b)
    h = handle(16, 8, 64, max_seqs=4)
    try:
        xa.launch(h)
        first_a = xa.result()
        xb.launch(h)
        first_b = xb.result()
        check(first_a, truth(a))
        check(first_b, truth(b))
        outs_a, outs_b = [], []
        for _ in range(4):
            xa.launch(h)
            xb.launch(h)
            outs_a.append(xa.out.clone())
            outs_b.append(xb.out.clone())
        h.check_device()
    finally:
        h.close()
    for oa, ob in zip(outs_a, outs_b):
        np.testing.assert_array_equal(oa.cpu().numpy().view(np.uint32), first_a.view(np.uint32))
        np.testing.assert_array_equal(ob.cpu().numpy().view(np.uint32), first_b.view(np.uint32))


def test_rows_outside_q_are_reported_not_written(cuda):
    """cu_q_lens naming rows past the n_tokens rows of q and out: that
    sequence is skipped and reported (NVATTN_ERR_OUT_OF_RANGE, detail = the
    offending end row); the other sequence is computed as usual.  The output
    buffer has spare rows past n_tokens, which must stay untouched."""
    import torch
    c = cases.prefill_case(930, 16, 8, [300, 200], [0, 0])
    x = Inputs(c)
    T = c.q.shape[0]
    bad_cu = c.cu_q.copy()
    bad_cu[2] = T + 20
    out = torch.full((T + 64, 16, 128), float("nan"), device="cuda")
    h = handle(16, 8, c.cache.num_blocks, max_seqs=2)
    try:
        h.prefill(c.layer, x.q, dev(bad_cu), x.qs, x.cl, x.bt, 320, x.k, x.v, out)
        torch.cuda.synchronize()
        st, detail = h.get_error()
    finally:
        h.close()
    assert st == nvattn.ERR_OUT_OF_RANGE and detail == T + 20
    got = out.cpu().numpy()
    assert np.isnan(got[300:]).all()
    check(got[:300], truth(c)[:300])
