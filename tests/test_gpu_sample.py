"""Device sampler (nvattn_sample) against the oracle's restatement of
ModelRunner::Sample (src/engine/model_runner.cpp:417-489).

Greedy rows: bit-exact tokens (penalty applied once per occurrence, first
index of the maximum, NaN rules).  Sampling rows: the token the exact (fp64)
inverse CDF gives for the same draw, for every draw farther than 2e-5 of the
total mass from a CDF step (the device and the reference both round within
that band), and a token whose step holds the draw within that band for the
others; with stratified draws, token counts within 2 of N*p."""
import os
import sys

import numpy as np
import pytest

import nvattn
from gpu_util import handle

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "oracle"))
import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu
QWEN3_VOCAB = 151936


def _run(h, logits, temps, pens, u, hist=None, off=None, stride=None):
    import torch
    n, V = logits.shape
    if stride is not None and stride != V:
        buf = torch.zeros((n, stride), dtype=torch.float32, device="cuda:0")
        buf[:, :V] = torch.from_numpy(logits)
        x = buf[:, :V]
    else:
        x = torch.from_numpy(np.ascontiguousarray(logits)).to("cuda:0")
    t = torch.from_numpy(np.asarray(temps, np.float32)).to("cuda:0")
    p = torch.from_numpy(np.asarray(pens, np.float32)).to("cuda:0")
    uu = torch.from_numpy(np.asarray(u, np.float32)).to("cuda:0")
    hh = None if hist is None else torch.from_numpy(np.asarray(hist, np.int32)).to("cuda:0")
    oo = None if off is None else torch.from_numpy(np.asarray(off, np.int64)).to("cuda:0")
    tok = torch.full((n,), -7, dtype=torch.int32, device="cuda:0")
    h.sample(x, t, p, uu, tok, hh, oo)
    torch.cuda.synchronize()
    return tok.cpu().numpy()


BAND = 2e-5  # fraction of the total mass within which a draw may fall on either side of a step


def _within_step(g, c, r):
    """Token g's CDF step [c[g-1], c[g]] holds r, up to BAND of the total."""
    lo = c[g - 1] if g > 0 else 0.0
    return lo - BAND * c[-1] <= r <= c[g] + BAND * c[-1]


def _histories(rng, n, V, max_len, repeat_frac=0.5):
    lens = rng.integers(0, max_len + 1, n)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    ids = rng.integers(0, V, int(off[-1])).astype(np.int32)
    # many repeats (a few hot ids) and some ids the reference skips
    hot = rng.integers(0, V, 8)
    mask = rng.random(ids.shape[0]) < repeat_frac
    ids[mask] = hot[rng.integers(0, 8, int(mask.sum()))]
    bad = rng.random(ids.shape[0]) < 0.01
    ids[bad] = rng.choice([-1, V, V + 100], int(bad.sum()))
    return ids, off


@pytest.mark.parametrize("n,V,stride,seed", [
    (1, QWEN3_VOCAB, None, 0), (37, QWEN3_VOCAB, None, 1), (300, 4097, None, 2),
    (16, 1000, 1003, 3), (5, 7, None, 4), (8, 4096 * 3, 4096 * 3 + 4, 5), (3, 1, None, 6),
    (4, 2, None, 7)])
def test_greedy_with_penalty_is_bit_exact(n, V, stride, seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 2, (n, V)).astype(np.float32)
    pens = rng.choice([1.0, 1.2, 1.5, 0.9], n).astype(np.float32)
    hist, off = _histories(rng, n, V, 3000)
    # put the history's ids on top so the penalty decides the argmax
    for s in range(n):
        ids = hist[off[s]:off[s + 1]]
        ids = ids[(ids >= 0) & (ids < V)]
        if ids.size:
            x[s, ids[:4]] = x[s].max() + rng.random(min(4, ids.size)).astype(np.float32)
    want = O.sample(x, np.zeros(n, np.float32), pens, np.zeros(n, np.float32), hist, off)
    h = handle(8, 8, 16, max_seqs=max(n, 1))
    try:
        got = _run(h, x, np.zeros(n), pens, np.zeros(n), hist, off, stride)
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()
    np.testing.assert_array_equal(got, want)


def test_edge_rows_nan_inf_ties():
    V = 9000
    rows = np.zeros((10, V), np.float32)
    rows[0, [3, 5000]] = 5.0                 # tie across chunks: first index
    rows[1, 0] = np.nan
    rows[1, 4] = 9.0
    rows[2, :] = -np.inf
    rows[3, 8000] = np.nan
    rows[3, 5] = 1.0
    rows[4, [6000, 8999]] = np.inf
    rows[5, 4100] = 7.0                      # max in the second chunk
    rows[6, :] = np.nan
    rows[7, 8999] = 3.0                      # max at the last element
    rows[8, :] = -np.inf
    rows[8, 4096] = -1e30
    rows[9, 4095:4097] = 2.0                 # tie straddling a chunk edge
    n = rows.shape[0]
    for temp in (0.0, 0.8):
        t = np.full(n, temp, np.float32)
        u = np.full(n, 0.5, np.float32)
        want = O.sample(rows, t, np.ones(n, np.float32), u)
        h = handle(8, 8, 16)
        try:
            got = _run(h, rows, t, np.ones(n), u)
            assert h.get_error() == (nvattn.OK, 0)
        finally:
            h.close()
        if temp == 0.0:
            np.testing.assert_array_equal(got, want)
        else:
            # rows whose reference sum is NaN give the last token; the others
            # are one-hot-ish (a single finite maximum dominates)
            for s in (1, 2, 3, 4, 6):
                assert got[s] == V - 1 == want[s], s
            assert got[8] == want[8] == 4096


@pytest.mark.parametrize("V,temps,scale", [(QWEN3_VOCAB, (0.6, 0.8, 1.0), 4.0),
                                           (5000, (0.5, 1.5), 3.0)])
def test_sampling_matches_exact_inverse_cdf(V, temps, scale):
    rng = np.random.default_rng(7)
    n = 128
    x = rng.normal(0, scale, (n, V)).astype(np.float32)
    t = rng.choice(temps, n).astype(np.float32)
    pens = np.full(n, 1.2, np.float32)
    hist, off = _histories(rng, n, V, 2000)
    u = ((np.arange(n) + 0.37) / n).astype(np.float32)
    h = handle(8, 8, 16, max_seqs=n)
    try:
        got = _run(h, x, t, pens, u, hist, off)
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()
    ref = O.sample(x, t, pens, u, hist, off)
    xp = O.penalize_rows(x, pens, hist, off).astype(np.float64)
    checked = agree_ref = 0
    for s in range(n):
        p = np.exp((xp[s] - xp[s].max()) / float(t[s]))
        c = np.cumsum(p)
        r = float(u[s]) * c[-1]
        i = int(np.searchsorted(c, r, side="left"))
        assert _within_step(int(got[s]), c, r), (s, got[s], i)
        lo = c[i - 1] if i > 0 else 0.0
        if min(abs(r - lo), abs(c[i] - r)) < BAND * c[-1]:
            continue
        checked += 1
        assert got[s] == i, (s, got[s], i)
        agree_ref += int(ref[s] == i)
    assert checked >= n * 0.85
    assert agree_ref >= checked * 0.9  # the reference chain, for context


def test_stratified_draws_follow_the_distribution():
    """Flat-ish logits, one row repeated under N stratified draws: each
    token's count is N*p within 2 (plus the draws that land within rounding
    of a step, at most one per step crossed)."""
    rng = np.random.default_rng(11)
    V, N = 1000, 4096
    row = rng.normal(0, 1, V).astype(np.float32)
    x = np.repeat(row[None], N, axis=0)
    u = ((np.arange(N) + 0.5) / N).astype(np.float32)
    h = handle(8, 8, 16, max_seqs=N, max_context=1024)
    try:
        got = _run(h, x, np.ones(N), np.ones(N), u)
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()
    p = np.exp(row.astype(np.float64) - row.max())
    p /= p.sum()
    counts = np.bincount(got, minlength=V)
    assert np.abs(counts - N * p).max() <= 2.0
    assert (np.diff(got) >= 0).all()  # monotone in u, as an inverse CDF is


def test_workspace_is_clean_between_calls():
    """Counts and bitmap words set by one call's histories are zeroed by it:
    a second call with other histories (and none) still matches."""
    rng = np.random.default_rng(3)
    n, V = 24, 20000
    h = handle(8, 8, 16, max_seqs=n)
    try:
        for it in range(3):
            x = rng.normal(0, 2, (n, V)).astype(np.float32)
            pens = np.full(n, 1.3, np.float32)
            hist, off = _histories(rng, n, V, 500, repeat_frac=0.9)
            for s in range(n):
                ids = hist[off[s]:off[s + 1]]
                ids = ids[(ids >= 0) & (ids < V)]
                if ids.size:
                    x[s, ids[0]] = x[s].max() + 0.01
            if it == 2:
                hist = off = None
            want = O.sample(x, np.zeros(n, np.float32), pens, np.zeros(n, np.float32), hist, off)
            got = _run(h, x, np.zeros(n), pens, np.zeros(n), hist, off)
            np.testing.assert_array_equal(got, want)
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()


@pytest.mark.parametrize("V", [QWEN3_VOCAB, 200000])
def test_penalty_counts_are_exact_past_saturation(V):
    """Ids seen 3, 20 (past the 4-bit count) and 300 (past the 8-bit
    histogram) times, in both count segments of a 200000-id vocabulary: a
    competitor one ulp below / above the oracle's penalised value flips the
    argmax if the device's count is one too high / too low."""
    pen = np.float32(1.01)
    reps = {0: 3, 1: 20, 2: 300}
    ids = {0: 17, 1: V // 2 + 5, 2: V - 9}
    rows, hists = [], []
    for kind in range(3):
        tok = ids[kind]
        for sign in (1.0, -1.0):
            for side in (-1, 1):
                x = np.random.default_rng(kind * 7 + (side > 0)).normal(0, 1, V).astype(np.float32)
                x[tok] = np.float32(50.0 * sign)
                hist = np.full(reps[kind], tok, np.int32)
                v = O.penalize_rows(x[None], np.array([pen], np.float32), hist,
                                    np.array([0, hist.size], np.int64))[0, tok]
                others = np.arange(V) != tok
                x[others] = np.minimum(x[others], v - np.float32(1.0))
                comp = V // 3 if side < 0 else 5
                x[comp] = np.nextafter(v, np.float32(-np.inf) if side < 0 else np.float32(np.inf))
                rows.append(x)
                hists.append(hist)
    x = np.stack(rows)
    n = x.shape[0]
    off = np.concatenate([[0], np.cumsum([hh.size for hh in hists])]).astype(np.int64)
    hist = np.concatenate(hists)
    pens = np.full(n, pen, np.float32)
    want = O.sample(x, np.zeros(n, np.float32), pens, np.zeros(n, np.float32), hist, off)
    h = handle(8, 8, 16, max_seqs=n)
    try:
        got = _run(h, x, np.zeros(n), pens, np.zeros(n), hist, off)
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()
    np.testing.assert_array_equal(got, want)
    # the construction makes the penalised id win exactly when side < 0
    for r in range(n):
        kind, rest = divmod(r, 4)
        assert (want[r] == ids[kind]) == (rest % 2 == 0), r


@pytest.mark.parametrize("u_bad", [1.0, -0.25, float("nan")])
def test_bad_draw_is_reported(u_bad):
    V, n = 300, 3
    x = np.zeros((n, V), np.float32)
    u = np.array([0.5, u_bad, 0.5], np.float32)
    h = handle(8, 8, 16)
    try:
        got = _run(h, x, np.ones(n), np.ones(n), u)
        assert h.get_error() == (nvattn.ERR_INVALID_ARG, 1)
    finally:
        h.close()
    assert got[1] == V - 1


def test_bad_history_offsets_are_reported():
    V, n = 300, 2
    x = np.zeros((n, V), np.float32)
    hist = np.arange(10, dtype=np.int32)
    off = np.array([0, 5, 3], np.int64)  # sequence 1 ends before it starts
    h = handle(8, 8, 16)
    try:
        _run(h, x, np.zeros(n), np.full(n, 1.5), np.zeros(n), hist, off)
        assert h.get_error() == (nvattn.ERR_INVALID_ARG, 1)
    finally:
        h.close()


def test_sampler_is_graph_capturable_after_first_call():
    import torch
    rng = np.random.default_rng(5)
    n, V = 16, QWEN3_VOCAB
    h = handle(8, 8, 16, max_seqs=n)
    try:
        x = torch.zeros((n, V), dtype=torch.float32, device="cuda:0")
        t = torch.full((n,), 0.8, device="cuda:0")
        p = torch.full((n,), 1.2, device="cuda:0")
        hist_np, off_np = _histories(rng, n, V, 300)
        hist = torch.from_numpy(hist_np).to("cuda:0")
        off = torch.from_numpy(off_np).to("cuda:0")
        u = torch.zeros(n, device="cuda:0")
        tok = torch.zeros(n, dtype=torch.int32, device="cuda:0")
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            h.sample(x, t, p, u, tok, hist, off, stream=s)  # allocates the workspace
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            h.sample(x, t, p, u, tok, hist, off, stream=s)
        for it in range(3):
            xs = rng.normal(0, 4, (n, V)).astype(np.float32)
            us = rng.random(n).astype(np.float32)
            x.copy_(torch.from_numpy(xs))
            u.copy_(torch.from_numpy(us))
            g.replay()
            torch.cuda.synchronize()
            got = tok.cpu().numpy()
            xp = O.penalize_rows(xs, np.full(n, 1.2, np.float32), hist_np, off_np)
            for r in range(n):
                pr = np.exp((xp[r].astype(np.float64) - xp[r].max()) / 0.8)
                c = np.cumsum(pr)
                assert _within_step(int(got[r]), c, float(us[r]) * c[-1]), r
        del g
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()


@pytest.mark.parametrize("V", [1, 2, 3])
def test_tiny_vocabularies_sample_like_the_reference(V):
    """One to three logits per row, temperature rows: with a single finite
    maximum far above the rest the inverse CDF gives it for any draw."""
    n = 6
    x = np.full((n, V), -50.0, np.float32)
    top = np.arange(n) % V
    x[np.arange(n), top] = 5.0
    t = np.full(n, 0.8, np.float32)
    u = np.linspace(0.05, 0.95, n).astype(np.float32)
    want = O.sample(x, t, np.ones(n, np.float32), u)
    h = handle(8, 8, 16)
    try:
        got = _run(h, x, t, np.ones(n), u)
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(got, top)
