"""The step protocol of nvattn_paged_decode_step_gather, checked over every
interleaving of the ranks' memory events (CPU; no GPU involved).

Each rank r, per gather step s, in its own order:
  W: stores its rows of step s into every rank's gathered buffer, parity s & 1
     (one event per destination; the decode launch's stores, fenced before R);
  R: adds one to every rank's completion counter (one event per counter);
  A: waits until its own counter reaches n_ranks * (s + 1);
  C: reads every rank's rows of step s from its own buffer (one event per
     source rank) -- nvattn_gather_read, issued before the next step.
The model explores all interleavings (memoised over states) and checks that
every read of step s sees step s's rows.  Reading step s - 1 after step s has
been issued -- what nvattn_gather_read rejects -- is shown to be unsafe by the
same search.
"""
import pytest


def _program(n, rank, steps, read_lag):
    """The event list of one rank; read_lag = 0 reads step s after its wait,
    read_lag = 1 reads step s - 1 there instead (the rejected pattern)."""
    ev = []
    for s in range(steps):
        ev += [("W", s, p) for p in range(n)]
        ev += [("R", s, p) for p in range(n)]
        ev.append(("A", s, None))
        t = s - read_lag
        if t >= 0:
            ev += [("C", t, p) for p in range(n)]
    return ev


def _explore(n, steps, read_lag):
    """Returns (states visited, first violation or None)."""
    progs = [_program(n, r, steps, read_lag) for r in range(n)]
    # state: (pcs, buffers, counters); buffers[r][parity][src] = step stored
    init = (tuple([0] * n), tuple(tuple(tuple([-1] * n) for _ in range(2)) for _ in range(n)),
            tuple([0] * n))
    seen = {init}
    stack = [init]
    while stack:
        pcs, bufs, cnt = stack.pop()
        for r in range(n):
            if pcs[r] == len(progs[r]):
                continue
            kind, s, p = progs[r][pcs[r]]
            nb, nc = bufs, cnt
            if kind == "W":
                b = [list(map(list, x)) for x in bufs]
                b[p][s & 1][r] = s
                nb = tuple(tuple(tuple(row) for row in x) for x in b)
            elif kind == "R":
                c = list(cnt)
                c[p] += 1
                nc = tuple(c)
            elif kind == "A":
                if cnt[r] < n * (s + 1):
                    continue  # blocked: another rank must move first
            else:  # C: rank r reads source p's rows of step s
                if bufs[r][s & 1][p] != s:
                    return len(seen), (r, s, p, bufs[r][s & 1][p])
            npcs = list(pcs)
            npcs[r] += 1
            st = (tuple(npcs), nb, nc)
            if st not in seen:
                seen.add(st)
                stack.append(st)
    return len(seen), None


@pytest.mark.parametrize("n,steps", [(2, 4), (3, 3)])
def test_latest_step_reads_always_see_that_step(n, steps):
    visited, bad = _explore(n, steps, read_lag=0)
    assert bad is None, f"rank {bad[0]} read step {bad[1]} of rank {bad[2]} and saw {bad[3]}"
    assert visited > 100


@pytest.mark.parametrize("n,steps", [(2, 4)])
def test_reading_the_previous_step_after_the_next_one_is_unsafe(n, steps):
    _, bad = _explore(n, steps, read_lag=1)
    assert bad is not None
    r, s, p, got = bad
    assert got == s + 2  # a peer's step s + 2 already overwrote that parity
