"""CPU tests of the oracle's restatement of ModelRunner::Sample
(src/engine/model_runner.cpp:417-489): repetition penalty once per
occurrence, greedy first-index argmax, temperature inverse-CDF sampling with a
given draw, and the libstdc++ generate_canonical<float> mapping of an mt19937
output.  Test infrastructure for the device sampler's parity tests."""
import os
import sys

import numpy as np
import pytest

import nvattn

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "oracle"))
import oracle as O  # noqa: E402


def py_penalize(row, penalty, hist):
    """The reference loop in Python float32 (model_runner.cpp:428-446)."""
    row = row.astype(np.float32).copy()
    p = np.float32(penalty)
    if penalty > 1.0:
        for t in hist:
            if 0 <= t < row.shape[0]:
                v = row[t]
                row[t] = np.float32(v * p) if v < 0 else np.float32(v / p)
    return row


def exact_inverse_cdf(row, temp, u):
    """First index whose exact (fp64) running probability sum reaches u*S."""
    x = row.astype(np.float64)
    p = np.exp((x - x.max()) / temp)
    c = np.cumsum(p)
    return int(np.searchsorted(c, u * c[-1], side="left")), c


def test_penalty_applies_once_per_occurrence():
    rng = np.random.default_rng(0)
    V = 500
    x = rng.normal(0, 3, (2, V)).astype(np.float32)
    hist = np.array([3, 3, 3, 7, -1, 500, 10**6, 9, 9], np.int32)
    off = np.array([0, 9, 9], np.int64)
    got = O.penalize_rows(x, np.array([1.3, 1.3], np.float32), hist, off)
    np.testing.assert_array_equal(got[0], py_penalize(x[0], 1.3, hist))
    np.testing.assert_array_equal(got[1], x[1])  # empty history


@pytest.mark.parametrize("penalty", [1.0, 0.5])
def test_penalty_at_most_one_is_ignored(penalty):
    x = np.linspace(-2, 2, 64, dtype=np.float32)[None]
    hist = np.arange(64, dtype=np.int32)
    got = O.penalize_rows(x, np.array([penalty], np.float32), hist, np.array([0, 64], np.int64))
    np.testing.assert_array_equal(got, x)


def test_greedy_first_index_and_nan_rules():
    V = 16
    rows = np.zeros((5, V), np.float32)
    rows[0, [3, 9]] = 5.0                 # tie: first index
    rows[1, 0] = np.nan                   # NaN at 0: the scan never moves
    rows[1, 4] = 9.0
    rows[2, :] = -np.inf                  # all -inf: 0
    rows[3, 2] = np.nan                   # NaN elsewhere is skipped
    rows[3, 5] = 1.0
    rows[4, [6, 11]] = np.inf             # first +inf
    tok = O.sample(rows, np.zeros(5, np.float32), np.ones(5, np.float32), np.zeros(5, np.float32))
    assert tok.tolist() == [3, 0, 0, 5, 6]


def test_temperature_nan_or_inf_gives_last_token():
    V = 16
    rows = np.zeros((4, V), np.float32)
    rows[0, 0] = np.nan
    rows[1, 7] = np.nan
    rows[2, 3] = np.inf
    rows[3, :] = -np.inf
    tok = O.sample(rows, np.full(4, 0.8, np.float32), np.ones(4, np.float32),
                   np.full(4, 0.5, np.float32))
    assert tok.tolist() == [V - 1] * 4


def test_temperature_sampling_matches_exact_inverse_cdf_away_from_steps():
    rng = np.random.default_rng(1)
    V, n = 4096, 64
    x = (rng.normal(0, 4, (n, V))).astype(np.float32)
    temps = rng.choice([0.5, 0.8, 1.0, 1.5], n).astype(np.float32)
    u = ((np.arange(n) + 0.5) / n).astype(np.float32)
    tok = O.sample(x, temps, np.ones(n, np.float32), u)
    checked = 0
    for s in range(n):
        i, c = exact_inverse_cdf(x[s], float(temps[s]), float(u[s]))
        r = float(u[s]) * c[-1]
        lo = c[i - 1] if i > 0 else 0.0
        if min(abs(r - lo), abs(c[i] - r)) < 1e-5 * c[-1]:
            continue
        checked += 1
        assert tok[s] == i, s
    assert checked >= n - 4


def test_canonical_float_matches_libstdcxx_mapping():
    assert O.canonical_float(0) == 0.0
    assert O.canonical_float(1 << 31) == 0.5
    top = float(np.nextafter(np.float32(1), np.float32(0)))
    assert O.canonical_float(0xFFFFFFFF) == top        # rounds to 1, clamped below 1
    assert O.canonical_float(0xFFFFFF7F) == top
    # numpy's legacy seeding of MT19937 is std::mt19937's: the C++ standard
    # ([rand.predef]) requires the 10000th output of a default-constructed
    # mt19937 (seed 5489) to be 4123659995
    bg = np.random.MT19937()
    bg._legacy_seeding(5489)
    raw = bg.random_raw(10000)
    assert int(raw[-1]) == 4123659995
    for r in raw[:64]:
        assert 0.0 <= O.canonical_float(int(r)) < 1.0


def test_sample_entry_point_validates_without_a_device():
    L = nvattn.lib()
    assert L.nvattn_sample(None, 1, 10, None, 10, None, None, None, None, None, None, None) == \
        nvattn.ERR_INVALID_ARG
