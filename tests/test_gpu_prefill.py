"""GPU parity of nvattn_paged_prefill (tcgen05 kernel) against the oracle.

The kernel takes f16 Q, converts the cache's bf16 K and V tiles to f16 (as
the reference's ggml_cast does), multiplies f16 Q and K on the tensor cores,
rounds the softmax probabilities P to f16 for the P.V product, and
accumulates in fp32.  The cases' queries are bf16 values, which f16 holds
exactly (but for magnitudes below 2^-17).  Tolerances (BF16 cache, FP32
accumulate):
  * against fp64 math on the same inputs: max-abs-err <= 2e-2 and
    mean-rel-err <= 1e-3 (sum|a-b| / sum|b|);
  * against the reference's dtype chain (oracle GGML mode): max-abs-err <= 2e-2
    and mean-rel-err no more than 1e-3 above the chain's own distance from
    exact math.
"""
import numpy as np
import pytest

import cases
import make_golden
import nvattn
import oracle as O
from gpu_util import dev, handle, prefill_q

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-3


def run_prefill(c: cases.PrefillCase, h=None, k=None, v=None, block_tables=None):
    import torch
    if h is None:
        h = handle(c.Hq, c.Hkv, c.cache.num_blocks, n_layer=c.cache.n_layer,
                   max_seqs=len(c.seq_lens))
    T = c.q.shape[0]
    out = torch.full((T, c.Hq, 128), float("nan"), device="cuda")
    max_q = int((c.seq_lens - c.q_starts).max())
    bt = c.block_tables if block_tables is None else block_tables
    h.prefill(c.layer, prefill_q(c.q), dev(c.cu_q), dev(c.q_starts), dev(c.seq_lens), dev(bt),
              max_q, dev(c.cache.k if k is None else k), dev(c.cache.v if v is None else v), out)
    torch.cuda.synchronize()
    return h, out.cpu().numpy()


def oracle_truth(c):
    p = cases.oracle_params(c.Hq, c.Hkv, c.cache)
    return O.paged_prefill(p, O.MODE_TRUTH, c.layer, c.q, c.cu_q, c.q_starts, c.seq_lens,
                           c.block_tables, c.cache.k, c.cache.v)


def check(got, ref):
    assert np.isfinite(got).all()
    mx, mr = O.err_stats(got, ref)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
    return mx, mr


def test_golden_prefill_prefix_hit(cuda):
    fx = np.load(make_golden.__file__.replace("make_golden.py", "prefill_prefix_hit.npz"))
    c = make_golden.prefill_inputs()
    h, got = run_prefill(c)
    h.check_device()
    check(got, fx["out_truth"])
    mx_g, mr_g = O.err_stats(got, fx["out_ggml"])
    _, chain = O.err_stats(fx["out_truth"], fx["out_ggml"])
    assert mx_g <= MAX_ABS and mr_g <= chain + MEAN_REL, (mx_g, mr_g, chain)


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (32, 8), (64, 8), (8, 8), (2, 1)])
def test_shapes_and_prefixes(cuda, Hq, Hkv):
    # (sequence length, cached prefix): no prefix, whole-block prefixes, and
    # chunked-prefill starts that are not block aligned
    lens = [1000, 700, 300, 129, 1, 600]
    starts = [0, 512, 44, 0, 0, 599]
    c = cases.prefill_case(Hq * 7 + Hkv, Hq, Hkv, lens, starts)
    h, got = run_prefill(c)
    h.check_device()
    check(got, oracle_truth(c))


def test_shared_prefix_blocks_config2_like(cuda):
    """Eight sequences share a 512-token prefix held in the same physical
    blocks (refcount 8), with suffixes of different lengths."""
    rng = np.random.default_rng(70)
    lens = rng.integers(520, 1300, 8).astype(np.int32)
    starts = np.full(8, 512, np.int32)
    c = cases.prefill_case(71, 16, 8, lens, starts)
    shared = c.block_tables[0, :2].copy()
    c.block_tables[:, :2] = shared
    h, got = run_prefill(c)
    h.check_device()
    check(got, oracle_truth(c))


def test_prefix_hit_rows_equal_full_prefill_rows(cuda):
    c = cases.prefill_case(72, 16, 8, [1500], [0])
    h, full = run_prefill(c)
    part = cases.PrefillCase(c.Hq, c.Hkv, c.seq_lens, np.array([1024], np.int32),
                             np.array([0, 476], np.int32), c.cache, c.block_tables,
                             np.ascontiguousarray(c.q[1024:]))
    _, got = run_prefill(part, h=h)
    # same keys, same row: the two launches differ only in tile alignment
    mx, _ = O.err_stats(got, full[1024:])
    assert mx <= 2e-3


def test_decode_matches_last_prefill_row(cuda):
    import torch
    c = cases.prefill_case(73, 32, 8, [2000, 777], [0, 0])
    h, pre = run_prefill(c)
    last = [int(c.cu_q[1]) - 1, int(c.cu_q[2]) - 1]
    out = torch.empty((2, 32, 128), device="cuda")
    h.decode(0, dev(np.ascontiguousarray(c.q[last])), dev(c.cache.k), dev(c.cache.v),
             dev(c.block_tables), dev(c.seq_lens), int(c.seq_lens.max()), out)
    dec = out.cpu().numpy()
    mx, mr = O.err_stats(pre[last], dec)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)


def test_nan_garbage_past_context_is_ignored(cuda):
    """Cache slots past a sequence's end may hold anything; they must not
    leak into the result (P = 0 must never meet NaN in P.V)."""
    c = cases.prefill_case(74, 16, 8, [300, 129], [0, 0], num_blocks=4)
    k, v = c.cache.k.copy(), c.cache.v.copy()
    for s, L in enumerate(c.seq_lens):
        for t in range(L, ((L + 255) // 256) * 256):
            b = c.block_tables[s, t // 256]
            k[0, b * 256 + t % 256] = 0x7fc1
            v[0, b * 256 + t % 256] = 0x7fc1
    h, got = run_prefill(c, k=k, v=v)
    h.check_device()
    check(got, oracle_truth(c))


def test_nan_garbage_past_context_is_ignored_by_decode(cuda):
    import torch
    dc = cases.decode_case(75, 16, 8, [300, 129, 70], num_blocks=5)
    k, v = dc.cache.k.copy(), dc.cache.v.copy()
    for s, L in enumerate(dc.lens):
        for t in range(L, ((L + 255) // 256) * 256):
            b = dc.block_tables[s, t // 256]
            k[0, b * 256 + t % 256] = 0x7fc1
            v[0, b * 256 + t % 256] = 0x7fc1
    h = handle(16, 8, dc.cache.num_blocks, max_seqs=3)
    out = torch.empty((3, 16, 128), device="cuda")
    h.decode(0, dev(dc.q), dev(k), dev(v), dev(dc.block_tables), dev(dc.lens),
             int(dc.lens.max()), out)
    h.check_device()
    p = cases.oracle_params(16, 8, dc.cache)
    ref = O.paged_decode(p, O.MODE_TRUTH, 0, dc.q, dc.cache.k, dc.cache.v, dc.block_tables,
                         dc.lens)
    check(out.cpu().numpy(), ref)


def test_long_chunk_over_long_prefix(cuda):
    """Chunked prefill: a 384-token chunk at positions [12288, 12672)."""
    c = cases.prefill_case(76, 64, 8, [12672], [12288])
    h, got = run_prefill(c)
    h.check_device()
    check(got, oracle_truth(c))


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (64, 8)])
def test_pv_precision_headroom(cuda, Hq, Hkv):
    """P is rounded to f16 (11 significant bits) for the P.V product, so the
    output's rounding noise stays well inside the 1e-3 bound (a bf16 P, with
    8 bits, would sit at ~1.4e-3 on these inputs)."""
    c = cases.prefill_case(78 + Hq, Hq, Hkv, [1000, 700, 300], [0, 512, 44])
    h, got = run_prefill(c)
    h.check_device()
    mx, mr = O.err_stats(got, oracle_truth(c))
    assert mx <= MAX_ABS and mr <= 6e-4, (mx, mr)


def test_bad_block_id_is_reported(cuda):
    c = cases.prefill_case(77, 16, 8, [600], [0])
    bt = c.block_tables.copy()
    bt[0, 1] = 10_000
    h, _ = run_prefill(c, block_tables=bt)
    st, detail = h.get_error()
    assert st == nvattn.ERR_OUT_OF_RANGE and detail == 10_000
