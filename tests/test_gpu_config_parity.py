"""GPU parity at the benchmark configurations' own shapes, and of whole steps
against the reference's own attention algorithm.

* Decode at the long-context workload's length (131,104 cached tokens, 64 q /
  8 kv heads): the split rule doubles the split past 2048 tokens there (a
  context needing more than the workspace's 64 splits), a path shorter
  contexts never reach.
* Decode over the large-batch workload's own context lengths (log-uniform in
  [1k, 32k], the draw the benchmark uses), its longest sequence included.
* Prefill of the chunked-prefill workload's chunk: 2048 new tokens at
  positions [129024, 131072) over a 129,024-token cached prefix, 64 q / 8 kv
  heads.  A query row at position P attends keys [0, P], which is what a
  decode of a sequence of length P + 1 computes; the oracle checks a sample of
  rows that way (the whole chunk would take the fp64 oracle minutes).
* A decode step and a prefill step as the reference runs them: the new tokens'
  K/V enter its attention as the graph's f32 rows (cast to F16 by
  BuildAttention), concatenated after the gathered history (decode:
  LoadHistoryKV + concat, model_runner.cpp:116-124, qwen3.cpp:648-661;
  prefill: the batch's own rows under FillCausalMask,
  model_runner.cpp:188-217, qwen3.cpp:461-531).  The library runs its fused
  norm/RoPE/store first and then attends the stored rows; the oracle runs the
  reference's concat-all algorithm on the f32 rows.

Bars (BF16 cache, FP32 accumulate): max-abs-err <= 2e-2 and mean-rel-err
(sum|a-b| / sum|b|) <= 1e-3 against exact (fp64) math; against the
reference's dtype chain, max-abs-err <= 2e-2 and mean-rel-err no more than
1e-3 above that chain's own distance from exact math.
"""
import math

import numpy as np
import pytest

import cases
import nvattn
import oracle as O
from gpu_util import dev, handle, prefill_q

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-3


def split_tokens(sm_count, Hkv, n_seqs, max_ctx, max_context_cfg, bs=256):
    """The decode split rule (tokens per split), restated to name the path a
    case takes: halve from 2048 until the grid fills the GPU, then double
    while a context needs more splits than the workspace holds."""
    max_splits = min((max_context_cfg + bs - 1) // bs, 64)
    split = 2048
    while split > bs and n_seqs * Hkv * math.ceil(max_ctx / split) < 8 * sm_count:
        split //= 2
    split = max(split, bs)
    while math.ceil(max_ctx / split) > max_splits:
        split *= 2
    return split


def decode_and_check(c, max_context_cfg):
    import torch
    h = handle(c.Hq, c.Hkv, c.cache.num_blocks, max_seqs=len(c.lens),
               max_context=max_context_cfg, max_position=max_context_cfg)
    out = torch.full((len(c.lens), c.Hq, 128), float("nan"), device="cuda")
    h.decode(0, dev(c.q), dev(c.cache.k), dev(c.cache.v), dev(c.block_tables), dev(c.lens),
             int(c.lens.max()), out)
    h.check_device()
    got = out.cpu().numpy()
    h.close()
    p = cases.oracle_params(c.Hq, c.Hkv, c.cache)
    truth = O.paged_decode(p, O.MODE_TRUTH, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens)
    assert np.isfinite(got).all()
    mx, mr = O.err_stats(got, truth)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
    return got, truth


def test_decode_131k_context_takes_the_doubled_split(cuda):
    import torch
    lens = np.array([131104, 4097], np.int32)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert split_tokens(sms, 8, len(lens), int(lens.max()), int(lens.max())) > 2048
    c = cases.decode_case(131, 64, 8, lens)
    decode_and_check(c, int(lens.max()))


def test_decode_large_batch_workload_lengths(cuda):
    """Eight of the 256 context lengths of the large-batch decode workload
    (numpy default_rng(0), log-uniform in [1024, 32768]): its longest and
    shortest sequences and six others, 32 q / 8 kv heads."""
    rng = np.random.default_rng(0)
    lens = np.exp(rng.uniform(math.log(1024), math.log(32768), 256)).astype(np.int64)
    order = np.argsort(lens)
    pick = np.concatenate([order[[-1, 0]], order[np.linspace(1, 254, 6).astype(int)]])
    sel = lens[pick].astype(np.int32)
    assert sel.max() > 30000 and sel.min() < 1100
    c = cases.decode_case(256, 32, 8, sel)
    decode_and_check(c, 32768)


def test_prefill_chunk_at_129024_sampled_rows(cuda):
    import torch
    Hq, Hkv, L, start = 64, 8, 131072, 129024
    c = cases.prefill_case(129, Hq, Hkv, [L], [start])
    h = handle(Hq, Hkv, c.cache.num_blocks, max_seqs=1, max_context=L, max_position=L)
    T = L - start
    out = torch.full((T, Hq, 128), float("nan"), device="cuda")
    h.prefill(0, prefill_q(c.q), dev(c.cu_q), dev(c.q_starts), dev(c.seq_lens),
              dev(c.block_tables), T, dev(c.cache.k), dev(c.cache.v), out)
    h.check_device()
    got = out.cpu().numpy()
    h.close()
    assert np.isfinite(got).all()
    rng = np.random.default_rng(7)
    rows = np.unique(np.concatenate([[0, 1, 127, 128, 255, 256, 1023, 1024, 2046, 2047],
                                     rng.choice(T, 14, replace=False)]))
    # row r at position start + r == a decode of length start + r + 1 (16
    # threads: each holds a 131k-key gather)
    p = cases.oracle_params(Hq, Hkv, c.cache, n_threads=16)
    bt = np.repeat(c.block_tables, len(rows), axis=0)
    ctx = (start + rows + 1).astype(np.int32)
    truth = O.paged_decode(p, O.MODE_TRUTH, 0, np.ascontiguousarray(c.q[rows]), c.cache.k,
                           c.cache.v, bt, ctx)
    mx, mr = O.err_stats(got[rows], truth)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)


def _norm_weights(rng):
    return (O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32)),
            O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32)))


def test_decode_step_against_the_reference_concat_algorithm(cuda):
    """The small-batch decode configuration (4 sequences of 37, 256, 513 and
    1000 tokens, 16 q / 8 kv heads, 64 blocks): fused store then decode on
    the GPU, against the reference's gather-all + concat + varlen-mask decode
    fed the new token's f32 K/V."""
    import torch
    Hq, Hkv = 16, 8
    c = cases.decode_case(900, Hq, Hkv, [37, 256, 513, 1000], num_blocks=64)
    rng = np.random.default_rng(901)
    B = len(c.lens)
    q = rng.standard_normal((B, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
    qw, kw = _norm_weights(rng)
    ctx, pos, slots = nvattn.plan_decode(c.lens, c.block_tables)
    h = handle(Hq, Hkv, c.cache.num_blocks, max_seqs=B)
    kc, vc, dq = dev(c.cache.k), dev(c.cache.v), dev(q)
    h.kv_store(0, dq, dev(k), dev(v), dev(qw), dev(kw), dev(pos), dev(slots), dq, kc, vc)
    out = torch.full((B, Hq, 128), float("nan"), device="cuda")
    h.decode(0, dq, kc, vc, dev(c.block_tables), dev(ctx), int(ctx.max()), out)
    h.check_device()
    got = out.cpu().numpy()
    h.close()

    p = cases.oracle_params(Hq, Hkv, c.cache)
    okc, ovc = c.cache.k.copy(), c.cache.v.copy()
    q_out, k_out = O.qk_norm_rope_store(p, 0, q, k, v, qw, kw, pos, slots, okc, ovc,
                                        want_k_out=True)
    assert np.array_equal(kc.cpu().numpy().view(np.uint16), okc)
    ref = O.concat_decode_ggml(p, 0, q_out, okc, ovc, c.block_tables, ctx, k_out, v)
    exact = O.paged_decode(p, O.MODE_TRUTH, 0, q_out, okc, ovc, c.block_tables, ctx,
                           new_k=k_out, new_v=v)
    _, chain = O.err_stats(ref, exact)
    mx, mr = O.err_stats(got, ref)
    assert mx <= MAX_ABS and mr <= chain + MEAN_REL, (mx, mr, chain)
    mx, mr = O.err_stats(got, exact)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)


def test_prefill_step_against_the_reference_concat_algorithm(cuda):
    """Three prompts without a cached prefix (16 q / 8 kv heads): fused store
    (f16 q) then prefill on the GPU, against the reference's prefill attention
    over the batch's own f32 rows cast to F16 under FillCausalMask.

    The library attends the rows as the BF16 cache holds them -- what every
    later step of either implementation reads -- while the reference's own
    step attends the unrounded graph rows; that storage rounding moves exact
    math by `storage` (measured here), so the bar against the reference's
    chain is chain + storage + 1e-3.  Against exact math on the stored rows
    the bar is the plain 1e-3."""
    import torch
    Hq, Hkv = 16, 8
    lens = np.array([300, 77, 513], np.int64)
    c = cases.decode_case(910, Hq, Hkv, lens, num_blocks=8)
    cu, qs, cl, pos, slot = nvattn.plan_prefill(lens, np.zeros(3, np.int64), c.block_tables)
    T = int(cu[-1])
    rng = np.random.default_rng(911)
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    qw, kw = _norm_weights(rng)
    h = handle(Hq, Hkv, c.cache.num_blocks, max_seqs=3)
    kc, vc = dev(c.cache.k), dev(c.cache.v)
    qh = torch.empty((T, Hq, 128), dtype=torch.float16, device="cuda")
    h.kv_store(0, dev(q), dev(k), dev(v), dev(qw), dev(kw), dev(pos), dev(slot), qh, kc, vc)
    out = torch.full((T, Hq, 128), float("nan"), device="cuda")
    h.prefill(0, qh, dev(cu), dev(qs), dev(cl), dev(c.block_tables), int(lens.max()), kc, vc, out)
    h.check_device()
    got = out.cpu().numpy()
    h.close()

    p = cases.oracle_params(Hq, Hkv, c.cache)
    okc, ovc = c.cache.k.copy(), c.cache.v.copy()
    q_out, k_out = O.qk_norm_rope_store(p, 0, q, k, v, qw, kw, pos, slot, okc, ovc,
                                        want_k_out=True)
    assert np.array_equal(kc.cpu().numpy().view(np.uint16), okc)
    ref = O.concat_prefill_ggml(p, q_out, cu, k_out, v)
    exact = O.paged_prefill(p, O.MODE_TRUTH, 0, q_out, cu, qs, cl, c.block_tables, okc, ovc,
                            new_k=k_out, new_v=v)
    stored = O.paged_prefill(p, O.MODE_TRUTH, 0, q_out, cu, qs, cl, c.block_tables, okc, ovc)
    _, chain = O.err_stats(ref, exact)
    _, storage = O.err_stats(stored, exact)
    mx, mr = O.err_stats(got, stored)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
    mx, mr = O.err_stats(got, ref)
    assert mx <= MAX_ABS and mr <= chain + storage + MEAN_REL, (mx, mr, chain, storage)


def _store_then_prefill(Hq, Hkv, lens, starts, seed, rows, num_blocks=None):
    """Fused store (f16 q, and with `rows` the step's f16 rows) then prefill
    on the GPU; returns the output and the oracle's view of the step."""
    import torch
    lens = np.asarray(lens, np.int64)
    starts = np.asarray(starts, np.int64)
    c = cases.decode_case(seed, Hq, Hkv, lens, num_blocks=num_blocks)
    cu, qs, cl, pos, slot = nvattn.plan_prefill(lens, starts, c.block_tables)
    T = int(cu[-1])
    rng = np.random.default_rng(seed + 1)
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    qw, kw = _norm_weights(rng)
    h = handle(Hq, Hkv, c.cache.num_blocks, max_seqs=len(lens))
    kc, vc = dev(c.cache.k), dev(c.cache.v)
    qh = torch.empty((T, Hq, 128), dtype=torch.float16, device="cuda")
    kr = torch.empty((T, Hkv, 128), dtype=torch.float16, device="cuda") if rows else None
    vr = torch.empty_like(kr) if rows else None
    h.kv_store(0, dev(q), dev(k), dev(v), dev(qw), dev(kw), dev(pos), dev(slot), qh, kc, vc,
               k_rows=kr, v_rows=vr)
    out = torch.full((T, Hq, 128), float("nan"), device="cuda")
    h.prefill(0, qh, dev(cu), dev(qs), dev(cl), dev(c.block_tables), int((cl - qs).max()), kc,
              vc, out, k_rows=kr, v_rows=vr)
    h.check_device()
    got = out.cpu().numpy()
    h.close()
    p = cases.oracle_params(Hq, Hkv, c.cache)
    okc, ovc = c.cache.k.copy(), c.cache.v.copy()
    q_out, k_out = O.qk_norm_rope_store(p, 0, q, k, v, qw, kw, pos, slot, okc, ovc,
                                        want_k_out=True)
    return got, p, (cu, qs, cl, c.block_tables, okc, ovc, q_out, k_out, v)


def test_prefill_step_with_the_steps_own_rows_meets_the_plain_bar(cuda):
    """With the step's own rows in f16 (nvattn_kv_store_qk_norm_rope_rows +
    nvattn_paged_prefill_rows) the prefill attends what the reference's step
    attends -- the graph rows cast to F16 -- so the plain bars hold against
    the reference's FillCausalMask attention over the batch's rows: mean-rel
    <= chain + 1e-3 (chain = its own distance from exact math) and <= 1e-3
    against exact math on the f32 rows."""
    got, p, (cu, qs, cl, bt, okc, ovc, q_out, k_out, v) = _store_then_prefill(
        16, 8, [300, 77, 513], [0, 0, 0], 920, rows=True, num_blocks=8)
    ref = O.concat_prefill_ggml(p, q_out, cu, k_out, v)
    exact = O.paged_prefill(p, O.MODE_TRUTH, 0, q_out, cu, qs, cl, bt, okc, ovc,
                            new_k=k_out, new_v=v)
    _, chain = O.err_stats(ref, exact)
    assert np.isfinite(got).all()
    mx, mr = O.err_stats(got, exact)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
    mx, mr = O.err_stats(got, ref)
    assert mx <= MAX_ABS and mr <= chain + MEAN_REL, (mx, mr, chain)


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (64, 8), (8, 8)])
def test_prefill_rows_with_a_cached_prefix_and_unaligned_starts(cuda, Hq, Hkv):
    """Prefix keys from the BF16 cache, the step's keys from its f16 rows:
    whole-block and unaligned prefix ends (a key tile that straddles the
    prefix end takes its later keys from the rows), a fully cached prompt
    (one row), against exact math on exactly those keys and values."""
    lens, starts = [600, 300, 1030, 1, 700], [512, 44, 1024, 0, 699]
    got, p, (cu, qs, cl, bt, okc, ovc, q_out, k_out, v) = _store_then_prefill(
        Hq, Hkv, lens, starts, 930 + Hq, rows=True)
    f16 = lambda a: a.astype(np.float16).astype(np.float32)
    exact = O.paged_prefill(p, O.MODE_TRUTH, 0, q_out, cu, qs, cl, bt, okc, ovc,
                            new_k=f16(k_out), new_v=f16(v))
    assert np.isfinite(got).all()
    mx, mr = O.err_stats(got, exact)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
