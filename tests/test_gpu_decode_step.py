"""GPU tests of the decode step (nvattn_paged_decode_step): the q/k RMSNorm +
NEOX RoPE and the store of each sequence's new token
(nvattn_kv_store_qk_norm_rope) and the paged decode (nvattn_paged_decode),
as one fused launch for grids up to 32 CTAs per SM and as those two launches
above.

Either form must equal the two calls bit for bit -- every stored K/V cache
row and every output row -- because the fused kernel runs the store's row
arithmetic (row_math.cuh) and the same attention; the tests also hold it to
the oracle (the reference's store semantics, exact attention) and check the
error reporting the step adds (in both forms).
"""
import numpy as np
import pytest

import cases
import nvattn
import oracle as O
from gpu_util import dev, handle

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-3


def _norm_weights(rng):
    return (O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32)),
            O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32)))


def _inputs(seed, Hq, Hkv, lens, num_blocks=None):
    c = cases.decode_case(seed, Hq, Hkv, lens, num_blocks=num_blocks)
    rng = np.random.default_rng(seed + 1)
    B = len(c.lens)
    q = rng.standard_normal((B, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
    qw, kw = _norm_weights(rng)
    ctx, pos, slots = nvattn.plan_decode(c.lens, c.block_tables)
    return c, q, k, v, qw, kw, ctx, pos, slots


def _two_calls(h, c, q, k, v, qw, kw, ctx, pos, slots):
    import torch
    kc, vc, dq = dev(c.cache.k), dev(c.cache.v), dev(q)
    h.kv_store(0, dq, dev(k), dev(v), dev(qw), dev(kw), dev(pos), dev(slots), dq, kc, vc)
    out = torch.full((len(ctx), c.Hq, 128), float("nan"), device="cuda")
    h.decode(0, dq, kc, vc, dev(c.block_tables), dev(ctx), int(ctx.max()), out)
    torch.cuda.synchronize()
    return out.cpu().numpy(), kc.cpu().numpy().view(np.uint16), vc.cpu().numpy().view(np.uint16)


def _fused(h, c, q, k, v, qw, kw, ctx, pos, slots, check=True):
    import torch
    kc, vc = dev(c.cache.k), dev(c.cache.v)
    out = torch.full((len(ctx), c.Hq, 128), float("nan"), device="cuda")
    h.decode_step(0, dev(q), dev(k), dev(v), dev(qw), dev(kw), dev(pos), dev(slots), kc, vc,
                  dev(c.block_tables), dev(ctx), int(ctx.max()), out, check=check)
    torch.cuda.synchronize()
    return out.cpu().numpy(), kc.cpu().numpy().view(np.uint16), vc.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("Hq,Hkv,lens", [
    (32, 8, [1, 37, 255, 256, 257, 1000, 2049, 5000]),   # GQA 4; 1 to 3 merged splits
    (16, 8, [37, 256, 513, 1000]),                        # the small-batch decode shape
    (64, 8, [129, 4097, 9000]),                           # GQA 8
    (8, 8, [300, 2048, 2300]),                            # no GQA
])
def test_fused_step_equals_store_then_decode_bit_for_bit(cuda, Hq, Hkv, lens):
    c, q, k, v, qw, kw, ctx, pos, slots = _inputs(1000 + Hq, Hq, Hkv, lens)
    h = handle(Hq, Hkv, c.cache.num_blocks, max_seqs=len(lens))
    ref_out, ref_k, ref_v = _two_calls(h, c, q, k, v, qw, kw, ctx, pos, slots)
    got_out, got_k, got_v = _fused(h, c, q, k, v, qw, kw, ctx, pos, slots)
    h.check_device()
    assert np.array_equal(got_k, ref_k) and np.array_equal(got_v, ref_v)
    assert np.array_equal(got_out.view(np.uint32), ref_out.view(np.uint32))
    # and against the oracle: the reference's store, exact attention
    p = cases.oracle_params(Hq, Hkv, c.cache)
    okc, ovc = c.cache.k.copy(), c.cache.v.copy()
    q_out = O.qk_norm_rope_store(p, 0, q, k, v, qw, kw, pos, slots, okc, ovc)
    assert np.array_equal(got_k, okc) and np.array_equal(got_v, ovc)
    exact = O.paged_decode(p, O.MODE_TRUTH, 0, q_out, okc, ovc, c.block_tables, ctx)
    mx, mr = O.err_stats(got_out, exact)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
    h.close()


def test_fused_step_skips_slot_minus_one(cuda):
    """slot -1 stores nothing (as the KV store) and attends the cache as it is."""
    c, q, k, v, qw, kw, ctx, pos, slots = _inputs(1100, 16, 8, [300, 700])
    slots = slots.copy()
    slots[1] = -1
    h = handle(16, 8, c.cache.num_blocks, max_seqs=2)
    ref_out, ref_k, ref_v = _two_calls(h, c, q, k, v, qw, kw, ctx, pos, slots)
    got_out, got_k, got_v = _fused(h, c, q, k, v, qw, kw, ctx, pos, slots)
    h.check_device()
    assert np.array_equal(got_k, ref_k) and np.array_equal(got_v, ref_v)
    assert np.array_equal(got_out.view(np.uint32), ref_out.view(np.uint32))
    h.close()


def test_fused_step_with_positions_other_than_the_last_token(cuda):
    """The fused kernel loads the RoPE row of position ctx-1 beside the query
    row; a step whose positions differ (an offset position scheme) reloads it
    and still equals the two calls bit for bit."""
    c, q, k, v, qw, kw, ctx, pos, slots = _inputs(1150, 32, 8, [40, 300, 2100, 5000])
    pos = (pos + np.array([7, 0, 1000, 30000], pos.dtype)).astype(pos.dtype)
    h = handle(32, 8, c.cache.num_blocks, max_seqs=4)
    ref_out, ref_k, ref_v = _two_calls(h, c, q, k, v, qw, kw, ctx, pos, slots)
    got_out, got_k, got_v = _fused(h, c, q, k, v, qw, kw, ctx, pos, slots)
    h.check_device()
    assert np.array_equal(got_k, ref_k) and np.array_equal(got_v, ref_v)
    assert np.array_equal(got_out.view(np.uint32), ref_out.view(np.uint32))
    h.close()


def test_fused_step_reports_a_slot_off_the_new_position(cuda):
    """A slot that is not the block table's slot of position ctx-1 is written
    (as the KV store would) but reported: the attention reads position ctx-1
    through the block table."""
    c, q, k, v, qw, kw, ctx, pos, slots = _inputs(1200, 16, 8, [300, 700], num_blocks=8)
    used = set(c.block_tables[c.block_tables >= 0].tolist())
    free = [b for b in range(c.cache.num_blocks) if b not in used]
    bad = slots.copy()
    bad[1] = free[0] * 256 + 5
    h = handle(16, 8, c.cache.num_blocks, max_seqs=2)
    _fused(h, c, q, k, v, qw, kw, ctx, pos, bad)
    st, detail = h.get_error()
    assert st == nvattn.ERR_INVALID_ARG and detail == bad[1]
    h.close()


def test_fused_step_reports_positions_outside_the_rope_table(cuda):
    c, q, k, v, qw, kw, ctx, pos, slots = _inputs(1300, 16, 8, [300, 700])
    bad = pos.copy()
    bad[0] = 50_000  # max_position 40960
    h = handle(16, 8, c.cache.num_blocks, max_seqs=2)
    _fused(h, c, q, k, v, qw, kw, ctx, bad, slots)
    st, detail = h.get_error()
    assert st == nvattn.ERR_OUT_OF_RANGE and detail == 50_000
    h.close()


def test_fused_step_replays_in_a_cuda_graph(cuda):
    """Captured once, replayed with new inputs in the same buffers: each
    replay equals an eager fused step on those inputs."""
    import torch
    c, q, k, v, qw, kw, ctx, pos, slots = _inputs(1400, 32, 8, [40, 600, 3000])
    h = handle(32, 8, c.cache.num_blocks, max_seqs=3)
    bufs = {n: dev(a) for n, a in (("q", q), ("k", k), ("v", v), ("qw", qw), ("kw", kw),
                                   ("pos", pos), ("slots", slots), ("ctx", ctx),
                                   ("bt", c.block_tables))}
    kc, vc = dev(c.cache.k), dev(c.cache.v)
    out = torch.zeros((3, 32, 128), device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        h.decode_step(0, bufs["q"], bufs["k"], bufs["v"], bufs["qw"], bufs["kw"], bufs["pos"],
                      bufs["slots"], kc, vc, bufs["bt"], bufs["ctx"], int(ctx.max()), out,
                      stream=s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        h.decode_step(0, bufs["q"], bufs["k"], bufs["v"], bufs["qw"], bufs["kw"], bufs["pos"],
                      bufs["slots"], kc, vc, bufs["bt"], bufs["ctx"], int(ctx.max()), out,
                      stream=s)
    rng = np.random.default_rng(1401)
    for _ in range(2):
        q2 = rng.standard_normal(q.shape, dtype=np.float32)
        k2 = rng.standard_normal(k.shape, dtype=np.float32)
        bufs["q"].copy_(torch.from_numpy(q2))
        bufs["k"].copy_(torch.from_numpy(k2))
        g.replay()
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        kc2, vc2 = kc.clone(), vc.clone()
        want = torch.zeros_like(out)
        h.decode_step(0, bufs["q"], bufs["k"], bufs["v"], bufs["qw"], bufs["kw"], bufs["pos"],
                      bufs["slots"], kc2, vc2, bufs["bt"], bufs["ctx"], int(ctx.max()), want)
        torch.cuda.synchronize()
        assert np.array_equal(got.view(np.uint32), want.cpu().numpy().view(np.uint32))
        assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    h.check_device()
    del g
    h.close()


def _expected_launches(sm, n_seqs, Hkv, max_ctx):
    """The step's rule restated: the decode's split (2048 tokens, halved while
    the grid would not fill the GPU eight times over, at least 256), then one
    launch while the grid stays within 32 CTAs per SM."""
    split = 2048
    while split > 256 and n_seqs * Hkv * -(-max_ctx // split) < 8 * sm:
        split //= 2
    return 1 if n_seqs * Hkv * max(1, -(-max_ctx // split)) <= 32 * sm else 2


def test_step_form_follows_the_grid(cuda):
    import torch
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    h = handle(32, 8, 64, max_seqs=512)
    assert h.decode_step_launches(0, 1000) == 0
    for n, L in ((4, 1000), (64, 32768), (128, 32768), (256, 32768), (512, 2048)):
        assert h.decode_step_launches(n, L) == _expected_launches(sm, n, 8, L), (n, L)
    for n, L in ((-1, 1000), (513, 1000), (4, 40961), (4, -1)):  # handle: 512 seqs, 40960
        with pytest.raises(nvattn.NvattnError):
            h.decode_step_launches(n, L)
    if sm == 148:  # B200: the large-batch workload's full grid and its 8-way shard
        assert h.decode_step_launches(256, 32768) == 2
        assert h.decode_step_launches(64, 32768) == 2   # the 4-way shard: 8,192
        assert h.decode_step_launches(32, 32768) == 1   # the 8-way shard: 4,096
    h.close()


def _two_launch_inputs(seed):
    """128 sequences, one of 32k tokens: 16,384 grid CTAs (two launches on a
    148-SM B200)."""
    lens = [32768] + np.random.default_rng(seed).integers(1, 600, 127).tolist()
    return _inputs(seed, 32, 8, lens)


def test_two_launch_step_equals_store_then_decode_bit_for_bit(cuda):
    import torch
    c, q, k, v, qw, kw, ctx, pos, slots = _two_launch_inputs(1500)
    h = handle(32, 8, c.cache.num_blocks, max_seqs=len(ctx))
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    assert h.decode_step_launches(len(ctx), int(ctx.max())) == _expected_launches(
        sm, len(ctx), 8, int(ctx.max()))
    ref_out, ref_k, ref_v = _two_calls(h, c, q, k, v, qw, kw, ctx, pos, slots)
    got_out, got_k, got_v = _fused(h, c, q, k, v, qw, kw, ctx, pos, slots)
    h.check_device()
    assert np.array_equal(got_k, ref_k) and np.array_equal(got_v, ref_v)
    assert np.array_equal(got_out.view(np.uint32), ref_out.view(np.uint32))
    h.close()


def test_two_launch_step_reports_a_slot_off_the_new_position(cuda):
    c, q, k, v, qw, kw, ctx, pos, slots = _two_launch_inputs(1600)
    used = set(c.block_tables[c.block_tables >= 0].tolist())
    free = [b for b in range(c.cache.num_blocks) if b not in used]
    bad = slots.copy()
    bad[3] = free[0] * 256 + 7
    h = handle(32, 8, c.cache.num_blocks, max_seqs=len(ctx))
    _fused(h, c, q, k, v, qw, kw, ctx, pos, bad)
    st, detail = h.get_error()
    assert st == nvattn.ERR_INVALID_ARG and detail == bad[3]
    h.close()
