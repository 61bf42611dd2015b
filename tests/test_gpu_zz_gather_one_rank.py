"""The decode step with the all-gather over peer memory
(nvattn_paged_decode_step_gather) as one rank on one GPU.

A one-rank gather runs the kernel path of the N-rank one -- every final
output row stored a second time, into the gathered buffer's step parity;
the launch's last final-row CTA releasing the step on the counter and
waiting until the count shows it -- with this rank's own buffer as the only
destination, so it needs no second GPU (the two-GPU run is
tests/test_gpu_peer_gather.py).  Its output rows and gathered rows must
equal the plain step's bit for bit, step after step, in both step forms
(one fused launch, and the store then the decode for grids above 32 CTAs
per SM), across a step with no sequences (released by a one-thread launch
instead), and only the latest step can be read back.

Collected after the other GPU parity tests: a failure here does not hide
theirs in a run that stops at the first failure.
"""
import ctypes

import numpy as np
import pytest

import cases
import nvattn
import oracle as O
from gpu_util import dev, handle

pytestmark = pytest.mark.gpu


def _inputs(seed, Hq, Hkv, lens, num_blocks=None):
    c = cases.decode_case(seed, Hq, Hkv, lens, num_blocks=num_blocks)
    rng = np.random.default_rng(seed + 1)
    B = len(c.lens)
    q = rng.standard_normal((B, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
    qw = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    kw = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    ctx, pos, slots = nvattn.plan_decode(c.lens, c.block_tables)
    return c, q, k, v, qw, kw, ctx, pos, slots


@pytest.mark.parametrize("Hq,Hkv,lens,launches", [
    (32, 8, [1, 37, 255, 256, 257, 1000, 2049, 5000], 1),  # one to three merged splits
    (32, 8, list(range(1, 601)), 2),                       # 600 x 8 one-split CTAs
])
def test_one_rank_gather_equals_the_plain_step(cuda, Hq, Hkv, lens, launches):
    import torch
    c, q, k, v, qw, kw, ctx, pos, slots = _inputs(3100 + len(lens), Hq, Hkv, lens)
    B, mc = len(lens), int(ctx.max())
    args = (dev(q), dev(k), dev(v), dev(qw), dev(kw), dev(pos), dev(slots))
    bt, dctx = dev(c.block_tables), dev(ctx)

    h = handle(Hq, Hkv, c.cache.num_blocks, max_seqs=B)
    assert h.decode_step_launches(B, mc) == launches
    kc, vc = dev(c.cache.k), dev(c.cache.v)
    ref = torch.full((B, Hq, 128), float("nan"), device="cuda")
    h.decode_step(0, *args, kc, vc, bt, dctx, mc, ref)
    torch.cuda.synchronize()
    h.check_device()
    ref_bits = ref.cpu().numpy().view(np.uint32)
    ref_k, ref_v = kc.cpu().numpy(), vc.cpu().numpy()

    hg = handle(Hq, Hkv, c.cache.num_blocks, max_seqs=B)
    hg.gather_connect([hg.gather_init(1, 0)])
    gkc, gvc = dev(c.cache.k), dev(c.cache.v)
    out = torch.empty((B, Hq, 128), device="cuda")
    got = torch.empty((1, B, Hq, 128), device="cuda")
    step = 0
    for rnd in range(4):
        if rnd == 2:
            # a step with no sequences: no decode launch, the one-thread
            # release in its place keeps the step count
            st = nvattn.lib().nvattn_paged_decode_step_gather(
                hg._h, 0, 0, *[ctypes.c_void_p(t.data_ptr()) for t in args],
                ctypes.c_void_p(gkc.data_ptr()), ctypes.c_void_p(gvc.data_ptr()),
                ctypes.c_void_p(bt.data_ptr()), c.block_tables.shape[1],
                ctypes.c_void_p(dctx.data_ptr()), mc, ctypes.c_void_p(out.data_ptr()), None)
            assert st == nvattn.OK, nvattn.status_string(st)
            step += 1
            continue
        out.fill_(float("nan"))
        got.fill_(float("nan"))
        # the same new rows at the same slots each step: the cache and the
        # outputs stay those of the plain step
        hg.decode_step_gather(0, *args, gkc, gvc, bt, dctx, mc, out)
        hg.gather_read(step, B, got)
        torch.cuda.synchronize()
        hg.check_device()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), ref_bits), rnd
        assert np.array_equal(got[0].cpu().numpy().view(np.uint32), ref_bits), rnd
        step += 1
    assert np.array_equal(gkc.cpu().numpy(), ref_k) and np.array_equal(gvc.cpu().numpy(), ref_v)
    # only the latest step can be read back
    with pytest.raises(nvattn.NvattnError):
        hg.gather_read(step - 2, B, got)
    hg.gather_read(step - 1, B, got)
    torch.cuda.synchronize()
    assert np.array_equal(got[0].cpu().numpy().view(np.uint32), ref_bits)
