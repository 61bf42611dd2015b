"""nvattn_paged_decode_noalloc: paged decode for callers that cannot
allocate device memory (an engine that has given nearly all of the GPU to its
KV cache, or a host that may not call cudaMalloc while serving a step).  The
entry point needs no handle and keeps its split-KV partials in a fixed 32 MiB
array inside the library; its results must equal those of the handle-based
nvattn_paged_decode, call after call, although every call reuses that array.

This file is named so that pytest collects it last.
"""
import numpy as np
import pytest

import cases
import nvattn
import oracle as O
from gpu_util import dev, handle

pytestmark = pytest.mark.gpu


def _cfg(Hq, Hkv, num_blocks, max_context=40960):
    return nvattn.qwen3_config(n_layer=1, n_q_heads=Hq, n_kv_heads=Hkv, num_blocks=num_blocks,
                               max_context=max_context, max_position=max_context, device=0)


def test_noalloc_decode_matches_handle_decode_on_consecutive_calls(cuda):
    import torch
    Hq, Hkv = 16, 8
    # two different problems of the same shape class, run back to back: the
    # second call must not see anything the first left in the shared scratch
    c1 = cases.decode_case(501, Hq, Hkv, [5000, 300, 9000], num_blocks=70)
    c2 = cases.decode_case(502, Hq, Hkv, [7000, 8191, 1], num_blocks=70)
    cfg = _cfg(Hq, Hkv, 70)
    h = handle(Hq, Hkv, 70, max_seqs=8)
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    for c in (c1, c2):
        args = (dev(c.q), dev(c.cache.k), dev(c.cache.v), dev(c.block_tables), dev(c.lens))
        mc = int(c.lens.max())
        ref = torch.full((3, Hq, 128), float("nan"), device="cuda")
        h.decode(0, *args, mc, ref)
        out = torch.full((3, Hq, 128), float("nan"), device="cuda")
        st = nvattn.decode_noalloc(cfg, 0, *args, mc, out, status=status)
        assert st == nvattn.OK, nvattn.status_string(st)
        torch.cuda.synchronize()
        h.check_device()
        got, want = out.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(got).all()
        # same kernel, same splits, same combine order: the same bits
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        assert int(status[0].item()) == nvattn.OK
        # and within the attention bars of exact (fp64) math
        p = cases.oracle_params(Hq, Hkv, c.cache)
        truth = O.paged_decode(p, O.MODE_TRUTH, 0, c.q, c.cache.k, c.cache.v, c.block_tables,
                               c.lens)
        mx, mr = O.err_stats(got, truth)
        assert mx <= 2e-2 and mr <= 1e-3, (mx, mr)


def test_noalloc_rejects_work_beyond_its_scratch(cuda):
    import torch
    Hq, Hkv, B, L = 32, 8, 512, 8192
    # the rejection depends on n_seqs, the heads and the split count only and
    # happens on the host before any kernel reads the cache, so a one-block
    # cache stands in for the (declared) 16,384-block one
    cfg = _cfg(Hq, Hkv, B * 32, max_context=L)
    q = torch.zeros((B, Hq, 128), device="cuda")
    kc = torch.zeros((256, Hkv, 128), dtype=torch.int16, device="cuda")
    bt = torch.zeros((B, 32), dtype=torch.int32, device="cuda")
    lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
    out = torch.zeros((B, Hq, 128), device="cuda")
    # 512 sequences x 32 heads x 4 splits x 520 B > 32 MiB
    st = nvattn.decode_noalloc(cfg, 0, q, kc, kc, bt, lens, L, out)
    assert st == nvattn.ERR_SCRATCH_LIMIT
    assert "32 MiB" in nvattn.status_string(st)
