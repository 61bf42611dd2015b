"""Device-side planners (nvattn_plan_prefill_device / nvattn_plan_decode_device)
against the host planners, bit for bit: positions, slot mapping, cu_q_lens,
q_starts and context lengths from device-resident sequence lengths, cached
prefix lengths and block tables -- the reference's PrepareInputs
(src/engine/model_runner.cpp:138-186) over BlockManager's tables
(src/engine/block_manager.cpp:96-184).  Errors are per sequence and come back
through get_error() with the sequence index as detail."""
import numpy as np
import pytest

import nvattn
from gpu_util import dev, handle

pytestmark = pytest.mark.gpu


def _random_tables(rng, lens, bs, max_blocks, n_blocks):
    bt = np.full((len(lens), max_blocks), -1, np.int32)
    perm = rng.permutation(n_blocks)
    k = 0
    for s, L in enumerate(lens):
        nb = -(-int(L) // bs)
        bt[s, :nb] = perm[k:k + nb]
        k += nb
    return bt


def _device_prefill(h, lens, cached, bt, max_tokens):
    import torch
    n = len(lens)
    out = dict(cu=torch.full((n + 1,), -7, dtype=torch.int32, device="cuda:0"),
               qs=torch.full((n,), -7, dtype=torch.int32, device="cuda:0"),
               cl=torch.full((n,), -7, dtype=torch.int32, device="cuda:0"),
               pos=torch.full((max(max_tokens, 1),), -7, dtype=torch.int32, device="cuda:0"),
               slot=torch.full((max(max_tokens, 1),), -7, dtype=torch.int32, device="cuda:0"))
    h.plan_prefill(dev(np.asarray(lens, np.int64)), dev(np.asarray(cached, np.int64)), dev(bt),
                   max_tokens, out["cu"], out["qs"], out["cl"], out["pos"], out["slot"])
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}


@pytest.mark.parametrize("n_seqs,bs,seed", [(1, 256, 0), (7, 256, 1), (64, 128, 2),
                                            (1500, 256, 3), (4096, 512, 4)])
def test_plan_prefill_device_matches_host(n_seqs, bs, seed):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 3000, n_seqs)
    # mix of no hit, block-aligned prefix hits and fully cached prompts
    kind = rng.integers(0, 3, n_seqs)
    cached = np.where(kind == 0, 0, np.where(kind == 1, (lens // bs) * bs // 2 // bs * bs, lens))
    max_blocks = int(-(-lens.max() // bs)) + 2
    n_blocks = int((-(-lens // bs)).sum()) + 5
    bt = _random_tables(rng, lens, bs, max_blocks, n_blocks)
    cu, qs, cl, pos, slot = nvattn.plan_prefill(lens, cached, bt, block_size=bs)
    T = int(cu[-1])
    h = handle(8, 8, n_blocks, block_size=bs, max_context=1024)
    try:
        d = _device_prefill(h, lens, cached, bt, T + 3)
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()
    np.testing.assert_array_equal(d["cu"], cu)
    np.testing.assert_array_equal(d["qs"], qs)
    np.testing.assert_array_equal(d["cl"], cl)
    np.testing.assert_array_equal(d["pos"][:T], pos)
    np.testing.assert_array_equal(d["slot"][:T], slot)
    # tokens past the planned total are left untouched
    assert (d["pos"][T:] == -7).all() and (d["slot"][T:] == -7).all()


def test_plan_prefill_device_fully_cached_prompt():
    bt = np.array([[4, 9]], np.int32)
    h = handle(8, 8, 16)
    try:
        d = _device_prefill(h, [512], [512], bt, 1)
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()
    assert list(d["cu"]) == [0, 1] and d["qs"][0] == 511 and d["cl"][0] == 512
    assert d["pos"][0] == 511 and d["slot"][0] == 9 * 256 + 255


def test_plan_prefill_device_empty_batch():
    import torch
    h = handle(8, 8, 16)
    try:
        cu = torch.full((1,), -7, dtype=torch.int32, device="cuda:0")
        empty64 = torch.zeros(0, dtype=torch.int64, device="cuda:0")
        bt = torch.zeros((0, 4), dtype=torch.int32, device="cuda:0")
        e32 = torch.zeros(0, dtype=torch.int32, device="cuda:0")
        h.plan_prefill(empty64, empty64, bt, 0, cu, e32, e32, e32, e32)
        torch.cuda.synchronize()
        assert cu.item() == 0
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()


@pytest.mark.parametrize("lens,cached,bt_rows,max_tokens,code,detail", [
    ([300, 100], [0, 0], [[1, -1], [3, -1]], 400, nvattn.ERR_OUT_OF_RANGE, 0),   # hole
    ([300, 600], [0, 0], [[1, 2], [3, 4]], 900, nvattn.ERR_INVALID_ARG, 1),      # > max_blocks
    ([300, 100], [0, 200], [[1, 2], [3, -1]], 400, nvattn.ERR_INVALID_ARG, 1),   # cached > len
    ([300, 0], [0, 0], [[1, 2], [3, -1]], 400, nvattn.ERR_INVALID_ARG, 1),       # empty prompt
    ([300, 100], [0, 0], [[1, 2], [3, -1]], 350, nvattn.ERR_INVALID_ARG, 1),     # > max_tokens
])
def test_plan_prefill_device_errors(lens, cached, bt_rows, max_tokens, code, detail):
    bt = np.array(bt_rows, np.int32)
    h = handle(8, 8, 16)
    try:
        _device_prefill(h, lens, cached, bt, max_tokens)
        assert h.get_error() == (code, detail)
        assert h.get_error() == (nvattn.OK, 0)  # reading the error clears it
    finally:
        h.close()
    if max_tokens >= sum(lens):  # the host wrapper sizes max_tokens itself
        with pytest.raises(nvattn.NvattnError) as e:
            nvattn.plan_prefill(lens, cached, bt)
        assert e.value.status == code


@pytest.mark.parametrize("n_seqs,bs,seed", [(1, 256, 0), (256, 256, 1), (3000, 128, 2)])
def test_plan_decode_device_matches_host(n_seqs, bs, seed):
    import torch
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 40000, n_seqs)
    max_blocks = int(-(-lens.max() // bs))
    n_blocks = int((-(-lens // bs)).sum())
    bt = _random_tables(rng, lens, bs, max_blocks, n_blocks)
    cl, pos, slot = nvattn.plan_decode(lens, bt, block_size=bs)
    h = handle(8, 8, n_blocks, block_size=bs, max_context=1024)
    try:
        o = [torch.full((n_seqs,), -7, dtype=torch.int32, device="cuda:0") for _ in range(3)]
        h.plan_decode(dev(lens.astype(np.int64)), dev(bt), *o)
        torch.cuda.synchronize()
        assert h.get_error() == (nvattn.OK, 0)
        got = [t.cpu().numpy() for t in o]
    finally:
        h.close()
    np.testing.assert_array_equal(got[0], cl)
    np.testing.assert_array_equal(got[1], pos)
    np.testing.assert_array_equal(got[2], slot)


@pytest.mark.parametrize("lens,bt_rows,code,detail", [
    ([257, 600], [[1, 2], [3, 4]], nvattn.ERR_INVALID_ARG, 1),   # position past the table
    ([257, 100], [[1, -1], [3, 4]], nvattn.ERR_OUT_OF_RANGE, 0),  # unallocated block
    ([0, 100], [[1, 2], [3, 4]], nvattn.ERR_INVALID_ARG, 0),      # empty sequence
])
def test_plan_decode_device_errors(lens, bt_rows, code, detail):
    import torch
    bt = np.array(bt_rows, np.int32)
    h = handle(8, 8, 16)
    try:
        o = [torch.zeros(2, dtype=torch.int32, device="cuda:0") for _ in range(3)]
        h.plan_decode(dev(np.asarray(lens, np.int64)), dev(bt), *o)
        st, d = h.get_error()
    finally:
        h.close()
    assert (st, d) == (code, detail)
    with pytest.raises(nvattn.NvattnError) as e:
        nvattn.plan_decode(lens, bt)
    assert e.value.status == code


def test_plan_device_is_graph_capturable():
    """The planners launch no allocation and no host sync, so a decode step
    (plan + attention) can be captured once and replayed with new lengths."""
    import torch
    bs, n = 256, 4
    lens = np.array([100, 257, 513, 1], np.int64)
    bt = np.arange(n * 4, dtype=np.int32).reshape(n, 4)
    h = handle(8, 8, 16)
    try:
        d_lens = dev(lens)
        d_bt = dev(bt)
        o = [torch.zeros(n, dtype=torch.int32, device="cuda:0") for _ in range(3)]
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            h.plan_decode(d_lens, d_bt, *o, stream=s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            h.plan_decode(d_lens, d_bt, *o, stream=s)
        for step in range(3):
            cur = lens + step
            d_lens.copy_(torch.from_numpy(cur))
            g.replay()
            torch.cuda.synchronize()
            cl, pos, slot = nvattn.plan_decode(cur, bt, block_size=bs)
            np.testing.assert_array_equal(o[0].cpu().numpy(), cl)
            np.testing.assert_array_equal(o[1].cpu().numpy(), pos)
            np.testing.assert_array_equal(o[2].cpu().numpy(), slot)
        del g
        assert h.get_error() == (nvattn.OK, 0)
    finally:
        h.close()
