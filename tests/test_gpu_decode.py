"""GPU parity of nvattn_paged_decode against the oracle.

Tolerances (BF16 inputs, FP32 accumulate):
  * against fp64 math (oracle TRUTH): max-abs-err <= 2e-2 and
    mean-rel-err <= 1e-3 (sum|a-b| / sum|b|); in practice ~1e-6.
  * against the reference's dtype chain (oracle GGML: f16 Q/K/V, f16 V
    accumulator): max-abs-err <= 2e-2, and mean-rel-err no more than 1e-3
    above the distance between that chain and exact math (the chain itself
    sits ~2e-3 from exact math at these shapes).
"""
import numpy as np
import pytest

import cases
import make_golden
import nvattn
import oracle as O
from gpu_util import dev, handle

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-3


def run_decode(c: cases.DecodeCase, h=None, block_tables=None, max_context=None, k=None, v=None):
    import torch
    if h is None:
        h = handle(c.Hq, c.Hkv, c.cache.num_blocks, n_layer=c.cache.n_layer,
                   max_seqs=max(len(c.lens), 1))
    bt = c.block_tables if block_tables is None else block_tables
    out = torch.full((len(c.lens), c.Hq, 128), float("nan"), device="cuda")
    mc = int(c.lens.max()) if max_context is None else max_context
    h.decode(c.layer, dev(c.q), dev(c.cache.k if k is None else k),
             dev(c.cache.v if v is None else v), dev(bt), dev(c.lens), mc, out)
    torch.cuda.synchronize()
    return h, out.cpu().numpy()


def check_truth(got, c):
    p = cases.oracle_params(c.Hq, c.Hkv, c.cache)
    ref = O.paged_decode(p, O.MODE_TRUTH, c.layer, c.q, c.cache.k, c.cache.v, c.block_tables,
                         c.lens)
    mx, mr = O.err_stats(got, ref)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)
    assert mx <= 1e-4, mx  # fp32 accumulation: far inside the tolerance
    return ref


def test_golden_decode_qwen3_0p6b(cuda):
    fx = np.load(make_golden.__file__.replace("make_golden.py", "decode_qwen3_0p6b.npz"))
    c = make_golden.decode_inputs()
    assert np.array_equal(make_golden._digest(c.q, c.cache.k, c.cache.v, c.block_tables, c.lens),
                          fx["inputs_sha256"])
    h, got = run_decode(c)
    h.check_device()
    mx, mr = O.err_stats(got, fx["out_truth"])
    assert mx <= 1e-4 and mr <= MEAN_REL
    mx_g, mr_g = O.err_stats(got, fx["out_ggml"])
    _, chain = O.err_stats(fx["out_truth"], fx["out_ggml"])
    assert mx_g <= MAX_ABS and mr_g <= chain + MEAN_REL, (mx_g, mr_g, chain)


@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (16, 8), (32, 8), (64, 8), (4, 1)])
def test_gqa_groups(cuda, Hq, Hkv):
    c = cases.decode_case(Hq + Hkv, Hq, Hkv, [1, 63, 64, 65, 255, 256, 257, 1000, 2049])
    h, got = run_decode(c)
    h.check_device()
    check_truth(got, c)


@pytest.mark.parametrize("lens", [[5000], [9000, 17, 12000], [40960], [3, 40000, 256, 511]])
def test_long_contexts_use_split_combine(cuda, lens):
    c = cases.decode_case(sum(lens), 32, 8, lens)
    h, got = run_decode(c)
    h.check_device()
    check_truth(got, c)


def test_many_sequences_config3_shape_sampled(cuda):
    """256 sequences of the large-batch decode shape (32 q / 8 kv heads),
    lengths log-uniform in [1, 2048] to keep the oracle quick."""
    rng = np.random.default_rng(33)
    lens = np.exp(rng.uniform(0, np.log(2048), 256)).astype(np.int32) + 1
    c = cases.decode_case(34, 32, 8, lens)
    h, got = run_decode(c)
    h.check_device()
    check_truth(got, c)


def test_block_permutation_gives_identical_bits(cuda):
    c = cases.decode_case(40, 16, 8, [700, 300, 1500], num_blocks=32)
    h, ref = run_decode(c)
    bt2 = c.block_tables.copy()
    k2, v2 = c.cache.k.copy(), c.cache.v.copy()
    used = set(c.block_tables[c.block_tables >= 0].tolist())
    free = [b for b in range(c.cache.num_blocks) if b not in used]
    for j in range(3):
        old, new = c.block_tables[0, j], free[j]
        k2[0, new * 256:(new + 1) * 256] = c.cache.k[0, old * 256:(old + 1) * 256]
        v2[0, new * 256:(new + 1) * 256] = c.cache.v[0, old * 256:(old + 1) * 256]
        k2[0, old * 256:(old + 1) * 256] = 0
        bt2[0, j] = new
    _, got = run_decode(c, h=h, block_tables=bt2, k=k2, v=v2)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_layer_offset_and_zero_context(cuda):
    c = cases.decode_case(41, 16, 8, [0, 300, 1], n_layer=3, layer=2)
    h, got = run_decode(c)
    h.check_device()
    assert not got[0].any()
    check_truth(got, c)


def test_bad_block_id_is_reported_not_faulted(cuda):
    c = cases.decode_case(42, 16, 8, [600, 100])
    bt = c.block_tables.copy()
    bt[0, 1] = c.cache.num_blocks + 5
    h, _ = run_decode(c, block_tables=bt)
    st, detail = h.get_error()
    assert st == nvattn.ERR_OUT_OF_RANGE and detail == c.cache.num_blocks + 5
    # the handle stays usable
    _, got = run_decode(c, h=h)
    assert h.get_error()[0] == nvattn.OK
    check_truth(got, c)


def test_context_above_declared_max_is_reported(cuda):
    c = cases.decode_case(43, 16, 8, [600, 100])
    h, _ = run_decode(c, max_context=512)
    st, detail = h.get_error()
    assert st == nvattn.ERR_OUT_OF_RANGE and detail == 600


def test_host_validation(cuda):
    import torch
    c = cases.decode_case(44, 16, 8, [10])
    h = handle(16, 8, c.cache.num_blocks, max_seqs=1)
    out = torch.empty((1, 16, 128), device="cuda")
    # max_context_len beyond the block table's reach
    st = h.decode(0, dev(c.q), dev(c.cache.k), dev(c.cache.v), dev(c.block_tables), dev(c.lens),
                  10_000, out, check=False)
    assert st == nvattn.ERR_INVALID_ARG
    # layer out of range
    st = h.decode(1, dev(c.q), dev(c.cache.k), dev(c.cache.v), dev(c.block_tables), dev(c.lens),
                  10, out, check=False)
    assert st == nvattn.ERR_INVALID_ARG


def test_descriptor_cache_with_more_cache_buffers_than_it_holds(cuda):
    """One handle decodes over 20 distinct K/V buffer pairs (40 bases, more
    than the 16 TMA descriptors a handle caches), twice over in different
    orders and once with K and V swapped: every launch must read the buffers
    it was given."""
    import torch
    Hq, Hkv, nb = 16, 8, 8
    h = handle(Hq, Hkv, nb, max_seqs=3)
    cs = [cases.decode_case(600 + i, Hq, Hkv, [300, 1, 900], num_blocks=nb) for i in range(20)]
    bufs = [(dev(c.cache.k), dev(c.cache.v)) for c in cs]
    p = cases.oracle_params(Hq, Hkv, cs[0].cache)
    order = list(range(20)) + [19 - i for i in range(20)] + [3, 17, 3, 0]
    for n, i in enumerate(order):
        c = cs[i]
        kd, vd = bufs[i]
        swap = n == len(order) - 1
        if swap:
            kd, vd = vd, kd
        out = torch.full((3, Hq, 128), float("nan"), device="cuda")
        h.decode(0, dev(c.q), kd, vd, dev(c.block_tables), dev(c.lens), 900, out)
        torch.cuda.synchronize()
        kh, vh = (c.cache.v, c.cache.k) if swap else (c.cache.k, c.cache.v)
        ref = O.paged_decode(p, O.MODE_TRUTH, 0, c.q, kh, vh, c.block_tables, c.lens)
        mx, mr = O.err_stats(out.cpu().numpy(), ref)
        assert mx <= 1e-4 and mr <= MEAN_REL, (n, i, mx, mr)
    h.check_device()


def test_split_tickets_rearm_across_launches_shapes_and_graph_replays(cuda):
    """The last split CTA of each (sequence, kv head) merges the partials and
    re-arms that pair's ticket; launches with other split counts, alternating
    batch shapes and CUDA-graph replays must each give the first launch's
    bits."""
    import torch
    Hq, Hkv = 32, 8
    ca = cases.decode_case(70, Hq, Hkv, [9000, 300, 20000, 4100], num_blocks=140)
    cb = cases.decode_case(71, Hq, Hkv, [700, 33000], num_blocks=140)
    h = handle(Hq, Hkv, 140, max_seqs=4, max_context=40960)

    def launch(c, out, stream=None):
        h.decode(0, ins[id(c)][0], ins[id(c)][1], ins[id(c)][2], ins[id(c)][3], ins[id(c)][4],
                 int(c.lens.max()), out, stream=stream)

    ins = {id(c): (dev(c.q), dev(c.cache.k), dev(c.cache.v), dev(c.block_tables), dev(c.lens))
           for c in (ca, cb)}
    outs = {id(c): torch.empty((len(c.lens), Hq, 128), device="cuda") for c in (ca, cb)}
    first = {}
    for rep in range(3):
        for c in (ca, cb):
            launch(c, outs[id(c)])
            torch.cuda.synchronize()
            bits = outs[id(c)].cpu().numpy().view(np.uint32).copy()
            if rep == 0:
                first[id(c)] = bits
                check_truth(outs[id(c)].cpu().numpy(), c)
            assert np.array_equal(bits, first[id(c)]), (rep, len(c.lens))
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            launch(ca, outs[id(ca)], stream=s)
            launch(cb, outs[id(cb)], stream=s)
    for _ in range(3):
        for c in (ca, cb):
            outs[id(c)].fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for c in (ca, cb):
            assert np.array_equal(outs[id(c)].cpu().numpy().view(np.uint32), first[id(c)])
    h.check_device()
