"""CPU tests of the oracle itself: known answers, IEEE edge cases, the
reference's concat-all decode and prefill algorithms, and the committed
golden fixtures.

Parity against the reference is unpinned (no reference tests exist and ggml
is not vendored); these tests pin the restatement instead.
"""
import os

import numpy as np
import pytest

import cases
import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def bits(f):
    return np.array([f], dtype=np.float32).view(np.uint32)[0]


def f32(u):
    return float(np.array([u], dtype=np.uint32).view(np.float32)[0])


# ---------------------------------------------------------------- conversions

@pytest.mark.parametrize("u,expect", [
    (0x3f800000, 0x3f80),  # 1.0
    (0x3f808000, 0x3f80),  # tie, even stays
    (0x3f818000, 0x3f82),  # tie, odd rounds up
    (0x3f808001, 0x3f81),  # above tie
    (0x3f807fff, 0x3f80),  # below tie
    (0x80000000, 0x8000),  # -0
    (0x7f800000, 0x7f80),  # +inf
    (0xff800000, 0xff80),  # -inf
    (0x7f7fffff, 0x7f80),  # max finite rounds to inf
    (0x00000001, 0x0000),  # smallest subnormal rounds to 0
    (0x00008000, 0x0000),  # subnormal tie to even (0)
    (0x00018000, 0x0002),  # subnormal tie to even (2)
    (0x7fc00001, 0x7fc0),  # quiet NaN keeps top payload
    (0x7f800001, 0x7fc0),  # signalling NaN forced quiet (| 64)
    (0xff812345, 0xffc1),
])
def test_bf16_rounding_edge_cases(u, expect):
    assert O.lib().orc_f32_to_bf16(f32(u)) == expect


def test_bf16_matches_torch_rne_on_random_values():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32),
                        (rng.standard_normal(1000) * 1e-39).astype(np.float32),
                        (rng.uniform(-3e38, 3e38, 1000)).astype(np.float32)])
    ours = O.f32_to_bf16(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)


@pytest.mark.parametrize("x,expect", [
    (1.0, 0x3c00), (-2.0, 0xc000), (65504.0, 0x7bff), (65520.0, 0x7c00), (65519.0, 0x7bff),
    (2.0 ** -14, 0x0400), (2.0 ** -24, 0x0001), (2.0 ** -25, 0x0000), (3 * 2.0 ** -26, 0x0001),
    (1.0 + 2.0 ** -11, 0x3c00), (1.0 + 3 * 2.0 ** -11, 0x3c02), (float("inf"), 0x7c00),
])
def test_f16_rounding_edge_cases(x, expect):
    assert O.lib().orc_f32_to_f16(x) == expect


def test_f16_roundtrip_matches_numpy():
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.standard_normal(50000), rng.standard_normal(5000) * 1e-5,
                        rng.uniform(-6.5e4, 6.5e4, 5000)]).astype(np.float32)
    ours = np.array([O.lib().orc_f32_to_f16(float(v)) for v in x], dtype=np.uint16)
    assert np.array_equal(ours, x.astype(np.float16).view(np.uint16))
    back = np.array([O.lib().orc_f16_to_f32(int(h)) for h in ours[:2000]], dtype=np.float32)
    assert np.array_equal(back, ours[:2000].view(np.float16).astype(np.float32))


# ---------------------------------------------------------------- RoPE

def test_rope_corr_dims_qwen3():
    dims = (ctypes_floats := np.zeros(2, np.float32))
    O.lib().orc_rope_corr_dims(128, 40960, O.ctypes.c_float(1e6), O.ctypes.c_float(32.0),
                               O.ctypes.c_float(1.0), ctypes_floats.ctypes.data_as(O.ctypes.c_void_p))
    assert list(dims) == [24.0, 41.0]


def test_rope_table_properties():
    p = O.params()
    t = O.rope_table(4096, p)
    assert np.all(t[0, :, 0] == 1.0) and np.all(t[0, :, 1] == 0.0)  # position 0: identity
    mag = t[..., 0].astype(np.float64) ** 2 + t[..., 1].astype(np.float64) ** 2
    assert np.abs(mag - 1).max() < 1e-6
    # pair 0 rotates by exactly the position (theta_scale^0 = 1)
    pos = np.arange(4096)
    assert np.allclose(t[:, 0, 0], np.cos(pos), atol=1e-6)
    # high pairs: theta = pos * 1e6^(-2i/128), up to float recurrence error
    i = 100 // 2
    th = pos * (1e6 ** (-2 * i / 128))
    assert np.allclose(t[:, i, 1], np.sin(th), atol=1e-4)


def test_norm_rope_store_identity_at_pos0_and_unit_weights():
    rng = np.random.default_rng(3)
    Hq, Hkv, T = 4, 2, 3
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=256)
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    w = O.f32_to_bf16(np.ones(128, np.float32))
    kc = np.zeros((1, 256, Hkv, 128), np.uint16)
    vc = np.zeros_like(kc)
    pos = np.zeros(T, np.int32)
    slots = np.array([5, -1, 7], np.int32)
    q_out, k_out = O.qk_norm_rope_store(p, 0, q, k, v, w, w, pos, slots, kc, vc, want_k_out=True)
    ref = q / np.sqrt((q.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-6)
    assert np.abs(q_out - ref).max() < 1e-5
    assert np.array_equal(kc[0, 5], O.f32_to_bf16(k_out[0]))
    assert np.array_equal(vc[0, 7], O.f32_to_bf16(v[2]))
    assert not kc[0, :5].any() and not kc[0, 6].any()  # slot -1 not stored


# ---------------------------------------------------------------- attention

@pytest.mark.parametrize("mode", [O.MODE_TRUTH, O.MODE_GGML])
def test_single_key_returns_v(mode):
    c = cases.decode_case(4, 4, 2, [1, 1])
    p = cases.oracle_params(4, 2, c.cache)
    out = O.paged_decode(p, mode, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens)
    for s in range(2):
        slot = c.block_tables[s, 0] * 256
        for h in range(4):
            v = O.bf16_to_f32(c.cache.v[0, slot, h // 2])
            tol = 0 if mode == O.MODE_TRUTH else 1e-3  # f16 V accumulator
            assert np.abs(out[s, h] - v).max() <= tol * np.abs(v).max()


@pytest.mark.parametrize("mode", [O.MODE_TRUTH, O.MODE_GGML])
def test_constant_keys_give_mean_of_v(mode):
    c = cases.decode_case(5, 2, 1, [300])
    slots = [c.block_tables[0, t // 256] * 256 + t % 256 for t in range(300)]
    c.cache.k[0, slots] = c.cache.k[0, slots[0]]
    p = cases.oracle_params(2, 1, c.cache)
    out = O.paged_decode(p, mode, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens)
    mean_v = O.bf16_to_f32(c.cache.v[0, slots, 0]).astype(np.float64).mean(0)
    tol = 1e-6 if mode == O.MODE_TRUTH else 3e-3
    assert np.abs(out[0, 0] - mean_v).max() < tol


def test_reference_concat_decode_is_bit_identical_to_paged_restatement():
    """The reference's decode algorithm (gather all histories, concat the new
    rows after them, varlen mask) visits each sequence's keys in the same order
    as the paged restatement, so the two agree bit for bit."""
    rng = np.random.default_rng(6)
    c = cases.decode_case(6, 16, 8, [37, 256, 513, 1000], num_blocks=64)
    p = cases.oracle_params(16, 8, c.cache)
    nk = rng.standard_normal((4, 8, 128), dtype=np.float32)
    nv = rng.standard_normal((4, 8, 128), dtype=np.float32)
    a = O.concat_decode_ggml(p, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens, nk, nv)
    b = O.paged_decode(p, O.MODE_GGML, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens,
                       nk, nv)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("Hq,Hkv,lens", [(16, 8, [300, 1, 129, 700]), (32, 8, [257, 511]),
                                         (8, 8, [1, 2, 3, 640]), (2, 1, [1000])])
def test_reference_concat_prefill_is_bit_identical_to_paged_restatement(Hq, Hkv, lens):
    """The reference's prefill (the batch's new tokens concatenated, f32 K/V
    padded and cast to F16, FillCausalMask's block-diagonal causal mask over
    the whole buffer) visits a row's keys in the same order as the paged
    restatement given the same f32 new rows; without a cached prefix the two
    agree bit for bit."""
    rng = np.random.default_rng(8 + Hq)
    c = cases.prefill_case(8 + Hq, Hq, Hkv, lens, [0] * len(lens))
    p = cases.oracle_params(Hq, Hkv, c.cache)
    T = int(c.cu_q[-1])
    nk = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    nv = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    a = O.concat_prefill_ggml(p, c.q, c.cu_q, nk, nv)
    b = O.paged_prefill(p, O.MODE_GGML, 0, c.q, c.cu_q, c.q_starts, c.seq_lens, c.block_tables,
                        c.cache.k, c.cache.v, nk, nv)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_reference_concat_prefill_ignores_a_cached_prefix():
    """With a cached prefix the reference's prefill attends only the batch's
    own tokens; the paged restatement (and the kernel) attend the prefix too,
    so the rows differ (by design, not a tolerance question)."""
    rng = np.random.default_rng(9)
    c = cases.prefill_case(9, 2, 1, [600], [256])
    p = cases.oracle_params(2, 1, c.cache)
    nk = rng.standard_normal((344, 1, 128), dtype=np.float32)
    nv = rng.standard_normal((344, 1, 128), dtype=np.float32)
    a = O.concat_prefill_ggml(p, c.q, c.cu_q, nk, nv)
    b = O.paged_prefill(p, O.MODE_GGML, 0, c.q, c.cu_q, c.q_starts, c.seq_lens, c.block_tables,
                        c.cache.k, c.cache.v, nk, nv)
    assert np.abs(a - b).max() > 1e-2


def test_block_permutation_invariance():
    c = cases.decode_case(7, 8, 4, [700, 129], num_blocks=12)
    p = cases.oracle_params(8, 4, c.cache)
    ref = O.paged_decode(p, O.MODE_TRUTH, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens)
    # move sequence 0's blocks to other physical ids
    bt2 = c.block_tables.copy()
    used = set(c.block_tables[c.block_tables >= 0].tolist())
    free = [b for b in range(c.cache.num_blocks) if b not in used]
    k2, v2 = c.cache.k.copy(), c.cache.v.copy()
    for j in range(3):
        old, new = c.block_tables[0, j], free[j]
        k2[0, new * 256:(new + 1) * 256] = c.cache.k[0, old * 256:(old + 1) * 256]
        v2[0, new * 256:(new + 1) * 256] = c.cache.v[0, old * 256:(old + 1) * 256]
        k2[0, old * 256:(old + 1) * 256] = 0
        bt2[0, j] = new
    out = O.paged_decode(p, O.MODE_TRUTH, 0, c.q, k2, v2, bt2, c.lens)
    assert np.array_equal(out, ref)


def test_decode_equals_last_prefill_row():
    c = cases.prefill_case(8, 4, 2, [600], [0])
    p = cases.oracle_params(4, 2, c.cache)
    pre = O.paged_prefill(p, O.MODE_TRUTH, 0, c.q, c.cu_q, c.q_starts, c.seq_lens,
                          c.block_tables, c.cache.k, c.cache.v)
    dec = O.paged_decode(p, O.MODE_TRUTH, 0, np.ascontiguousarray(c.q[-1:]), c.cache.k,
                         c.cache.v, c.block_tables, c.seq_lens)
    assert np.array_equal(pre[-1], dec[0])


def test_prefix_hit_rows_equal_full_prefill_rows():
    c = cases.prefill_case(9, 4, 2, [700], [0])
    p = cases.oracle_params(4, 2, c.cache)
    full = O.paged_prefill(p, O.MODE_TRUTH, 0, c.q, c.cu_q, c.q_starts, c.seq_lens,
                           c.block_tables, c.cache.k, c.cache.v)
    qs = np.array([512], np.int32)
    cu = np.array([0, 188], np.int32)
    part = O.paged_prefill(p, O.MODE_TRUTH, 0, np.ascontiguousarray(c.q[512:]), cu, qs,
                           c.seq_lens, c.block_tables, c.cache.k, c.cache.v)
    assert np.array_equal(part, full[512:])


def test_ggml_chain_distance_from_exact_math():
    """Documents how far the reference's dtype chain (f16 K/V/Q, f16 V
    accumulator) sits from fp64 math at the decode workload's shape."""
    c = cases.decode_case(10, 16, 8, [37, 256, 513, 1000], num_blocks=64)
    p = cases.oracle_params(16, 8, c.cache)
    t = O.paged_decode(p, O.MODE_TRUTH, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens)
    g = O.paged_decode(p, O.MODE_GGML, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens)
    mx, mr = O.err_stats(g, t)
    assert mx < 2e-2
    assert mr < 4e-3


# ---------------------------------------------------------------- golden fixtures

def _load(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.mark.parametrize("name", ["decode_qwen3_0p6b.npz", "kv_store_qwen3_0p6b.npz",
                                  "prefill_prefix_hit.npz"])
def test_oracle_reproduces_golden_fixture(name):
    import make_golden
    fx = _load(name)
    again = make_golden.BUILDERS[name]()
    for key in fx.files:
        assert np.array_equal(fx[key], again[key]), key
