"""GPU parity of nvattn_kv_store_qk_norm_rope against the oracle: the normed,
rotated q (f32, bf16 and f16) and the bf16 K/V cache rows must match bit for bit
(StorePrefillKV / AppendDecodeKV semantics, model_runner.cpp:248-415)."""
import numpy as np
import pytest

import make_golden
import nvattn
import oracle as O
from gpu_util import dev, handle, host_bits

pytestmark = pytest.mark.gpu


def run_store(h, layer, q, k, v, qw, kw, pos, slots, n_slots, Hkv, n_layer=1, q_dtype="f32",
              cache_fill=0):
    import torch
    kc = torch.full((n_layer, n_slots, Hkv, 128), cache_fill, dtype=torch.int16, device="cuda")
    vc = torch.full_like(kc, cache_fill)
    dq = dev(q)
    dt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[q_dtype]
    qo = torch.empty(q.shape, dtype=dt, device="cuda")
    h.kv_store(layer, dq, dev(k), dev(v), dev(qw), dev(kw), dev(pos), dev(slots), qo, kc, vc)
    torch.cuda.synchronize()
    return qo, kc, vc


def test_golden_fixture_bit_exact(cuda):
    fx = np.load(make_golden.__file__.replace("make_golden.py", "kv_store_qwen3_0p6b.npz"))
    q, k, v, qw, kw, pos, slots = make_golden.store_inputs()
    assert np.array_equal(make_golden._digest(q, k, v, qw, kw, pos, slots), fx["inputs_sha256"])
    h = handle(16, 8, 2)
    qo, kc, vc = run_store(h, 0, q, k, v, qw, kw, pos, slots, 512, 8)
    h.check_device()
    assert np.array_equal(qo.cpu().numpy().view(np.uint32), fx["q_out"].view(np.uint32))
    assert np.array_equal(host_bits(kc)[0, slots], fx["k_rows"])
    assert np.array_equal(host_bits(vc)[0, slots], fx["v_rows"])


# (8, 1, 20000): ten rows per token, so an 8-lane group's run of rows crosses
# token boundaries and the (cos, sin) reload path is exercised.  The
# register-row kernel's forms: one row per group up to three blocks' worth
# of groups per SM ((64, 8, 129), (8, 1, 513)), two rows per group above
# that ((64, 8, 256): 20,480 rows); larger batches take the staged kernel.
@pytest.mark.parametrize("Hq,Hkv,T", [(16, 8, 3000), (32, 8, 777), (8, 1, 513), (64, 8, 129),
                                      (64, 8, 256), (8, 1, 20000)])
@pytest.mark.parametrize("q_dtype", ["f32", "bf16", "f16"])
def test_random_tokens_bit_exact(cuda, Hq, Hkv, T, q_dtype):
    rng = np.random.default_rng(Hq * 1000 + T)
    n_layer, layer, num_blocks = 3, 1, (T + 255) // 256 + 2
    n_slots = num_blocks * 256
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = (rng.standard_normal((T, Hkv, 128)) * rng.uniform(0.01, 30, (T, Hkv, 1))).astype(np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    qw = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    kw = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    pos = rng.integers(0, 40960, T).astype(np.int32)
    slots = rng.permutation(n_slots)[:T].astype(np.int32)
    h = handle(Hq, Hkv, num_blocks, n_layer=n_layer)
    qo, kc, vc = run_store(h, layer, q, k, v, qw, kw, pos, slots, n_slots, Hkv, n_layer, q_dtype)
    h.check_device()
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=n_slots)
    okc = np.zeros((n_layer, n_slots, Hkv, 128), np.uint16)
    ovc = np.zeros_like(okc)
    oq = O.qk_norm_rope_store(p, layer, q, k, v, qw, kw, pos, slots, okc, ovc)
    if q_dtype == "bf16":
        import torch
        assert np.array_equal(host_bits(qo.view(torch.int16)), O.f32_to_bf16(oq))
    elif q_dtype == "f16":
        # round to nearest even (numpy's f32 -> f16 cast; the inputs are finite)
        assert np.array_equal(qo.cpu().numpy().view(np.uint16), oq.astype(np.float16).view(np.uint16))
    else:
        assert np.array_equal(qo.cpu().numpy().view(np.uint32), oq.view(np.uint32))
    got_k, got_v = host_bits(kc), host_bits(vc)
    assert np.array_equal(got_k, okc)  # other layers and unused slots untouched (zero)
    assert np.array_equal(got_v, ovc)


def test_negative_slot_is_skipped_and_bad_slot_is_reported(cuda):
    rng = np.random.default_rng(5)
    T, Hq, Hkv = 4, 16, 8
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    w = O.f32_to_bf16(np.ones(128, np.float32))
    pos = np.array([1, 2, 3, 4], np.int32)
    h = handle(Hq, Hkv, 1)
    _, kc, _ = run_store(h, 0, q, k, v, w, w, pos, np.array([0, -1, 2, 3], np.int32), 256, Hkv)
    assert h.get_error()[0] == nvattn.OK
    kb = host_bits(kc)
    assert not kb[0, 1].any() and kb[0, 0].any()
    _, kc, _ = run_store(h, 0, q, k, v, w, w, pos, np.array([0, 1, 256, 3], np.int32), 256, Hkv)
    st, detail = h.get_error()
    assert st == nvattn.ERR_OUT_OF_RANGE and detail == 256
    _, kc, _ = run_store(h, 0, q, k, v, w, w, np.array([0, 1, 40960, 3], np.int32),
                         np.array([0, 1, 2, 3], np.int32), 256, Hkv)
    st, detail = h.get_error()
    assert st == nvattn.ERR_OUT_OF_RANGE and detail == 40960
    assert h.get_error()[0] == nvattn.OK  # cleared after reading


# 300 tokens take the register-row kernel, 3000 the bulk-copy staged kernel
@pytest.mark.parametrize("T", [300, 3000])
def test_in_place_f32_q(cuda, T):
    import torch
    rng = np.random.default_rng(6)
    Hq, Hkv = 16, 8
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    w = O.f32_to_bf16(np.ones(128, np.float32))
    pos = np.arange(T, dtype=np.int32)
    slots = np.arange(T, dtype=np.int32)
    nb = (T + 255) // 256
    h = handle(Hq, Hkv, nb)
    dq = dev(q)
    kc = torch.zeros((1, nb * 256, Hkv, 128), dtype=torch.int16, device="cuda")
    vc = torch.zeros_like(kc)
    h.kv_store(0, dq, dev(k), dev(v), dev(w), dev(w), dev(pos), dev(slots), dq, kc, vc)
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=nb * 256)
    okc = np.zeros((1, nb * 256, Hkv, 128), np.uint16)
    ovc = np.zeros_like(okc)
    oq = O.qk_norm_rope_store(p, 0, q, k, v, w, w, pos, slots, okc, ovc)
    assert np.array_equal(host_bits(kc), okc)
    assert np.array_equal(host_bits(vc), ovc)
    assert np.array_equal(dq.cpu().numpy().view(np.uint32), oq.view(np.uint32))


@pytest.mark.parametrize("T", [64, 2000])
def test_rms_mean_on_rounding_midpoint_uses_sequential_sum(cuda, T):
    """Rows whose sum of squares / 128 sits exactly on a float rounding
    midpoint (1 + 2^-24): the kernel's 8-lane tree sum is flagged as
    ambiguous there and redone in the reference's index order."""
    rng = np.random.default_rng(8)
    Hq, Hkv = 16, 8
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    mid = np.ones(128, np.float32)
    mid[77] = np.float32(1 + 2.0 ** -18)  # square rounds to 1 + 2^-17 exactly
    q[::3, 5] = mid
    k[1::5, 2] = mid[::-1]
    w = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    pos = rng.integers(0, 40960, T).astype(np.int32)
    slots = np.arange(T, dtype=np.int32)
    nb = (T + 255) // 256
    h = handle(Hq, Hkv, nb)
    qo, kc, vc = run_store(h, 0, q, k, v, w, w, pos, slots, nb * 256, Hkv)
    h.check_device()
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=nb * 256)
    okc = np.zeros((1, nb * 256, Hkv, 128), np.uint16)
    ovc = np.zeros_like(okc)
    oq = O.qk_norm_rope_store(p, 0, q, k, v, w, w, pos, slots, okc, ovc)
    assert np.array_equal(qo.cpu().numpy().view(np.uint32), oq.view(np.uint32))
    assert np.array_equal(host_bits(kc), okc)
    assert np.array_equal(host_bits(vc), ovc)


def test_staged_path_reports_bad_position_and_slot(cuda):
    """The bulk-copy path (thousands of tokens): a token with an out-of-range
    position stores nothing and is reported; negative slots are skipped."""
    rng = np.random.default_rng(9)
    T, Hq, Hkv = 4000, 16, 8
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    w = O.f32_to_bf16(np.ones(128, np.float32))
    pos = np.arange(T, dtype=np.int32)
    slots = np.arange(T, dtype=np.int32)
    slots[17] = -1
    pos[2345] = 40960
    nb = (T + 255) // 256
    h = handle(Hq, Hkv, nb)
    qo, kc, vc = run_store(h, 0, q, k, v, w, w, pos, slots, nb * 256, Hkv)
    st, detail = h.get_error()
    assert st == nvattn.ERR_OUT_OF_RANGE and detail == 40960
    kb, vb = host_bits(kc), host_bits(vc)
    assert not kb[0, 2345].any() and not vb[0, 2345].any()
    assert not kb[0, 17].any() and not vb[0, 17].any()
    good = np.ones(T, bool)
    good[[17, 2345]] = False
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=nb * 256)
    okc = np.zeros((1, nb * 256, Hkv, 128), np.uint16)
    ovc = np.zeros_like(okc)
    pos_ok = pos.copy()
    pos_ok[2345] = 0
    oq = O.qk_norm_rope_store(p, 0, q, k, v, w, w, pos_ok, slots, okc, ovc)
    sl = slots[good]
    assert np.array_equal(kb[0, sl], okc[0, sl]) and np.array_equal(vb[0, sl], ovc[0, sl])
    got_q = qo.cpu().numpy().view(np.uint32)
    assert np.array_equal(got_q[good], oq.view(np.uint32)[good])


@pytest.mark.parametrize("T", [64, 3000])
def test_non_finite_rows(cuda, T):
    """NaN and inf inputs.  V rows are stored as-is, so their bf16 bits must
    match ggml's rule exactly (a NaN keeps its payload and is made quiet).
    A normed row containing inf or NaN becomes (partly) NaN; NaN payloads from
    arithmetic differ between CPU and GPU, so there only the NaN positions and
    the finite values are compared."""
    rng = np.random.default_rng(10)
    Hq, Hkv = 16, 8
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v[3, 1, 7] = np.uint32(0x7fa00001).view(np.float32)  # signaling NaN payload
    v[5, 0, 100] = np.inf
    v[6, 7, 0] = -np.inf
    k[9, 2, 64] = np.inf
    k[11, 4, 5] = np.nan
    q[13, 6, 127] = -np.inf
    w = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    pos = rng.integers(0, 40960, T).astype(np.int32)
    slots = np.arange(T, dtype=np.int32)
    nb = (T + 255) // 256
    h = handle(Hq, Hkv, nb)
    qo, kc, vc = run_store(h, 0, q, k, v, w, w, pos, slots, nb * 256, Hkv)
    h.check_device()
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=nb * 256)
    okc = np.zeros((1, nb * 256, Hkv, 128), np.uint16)
    ovc = np.zeros_like(okc)
    oq = O.qk_norm_rope_store(p, 0, q, k, v, w, w, pos, slots, okc, ovc)
    assert np.array_equal(host_bits(vc), ovc)
    gk, ok = host_bits(kc), okc
    gnan = (gk & 0x7fff) > 0x7f80
    onan = (ok & 0x7fff) > 0x7f80
    assert np.array_equal(gnan, onan) and gnan[0, 9, 2].any() and gnan[0, 11, 4].all()
    assert np.array_equal(gk[~gnan], ok[~onan])
    gq = qo.cpu().numpy()
    assert np.array_equal(np.isnan(gq), np.isnan(oq)) and np.isnan(gq[13, 6]).any()
    fin = ~np.isnan(gq)
    assert np.array_equal(gq[fin].view(np.uint32), oq[fin].view(np.uint32))


@pytest.mark.parametrize("T", [300, 3000])  # register-row kernel, staged kernel
def test_step_rows_in_f16(cuda, T):
    """nvattn_kv_store_qk_norm_rope_rows also writes the step's own K (normed,
    rotated) and V rows as f16: the reference's F16 cast of its graph rows,
    bit for bit; everything else equals the plain store's."""
    import torch
    rng = np.random.default_rng(900 + T)
    Hq, Hkv = 16, 8
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    qw = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    kw = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    nb = (T + 255) // 256 + 1
    pos = rng.integers(0, 40960, T).astype(np.int32)
    slots = rng.permutation(nb * 256)[:T].astype(np.int32)
    slots[:3] = -1  # rows are written whatever the slot
    h = handle(Hq, Hkv, nb)
    kc = torch.zeros((1, nb * 256, Hkv, 128), dtype=torch.int16, device="cuda")
    vc = torch.zeros_like(kc)
    qo = torch.empty((T, Hq, 128), dtype=torch.float16, device="cuda")
    kr = torch.empty((T, Hkv, 128), dtype=torch.float16, device="cuda")
    vr = torch.empty_like(kr)
    h.kv_store(0, dev(q), dev(k), dev(v), dev(qw), dev(kw), dev(pos), dev(slots), qo, kc, vc,
               k_rows=kr, v_rows=vr)
    h.check_device()
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=nb * 256)
    okc = np.zeros((1, nb * 256, Hkv, 128), np.uint16)
    ovc = np.zeros_like(okc)
    oq, ok = O.qk_norm_rope_store(p, 0, q, k, v, qw, kw, pos, slots, okc, ovc, want_k_out=True)
    f16 = lambda a: a.astype(np.float16).view(np.uint16)
    assert np.array_equal(kr.cpu().numpy().view(np.uint16), f16(ok))
    assert np.array_equal(vr.cpu().numpy().view(np.uint16), f16(v))
    assert np.array_equal(qo.cpu().numpy().view(np.uint16), f16(oq))
    assert np.array_equal(host_bits(kc), okc) and np.array_equal(host_bits(vc), ovc)
