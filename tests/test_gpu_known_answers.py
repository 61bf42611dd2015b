"""Known-answer tests of the CUDA attention kernels, independent of the oracle.

Closed forms that hold for any queries:
  * a context of one key: the softmax is 1, so the output row is that key's
    V row (to f32 rounding: the kernels form x = s*scale - max with one
    fused multiply-add, so p = 2^x is 1 within an ulp, and O = p*V / p);
  * identical keys: every score equals the row maximum, so every probability
    is 1 (within an ulp, as above) and the output is the mean of the visible
    V rows; beyond that only the f32 summation order differs from the exact
    mean;
  * prefill row 0 of a prompt without a cached prefix attends key 0 only.
Decode runs on split-KV lengths (the in-kernel merge included) and prefill on
prefix hits, unaligned prefix ends and GQA groups of 1, 2 and 8.
"""
import numpy as np
import pytest

import cases
import oracle as O
from gpu_util import dev, handle, prefill_q

pytestmark = pytest.mark.gpu

BS = 256


def _slot(bt, s, pos):
    return int(bt[s, pos // BS]) * BS + pos % BS


def _v_rows(c_cache, layer, bt, s, n, kvh):
    """f32 V rows of positions [0, n) of sequence s, kv head kvh."""
    slots = [_slot(bt, s, p) for p in range(n)]
    return O.bf16_to_f32(c_cache.v[layer, slots, kvh, :]).astype(np.float64)


def _decode(c, h=None):
    import torch
    h = h or handle(c.Hq, c.Hkv, c.cache.num_blocks, max_seqs=len(c.lens))
    out = torch.full((len(c.lens), c.Hq, 128), float("nan"), device="cuda")
    h.decode(0, dev(c.q), dev(c.cache.k), dev(c.cache.v), dev(c.block_tables), dev(c.lens),
             int(c.lens.max()), out)
    torch.cuda.synchronize()
    h.check_device()
    return out.cpu().numpy().astype(np.float64)


def _prefill(c):
    import torch
    h = handle(c.Hq, c.Hkv, c.cache.num_blocks, max_seqs=len(c.seq_lens))
    out = torch.full((c.q.shape[0], c.Hq, 128), float("nan"), device="cuda")
    h.prefill(0, prefill_q(c.q), dev(c.cu_q), dev(c.q_starts), dev(c.seq_lens),
              dev(c.block_tables), int((c.seq_lens - c.q_starts).max()), dev(c.cache.k),
              dev(c.cache.v), out)
    torch.cuda.synchronize()
    h.check_device()
    return out.cpu().numpy().astype(np.float64)


def _constant_keys(cache, seed):
    """Every K row of each kv head set to one random bf16 vector."""
    rng = np.random.default_rng(seed)
    kvec = O.f32_to_bf16(rng.standard_normal((cache.Hkv, 128), dtype=np.float32))
    cache.k[:] = kvec[None, None, :, :]


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (32, 8), (8, 8)])
def test_decode_single_key_returns_its_v_row(cuda, Hq, Hkv):
    c = cases.decode_case(901, Hq, Hkv, [1, 1, 1, 1, 1])
    got = _decode(c)
    G = Hq // Hkv
    for s in range(len(c.lens)):
        for hq in range(Hq):
            want = _v_rows(c.cache, 0, c.block_tables, s, 1, hq // G)[0]
            np.testing.assert_allclose(got[s, hq], want, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (16, 8)])
def test_decode_identical_keys_give_the_mean_of_v(cuda, Hq, Hkv):
    # lengths across the 2048-token splits: one, two and five splits merged
    lens = [1, 255, 256, 257, 2048, 2049, 5000, 9001]
    c = cases.decode_case(902, Hq, Hkv, lens)
    _constant_keys(c.cache, 903)
    got = _decode(c)
    G = Hq // Hkv
    for s, L in enumerate(lens):
        for kvh in range(Hkv):
            want = _v_rows(c.cache, 0, c.block_tables, s, L, kvh).mean(axis=0)
            rows = got[s, kvh * G:(kvh + 1) * G]
            err = np.abs(rows - want[None, :]).max()
            assert err <= 1e-5, (s, L, kvh, err)


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (64, 8), (8, 8)])
def test_prefill_first_row_returns_v_of_key0(cuda, Hq, Hkv):
    c = cases.prefill_case(904, Hq, Hkv, [300, 129, 1], [0, 0, 0])
    got = _prefill(c)
    G = Hq // Hkv
    for s in range(len(c.seq_lens)):
        r = int(c.cu_q[s])  # the prompt's first row, position 0
        for hq in range(Hq):
            want = _v_rows(c.cache, 0, c.block_tables, s, 1, hq // G)[0]
            # V is converted bf16 -> f16 (exact but for |v| below 2^-14)
            np.testing.assert_allclose(got[r, hq], want, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (64, 8), (8, 8)])
def test_prefill_identical_keys_give_causal_prefix_means(cuda, Hq, Hkv):
    # no prefix, a block-aligned prefix hit, an unaligned chunk start
    seq_lens, q_starts = [700, 1300, 900], [0, 512, 333]
    c = cases.prefill_case(905, Hq, Hkv, seq_lens, q_starts)
    _constant_keys(c.cache, 906)
    got = _prefill(c)
    G = Hq // Hkv
    for s, (L, q0) in enumerate(zip(seq_lens, q_starts)):
        for kvh in range(Hkv):
            v = _v_rows(c.cache, 0, c.block_tables, s, L, kvh)
            means = np.cumsum(v, axis=0) / np.arange(1, L + 1)[:, None]
            rows = got[c.cu_q[s]:c.cu_q[s + 1], kvh * G:(kvh + 1) * G]  # [n_new][G][128]
            err = np.abs(rows - means[q0:L, None, :]).max()
            assert err <= 1e-5, (s, kvh, err)
