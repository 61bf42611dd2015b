"""The oracle against a second, independently written statement of the same
Qwen3 attention block: Hugging Face transformers' modeling_qwen3
(Qwen3RMSNorm, Qwen3RotaryEmbedding + apply_rotary_pos_emb,
eager_attention_forward with repeat_kv), as installed.  It is not the
reference's code -- ggml computes the reference's attention -- but it pins
the semantics a restatement could get wrong without any golden vector
noticing: the NEOX pairing (i, i + 64), the rope base 1e6 over 128 dims, eps
1e-6 inside the square root, the norm weight applied after the scale, the
GQA mapping kv = q / (Hq / Hkv), the 1/sqrt(128) scale and the causal limit
with a cached prefix (qwen3.cpp:497-514, 627-641, 377-405).  A slip in any of
them moves outputs by O(1); the tolerances below only admit float32 rounding
(RoPE angles lose up to ~1.75e-7 * position radians in float32 on both sides).
Skipped where transformers is missing.
"""
import types

import numpy as np
import pytest

import cases
import oracle as O

m = pytest.importorskip("transformers.models.qwen3.modeling_qwen3")
torch = pytest.importorskip("torch")


def _hf_config(Hq, Hkv):
    from transformers import Qwen3Config
    return Qwen3Config(hidden_size=Hq * 128, num_attention_heads=Hq, num_key_value_heads=Hkv,
                       head_dim=128, rms_norm_eps=1e-6, max_position_embeddings=40960,
                       rope_parameters={"rope_type": "default", "rope_theta": 1e6})


def _hf_norm_rope(cfg, x, w_bits, pos):
    """x f32 [T][H][128] -> RMSNorm(weight) then RoPE at pos, as modeling_qwen3."""
    norm = m.Qwen3RMSNorm(128, eps=cfg.rms_norm_eps)
    norm.weight.data = torch.from_numpy(O.bf16_to_f32(w_bits))
    rot = m.Qwen3RotaryEmbedding(cfg)
    with torch.no_grad():
        xt = norm(torch.from_numpy(x)).transpose(0, 1)[None]  # [1][H][T][128]
        cos, sin = rot(xt, torch.from_numpy(pos.astype(np.int64))[None])
        y, _ = m.apply_rotary_pos_emb(xt, xt, cos, sin)
    return y[0].transpose(0, 1).numpy()


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (32, 8), (64, 8)])
def test_norm_rope_matches_hf_qwen3(Hq, Hkv):
    rng = np.random.default_rng(40 + Hq)
    T = 96
    q = 3 * rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = 3 * rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    wq = O.f32_to_bf16(rng.normal(1, 0.1, 128).astype(np.float32))
    wk = O.f32_to_bf16(rng.normal(1, 0.1, 128).astype(np.float32))
    pos = np.concatenate([np.arange(32), np.sort(rng.integers(32, 40960, T - 32))]).astype(np.int32)
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=256)
    kc = np.zeros((1, 256, Hkv, 128), np.uint16)
    vc = np.zeros_like(kc)
    q_out, k_out = O.qk_norm_rope_store(p, 0, q, k, v, wq, wk, pos, np.full(T, -1, np.int32),
                                        kc, vc, want_k_out=True)
    cfg = _hf_config(Hq, Hkv)
    for ours, x, w in ((q_out, q, wq), (k_out, k, wk)):
        hf = _hf_norm_rope(cfg, x, w, pos)
        d = np.abs(ours.astype(np.float64) - hf)
        # a rotation error of dtheta moves an element by up to dtheta times its
        # NEOX pair's magnitude; both sides round the angle in float32
        # (measured dtheta <= 1.75e-7 * position)
        pair = np.sqrt(hf[..., :64] ** 2 + hf[..., 64:] ** 2)
        pair = np.concatenate([pair, pair], axis=-1)
        bound = 5e-5 + 3e-7 * pos.astype(np.float64)[:, None, None] * pair
        assert (d <= bound).all(), (float(d.max()), int(pos[np.argmax(d.max(axis=(1, 2)))]))
        assert d[:32].max() < 5e-5  # low positions: only the norm's rounding


def _hf_attention(Hq, Hkv, q, k, v, q_start):
    """q f64 [Tq][Hq][128] at positions q_start + i; k, v f64 [L][Hkv][128] for
    positions [0, L).  Causal: row i sees keys [0, q_start + i]."""
    Tq, L = q.shape[0], k.shape[0]
    mod = types.SimpleNamespace(num_key_value_groups=Hq // Hkv, training=False)
    mask = np.where(np.arange(L)[None, :] <= (q_start + np.arange(Tq))[:, None], 0.0, -np.inf)
    qt = torch.from_numpy(q).transpose(0, 1)[None]
    kt = torch.from_numpy(k).transpose(0, 1)[None]
    vt = torch.from_numpy(v).transpose(0, 1)[None]
    out, _ = m.eager_attention_forward(mod, qt, kt, vt, torch.from_numpy(mask)[None, None],
                                       scaling=1.0 / np.sqrt(128.0))
    return out[0].numpy()  # [Tq][Hq][128]


@pytest.mark.parametrize("Hq,Hkv", [(16, 8), (32, 8), (8, 1)])
def test_paged_prefill_matches_hf_qwen3_attention(Hq, Hkv):
    """Three prompts, one with a two-block cached prefix: the oracle's exact
    paged prefill over the block table equals transformers' eager attention
    over each sequence's contiguous K/V with the causal limit."""
    c = cases.prefill_case(77 + Hq, Hq, Hkv, [300, 700, 129], [0, 512, 0])
    p = cases.oracle_params(Hq, Hkv, c.cache)
    out = O.paged_prefill(p, O.MODE_TRUTH, 0, c.q, c.cu_q, c.q_starts, c.seq_lens,
                          c.block_tables, c.cache.k, c.cache.v)
    for s, L in enumerate(c.seq_lens):
        L = int(L)
        slots = (c.block_tables[s, np.arange(L) // 256].astype(np.int64) * 256
                 + np.arange(L) % 256)
        k = O.bf16_to_f32(c.cache.k[0, slots]).astype(np.float64)
        v = O.bf16_to_f32(c.cache.v[0, slots]).astype(np.float64)
        r0, r1 = int(c.cu_q[s]), int(c.cu_q[s + 1])
        hf = _hf_attention(Hq, Hkv, c.q[r0:r1].astype(np.float64), k, v, int(c.q_starts[s]))
        mx, mr = O.err_stats(out[r0:r1], hf)
        # transformers takes the softmax in float32: ~1e-7 relative
        assert mx < 1e-5 and mr < 1e-6, (s, mx, mr)


def test_paged_decode_matches_hf_qwen3_attention():
    """One new token per sequence attending its whole context (the decode
    step's last row) against transformers' attention for a single query."""
    Hq, Hkv = 32, 8
    c = cases.decode_case(91, Hq, Hkv, [1, 255, 256, 1000])
    p = cases.oracle_params(Hq, Hkv, c.cache)
    out = O.paged_decode(p, O.MODE_TRUTH, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens)
    for s, L in enumerate(c.lens):
        L = int(L)
        slots = (c.block_tables[s, np.arange(L) // 256].astype(np.int64) * 256
                 + np.arange(L) % 256)
        k = O.bf16_to_f32(c.cache.k[0, slots]).astype(np.float64)
        v = O.bf16_to_f32(c.cache.v[0, slots]).astype(np.float64)
        hf = _hf_attention(Hq, Hkv, c.q[s:s + 1].astype(np.float64), k, v, L - 1)
        mx, mr = O.err_stats(out[s:s + 1], hf)
        assert mx < 1e-5 and mr < 1e-6, (s, mx, mr)
