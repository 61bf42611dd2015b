"""GPU test of the model-step harness (nano-vllm.cpp_b200/python/model_runner.py):
ModelRunner::Run's decode step for the Qwen3 architecture with the attention
path served by libnvattn (nvattn_paged_decode_step: the store of the new
token and the paged decode in one launch) and greedy sampling by
nvattn_sample, over three decode steps of six sequences (two of which cross
a block boundary, so BlockManager::Append hands them a new block).

Two checks:
  * every layer of every step: the library's attention output against the
    oracle's (the reference's store semantics, exact attention) on the same
    q/k/v, within the attention bars (max-abs 2e-2, mean-rel 1e-3), the raw
    q left unmodified, and after the last step the whole K/V cache (all
    layers) bit-exact with the oracle's;
  * the greedy tokens against a second run of the same loop whose attention
    is the oracle, teacher-forced with that run's tokens.  bf16 rounding of
    the activations before every projection (as in ggml's mul_mat) makes the
    logits move by ~3e-3 mean-rel under a 1e-6 change of the attention
    output, so tokens are compared where the oracle run's top two logits are
    further apart than the two runs' largest logit difference, and the
    logits are held to 2e-2 mean-rel.
"""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_REL = 1e-3


def test_decode_steps_match_the_oracle(cuda):
    import torch
    import model_runner as MR
    dev = torch.device("cuda:0")
    shape = MR.Qwen3Shape(n_layer=3)
    w = MR.Qwen3Weights(shape, dev, seed=11, norm_mean=1.0)
    rng = np.random.default_rng(12)
    lens = np.array([256, 511, 1300, 700, 257, 1023], np.int64)
    steps = 3
    need = int(((lens + steps + 255) // 256).sum())
    num_blocks, max_blocks = need + 4, int((lens.max() + steps + 255) // 256)
    n_slots = num_blocks * 256
    cache_shape = (shape.n_layer, n_slots, shape.n_kv_heads, shape.head_dim)
    kc = O.f32_to_bf16(rng.standard_normal(cache_shape, dtype=np.float32))
    vc = O.f32_to_bf16(rng.standard_normal(cache_shape, dtype=np.float32))
    B = len(lens)
    p = O.params(n_q_heads=shape.n_q_heads, n_kv_heads=shape.n_kv_heads, n_slots=n_slots)

    def norm_bits(t):
        return t.view(torch.int16).cpu().numpy().view(np.uint16)

    # -- the library run, each layer's attention shadowed by the oracle
    lib = MR.DecodeRunner(shape, w, num_blocks, B, max_blocks, dev)
    lib.allocate(B)
    lib.k_cache.copy_(torch.from_numpy(kc.view(np.int16)))
    lib.v_cache.copy_(torch.from_numpy(vc.view(np.int16)))
    skc, svc = kc.copy(), vc.copy()
    worst = [0.0, 0.0]

    def checked_attention(layer, q, k, v, stream=None):
        qh, kh, vh = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
        out = lib.library_attention(layer, q, k, v, stream).cpu().numpy()
        b, L = lib.bufs, w.layers[layer]
        pos, slots, ctx, bt = (t.cpu().numpy() for t in (b["pos"], b["slots"], b["ctx"], b["bt"]))
        # the fused step leaves q as it was (the normed q stays on chip)
        assert np.array_equal(q.cpu().numpy().view(np.uint32), qh.view(np.uint32))
        q_out = O.qk_norm_rope_store(p, layer, qh, kh, vh, norm_bits(L["q_norm"]),
                                     norm_bits(L["k_norm"]), pos, slots, skc, svc)
        ref = O.paged_decode(p, O.MODE_TRUTH, layer, q_out, skc, svc, bt, ctx)
        mx, mr = O.err_stats(out, ref)
        assert mx <= MAX_ABS and mr <= MEAN_REL, (layer, mx, mr)
        worst[0], worst[1] = max(worst[0], mx), max(worst[1], mr)
        return lib.bufs["attn"]

    lib.attention = checked_attention

    # -- the same loop with the oracle as its attention path
    ref = MR.DecodeRunner(shape, w, num_blocks, B, max_blocks, dev)
    ref.allocate(B)
    okc, ovc = kc.copy(), vc.copy()

    def oracle_attention(layer, q, k, v, stream=None):
        b, L = ref.bufs, w.layers[layer]
        pos, slots, ctx, bt = (t.cpu().numpy() for t in (b["pos"], b["slots"], b["ctx"], b["bt"]))
        q_out = O.qk_norm_rope_store(p, layer, q.cpu().numpy(), k.cpu().numpy(),
                                     v.cpu().numpy(), norm_bits(L["q_norm"]),
                                     norm_bits(L["k_norm"]), pos, slots, okc, ovc)
        out = O.paged_decode(p, O.MODE_TRUTH, layer, q_out, okc, ovc, bt, ctx)
        return torch.from_numpy(out).to(dev)

    ref.attention = oracle_attention
    t_lib = MR.BlockTables(lens, num_blocks, max_blocks, seed=13)
    t_ref = MR.BlockTables(lens, num_blocks, max_blocks, seed=13)
    tokens = rng.integers(0, shape.vocab, B)
    compared = 0
    for step in range(steps):
        lib.set_inputs(tokens, t_lib)
        ref.set_inputs(tokens, t_ref)
        got = lib.forward().cpu().numpy()
        want = ref.forward().cpu().numpy()
        lib.h.check_device(f"step {step}")
        lg, lw = lib.bufs["logits"].cpu().numpy(), ref.bufs["logits"].cpu().numpy()
        assert np.array_equal(got, lg.argmax(axis=1))  # greedy = first index of the max
        assert np.array_equal(want, lw.argmax(axis=1))
        mx, mr = O.err_stats(lg, lw)
        assert mr <= 2e-2, (step, mx, mr)
        top2 = np.sort(lw, axis=1)[:, -2:]
        clear = (top2[:, 1] - top2[:, 0]) > mx
        assert np.array_equal(got[clear], want[clear]), (step, got, want)
        compared += int(clear.sum())
        tokens = want
        t_lib.append_token()
        t_ref.append_token()
    assert compared >= B * steps // 2, compared
    # every stored row of every layer (incl. the blocks taken during the steps)
    assert np.array_equal(lib.k_cache.cpu().numpy().view(np.uint16), skc)
    assert np.array_equal(lib.v_cache.cpu().numpy().view(np.uint16), svc)
    lib.close()
    ref.close()
