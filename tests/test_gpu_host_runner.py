"""GPU test of the C++ host layer (nano-vllm.cpp_b200/host/attention_runner.*),
the ModelRunner-shaped caller of the C ABI (model_runner.cpp:25-186).

nano-vllm.cpp_b200/bin/runner_check drives AttentionRunner through one prefill
step (three sequences, one with a two-block prefix-cache hit), one decode
step on layer 1 of a 2-layer cache, and two Sample calls, and dumps every
input and output; this test recomputes them with the oracle: the runner's
positions and slot mapping equal the planner's, the stored K/V rows are
bit-exact, the attention outputs meet the attention tolerances, the draws
are the reference's mt19937 draws and the sampled tokens equal
ModelRunner::Sample's."""
import os
import subprocess

import numpy as np
import pytest

import nvattn
import oracle as O

pytestmark = pytest.mark.gpu

BIN = os.path.join(nvattn.PKG_DIR, "bin", "runner_check")
MAX_ABS = 2e-2
MEAN_REL = 1e-3
DT = {"f32": np.float32, "u16": np.uint16, "i32": np.int32}


def load(d):
    arrs = {}
    with open(os.path.join(d, "manifest.txt")) as f:
        for line in f:
            name, dt, *shape = line.split()
            arrs[name] = np.fromfile(os.path.join(d, name + ".bin"),
                                     dtype=DT[dt]).reshape([int(x) for x in shape])
    return arrs


def test_host_runner_prefill_then_decode(cuda, tmp_path):
    assert os.path.exists(BIN), "runner_check not built (run __graft_entry__.build())"
    r = subprocess.run([BIN, str(tmp_path), "3"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    a = load(str(tmp_path))
    layer, Hq, Hkv = 1, 16, 8
    n_slots = a["k_cache0"].shape[1]
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=n_slots)
    kc = a["k_cache0"].copy()
    vc = a["v_cache0"].copy()

    # ---- prefill step ----
    lens = a["prefill_seq_lens"].astype(np.int64)
    cached = a["prefill_num_cached"].astype(np.int64)
    bt = a["prefill_block_tables"]
    cu, qs, cl, pos, slot = nvattn.plan_prefill(lens, cached, bt)
    assert np.array_equal(a["prefill_positions"], pos)
    assert np.array_equal(a["prefill_slots"], slot)
    oq = O.qk_norm_rope_store(p, layer, a["prefill_q"], a["prefill_k"], a["prefill_v"],
                              a["q_norm_w"], a["k_norm_w"], pos, slot, kc, vc)
    assert np.array_equal(a["prefill_k_cache"], kc)  # rows written, everything else kept
    assert np.array_equal(a["prefill_v_cache"], vc)
    # exact math on the f32 normed/rotated q (the runner hands the prefill f16 q)
    ref = O.paged_prefill(p, O.MODE_TRUTH, layer, oq, cu, qs, cl, bt, kc, vc)
    mx, mr = O.err_stats(a["prefill_out"], ref)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)

    # ---- decode step: one new token per sequence ----
    lens = a["decode_seq_lens"].astype(np.int64)
    bt = a["decode_block_tables"]
    cl, pos, slot = nvattn.plan_decode(lens, bt)
    assert np.array_equal(a["decode_positions"], pos)
    assert np.array_equal(a["decode_slots"], slot)
    oq = O.qk_norm_rope_store(p, layer, a["decode_q"], a["decode_k"], a["decode_v"],
                              a["q_norm_w"], a["k_norm_w"], pos, slot, kc, vc)
    # the decode step reads q and writes no q back
    assert np.array_equal(a["decode_q_after"].view(np.uint32), a["decode_q"].view(np.uint32))
    assert np.array_equal(a["decode_k_cache"], kc)
    assert np.array_equal(a["decode_v_cache"], vc)
    ref = O.paged_decode(p, O.MODE_TRUTH, layer, oq, kc, vc, bt, cl)
    mx, mr = O.err_stats(a["decode_out"], ref)
    assert mx <= MAX_ABS and mr <= MEAN_REL, (mx, mr)

    # ---- sampling: AttentionRunner::Sample, twice on the same logits ----
    logits = a["sample_logits"]
    temps, pens = a["sample_temperatures"], a["sample_penalties"]
    offs = a["sample_history_offsets"].astype(np.int64)
    hist = a["sample_history"]
    # the draws are the reference's: one generate_canonical<float> of the
    # runner's mt19937 (default seed 5489) per temperature row, in row order
    bg = np.random.MT19937()
    bg._legacy_seeding(5489)
    raw = bg.random_raw(2)
    u = a["sample_uniforms"]
    assert u[0, 0] == u[0, 2] == u[1, 0] == u[1, 2] == 0.0
    assert u[0, 1] == np.float32(O.canonical_float(int(raw[0])))
    assert u[1, 1] == np.float32(O.canonical_float(int(raw[1])))
    for call in range(2):
        want = O.sample(logits, temps, pens, u[call], hist, offs)
        np.testing.assert_array_equal(a["sample_tokens"][call], want)
    assert a["sample_tokens"][0, 1] == 4321
