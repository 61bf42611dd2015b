"""CPU tests of the C ABI boundary: the library loads, exports every entry
point include/nvattn.h declares, validates arguments before touching a
device, and plans positions / slots exactly as ModelRunner::PrepareInputs
does (model_runner.cpp:138-186, 286-288, 402-405)."""
import ctypes
import os
import re

import numpy as np
import pytest

import nvattn

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "nvattn.h")).read()
    return sorted(set(re.findall(r"NVATTN_API\s+[\w\s\*]*?\b(nvattn_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    syms = header_symbols()
    assert len(syms) >= 11
    L = nvattn.lib()
    for s in syms:
        assert hasattr(L, s), s
    assert sorted(nvattn.EXPORTED) == sorted(syms)


def test_version_and_status_strings():
    assert nvattn.version() == (0, 5)
    for s in range(7):
        assert nvattn.status_string(s)
    assert nvattn.status_string(99) == "unknown status"


def test_config_defaults_are_qwen3():
    c = nvattn.qwen3_config()
    assert (c.n_layer, c.n_q_heads, c.n_kv_heads, c.head_dim, c.block_size) == (28, 16, 8, 128, 256)
    assert c.num_blocks == 160 and c.max_position == 40960
    assert abs(c.scale - 1 / np.sqrt(128)) < 1e-7
    assert c.rope_theta == 1e6 and c.rope_n_ctx_orig == 40960


@pytest.mark.parametrize("field,value,status", [
    ("head_dim", 64, nvattn.ERR_UNSUPPORTED),
    ("block_size", 16, nvattn.ERR_UNSUPPORTED),
    ("n_q_heads", 12, nvattn.ERR_INVALID_ARG),  # not a multiple of n_kv_heads
    ("n_q_heads", 24, nvattn.ERR_UNSUPPORTED),  # GQA group of 3
    ("num_blocks", 0, nvattn.ERR_INVALID_ARG),
    ("n_layer", 0, nvattn.ERR_INVALID_ARG),
])
def test_create_rejects_bad_config_without_a_device(field, value, status):
    c = nvattn.qwen3_config(**{field: value})
    h = ctypes.c_void_p()
    assert nvattn.lib().nvattn_create(ctypes.byref(c), ctypes.byref(h)) == status
    assert not h.value


def test_null_handle_is_rejected():
    L = nvattn.lib()
    assert L.nvattn_plan_prefill_device(None, 1, None, None, None, 4, 16, None, None, None, None,
                                        None, None) == nvattn.ERR_INVALID_ARG
    assert L.nvattn_plan_decode_device(None, 1, None, None, 4, None, None, None, None) == \
        nvattn.ERR_INVALID_ARG
    assert L.nvattn_paged_decode(None, 0, 1, None, None, None, None, 1, None, 1, None, None) == \
        nvattn.ERR_INVALID_ARG
    assert L.nvattn_get_error(None, None) == nvattn.ERR_INVALID_ARG
    assert L.nvattn_destroy(None) == nvattn.OK


def test_gather_entry_points_reject_a_null_handle():
    """The peer-memory gather's entry points check their handle before any
    device work: a null handle is an argument error."""
    L = nvattn.lib()
    buf = ctypes.create_string_buffer(nvattn.IPC_HANDLE_BYTES * 2)
    assert L.nvattn_gather_init(None, 2, 0, buf) == nvattn.ERR_INVALID_ARG
    assert L.nvattn_gather_connect(None, buf) == nvattn.ERR_INVALID_ARG
    assert L.nvattn_paged_decode_step_gather(None, 0, 1, *([None] * 10), 1, None, 1, None,
                                             None) == nvattn.ERR_INVALID_ARG
    assert L.nvattn_gather_read(None, 0, 1, None, None) == nvattn.ERR_INVALID_ARG


def reference_prepare_inputs(seq_lens, num_cached, block_tables, bs=256):
    """ModelRunner::PrepareInputs + the StorePrefillKV slot formula, in Python."""
    positions, slots, cu = [], [], [0]
    for s, L in enumerate(seq_lens):
        start = num_cached[s]
        for pos in range(start, L):
            positions.append(pos)
            slots.append(block_tables[s][pos // bs] * bs + pos % bs)
        cu.append(len(positions))
    return positions, slots, cu


def test_plan_prefill_matches_prepare_inputs():
    rng = np.random.default_rng(0)
    lens = np.array([600, 1, 256, 1030], np.int64)
    cached = np.array([512, 0, 0, 1024], np.int64)
    bt = np.full((4, 5), -1, np.int32)
    perm = rng.permutation(64)
    o = 0
    for s, L in enumerate(lens):
        n = (L + 255) // 256
        bt[s, :n] = perm[o:o + n]
        o += n
    cu, qs, cl, pos, slot = nvattn.plan_prefill(lens, cached, bt)
    rp, rs, rc = reference_prepare_inputs(lens.tolist(), cached.tolist(), bt.tolist())
    assert pos.tolist() == rp and slot.tolist() == rs and cu.tolist() == rc
    assert qs.tolist() == cached.tolist() and cl.tolist() == lens.tolist()


def test_plan_prefill_fully_cached_prompt_recomputes_last_token():
    bt = np.array([[3, 7]], np.int32)
    cu, qs, cl, pos, slot = nvattn.plan_prefill([512], [512], bt)
    assert cu.tolist() == [0, 1] and qs.tolist() == [511] and pos.tolist() == [511]
    assert slot.tolist() == [7 * 256 + 255]


def test_plan_rejects_missing_blocks():
    bt = np.array([[3, -1]], np.int32)
    with pytest.raises(nvattn.NvattnError):
        nvattn.plan_prefill([300], [0], bt)
    with pytest.raises(nvattn.NvattnError):
        nvattn.plan_decode([600], bt)  # needs a third block


def test_plan_decode_matches_append_decode_kv():
    bt = np.array([[5, 9, 2], [1, -1, -1]], np.int32)
    cl, pos, slot = nvattn.plan_decode([513, 256], bt)
    assert cl.tolist() == [513, 256] and pos.tolist() == [512, 255]
    assert slot.tolist() == [2 * 256 + 0, 1 * 256 + 255]


def test_decode_rejects_more_sequences_than_one_launch_holds():
    """A decode launch covers at most 65535 sequences (its grid's z extent);
    both decode entry points reject more as an argument error before they
    touch a device."""
    cfg = nvattn.qwen3_config(n_layer=1, max_seqs=70000)
    dummy = ctypes.c_void_p(1 << 20)  # aligned, never dereferenced
    L = nvattn.lib()
    st = L.nvattn_paged_decode_noalloc(ctypes.byref(cfg), 0, 65536, dummy, dummy, dummy, dummy, 4,
                                       dummy, 1024, dummy, None, None)
    assert st == nvattn.ERR_INVALID_ARG
