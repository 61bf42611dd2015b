"""ctypes wrapper around the C oracle (oracle/nvattn_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by the smoke check and by the
CPU-baseline leg of bench.py, never by the library.  Parity against the
reference (nano-vllm.cpp) is unpinned: the reference ships no tests and its
ggml dependency is not vendored; see nvattn_oracle.h for what is restated.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

MODE_TRUTH = 0
MODE_GGML = 1


class OrcParams(ctypes.Structure):
    _fields_ = [
        ("n_q_heads", ctypes.c_int),
        ("n_kv_heads", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("block_size", ctypes.c_int),
        ("n_slots", ctypes.c_int64),
        ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("rope_freq_scale", ctypes.c_float),
        ("rope_ext_factor", ctypes.c_float),
        ("rope_attn_factor", ctypes.c_float),
        ("rope_beta_fast", ctypes.c_float),
        ("rope_beta_slow", ctypes.c_float),
        ("rope_n_ctx_orig", ctypes.c_int),
        ("scale", ctypes.c_float),
        ("n_threads", ctypes.c_int),
    ]


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.orc_f32_to_bf16.restype = ctypes.c_uint16
        _lib.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        _lib.orc_bf16_to_f32.restype = ctypes.c_float
        _lib.orc_bf16_to_f32.argtypes = [ctypes.c_uint16]
        _lib.orc_f32_to_f16.restype = ctypes.c_uint16
        _lib.orc_f32_to_f16.argtypes = [ctypes.c_float]
        _lib.orc_f16_to_f32.restype = ctypes.c_float
        _lib.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
    return _lib


def params(n_q_heads=16, n_kv_heads=8, head_dim=128, block_size=256, n_slots=0,
           rms_eps=1e-6, rope_theta=1e6, rope_freq_scale=1.0, rope_ext_factor=1.0,
           rope_attn_factor=1.0, rope_beta_fast=32.0, rope_beta_slow=1.0,
           rope_n_ctx_orig=40960, scale=None, n_threads=0) -> OrcParams:
    """Qwen3 defaults (qwen3.h:30-56)."""
    if scale is None:
        scale = float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))
    return OrcParams(n_q_heads, n_kv_heads, head_dim, block_size, n_slots, rms_eps,
                     rope_theta, rope_freq_scale, rope_ext_factor, rope_attn_factor,
                     rope_beta_fast, rope_beta_slow, rope_n_ctx_orig, scale, n_threads)


def _p(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_bf16_row(_p(x), _p(y), ctypes.c_int64(x.size))
    return y


def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.empty(x.shape, dtype=np.float32)
    lib().orc_bf16_to_f32_row(_p(x), _p(y), ctypes.c_int64(x.size))
    return y


def rope_table(n_pos: int, p: OrcParams) -> np.ndarray:
    t = np.empty((n_pos, p.head_dim // 2, 2), dtype=np.float32)
    lib().orc_rope_table(ctypes.c_int(n_pos), ctypes.byref(p), _p(t))
    return t


def qk_norm_rope_store(p, layer, q, k, v, q_norm_w, k_norm_w, positions, slots,
                       k_cache, v_cache, want_k_out=False):
    """In place on k_cache/v_cache (uint16 bf16 bits); returns q_out[, k_out]."""
    T = positions.shape[0]
    q_out = np.empty_like(q, dtype=np.float32)
    k_out = np.empty_like(k, dtype=np.float32) if want_k_out else None
    lib().orc_qk_norm_rope_store(
        ctypes.byref(p), ctypes.c_int(layer), ctypes.c_int(T), _p(q), _p(k), _p(v),
        _p(q_norm_w), _p(k_norm_w), _p(positions), _p(slots), _p(q_out), _p(k_out),
        _p(k_cache), _p(v_cache))
    return (q_out, k_out) if want_k_out else q_out


def paged_decode(p, mode, layer, q, k_cache, v_cache, block_tables, context_lens,
                 new_k=None, new_v=None):
    B = context_lens.shape[0]
    out = np.empty((B, p.n_q_heads, p.head_dim), dtype=np.float32)
    lib().orc_paged_decode(
        ctypes.byref(p), ctypes.c_int(mode), ctypes.c_int(layer), ctypes.c_int(B),
        _p(q), _p(k_cache), _p(v_cache), _p(block_tables),
        ctypes.c_int(block_tables.shape[1]), _p(context_lens), _p(new_k), _p(new_v),
        _p(out))
    return out


def paged_prefill(p, mode, layer, q, cu_q, q_start, context_lens, block_tables,
                  k_cache, v_cache, new_k=None, new_v=None):
    B = context_lens.shape[0]
    T = int(cu_q[-1])
    out = np.empty((T, p.n_q_heads, p.head_dim), dtype=np.float32)
    lib().orc_paged_prefill(
        ctypes.byref(p), ctypes.c_int(mode), ctypes.c_int(layer), ctypes.c_int(B),
        _p(q), _p(cu_q), _p(q_start), _p(context_lens), _p(block_tables),
        ctypes.c_int(block_tables.shape[1]), _p(k_cache), _p(v_cache), _p(new_k),
        _p(new_v), _p(out))
    return out


def concat_decode_ggml(p, layer, q, k_cache, v_cache, block_tables, context_lens,
                       new_k, new_v):
    B = context_lens.shape[0]
    out = np.empty((B, p.n_q_heads, p.head_dim), dtype=np.float32)
    lib().orc_concat_decode_ggml(
        ctypes.byref(p), ctypes.c_int(layer), ctypes.c_int(B), _p(q), _p(k_cache),
        _p(v_cache), _p(block_tables), ctypes.c_int(block_tables.shape[1]),
        _p(context_lens), _p(new_k), _p(new_v), _p(out))
    return out


def concat_prefill_ggml(p, q, cu_q, new_k, new_v):
    """The reference's prefill attention over the batch's concatenated new
    tokens (FillCausalMask, model_runner.cpp:188-217; qwen3.cpp:461-531)."""
    T = int(cu_q[-1])
    out = np.empty((T, p.n_q_heads, p.head_dim), dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.float32)
    new_k = np.ascontiguousarray(new_k, dtype=np.float32)
    new_v = np.ascontiguousarray(new_v, dtype=np.float32)
    cu_q = np.ascontiguousarray(cu_q, dtype=np.int32)
    lib().orc_concat_prefill_ggml(ctypes.byref(p), ctypes.c_int(len(cu_q) - 1), _p(cu_q), _p(q),
                                  _p(new_k), _p(new_v), _p(out))
    return out


def _hist_args(history, history_offsets):
    if history is None:
        return None, None, None
    h = np.ascontiguousarray(history, dtype=np.int32)
    o = np.ascontiguousarray(history_offsets, dtype=np.int64)
    return h, o, _p(h)


def penalize_rows(logits, penalties, history=None, history_offsets=None):
    """Repetition-penalised copy of each logits row (model_runner.cpp:428-446)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    n, V = x.shape
    pen = np.ascontiguousarray(penalties, dtype=np.float32)
    h, o, hp = _hist_args(history, history_offsets)
    out = np.empty_like(x)
    lib().orc_penalize_rows(ctypes.c_int(n), ctypes.c_int(V), _p(x), ctypes.c_int64(V), _p(pen),
                            hp, None if o is None else _p(o), _p(out))
    return out


def sample(logits, temperatures, penalties, uniforms, history=None, history_offsets=None):
    """ModelRunner::Sample (model_runner.cpp:417-489) with the uniform draws
    given: the reference's float chain, token per row."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    n, V = x.shape
    t = np.ascontiguousarray(temperatures, dtype=np.float32)
    pen = np.ascontiguousarray(penalties, dtype=np.float32)
    u = np.ascontiguousarray(uniforms, dtype=np.float32)
    h, o, hp = _hist_args(history, history_offsets)
    out = np.empty(n, np.int32)
    lib().orc_sample(ctypes.c_int(n), ctypes.c_int(V), _p(x), ctypes.c_int64(V), _p(t), _p(pen),
                     hp, None if o is None else _p(o), _p(u), _p(out))
    return out


def canonical_float(x: int) -> float:
    """generate_canonical<float> of one 32-bit mt19937 output (libstdc++)."""
    f = lib().orc_canonical_float
    f.restype = ctypes.c_float
    f.argtypes = [ctypes.c_uint32]
    return float(f(x))


def err_stats(got: np.ndarray, ref: np.ndarray):
    """(max-abs-err, mean-rel-err = sum|got-ref| / sum|ref|)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    diff = np.abs(got - ref)
    denom = np.abs(ref).sum()
    return float(diff.max(initial=0.0)), float(diff.sum() / denom) if denom > 0 else 0.0
