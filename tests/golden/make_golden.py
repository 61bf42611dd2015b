"""Generates the golden fixtures in this directory from the C oracle.

    python tests/golden/make_golden.py          # rewrite all fixtures

Each fixture stores the seed, the shape parameters, a SHA-256 of the
regenerated inputs (so a change in numpy's random stream is detected rather
than silently compared), and the oracle outputs.  The reference itself ships
no tests or golden vectors and cannot be built here (its ggml submodule is
not vendored), so these fixtures pin the oracle and the CUDA kernels against
each other over time; they are not reference outputs.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import cases  # noqa: E402
import oracle as O  # noqa: E402


def _digest(*arrays) -> np.ndarray:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return np.frombuffer(h.digest(), dtype=np.uint8).copy()


# ---- decode, Qwen3-0.6B attention shape (16 q / 8 kv heads, 4 sequences) ----
DECODE_SEED = 20241
DECODE_LENS = [37, 256, 513, 1000]


def decode_inputs():
    return cases.decode_case(DECODE_SEED, 16, 8, DECODE_LENS, num_blocks=12)


def build_decode():
    c = decode_inputs()
    p = cases.oracle_params(16, 8, c.cache)
    args = (c.q, c.cache.k, c.cache.v, c.block_tables, c.lens)
    return {
        "seed": np.array(DECODE_SEED), "lens": c.lens,
        "inputs_sha256": _digest(*args),
        "out_truth": O.paged_decode(p, O.MODE_TRUTH, 0, *args),
        "out_ggml": O.paged_decode(p, O.MODE_GGML, 0, *args),
    }


# ---- fused q/k norm + RoPE + KV store (8 tokens, 16 q / 8 kv heads) ----
STORE_SEED = 20242
STORE_T = 8


def store_inputs():
    rng = np.random.default_rng(STORE_SEED)
    T, Hq, Hkv = STORE_T, 16, 8
    q = rng.standard_normal((T, Hq, 128), dtype=np.float32)
    k = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    v = rng.standard_normal((T, Hkv, 128), dtype=np.float32)
    qw = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    kw = O.f32_to_bf16((1 + 0.02 * rng.standard_normal(128)).astype(np.float32))
    pos = np.array([0, 1, 255, 256, 1023, 4096, 40000, 40959], np.int32)
    slots = rng.permutation(2 * 256)[:T].astype(np.int32)
    return q, k, v, qw, kw, pos, slots


def build_store():
    q, k, v, qw, kw, pos, slots = store_inputs()
    p = O.params(n_q_heads=16, n_kv_heads=8, n_slots=2 * 256)
    kc = np.zeros((1, 512, 8, 128), np.uint16)
    vc = np.zeros_like(kc)
    q_out = O.qk_norm_rope_store(p, 0, q, k, v, qw, kw, pos, slots, kc, vc)
    return {
        "seed": np.array(STORE_SEED), "inputs_sha256": _digest(q, k, v, qw, kw, pos, slots),
        "q_out": q_out, "k_rows": kc[0, slots], "v_rows": vc[0, slots],
    }


# ---- causal prefill with a cached prefix (4 q / 2 kv heads) ----
PREFILL_SEED = 20243
PREFILL_LENS = [270, 40]
PREFILL_STARTS = [256, 0]


def prefill_inputs():
    return cases.prefill_case(PREFILL_SEED, 4, 2, PREFILL_LENS, PREFILL_STARTS, num_blocks=4)


def build_prefill():
    c = prefill_inputs()
    p = cases.oracle_params(4, 2, c.cache)
    args = (c.q, c.cu_q, c.q_starts, c.seq_lens, c.block_tables, c.cache.k, c.cache.v)
    return {
        "seed": np.array(PREFILL_SEED), "inputs_sha256": _digest(*args),
        "out_truth": O.paged_prefill(p, O.MODE_TRUTH, 0, *args),
        "out_ggml": O.paged_prefill(p, O.MODE_GGML, 0, *args),
    }


BUILDERS = {
    "decode_qwen3_0p6b.npz": build_decode,
    "kv_store_qwen3_0p6b.npz": build_store,
    "prefill_prefix_hit.npz": build_prefill,
}


def main():
    for name, fn in BUILDERS.items():
        np.savez_compressed(os.path.join(HERE, name), **fn())
        print("wrote", name)


if __name__ == "__main__":
    main()
