"""Seeded synthetic inputs shared by the CPU and GPU tests.

Shapes follow the workloads the reference's attention path serves: Qwen3
heads of 128 dims, 256-token KV blocks, block tables that are seeded random
permutations of the physical block ids (BlockManager hands out free ids,
block_manager.cpp:96-142).  K/V cache values are N(0,1) rounded to bf16;
queries are N(0,1) f32.
"""
from __future__ import annotations

import dataclasses

import numpy as np

import oracle as O

D = 128
BS = 256


@dataclasses.dataclass
class PagedCache:
    Hkv: int
    num_blocks: int
    n_layer: int
    k: np.ndarray  # uint16 bf16 bits [n_layer][num_blocks*BS][Hkv][D]
    v: np.ndarray

    @property
    def n_slots(self):
        return self.num_blocks * BS


def make_cache(rng, Hkv, num_blocks, n_layer=1):
    shape = (n_layer, num_blocks * BS, Hkv, D)
    k = O.f32_to_bf16(rng.standard_normal(shape, dtype=np.float32))
    v = O.f32_to_bf16(rng.standard_normal(shape, dtype=np.float32))
    return PagedCache(Hkv, num_blocks, n_layer, k, v)


def make_block_tables(rng, lens, num_blocks, extra_cols=0):
    """Each sequence takes ceil(L/BS) ids, in order, from one seeded
    permutation of [0, num_blocks)."""
    need = [(int(L) + BS - 1) // BS for L in lens]
    assert sum(need) <= num_blocks, "pool too small"
    perm = rng.permutation(num_blocks).astype(np.int32)
    max_blocks = max(max(need), 1) + extra_cols
    bt = np.full((len(lens), max_blocks), -1, dtype=np.int32)
    off = 0
    for s, n in enumerate(need):
        bt[s, :n] = perm[off:off + n]
        off += n
    return bt


def oracle_params(Hq, Hkv, cache: PagedCache, n_threads=0):
    return O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=cache.n_slots, n_threads=n_threads)


@dataclasses.dataclass
class DecodeCase:
    Hq: int
    Hkv: int
    lens: np.ndarray  # int32 [B]
    cache: PagedCache
    block_tables: np.ndarray  # int32 [B][max_blocks]
    q: np.ndarray  # f32 [B][Hq][D]
    layer: int = 0


def decode_case(seed, Hq, Hkv, lens, num_blocks=None, n_layer=1, layer=0, extra_cols=0):
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, dtype=np.int32)
    need = int(sum((int(L) + BS - 1) // BS for L in lens))
    if num_blocks is None:
        num_blocks = max(need + need // 8 + 1, 2)
    cache = make_cache(rng, Hkv, num_blocks, n_layer)
    bt = make_block_tables(rng, lens, num_blocks, extra_cols)
    q = rng.standard_normal((len(lens), Hq, D), dtype=np.float32)
    return DecodeCase(Hq, Hkv, lens, cache, bt, q, layer)


@dataclasses.dataclass
class PrefillCase:
    Hq: int
    Hkv: int
    seq_lens: np.ndarray  # int32 [B]: SequenceLen
    q_starts: np.ndarray  # int32 [B]: cached prefix length
    cu_q: np.ndarray  # int32 [B+1]
    cache: PagedCache
    block_tables: np.ndarray
    q: np.ndarray  # f32 [T][Hq][D], values exactly representable in bf16
    layer: int = 0


def prefill_case(seed, Hq, Hkv, seq_lens, q_starts, num_blocks=None, n_layer=1, layer=0):
    rng = np.random.default_rng(seed)
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    q_starts = np.asarray(q_starts, dtype=np.int32)
    need = int(sum((int(L) + BS - 1) // BS for L in seq_lens))
    if num_blocks is None:
        num_blocks = max(need + need // 8 + 1, 2)
    cache = make_cache(rng, Hkv, num_blocks, n_layer)
    bt = make_block_tables(rng, seq_lens, num_blocks)
    n_new = seq_lens - q_starts
    cu = np.zeros(len(seq_lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(n_new)
    T = int(cu[-1])
    q = O.bf16_to_f32(O.f32_to_bf16(rng.standard_normal((T, Hq, D), dtype=np.float32)))
    return PrefillCase(Hq, Hkv, seq_lens, q_starts, cu, cache, bt, q, layer)


def bf16_bits_to_i16(a: np.ndarray) -> np.ndarray:
    """uint16 bf16 bits viewed as int16 (a dtype torch moves to the GPU)."""
    return a.view(np.int16)
