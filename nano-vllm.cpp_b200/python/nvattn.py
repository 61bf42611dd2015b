"""Python binding of libnvattn through its C ABI (include/nvattn.h), via ctypes.

This is the ctypes stub a Python caller (tests, benchmarks) uses; tensors are
passed as raw device pointers, so no framework type crosses the ABI.  The
library is loaded from nano-vllm.cpp_b200/lib/libnvattn.so and there is no
fallback: a missing library raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.dirname(_HERE)
LIB_PATH = os.path.join(PKG_DIR, "lib", "libnvattn.so")

OK = 0
ERR_INVALID_ARG = 1
ERR_OUT_OF_RANGE = 2
ERR_CUDA = 3
ERR_TIMEOUT = 4
ERR_UNSUPPORTED = 5
ERR_NO_MEMORY = 6

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

EXPORTED = [
    "nvattn_config_init_qwen3", "nvattn_create", "nvattn_destroy", "nvattn_status_string",
    "nvattn_version", "nvattn_get_error", "nvattn_plan_prefill", "nvattn_plan_decode",
    "nvattn_kv_store_qk_norm_rope", "nvattn_paged_decode", "nvattn_paged_prefill",
    "nvattn_paged_decode_noalloc", "nvattn_plan_prefill_device", "nvattn_plan_decode_device",
    "nvattn_sample", "nvattn_schedule_prefill_chunks", "nvattn_kv_store_qk_norm_rope_rows",
    "nvattn_paged_prefill_rows", "nvattn_paged_decode_step", "nvattn_paged_decode_step_launches",
    "nvattn_gather_init", "nvattn_gather_connect", "nvattn_paged_decode_step_gather",
    "nvattn_gather_read",
]
IPC_HANDLE_BYTES = 128
ERR_SCRATCH_LIMIT = 7


class NvattnError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} ({status})")


class Config(ctypes.Structure):
    _fields_ = [
        ("n_layer", ctypes.c_int),
        ("n_q_heads", ctypes.c_int),
        ("n_kv_heads", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("block_size", ctypes.c_int),
        ("num_blocks", ctypes.c_int64),
        ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("rope_freq_scale", ctypes.c_float),
        ("rope_ext_factor", ctypes.c_float),
        ("rope_attn_factor", ctypes.c_float),
        ("rope_beta_fast", ctypes.c_float),
        ("rope_beta_slow", ctypes.c_float),
        ("rope_n_ctx_orig", ctypes.c_int),
        ("scale", ctypes.c_float),
        ("max_position", ctypes.c_int),
        ("max_seqs", ctypes.c_int),
        ("max_context", ctypes.c_int),
        ("device", ctypes.c_int),
    ]


_lib = None
_vp = ctypes.c_void_p
_i32 = ctypes.c_int
_i64 = ctypes.c_int64


def lib():
    """Loads libnvattn.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"libnvattn not built: {LIB_PATH} (run __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        L.nvattn_config_init_qwen3.argtypes = [ctypes.POINTER(Config)]
        L.nvattn_config_init_qwen3.restype = None
        L.nvattn_create.argtypes = [ctypes.POINTER(Config), ctypes.POINTER(_vp)]
        L.nvattn_destroy.argtypes = [_vp]
        L.nvattn_status_string.argtypes = [_i32]
        L.nvattn_status_string.restype = ctypes.c_char_p
        L.nvattn_version.argtypes = [ctypes.POINTER(_i32), ctypes.POINTER(_i32)]
        L.nvattn_version.restype = None
        L.nvattn_get_error.argtypes = [_vp, ctypes.POINTER(_i64)]
        L.nvattn_plan_prefill.argtypes = [_i32, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp,
                                          _vp, _vp]
        L.nvattn_plan_decode.argtypes = [_i32, _vp, _vp, _i32, _i32, _vp, _vp, _vp]
        L.nvattn_plan_prefill_device.argtypes = [_vp, _i32, _vp, _vp, _vp, _i32, _i32, _vp, _vp,
                                                 _vp, _vp, _vp, _vp]
        L.nvattn_plan_decode_device.argtypes = [_vp, _i32, _vp, _vp, _i32, _vp, _vp, _vp, _vp]
        L.nvattn_sample.argtypes = [_vp, _i32, _i32, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]
        L.nvattn_schedule_prefill_chunks.argtypes = [_i32, _vp, _vp, _vp, _i32, _i64, _i32,
                                                     _i64, _vp, _vp, _vp,
                                                     ctypes.POINTER(_i32)]
        L.nvattn_kv_store_qk_norm_rope.argtypes = [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp,
                                                   _vp, _vp, _i32, _vp, _vp, _vp]
        L.nvattn_kv_store_qk_norm_rope_rows.argtypes = [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp,
                                                        _vp, _vp, _vp, _i32, _vp, _vp, _vp, _vp,
                                                        _vp]
        L.nvattn_paged_prefill_rows.argtypes = [_vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp,
                                                _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp]
        L.nvattn_paged_decode_step.argtypes = [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                               _vp, _vp, _vp, _i32, _vp, _i32, _vp, _vp]
        L.nvattn_paged_decode_step.restype = _i32
        L.nvattn_paged_decode_step_launches.argtypes = [_vp, _i32, _i32, ctypes.POINTER(_i32)]
        L.nvattn_gather_init.argtypes = [_vp, _i32, _i32, ctypes.c_char_p]
        L.nvattn_gather_connect.argtypes = [_vp, ctypes.c_char_p]
        L.nvattn_paged_decode_step_gather.argtypes = L.nvattn_paged_decode_step.argtypes
        L.nvattn_gather_read.argtypes = [_vp, ctypes.c_uint, _i32, _vp, _vp]
        L.nvattn_paged_decode.argtypes = [_vp, _i32, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _i32,
                                          _vp, _vp]
        L.nvattn_paged_prefill.argtypes = [_vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _i32,
                                           _i32, _vp, _vp, _vp, _vp]
        L.nvattn_paged_decode_noalloc.argtypes = [ctypes.POINTER(Config), _i32, _i32, _vp, _vp,
                                                  _vp, _vp, _i32, _vp, _i32, _vp, _vp, _vp]
        # every other entry point returns nvattn_status (ctypes' default c_int)
        _lib = L
    return _lib


def status_string(s: int) -> str:
    return lib().nvattn_status_string(int(s)).decode()


def version():
    a, b = _i32(), _i32()
    lib().nvattn_version(ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def qwen3_config(**overrides) -> Config:
    c = Config()
    lib().nvattn_config_init_qwen3(ctypes.byref(c))
    for k, v in overrides.items():
        setattr(c, k, v)
    return c


def _check(st: int, what: str):
    if st != OK:
        raise NvattnError(st, what)


def _ptr(t):
    """Raw address of a tensor-like (anything with data_ptr()) or None."""
    if t is None:
        return None
    return _vp(t.data_ptr())


def _np_ptr(a):
    return a.ctypes.data_as(_vp)


def _stream_ptr(stream):
    if stream is None:
        return None
    return _vp(int(stream.cuda_stream) if hasattr(stream, "cuda_stream") else int(stream))


class Handle:
    """One libnvattn handle (one device)."""

    def __init__(self, cfg: Config):
        self.cfg = cfg
        h = _vp()
        _check(lib().nvattn_create(ctypes.byref(cfg), ctypes.byref(h)), "nvattn_create")
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().nvattn_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def get_error(self):
        """Returns (status, detail) recorded by kernels since the last call (syncs)."""
        d = _i64()
        st = lib().nvattn_get_error(self._h, ctypes.byref(d))
        return st, d.value

    def check_device(self, what="kernel"):
        st, d = self.get_error()
        if st != OK:
            raise NvattnError(st, f"{what} (detail {d})")

    def plan_prefill(self, seq_lens, num_cached, block_tables, max_tokens, cu_q, q_starts,
                     context_lens, positions, slot_mapping, stream=None, check=True):
        """nvattn_plan_prefill_device: the host planner's outputs computed on the
        device from device tensors (seq_lens/num_cached int64, block_tables
        int32 [n_seqs][max_blocks]); per-sequence errors land in get_error()."""
        st = lib().nvattn_plan_prefill_device(
            self._h, seq_lens.shape[0], _ptr(seq_lens), _ptr(num_cached), _ptr(block_tables),
            block_tables.shape[1], int(max_tokens), _ptr(cu_q), _ptr(q_starts),
            _ptr(context_lens), _ptr(positions), _ptr(slot_mapping), _stream_ptr(stream))
        if check:
            _check(st, "nvattn_plan_prefill_device")
        return st

    def plan_decode(self, seq_lens, block_tables, context_lens, positions, slot_mapping,
                    stream=None, check=True):
        """nvattn_plan_decode_device: one decode token per sequence, on the device."""
        st = lib().nvattn_plan_decode_device(
            self._h, seq_lens.shape[0], _ptr(seq_lens), _ptr(block_tables),
            block_tables.shape[1], _ptr(context_lens), _ptr(positions), _ptr(slot_mapping),
            _stream_ptr(stream))
        if check:
            _check(st, "nvattn_plan_decode_device")
        return st

    def sample(self, logits, temperatures, penalties, uniforms, tokens, history=None,
               history_offsets=None, stream=None, check=True):
        """nvattn_sample: one token per logits row ([n_seqs][row_stride] f32,
        the first n_vocab = logits.shape[1] columns used) into tokens (int32);
        history (int32 ids) / history_offsets (int64, n_seqs+1) feed the
        repetition penalty."""
        n, V = logits.shape
        st = lib().nvattn_sample(
            self._h, n, V, _ptr(logits), logits.stride(0), _ptr(temperatures), _ptr(penalties),
            _ptr(history), _ptr(history_offsets), _ptr(uniforms), _ptr(tokens),
            _stream_ptr(stream))
        if check:
            _check(st, "nvattn_sample")
        return st

    def kv_store(self, layer, q, k, v, q_norm_w, k_norm_w, positions, slots, q_out, k_cache,
                 v_cache, stream=None, check=True, k_rows=None, v_rows=None):
        """nvattn_kv_store_qk_norm_rope; with k_rows / v_rows (f16 [T][Hkv][128])
        nvattn_kv_store_qk_norm_rope_rows, which also writes the step's rows."""
        import torch
        dt = {torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}.get(q_out.dtype, DTYPE_F32)
        args = (self._h, layer, positions.shape[0], _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm_w),
                _ptr(k_norm_w), _ptr(positions), _ptr(slots), _ptr(q_out), dt, _ptr(k_cache),
                _ptr(v_cache))
        if k_rows is None:
            st = lib().nvattn_kv_store_qk_norm_rope(*args, _stream_ptr(stream))
        else:
            st = lib().nvattn_kv_store_qk_norm_rope_rows(*args, _ptr(k_rows), _ptr(v_rows),
                                                         _stream_ptr(stream))
        if check:
            _check(st, "nvattn_kv_store_qk_norm_rope")
        return st

    def decode(self, layer, q, k_cache, v_cache, block_tables, context_lens, max_context_len,
               out, stream=None, check=True):
        st = lib().nvattn_paged_decode(
            self._h, layer, context_lens.shape[0], _ptr(q), _ptr(k_cache), _ptr(v_cache),
            _ptr(block_tables), block_tables.shape[1], _ptr(context_lens), int(max_context_len),
            _ptr(out), _stream_ptr(stream))
        if check:
            _check(st, "nvattn_paged_decode")
        return st

    def decode_step(self, layer, q, k, v, q_norm_w, k_norm_w, positions, slots, k_cache, v_cache,
                    block_tables, context_lens, max_context_len, out, stream=None, check=True):
        """nvattn_paged_decode_step: the store of the new token (q/k norm +
        RoPE) and the decode, in one launch or two (decode_step_launches);
        q, k, v are the raw f32 projections."""
        st = lib().nvattn_paged_decode_step(
            self._h, layer, context_lens.shape[0], _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm_w),
            _ptr(k_norm_w), _ptr(positions), _ptr(slots), _ptr(k_cache), _ptr(v_cache),
            _ptr(block_tables), block_tables.shape[1], _ptr(context_lens), int(max_context_len),
            _ptr(out), _stream_ptr(stream))
        if check:
            _check(st, "nvattn_paged_decode_step")
        return st

    # ---- the decode step with the all-gather over peer memory ----
    def gather_init(self, n_ranks, rank):
        """This rank's gathered buffer; returns its IPC handle (bytes) for the
        other ranks."""
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        _check(lib().nvattn_gather_init(self._h, n_ranks, rank, buf), "nvattn_gather_init")
        return buf.raw

    def gather_connect(self, handles):
        """handles: every rank's gather_init bytes, in rank order."""
        blob = b"".join(handles)
        _check(lib().nvattn_gather_connect(self._h, blob), "nvattn_gather_connect")

    def decode_step_gather(self, layer, q, k, v, q_norm_w, k_norm_w, positions, slots, k_cache,
                           v_cache, block_tables, context_lens, max_context_len, out,
                           stream=None, check=True):
        """decode_step whose output rows also land in every rank's gathered
        buffer (a collective; see nvattn_paged_decode_step_gather)."""
        st = lib().nvattn_paged_decode_step_gather(
            self._h, layer, context_lens.shape[0], _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm_w),
            _ptr(k_norm_w), _ptr(positions), _ptr(slots), _ptr(k_cache), _ptr(v_cache),
            _ptr(block_tables), block_tables.shape[1], _ptr(context_lens), int(max_context_len),
            _ptr(out), _stream_ptr(stream))
        if check:
            _check(st, "nvattn_paged_decode_step_gather")
        return st

    def gather_read(self, step, n_seqs, out, stream=None):
        """Copies gather step `step`'s rows into out [n_ranks][n_seqs][Hq][128] f32;
        `step` must be the latest gather step this handle took, read before
        its next one."""
        _check(lib().nvattn_gather_read(self._h, step, n_seqs, _ptr(out), _stream_ptr(stream)),
               "nvattn_gather_read")

    def decode_step_launches(self, n_seqs, max_context_len):
        """Kernel launches decode_step makes for this batch shape: 1 (fused),
        2 (the KV store, then the decode) or 0 (no sequences)."""
        n = _i32()
        _check(lib().nvattn_paged_decode_step_launches(self._h, n_seqs, max_context_len,
                                                       ctypes.byref(n)),
               "nvattn_paged_decode_step_launches")
        return n.value

    def prefill(self, layer, q, cu_q, q_starts, context_lens, block_tables, max_q_len, k_cache,
                v_cache, out, stream=None, check=True, k_rows=None, v_rows=None):
        """nvattn_paged_prefill; with k_rows / v_rows (the step's f16 rows)
        nvattn_paged_prefill_rows."""
        args = (self._h, layer, context_lens.shape[0], q.shape[0], _ptr(q), _ptr(cu_q),
                _ptr(q_starts), _ptr(context_lens), _ptr(block_tables), block_tables.shape[1],
                int(max_q_len), _ptr(k_cache), _ptr(v_cache))
        if k_rows is None:
            st = lib().nvattn_paged_prefill(*args, _ptr(out), _stream_ptr(stream))
        else:
            st = lib().nvattn_paged_prefill_rows(*args, _ptr(k_rows), _ptr(v_rows), _ptr(out),
                                                 _stream_ptr(stream))
        if check:
            _check(st, "nvattn_paged_prefill")
        return st


def decode_noalloc(cfg, layer, q, k_cache, v_cache, block_tables, context_lens,
                   max_context_len, out, status=None, stream=None):
    """nvattn_paged_decode_noalloc: decode without a handle and without any
    device allocation (split-KV partials go to the library's fixed 32 MiB
    scratch).  `status` (optional) is a caller-owned 16-byte device buffer
    (e.g. torch.zeros(4, dtype=torch.int32, device=...)) that receives the
    first error a kernel detects.  Returns the status code."""
    return lib().nvattn_paged_decode_noalloc(
        ctypes.byref(cfg), layer, context_lens.shape[0], _ptr(q), _ptr(k_cache), _ptr(v_cache),
        _ptr(block_tables), block_tables.shape[1], _ptr(context_lens), int(max_context_len),
        _ptr(out), _ptr(status), _stream_ptr(stream))


def kv_head_shard(n_q_heads, n_kv_heads, world, rank):
    """KV-head sharding across `world` GPUs: rank r owns kv heads
    [r*Hkv/N, (r+1)*Hkv/N) and the GQA q heads that read them (consecutive q
    heads share a kv head, as ggml's broadcast does).  Returns
    (kv_begin, kv_end, q_begin, q_end)."""
    if world <= 0 or not 0 <= rank < world or n_kv_heads % world or n_q_heads % n_kv_heads:
        raise ValueError("kv heads must split evenly across ranks")
    per = n_kv_heads // world
    g = n_q_heads // n_kv_heads
    return rank * per, (rank + 1) * per, rank * per * g, (rank + 1) * per * g


def gather_heads(shards):
    """Concatenates per-rank outputs [tokens][Hq/N][d] along the head axis into
    [tokens][Hq][d] (the layout BuildAttention hands to o_proj)."""
    import numpy as np
    return np.concatenate(shards, axis=1)


def plan_prefill(seq_lens, num_cached, block_tables, block_size=256):
    """Host planner (no device work): numpy in, numpy out."""
    import numpy as np
    seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int64)
    num_cached = np.ascontiguousarray(num_cached, dtype=np.int64)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    n = seq_lens.shape[0]
    cap = int(np.maximum(seq_lens - num_cached, 1).sum())
    cu = np.zeros(n + 1, np.int32)
    qs = np.zeros(n, np.int32)
    cl = np.zeros(n, np.int32)
    pos = np.zeros(cap, np.int32)
    slot = np.zeros(cap, np.int32)
    st = lib().nvattn_plan_prefill(n, _np_ptr(seq_lens), _np_ptr(num_cached), _np_ptr(bt),
                                   bt.shape[1], block_size, cap, _np_ptr(cu), _np_ptr(qs),
                                   _np_ptr(cl), _np_ptr(pos), _np_ptr(slot))
    _check(st, "nvattn_plan_prefill")
    T = int(cu[-1])
    return cu, qs, cl, pos[:T], slot[:T]


def schedule_prefill_chunks(prompt_lens, done, held_blocks, free_blocks, max_num_seqs,
                            max_num_batched_tokens, block_size=256):
    """nvattn_schedule_prefill_chunks: one step's chunked prefill admission.
    Returns (selected sequence indices, chunk ends, new blocks per chunk)."""
    import numpy as np
    lens = np.ascontiguousarray(prompt_lens, dtype=np.int64)
    dn = np.ascontiguousarray(done, dtype=np.int64)
    hb = np.ascontiguousarray(held_blocks, dtype=np.int64)
    n = lens.shape[0]
    sel = np.zeros(max(n, 1), np.int32)
    end = np.zeros(max(n, 1), np.int64)
    nb = np.zeros(max(n, 1), np.int64)
    k = _i32()
    st = lib().nvattn_schedule_prefill_chunks(n, _np_ptr(lens), _np_ptr(dn), _np_ptr(hb),
                                              block_size, int(free_blocks), int(max_num_seqs),
                                              int(max_num_batched_tokens), _np_ptr(sel),
                                              _np_ptr(end), _np_ptr(nb), ctypes.byref(k))
    _check(st, "nvattn_schedule_prefill_chunks")
    return sel[:k.value], end[:k.value], nb[:k.value]


def plan_decode(seq_lens, block_tables, block_size=256):
    import numpy as np
    seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int64)
    bt = np.ascontiguousarray(block_tables, dtype=np.int32)
    n = seq_lens.shape[0]
    cl = np.zeros(n, np.int32)
    pos = np.zeros(n, np.int32)
    slot = np.zeros(n, np.int32)
    st = lib().nvattn_plan_decode(n, _np_ptr(seq_lens), _np_ptr(bt), bt.shape[1], block_size,
                                  _np_ptr(cl), _np_ptr(pos), _np_ptr(slot))
    _check(st, "nvattn_plan_decode")
    return cl, pos, slot
