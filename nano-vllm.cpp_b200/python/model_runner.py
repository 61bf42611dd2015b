"""The reference's decode step with the ggml graph cut at the attention node.

ModelRunner::Run for a decode batch (src/engine/model_runner.cpp:25-136) over
Qwen3Model::BuildDecodeGraph (src/models/qwen3.cpp:573-686), for the Qwen3
architecture, with the hot path served by libnvattn through its C ABI:

  reference                                          here
  -------------------------------------------------  -----------------------------
  PrepareInputs positions / slots (:138-186)         nvattn.plan_decode (host)
  q/k RMSNorm + NEOX RoPE (qwen3.cpp:619-641),       nvattn_paged_decode_step
    AppendDecodeKV (model_runner.cpp:380-415),          (one launch)
    LoadHistoryKV + concat + FillVarlenMask +
    BuildAttention (:300-376; qwen3.cpp:648-662)
  Sample, greedy (model_runner.cpp:417-489)          nvattn_sample

The layers outside attention -- token embedding (get_rows), RMSNorm, the
q/k/v/o projections, the SwiGLU FFN, the residual adds, the output norm and
lm_head (qwen3.cpp:580-686) -- run as torch / cuBLAS ops on the GPU in the
order the reference's graph runs them ("not-ggml": ggml, which holds those
ops in the reference, is not vendored).  As in ggml's mul_mat with bf16
weights, activations are rounded to bf16, products accumulate in f32 and
the outputs stay f32; the residual stream and the norms are f32.

The attention path is a parameter (`attention`): the library by default; a
test substitutes the CPU oracle to compare whole steps.  Block tables follow
BlockManager::Append (block_manager.cpp:162-184): a sequence takes a new
block when its length reaches a multiple of the block size plus one.
"""
from __future__ import annotations

import dataclasses

import numpy as np

import nvattn

BS = 256


@dataclasses.dataclass
class Qwen3Shape:
    """Qwen3Hparams (qwen3.h:30-56); defaults are Qwen3-0.6B."""
    n_layer: int = 28
    hidden: int = 1024
    n_q_heads: int = 16
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 3072
    vocab: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6


class Qwen3Weights:
    """Random bf16 weights of the architecture, N(mean, std) per tensor
    (matrices stored [in, out] so activations multiply from the left)."""

    def __init__(self, shape: Qwen3Shape, device, seed=0, std=0.02, norm_mean=0.0):
        import torch
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        H, D, F = shape.hidden, shape.head_dim, shape.ffn
        Hq, Hkv = shape.n_q_heads, shape.n_kv_heads

        def mat(*s):
            return (torch.randn(s, generator=g, device=device) * std).to(torch.bfloat16)

        def norm(n):
            return (norm_mean + std * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)

        self.embed = mat(shape.vocab, H)
        self.layers = []
        for _ in range(shape.n_layer):
            self.layers.append({
                "attn_norm": norm(H), "wq": mat(H, Hq * D), "wk": mat(H, Hkv * D),
                "wv": mat(H, Hkv * D), "q_norm": norm(D), "k_norm": norm(D),
                "wo": mat(Hq * D, H), "ffn_norm": norm(H), "w_gate": mat(H, F),
                "w_up": mat(H, F), "w_down": mat(F, H),
            })
        self.out_norm = norm(H)
        self.lm_head = mat(H, shape.vocab)


class BlockTables:
    """Per-sequence block tables over a pool of physical blocks, grown the
    way BlockManager::Append does (one new block when a sequence's length
    becomes a multiple of the block size plus one).  The pool is a seeded
    permutation of the block ids, handed out in order."""

    def __init__(self, seq_lens, num_blocks, max_blocks, seed=0):
        rng = np.random.default_rng(seed)
        self.free = list(rng.permutation(num_blocks).astype(np.int32)[::-1])
        self.lens = np.asarray(seq_lens, np.int64).copy()
        self.table = np.full((len(self.lens), max_blocks), -1, np.int32)
        for s, L in enumerate(self.lens):
            for b in range((int(L) + BS - 1) // BS):
                self.table[s, b] = self.free.pop()

    def append_token(self):
        """Every sequence grows by one token (the decode step's new token)."""
        for s in range(len(self.lens)):
            self.lens[s] += 1
            if self.lens[s] % BS == 1:
                self.table[s, (self.lens[s] - 1) // BS] = self.free.pop()


def mm(a, w):
    """bf16 activations x bf16 weights -> f32 (cuBLAS, f32 accumulation)."""
    import torch
    return torch.mm(a, w, out_dtype=torch.float32)


def rms_norm(x, w, eps):
    """ggml_rms_norm then ggml_mul by the weight cast to f32 (f32 math)."""
    import torch
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * w.float()


class DecodeRunner:
    """One decode step of a batch through all layers (ModelRunner::Run,
    decode branch) with the KV cache in the reference's layout:
    [n_layer][num_blocks * 256][n_kv_heads][head_dim] bf16, K and V."""

    def __init__(self, shape: Qwen3Shape, weights: Qwen3Weights, num_blocks, max_seqs,
                 max_blocks, device, attention=None):
        import torch
        self.shape, self.w, self.device = shape, weights, device
        self.max_blocks = max_blocks
        self.max_context = max_blocks * BS
        cfg = nvattn.qwen3_config(n_layer=shape.n_layer, n_q_heads=shape.n_q_heads,
                                  n_kv_heads=shape.n_kv_heads, num_blocks=num_blocks,
                                  max_seqs=max_seqs, max_context=self.max_context,
                                  max_position=self.max_context, rms_eps=shape.rms_eps,
                                  rope_theta=shape.rope_theta, device=device.index or 0)
        self.h = nvattn.Handle(cfg)
        n_slots = num_blocks * BS
        self.k_cache = torch.zeros((shape.n_layer, n_slots, shape.n_kv_heads, shape.head_dim),
                                   dtype=torch.int16, device=device)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.attention = attention or self.library_attention
        # per-step device inputs (fixed addresses, so a captured step replays)
        self.bufs = None
        self.attn_events = None  # [(start, end)] per layer when timing

    def allocate(self, n_seqs):
        import torch
        dev = self.device
        self.bufs = {
            "tokens": torch.zeros(n_seqs, dtype=torch.int64, device=dev),
            "ctx": torch.zeros(n_seqs, dtype=torch.int32, device=dev),
            "pos": torch.zeros(n_seqs, dtype=torch.int32, device=dev),
            "slots": torch.zeros(n_seqs, dtype=torch.int32, device=dev),
            "bt": torch.zeros((n_seqs, self.max_blocks), dtype=torch.int32, device=dev),
            "attn": torch.empty((n_seqs, self.shape.n_q_heads, self.shape.head_dim), device=dev),
            "next": torch.zeros(n_seqs, dtype=torch.int32, device=dev),
            "logits": torch.empty((n_seqs, self.shape.vocab), device=dev),
            "temps": torch.zeros(n_seqs, device=dev),
            "pens": torch.ones(n_seqs, device=dev),
            "draws": torch.zeros(n_seqs, device=dev),
        }
        return self.bufs

    def library_attention(self, layer, q, k, v, stream=None):
        """q/k norm + RoPE, the store of the new K/V rows and the paged decode
        in one launch (nvattn_paged_decode_step), on the caller's current
        stream; q, k, v are the raw projections (not modified)."""
        import torch
        stream = stream or torch.cuda.current_stream(self.device)
        b, L = self.bufs, self.w.layers[layer]
        self.h.decode_step(layer, q, k, v, L["q_norm"].view(torch_int16()),
                           L["k_norm"].view(torch_int16()), b["pos"], b["slots"], self.k_cache,
                           self.v_cache, b["bt"], b["ctx"], self.max_context, b["attn"],
                           stream=stream)
        return b["attn"]

    def set_inputs(self, tokens, tables: BlockTables):
        """Host side of the step: PrepareInputs' positions / slots (the new
        token of each sequence at position len - 1) and the block tables,
        copied into the step's device buffers."""
        import torch
        ctx, pos, slots = nvattn.plan_decode(tables.lens, tables.table)
        b = self.bufs
        for name, arr in (("ctx", ctx), ("pos", pos), ("slots", slots), ("bt", tables.table)):
            b[name].copy_(torch.from_numpy(np.ascontiguousarray(arr)), non_blocking=True)
        if tokens is not None:
            b["tokens"].copy_(torch.as_tensor(np.asarray(tokens, np.int64)), non_blocking=True)

    def forward(self, stream=None):
        """The step's device work on the current buffers: every layer, the
        output norm, lm_head and greedy sampling into bufs['next']."""
        import torch
        import torch.nn.functional as F
        sh, W, b = self.shape, self.w, self.bufs
        n, H = b["tokens"].shape[0], sh.hidden
        Hq, Hkv, D = sh.n_q_heads, sh.n_kv_heads, sh.head_dim
        x = W.embed.index_select(0, b["tokens"]).float()  # get_rows + cast to f32
        for layer, L in enumerate(W.layers):
            res = x
            hb = rms_norm(x, L["attn_norm"], sh.rms_eps).to(torch.bfloat16)
            q = mm(hb, L["wq"]).view(n, Hq, D)
            k = mm(hb, L["wk"]).view(n, Hkv, D)
            v = mm(hb, L["wv"]).view(n, Hkv, D)
            ev = self.attn_events[layer] if self.attn_events else None
            if ev:
                ev[0].record()
            attn = self.attention(layer, q, k, v, stream)
            if ev:
                ev[1].record()
            x = mm(attn.reshape(n, Hq * D).to(torch.bfloat16), L["wo"]) + res
            res = x
            hb = rms_norm(x, L["ffn_norm"], sh.rms_eps).to(torch.bfloat16)
            gate = mm(hb, L["w_gate"])
            up = mm(hb, L["w_up"])
            x = mm((F.silu(gate) * up).to(torch.bfloat16), L["w_down"]) + res
        hb = rms_norm(x, W.out_norm, sh.rms_eps).to(torch.bfloat16)
        b["logits"].copy_(mm(hb, W.lm_head))
        self.h.sample(b["logits"], b["temps"], b["pens"], b["draws"], b["next"],
                      stream=stream or torch.cuda.current_stream(self.device))
        return b["next"]

    def close(self):
        self.h.close()


def torch_int16():
    import torch
    return torch.int16
