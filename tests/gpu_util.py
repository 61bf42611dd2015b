"""Helpers for the GPU parity tests: handles sized for a case, and moving
numpy inputs to the device (bf16 bit patterns travel as int16)."""
import numpy as np

import nvattn


def handle(Hq, Hkv, num_blocks, n_layer=1, max_seqs=512, max_context=40960,
           max_position=40960, device=0, **overrides):
    cfg = nvattn.qwen3_config(n_layer=n_layer, n_q_heads=Hq, n_kv_heads=Hkv,
                              num_blocks=num_blocks, max_seqs=max_seqs, max_context=max_context,
                              max_position=max_position, device=device, **overrides)
    return nvattn.Handle(cfg)


def dev(a, device="cuda:0"):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a).to(device)


def host_bits(t):
    """Device int16 tensor of bf16 bits -> numpy uint16."""
    return t.cpu().numpy().view(np.uint16)


def prefill_q(q, device="cuda:0"):
    """Query rows for nvattn_paged_prefill: f16 on the device (round to
    nearest even; the test cases' bf16-exact values are f16-exact except
    magnitudes below 2^-17)."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(q, dtype=np.float32).astype(np.float16)).to(device)
