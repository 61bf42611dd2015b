"""Benchmark of the paged-attention hot path (libnvattn) on B200.

Workload (one step = one decode layer-step): 256 sequences, Qwen3-8B
attention shape (32 q heads, 8 kv heads, head_dim 128, 256-token blocks,
BF16 KV), context lengths log-uniform in [1k, 32k] (seeded), block tables
from a seeded permutation of a pool 10% larger than needed, Q/K/V N(0,1).
A step is one nvattn_paged_decode_step call: the new token's q/k RMSNorm +
RoPE, the slot_mapping store of its K/V rows, then paged split-KV decode over
all cached tokens -- one fused launch, or the store and decode launches when
the decode grid is large (the full workload on one GPU); the explicit two
calls (nvattn_kv_store_qk_norm_rope, nvattn_paged_decode) are timed beside
it.  With --gpus N the 8 kv heads are sharded N ways (rank r owns kv
heads [r*8/N, (r+1)*8/N) and their q heads) -- strong scaling, no collective
on the data path; a second timed loop adds the optional all-gather of the
head outputs and checks the gathered rows against the oracle
(--no-allgather skips it).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.  `value` is whole-job decode tokens/s with
inputs resident in HBM; `e2e` is the same metric through the C ABI with the
step's inputs copied from pinned host memory and the output copied back
inside the timed region.  `--impl reference` times the CPU restatement of the
reference's attention (its ggml dtype chain, paged form) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nano-vllm.cpp_b200", "python"))

METRIC = "paged decode-attn tokens/s + HBM GB/s vs 8 TB/s; prefill-attn TFLOPS vs peak"
WORKLOAD = "decode_qwen3_8b_attn_256seq_ctx1k-32k"
N_SEQS, HQ, HKV, D, BS = 256, 32, 8, 128, 256
SEED = 0

# DRAM traffic per step of this workload on one GPU (dram__bytes_read.sum +
# dram__bytes_write.sum), where the step runs as the store launch and the
# decode launch.  The decode kernel: an ncu capture of the first 32 sequences
# moved 1.3774 GB (1.3722 read, 0.0052 written) for 1.3632 GB of algorithmic
# bytes (x1.0104), scaled to the full launch's 10.987 GB = 11.101 GB; the
# store launch adds its 11.7 MB (each byte read or written once).  (The fused
# one-launch kernel on the same 32-sequence capture: 1.3771 GB, x1.0099 of
# its algorithmic bytes.)
NCU_TRAFFIC_BYTES_N1 = 11.113e9

# sm__pipe_tensor_cycles_active of paged_prefill_kernel, fraction of elapsed
# cycles, from ncu captures of the CTA-pair kernel with f16 Q/K/V: the chunk
# shape (2 x 2048 new tokens at [30720, 32768), 32B heads; full capture) and
# the prefix-hit workload itself (one launch; 42.2 % of the SMs' active
# cycles, the SMs active 88.6 % of the launch).
NCU_PREFILL_TENSOR_ACTIVE = 0.556
NCU_PREFIX_HIT_TENSOR_ACTIVE = 0.374


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def workload(rng_seed=SEED, n_seqs=N_SEQS):
    """Context lengths, block tables and pool size.  n_seqs < 256 keeps the
    first n_seqs lengths of the same draw (a smaller case for profiling)."""
    rng = np.random.default_rng(rng_seed)
    lens = np.exp(rng.uniform(math.log(1024), math.log(32768), N_SEQS)).astype(np.int64)
    lens = lens[:n_seqs]
    need = (lens + BS - 1) // BS
    num_blocks = int(need.sum() * 1.1) + 1
    perm = rng.permutation(num_blocks).astype(np.int32)
    max_blocks = int(need.max())
    bt = np.full((n_seqs, max_blocks), -1, np.int32)
    off = 0
    for s in range(n_seqs):
        bt[s, :need[s]] = perm[off:off + need[s]]
        off += int(need[s])
    return lens, bt, num_blocks


def prefill_workload(kind):
    """(name, Hq, Hkv, seq_lens, cached prefix per sequence, block tables,
    num_blocks) for the two prefill workloads.

    prefix_hit: Qwen3-0.6B attention shape, 8 sequences with prompt lengths
      uniform in [512, 4096]; the first 1024 tokens (4 blocks) are a prefix
      already in the cache and shared by all 8 (refcount 8); a prompt of at
      most 1024 tokens hits 256*floor((L-1)/256) tokens of the same blocks.
    chunk: Qwen3-32B attention shape (64 q / 8 kv heads), 16 sequences whose
      cached context is 129024 tokens; one 2048-token chunk each at positions
      [129024, 131072)."""
    rng = np.random.default_rng(SEED + 2)
    if kind == "prefix_hit":
        name, Hq, Hkv = "prefill_prefix_hit_qwen3_0p6b_8seq", 16, 8
        lens = rng.integers(512, 4097, 8).astype(np.int64)
        cached = np.where(lens > 1024, 1024, 256 * ((lens - 1) // 256)).astype(np.int64)
        n_shared = 4
    elif kind == "chunk_small":
        # profiling-sized case of the chunk workload: 2 sequences, 32k context
        name, Hq, Hkv = "chunked_prefill_qwen3_32b_2x2048_at_30720", 64, 8
        lens = np.full(2, 32768, np.int64)
        cached = np.full(2, 30720, np.int64)
        n_shared = 0
    else:
        name, Hq, Hkv = "chunked_prefill_qwen3_32b_16x2048_at_129024", 64, 8
        lens = np.full(16, 131072, np.int64)
        cached = np.full(16, 129024, np.int64)
        n_shared = 0
    need = (lens + BS - 1) // BS
    n_hit = cached // BS if n_shared else np.zeros_like(cached)  # blocks taken from the prefix
    num_blocks = int(n_shared + (need - n_hit).sum() + 8)
    perm = rng.permutation(num_blocks).astype(np.int32)
    shared, pool = perm[:n_shared], perm[n_shared:]
    bt = np.full((len(lens), int(need.max())), -1, np.int32)
    off = 0
    for s in range(len(lens)):
        ns = int(n_hit[s])
        bt[s, :ns] = shared[:ns]
        bt[s, ns:need[s]] = pool[off:off + need[s] - ns]
        off += int(need[s] - ns)
    return name, Hq, Hkv, lens, cached, bt, num_blocks


def bench_prefill(kind, args, world, rank, device):
    """Times one prefill layer-step (fused q/k norm + RoPE + suffix K/V store,
    then causal paged prefill over prefix + suffix) on this rank's kv-head
    shard.  Returns (fields, per-rank prefill ms, per-rank step ms)."""
    import torch
    import nvattn
    name, Hq, Hkv, lens, cached, bt_np, num_blocks = prefill_workload(kind)
    hq, hkv = Hq // world, Hkv // world
    cu, qs, cl, pos_np, slot_np = nvattn.plan_prefill(lens, cached, bt_np)
    T = int(cu[-1])
    max_q = int((cl - qs).max())
    max_ctx = int(cl.max())
    cfg = nvattn.qwen3_config(n_layer=1, n_q_heads=hq, n_kv_heads=hkv, num_blocks=num_blocks,
                              max_seqs=len(lens), max_context=max_ctx, max_position=max_ctx,
                              device=device.index)
    h = nvattn.Handle(cfg)
    gen = torch.Generator(device=device)
    gen.manual_seed(2000 + rank)
    n_slots = num_blocks * BS
    kc = torch.empty((n_slots, hkv, D), dtype=torch.bfloat16, device=device)
    vc = torch.empty_like(kc)
    for t in (kc, vc):
        for i in range(0, n_slots, 1 << 16):
            t[i:i + (1 << 16)].copy_(torch.randn((min(1 << 16, n_slots - i), hkv, D),
                                                 generator=gen, device=device))
    q = torch.randn((T, hq, D), generator=gen, device=device)
    k = torch.randn((T, hkv, D), generator=gen, device=device)
    v = torch.randn((T, hkv, D), generator=gen, device=device)
    qw = (1 + 0.02 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16)
    kw = (1 + 0.02 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16)
    qb = torch.empty((T, hq, D), dtype=torch.float16, device=device)
    out = torch.empty((T, hq, D), device=device)
    d = {n: torch.from_numpy(a).to(device) for n, a in
         (("cu", cu), ("qs", qs), ("cl", cl), ("pos", pos_np), ("slot", slot_np), ("bt", bt_np))}
    stream = torch.cuda.current_stream(device)
    kc16, vc16 = kc.view(torch.int16), vc.view(torch.int16)
    qw16, kw16 = qw.view(torch.int16), kw.view(torch.int16)
    evs = []

    def step():
        z, a, b = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        z.record(stream)
        h.kv_store(0, q, k, v, qw16, kw16, d["pos"], d["slot"], qb, kc16, vc16, stream=stream)
        a.record(stream)
        h.prefill(0, qb, d["cu"], d["qs"], d["cl"], d["bt"], max_q, kc16, vc16, out,
                  stream=stream)
        b.record(stream)
        evs.append((z, a, b))

    steps = max(2, args.prefill_steps)
    clocks = ClockSampler(device.index)
    clocks.start()
    for _ in range(max(3, min(args.warmup, 5))):
        step()
    torch.cuda.synchronize(device)
    h.check_device(f"prefill warmup {name}")
    evs.clear()
    mark = clocks.mark()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[device.index])
    t0.record(stream)
    for _ in range(steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop(mark)
    h.check_device(f"prefill {name}")
    step_ms = t0.elapsed_time(t1) / steps
    pre_ms = sum(a.elapsed_time(b) for _, a, b in evs) / len(evs)
    store_ms = sum(z.elapsed_time(a) for z, a, _ in evs) / len(evs)
    # algorithmic causal FLOPs (whole job, all heads): 4*d*Hq per visible (q, k) pair
    pairs = sum(int(((np.arange(qs[s], cl[s]) + 1)).sum()) for s in range(len(lens)))
    flops = 4.0 * D * Hq * pairs
    cpu = None
    if kind == "prefix_hit" and world == 1 and rank == 0 and not args.no_cpu_baseline:
        # the same prefill (the cache as the last step left it) on the host
        # cores: the oracle's restatement of the reference's dtype chain
        # (bf16 K -> f16, f32 scores and softmax, f16 V accumulator)
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        cores = os.cpu_count() or 1
        p = O.params(n_q_heads=hq, n_kv_heads=hkv, n_slots=n_slots, n_threads=cores)
        kh = kc16.cpu().numpy().view(np.uint16)[None]
        vh = vc16.cpu().numpy().view(np.uint16)[None]
        qh = qb.float().cpu().numpy()
        t_cpu = time.perf_counter()
        O.paged_prefill(p, O.MODE_GGML, 0, qh, cu.astype(np.int32), qs.astype(np.int32),
                        cl.astype(np.int32), bt_np, kh, vh)
        t_cpu = time.perf_counter() - t_cpu
        # the reference's own prefill algorithm on the same host cores: the
        # batch's new tokens concatenated, masked attention over the padded
        # buffer; it attends no cached prefix, so it does less work than the
        # path above (timing only; the f32 rows are the store's inputs)
        t_ref = time.perf_counter()
        O.concat_prefill_ggml(p, qh, cu.astype(np.int32), k.cpu().numpy(), v.cpu().numpy())
        t_ref = time.perf_counter() - t_ref
        cpu = {"cores": cores, "kind": "port", "ms": t_cpu * 1e3,
               "tflops": flops / world / t_cpu / 1e12,
               "reference_concat_ms": t_ref * 1e3,
               "sample": "the whole workload, once (oracle GGML-mode paged prefill; and the "
                         "reference's concat-all prefill, which ignores the cached prefix)"}
    h.close()
    fields = {"workload": name, "q_heads": Hq, "kv_heads": Hkv, "n_seqs": len(lens),
              "new_tokens": T, "sum_context": int(cl.sum()), "flops_per_step": flops,
              "steps": steps, "precision": "f16 Q x f16 K, f16 P x f16 V (K, V converted in smem), f32 accumulation",
              "kv_store": kv_store_roofline(T, hq, hkv, store_ms, q_out_bytes=2),
              "clocks": clk}
    if cpu is not None:
        fields["cpu"] = cpu
    return fields, pre_ms, step_ms


def bench_prefill_chunked(args, world, rank, device):
    """Chunked prefill against one-shot prefill: Qwen3-8B attention shape (32 q
    / 8 kv heads), 8 prompts of 8192 new tokens, nothing cached.  One shot:
    the fused q/k norm + RoPE + K/V store of all 65,536 tokens, then one
    causal prefill.  Chunked: nvattn_schedule_prefill_chunks with a 3,000
    token budget per step (22 steps; chunks start mid-block and a step can
    end one prompt and begin the next); each step stores its chunks' K/V and
    runs their prefill over everything cached so far.  Per-step inputs (q/k/v rows, plans) are built before the
    timed region; both runs time device work only.  Reports both totals, the
    longest step and TFLOP/s of the algorithmic causal FLOPs."""
    import torch
    import nvattn
    Hq, Hkv, n, L, budget = 32, 8, 8, 8192, 3000
    hq, hkv = Hq // world, Hkv // world
    lens = np.full(n, L, np.int64)
    need = (lens + BS - 1) // BS
    num_blocks = int(need.sum()) + 8
    rng = np.random.default_rng(SEED + 6)
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt_np = perm[:int(need.sum())].reshape(n, int(need.max()))
    cfg = nvattn.qwen3_config(n_layer=1, n_q_heads=hq, n_kv_heads=hkv, num_blocks=num_blocks,
                              max_seqs=n, max_context=L, max_position=L, device=device.index)
    h = nvattn.Handle(cfg)
    gen = torch.Generator(device=device)
    gen.manual_seed(6000 + rank)
    n_slots = num_blocks * BS
    kc = torch.zeros((n_slots, hkv, D), dtype=torch.int16, device=device)
    vc = torch.zeros_like(kc)
    T = int(lens.sum())
    q = torch.randn((T, hq, D), generator=gen, device=device)  # token t of seq s at s*L + t
    k = torch.randn((T, hkv, D), generator=gen, device=device)
    v = torch.randn((T, hkv, D), generator=gen, device=device)
    w16 = (1 + 0.02 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16).view(
        torch.int16)
    stream = torch.cuda.current_stream(device)

    def make_step(seqs, starts, ends):
        cu, qs, cl, pos, slot = nvattn.plan_prefill(ends, starts, bt_np[seqs])
        rows = np.concatenate([s * L + np.arange(a, b) for s, a, b in zip(seqs, starts, ends)])
        idx = torch.from_numpy(rows).to(device)
        t = {"q": q.index_select(0, idx), "k": k.index_select(0, idx),
             "v": v.index_select(0, idx)}
        t["qb"] = torch.empty(t["q"].shape, dtype=torch.float16, device=device)
        t["out"] = torch.empty(t["q"].shape, device=device)
        for name, arr in (("cu", cu), ("qs", qs), ("cl", cl), ("pos", pos), ("slot", slot),
                          ("bt", np.ascontiguousarray(bt_np[seqs]))):
            t[name] = torch.from_numpy(arr).to(device)
        t["max_q"] = int((cl - qs).max())
        return t

    def run(t):
        h.kv_store(0, t["q"], t["k"], t["v"], w16, w16, t["pos"], t["slot"], t["qb"], kc, vc,
                   stream=stream)
        h.prefill(0, t["qb"], t["cu"], t["qs"], t["cl"], t["bt"], t["max_q"], kc, vc, t["out"],
                  stream=stream)

    one = make_step(list(range(n)), [0] * n, [L] * n)
    chunks, done, held, free = [], np.zeros(n, np.int64), np.zeros(n, np.int64), num_blocks
    while (done < lens).any():
        idx = np.array([s for s in range(n) if done[s] < lens[s]])
        sel, ends, adds = nvattn.schedule_prefill_chunks(lens[idx], done[idx], held[idx], free,
                                                         256, budget)
        seqs = [int(idx[i]) for i in sel]
        chunks.append(make_step(seqs, [int(done[s]) for s in seqs], ends.tolist()))
        for s, e, a_ in zip(seqs, ends.tolist(), adds.tolist()):
            done[s], held[s] = e, held[s] + a_
            free -= a_

    def timed(steps_list, reps):
        for _ in range(2):
            for t in steps_list:
                run(t)
        torch.cuda.synchronize(device)
        evs = []
        for _ in range(reps):
            for t in steps_list:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                run(t)
                b.record(stream)
                evs.append((a, b))
        torch.cuda.synchronize(device)
        per = [a.elapsed_time(b) for a, b in evs]
        k_ = len(steps_list)
        totals = [sum(per[r * k_:(r + 1) * k_]) for r in range(reps)]
        return sum(totals) / reps, max(per)

    one_ms, _ = timed([one], 3)
    ch_ms, ch_max = timed(chunks, 3)
    h.check_device("prefill_chunked")
    tv = torch.tensor([one_ms, ch_ms, ch_max], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(tv, op=dist.ReduceOp.MAX)
    one_ms, ch_ms, ch_max = tv.tolist()
    h.close()
    flops = 4.0 * D * Hq * n * (L * (L + 1) // 2)
    return {"workload": "prefill_chunked_qwen3_8b_8x8192_budget3000", "q_heads": Hq,
            "kv_heads": Hkv, "n_seqs": n, "prompt_len": L, "token_budget": budget,
            "steps": len(chunks), "one_shot_ms": one_ms, "chunked_total_ms": ch_ms,
            "chunked_max_step_ms": ch_max, "chunked_over_one_shot": ch_ms / one_ms,
            "one_shot_tflops": flops / (one_ms / 1e3) / 1e12,
            "chunked_tflops": flops / (ch_ms / 1e3) / 1e12,
            "note": "store + prefill per step, device time"}


def kv_store_roofline(T, hq, hkv, ms, q_out_bytes):
    """Algorithmic bytes of the fused q/k norm + RoPE + K/V store on one GPU:
    read q, k, v (f32) and one RoPE row per token, write q (f32 or bf16) and
    the bf16 K/V rows; positions and slots 8 B per token."""
    hbm_peak, _, kind = peaks()
    per_tok = (hq + 2 * hkv) * D * 4 + D * 4 + hq * D * q_out_bytes + 2 * hkv * D * 2 + 8
    gbs = T * per_tok / (ms / 1e3) / 1e9
    return {"bound": "hbm", "kernel": "kv_store_qk_norm_rope", "tokens": T, "ms": ms,
            "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
            "peak_source": kind, "bytes_per_token": per_tok, "frac_of_8tbs": gbs / 8000.0}


def bench_decode_small(args, world, rank, device):
    """Small decode batch: 4 sequences of 37, 256, 513 and 1000 tokens (the new
    token included), Qwen3-0.6B attention heads (16 q / 8 kv), 64 physical
    blocks of a permuted pool, kv-head sharded.  Far too small to approach the
    HBM roofline (7.4 MB of K/V); reports the step's device time (store +
    decode, eager and as a CUDA graph; the fused decode step likewise), the
    decode launch's own device time and its GB/s.  On one GPU it also times, on the host
    cores, the oracle's paged decode in the reference's dtype chain and the
    reference's own decode algorithm (gather every history, append the new
    rows, masked attention over the concatenation) on the same inputs."""
    import torch
    import nvattn
    Hq, Hkv, B = 16, 8, 4
    hq, hkv = Hq // world, Hkv // world
    lens = np.array([37, 256, 513, 1000], np.int64)
    num_blocks = 64
    rng = np.random.default_rng(SEED + 4)
    perm = rng.permutation(num_blocks).astype(np.int32)
    need = (lens + BS - 1) // BS
    bt_np = np.full((B, int(need.max())), -1, np.int32)
    off = 0
    for s_ in range(B):
        bt_np[s_, :need[s_]] = perm[off:off + need[s_]]
        off += int(need[s_])
    cfg = nvattn.qwen3_config(n_layer=1, n_q_heads=hq, n_kv_heads=hkv, num_blocks=num_blocks,
                              max_seqs=B, max_context=int(lens.max()), device=device.index)
    h = nvattn.Handle(cfg)
    gen = torch.Generator(device=device)
    gen.manual_seed(4000 + rank)
    n_slots = num_blocks * BS
    kc = torch.randn((1, n_slots, hkv, D), generator=gen, device=device).to(torch.bfloat16)
    vc = torch.randn((1, n_slots, hkv, D), generator=gen, device=device).to(torch.bfloat16)
    cl, pos_np, slot_np = nvattn.plan_decode(lens, bt_np)
    bt, ctx = torch.from_numpy(bt_np).to(device), torch.from_numpy(cl).to(device)
    pos, slots = torch.from_numpy(pos_np).to(device), torch.from_numpy(slot_np).to(device)
    q0 = torch.randn((B, hq, D), generator=gen, device=device)
    kn = torch.randn((B, hkv, D), generator=gen, device=device)
    vn = torch.randn((B, hkv, D), generator=gen, device=device)
    w16 = (1 + 0.02 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16).view(
        torch.int16)
    q, out = torch.empty_like(q0), torch.empty((B, hq, D), device=device)
    kc16, vc16 = kc.view(torch.int16), vc.view(torch.int16)
    stream = torch.cuda.current_stream(device)

    def step():
        q.copy_(q0)
        h.kv_store(0, q, kn, vn, w16, w16, pos, slots, q, kc16, vc16, stream=stream)
        h.decode(0, q, kc16, vc16, bt, ctx, int(lens.max()), out, stream=stream)

    def queue_ahead():
        # a ~10 ms spin kernel holds the stream while the host issues the
        # timed calls, so the events around them see back-to-back device work
        torch.cuda._sleep(20_000_000)

    def loop_ms(body, n, queued):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if queued:
            queue_ahead()
        a.record(stream)
        for _ in range(n):
            body()
        b.record(stream)
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / n

    for _ in range(5):
        step()
    torch.cuda.synchronize(device)
    h.check_device("decode_small warmup")
    steps = 50
    # the step paced by the host (each call waits for Python to issue it),
    # then its device time (the same calls queued ahead of the device)
    host_ms = loop_ms(step, steps, queued=False)
    step_ms = loop_ms(step, steps, queued=True)
    h.check_device("decode_small")
    # The same step captured once in a CUDA graph and replayed (what a C++
    # caller or a graph-capturing engine issues).  A decode engine that keeps
    # its sequence lengths on the device can also capture the step's
    # planning: the second graph derives positions, slots and context lengths
    # with the device planner before the store and decode.
    d_lens = torch.from_numpy(lens).to(device)
    ctx_p, pos_p, slots_p = (torch.empty(B, dtype=torch.int32, device=device) for _ in range(3))

    def plain_body(cs):
        q.copy_(q0)
        h.kv_store(0, q, kn, vn, w16, w16, pos, slots, q, kc16, vc16, stream=cs)
        h.decode(0, q, kc16, vc16, bt, ctx, int(lens.max()), out, stream=cs)

    def planned_body(cs):
        h.plan_decode(d_lens, bt, ctx_p, pos_p, slots_p, stream=cs)
        q.copy_(q0)
        h.kv_store(0, q, kn, vn, w16, w16, pos_p, slots_p, q, kc16, vc16, stream=cs)
        h.decode(0, q, kc16, vc16, bt, ctx_p, int(lens.max()), out, stream=cs)

    def graph_us_of(body):
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                body(torch.cuda.current_stream(device))
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize(device)
            ga, gb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            queue_ahead()
            ga.record(stream)
            for _ in range(steps):
                g.replay()
            gb.record(stream)
            torch.cuda.synchronize(device)
            h.check_device("decode_small graph")
            del g
            return ga.elapsed_time(gb) / steps * 1e3
        except Exception as e:  # noqa: BLE001 -- reported, not fatal
            return f"capture failed: {e}"

    # The fused step (nvattn_paged_decode_step): the store and the decode in
    # one launch, reading the raw q (q0) and writing no q back.
    def fused_body(cs):
        h.decode_step(0, q0, kn, vn, w16, w16, pos, slots, kc16, vc16, bt, ctx, int(lens.max()),
                      out, stream=cs)

    def fused_planned_body(cs):
        h.plan_decode(d_lens, bt, ctx_p, pos_p, slots_p, stream=cs)
        h.decode_step(0, q0, kn, vn, w16, w16, pos_p, slots_p, kc16, vc16, bt, ctx_p,
                      int(lens.max()), out, stream=cs)

    planned_body(stream)
    fused_planned_body(stream)
    torch.cuda.synchronize(device)
    h.check_device("decode_small planned warmup")
    fz, fb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    queue_ahead()
    fz.record(stream)
    for _ in range(steps):
        fused_body(stream)
    fb.record(stream)
    torch.cuda.synchronize(device)
    h.check_device("decode_small fused")
    fused_us = fz.elapsed_time(fb) / steps * 1e3

    # the decode launch alone: 20 launches captured in one graph, replayed
    # queued ahead (per-launch device time, no events between launches)
    def decode_body20(cs):
        for _ in range(20):
            h.decode(0, q, kc16, vc16, bt, ctx, int(lens.max()), out, stream=cs)

    graph_us, planned_us = graph_us_of(plain_body), graph_us_of(planned_body)
    fgraph_us, fplanned_us = graph_us_of(fused_body), graph_us_of(fused_planned_body)
    dec20_us = graph_us_of(decode_body20)
    vals = (graph_us, planned_us, fgraph_us, fplanned_us, fused_us, dec20_us,
            host_ms * 1e3, step_ms * 1e3)
    gt = torch.tensor([v if isinstance(v, float) else -1.0 for v in vals],
                      dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
    graph_us, planned_us, fgraph_us, fplanned_us, fused_us, dec20_us, host_us, step_us = (
        gt[i].item() if isinstance(v, float) else v for i, v in enumerate(vals))
    # a failed capture is reported in its field; the decode time is then NaN
    dec_ms = dec20_us / 20 / 1e3 if isinstance(dec20_us, float) else float("nan")
    hbm_peak, _, kind = peaks()
    alg = int(lens.sum()) * hkv * D * 2 * 2 + B * hq * D * 4 * 2 + int(need.sum()) * 4 + B * 4
    gbs = alg / (dec_ms / 1e3) / 1e9
    res = {"workload": "decode_qwen3_0p6b_attn_4seq_len37-1000", "q_heads": Hq, "kv_heads": Hkv,
           "lens": lens.tolist(), "steps": steps, "step_us": step_us,
           "host_paced_step_us": host_us,
           "graph_step_us": graph_us, "graph_step_device_planned_us": planned_us,
           "decode_us": dec_ms * 1e3,
           "timing": "device time with the host queued ahead (a spin kernel first), events "
                     "around whole loops; decode_us: 20 decode launches per graph replay; "
                     "host_paced_step_us: the eager step as Python issues it",
           "fused_step_us": fused_us, "fused_graph_step_us": fgraph_us,
           "fused_graph_step_device_planned_us": fplanned_us,
           "roofline": {"bound": "hbm", "kernel": "paged_decode (split-KV, merged in-kernel by the last split)",
                        "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                        "frac": gbs / hbm_peak, "peak_source": kind, "algorithmic_bytes": alg,
                        "frac_of_8tbs": gbs / 8000.0}}
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        cores = os.cpu_count() or 1
        # the cache before this step's store: regenerate it with the same seed
        gen.manual_seed(4000 + rank)
        kh = torch.randn((1, n_slots, hkv, D), generator=gen, device=device).to(
            torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)
        vh = torch.randn((1, n_slots, hkv, D), generator=gen, device=device).to(
            torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)
        p = O.params(n_q_heads=hq, n_kv_heads=hkv, n_slots=n_slots, n_threads=cores)
        qh, knh, vnh = q.cpu().numpy(), kn.cpu().numpy(), vn.cpu().numpy()
        lens32 = lens.astype(np.int32)

        def timed(fn):
            n, t0 = 0, time.perf_counter()
            while True:
                fn()
                n += 1
                dt = time.perf_counter() - t0
                if dt >= 0.5 or n >= 200:
                    return dt / n

        res["cpu"] = {
            "cores": cores,
            "oracle_paged_ggml_us": 1e6 * timed(lambda: O.paged_decode(
                p, O.MODE_GGML, 0, qh, kh, vh, bt_np, lens32, knh, vnh)),
            "reference_concat_all_us": 1e6 * timed(lambda: O.concat_decode_ggml(
                p, 0, qh, kh, vh, bt_np, lens32, knh, vnh)),
            "note": "host cores; the reference algorithm's gather/concat/mask restated by the "
                    "oracle (ggml itself is absent)"}
    h.close()
    return res


def bench_decode_long(args, world, rank, device):
    """Secondary decode workload: the Qwen3-32B attention shape (64 q / 8 kv
    heads) with 16 sequences at 131104 cached tokens (the middle of the 64
    decode steps that follow the 2048-token chunk), kv-head sharded like the
    headline workload.  Device-resident inputs; returns a JSON-ready dict."""
    import torch
    import nvattn
    Hq, Hkv, B, L = 64, 8, 16, 131104
    hq, hkv = Hq // world, Hkv // world
    need = (L + BS - 1) // BS
    num_blocks = B * need + 8
    rng = np.random.default_rng(SEED + 3)
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt_np = perm[:B * need].reshape(B, need)
    lens = np.full(B, L, np.int64)
    cfg = nvattn.qwen3_config(n_layer=1, n_q_heads=hq, n_kv_heads=hkv, num_blocks=num_blocks,
                              max_seqs=B, max_context=L, max_position=L, device=device.index)
    h = nvattn.Handle(cfg)
    gen = torch.Generator(device=device)
    gen.manual_seed(3000 + rank)
    n_slots = num_blocks * BS
    kc = torch.empty((n_slots, hkv, D), dtype=torch.bfloat16, device=device)
    vc = torch.empty_like(kc)
    for t in (kc, vc):
        for i in range(0, n_slots, 1 << 16):
            t[i:i + (1 << 16)].copy_(torch.randn((min(1 << 16, n_slots - i), hkv, D),
                                                 generator=gen, device=device))
    cl, pos_np, slot_np = nvattn.plan_decode(lens, bt_np)
    bt, ctx = torch.from_numpy(bt_np).to(device), torch.from_numpy(cl).to(device)
    pos, slots = torch.from_numpy(pos_np).to(device), torch.from_numpy(slot_np).to(device)
    q0 = torch.randn((B, hq, D), generator=gen, device=device)
    kn = torch.randn((B, hkv, D), generator=gen, device=device)
    vn = torch.randn((B, hkv, D), generator=gen, device=device)
    w16 = (1 + 0.02 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16).view(
        torch.int16)
    q, out = torch.empty_like(q0), torch.empty((B, hq, D), device=device)
    kc16, vc16 = kc.view(torch.int16), vc.view(torch.int16)
    stream = torch.cuda.current_stream(device)
    evs = []

    def step():
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        q.copy_(q0)
        h.kv_store(0, q, kn, vn, w16, w16, pos, slots, q, kc16, vc16, stream=stream)
        a.record(stream)
        h.decode(0, q, kc16, vc16, bt, ctx, L, out, stream=stream)
        b.record(stream)
        evs.append((a, b))

    for _ in range(3):
        step()
    torch.cuda.synchronize(device)
    h.check_device("decode_long warmup")
    evs.clear()
    steps = max(5, args.prefill_steps * 2)
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[device.index])
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(device)
    h.check_device("decode_long")
    h.close()
    t = torch.tensor([t0.elapsed_time(t1) / steps,
                      sum(a.elapsed_time(b) for a, b in evs) / len(evs)],
                     dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, dec_ms = t.tolist()
    hbm_peak, _, kind = peaks()
    alg = B * L * hkv * D * 2 * 2 + B * hq * D * 4 * 2 + B * need * 4 + B * 4
    gbs = alg / (dec_ms / 1e3) / 1e9
    return {"workload": "decode_qwen3_32b_attn_16seq_ctx131104", "q_heads": Hq, "kv_heads": Hkv,
            "n_seqs": B, "context": L, "steps": steps, "ms_per_step": step_ms,
            "tokens_per_s": B / (step_ms / 1e3),
            "roofline": {"bound": "hbm", "kernel": "paged_decode (split-KV, merged in-kernel by the last split)",
                         "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": gbs / hbm_peak, "peak_source": kind, "decode_ms": dec_ms,
                         "algorithmic_bytes": alg, "frac_of_8tbs": gbs / 8000.0}}


def bench_model_step(args, world, rank, device):
    """The full-model decode step (one GPU): Qwen3-0.6B architecture, 28
    layers, hidden 1024, 16 q / 8 kv heads, FFN 3072, vocabulary 151936,
    random N(0, 0.02) bf16 weights, 64 sequences with contexts uniform in
    [256, 8192] (seeded), greedy sampling.  ModelRunner::Run's decode step
    (nano-vllm.cpp_b200/python/model_runner.py): libnvattn serves the fused
    store, paged decode and sampling; embedding, norms, projections, FFN and
    lm_head run as torch / cuBLAS ops ("not-ggml" -- the reference's ggml is
    not vendored).  The step (all layers + sampling) is captured once in a
    CUDA graph; each timed step writes the host planner's positions / slots /
    block tables and the input tokens into the step's device buffers, replays
    the graph and reads the 64 tokens back, which feed the next step.  The
    attention share is a separate graph holding only the 28 layers' store +
    decode, timed alone."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "nano-vllm.cpp_b200", "python"))
    import model_runner as MR
    shape = MR.Qwen3Shape()
    B, steps, warm = 64, max(10, min(args.steps, 50)), 3
    rng = np.random.default_rng(SEED + 8)
    lens = rng.integers(256, 8193, B).astype(np.int64)
    max_blocks = int((lens.max() + steps + warm + 2 + BS - 1) // BS)
    num_blocks = int(((lens + steps + warm + 2 + BS - 1) // BS).sum()) + 8
    w = MR.Qwen3Weights(shape, device, seed=8)
    run = MR.DecodeRunner(shape, w, num_blocks, B, max_blocks, device)
    bufs = run.allocate(B)
    gen = torch.Generator(device=device)
    gen.manual_seed(8000)
    for t in (run.k_cache, run.v_cache):
        for layer in range(shape.n_layer):
            t[layer].copy_(torch.randn(t[layer].shape, generator=gen, device=device)
                           .to(torch.bfloat16).view(torch.int16))
    tables = MR.BlockTables(lens, num_blocks, max_blocks, seed=SEED + 9)
    tokens = rng.integers(0, shape.vocab, B)
    stream = torch.cuda.current_stream(device)
    run.set_inputs(tokens, tables)
    run.forward()  # eager warm-up (kernel attributes, workspaces)
    torch.cuda.synchronize(device)
    run.h.check_device("model_step eager")
    side = torch.cuda.Stream(device=device)
    side.wait_stream(stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            run.forward(stream=side)
    stream.wait_stream(side)
    host_next = torch.empty(B, dtype=torch.int32).pin_memory()

    def one_step():
        run.set_inputs(tokens, tables)
        g.replay()
        host_next.copy_(bufs["next"], non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
        tables.append_token()
        return host_next.numpy().copy()

    for _ in range(warm):
        tokens = one_step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall = time.perf_counter()
    e0.record(stream)
    dev_ms = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        run.set_inputs(tokens, tables)
        a.record(stream)
        g.replay()
        b.record(stream)
        host_next.copy_(bufs["next"], non_blocking=True)
        stream.synchronize()
        dev_ms.append(a.elapsed_time(b))
        tables.append_token()
        tokens = host_next.numpy().copy()
    e1.record(stream)
    torch.cuda.synchronize(device)
    wall = time.perf_counter() - t_wall
    e2e_ms = e0.elapsed_time(e1) / steps
    run.h.check_device("model_step")
    # attention alone: the 28 layers' fused store + decode on the same inputs
    q = torch.randn((B, shape.n_q_heads, shape.head_dim), generator=gen, device=device)
    kv = torch.randn((B, shape.n_kv_heads, shape.head_dim), generator=gen, device=device)
    qs = [q.clone() for _ in range(shape.n_layer)]
    run.set_inputs(tokens, tables)
    ga = torch.cuda.CUDAGraph()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        with torch.cuda.graph(ga, stream=side):
            for layer in range(shape.n_layer):
                run.library_attention(layer, qs[layer], kv, kv, stream=side)
    stream.wait_stream(side)
    ga.replay()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(5):
        ga.replay()
    b.record(stream)
    torch.cuda.synchronize(device)
    attn_ms = a.elapsed_time(b) / 5
    run.h.check_device("model_step attention")
    step_ms = statistics.median(dev_ms)
    kv_bytes = int(tables.lens.sum()) * shape.n_kv_heads * shape.head_dim * 2 * 2 * shape.n_layer
    del g, ga
    run.close()
    return {"workload": "decode_step_qwen3_0p6b_arch_28layers_64seq_ctx256-8192",
            "ops_outside_attention": "not-ggml: torch / cuBLAS (bf16 weights, f32 residual)",
            "n_layer": shape.n_layer, "n_seqs": B, "steps": steps,
            "sum_context_start": int(lens.sum()),
            "step_ms": step_ms, "tokens_per_s": B / (step_ms / 1e3),
            "e2e": {"ms_per_step": e2e_ms, "tokens_per_s": B / (e2e_ms / 1e3),
                    "note": "host planner + H2D inputs + graph replay + D2H tokens per step"},
            "wall_tokens_per_s": B * steps / wall,
            "attention_ms": attn_ms, "attention_share": attn_ms / step_ms,
            "attention_kv_gb_per_step": kv_bytes / 1e9,
            "attention_gbs": kv_bytes / (attn_ms / 1e3) / 1e9}


def bench_kv_store(args, world, rank, device):
    """The decode step's KV store alone (for profiling): the headline
    workload's 256 new tokens (this rank's shard of 32 q / 8 kv heads),
    random positions and slots in a 64-block cache, 50 launches queued behind
    a spin kernel and timed with CUDA events (device time per launch)."""
    import torch
    import nvattn
    T, ways = N_SEQS, (world if world > 1 else max(1, args.shard_of))
    hq, hkv = HQ // ways, HKV // ways
    cfg = nvattn.qwen3_config(n_layer=1, n_q_heads=hq, n_kv_heads=hkv, num_blocks=64,
                              max_seqs=T, max_context=8192, max_position=40960,
                              device=device.index)
    h = nvattn.Handle(cfg)
    gen = torch.Generator(device=device)
    gen.manual_seed(5000 + rank)
    kc = torch.zeros((64 * BS, hkv, D), dtype=torch.int16, device=device)
    vc = torch.zeros_like(kc)
    q = torch.randn((T, hq, D), generator=gen, device=device)
    k = torch.randn((T, hkv, D), generator=gen, device=device)
    v = torch.randn((T, hkv, D), generator=gen, device=device)
    w = (1 + 0.02 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16).view(
        torch.int16)
    pos = torch.randint(0, 32768, (T,), generator=gen, dtype=torch.int32, device=device)
    slots = torch.randperm(64 * BS, generator=gen, device=device)[:T].to(torch.int32)
    qo = torch.empty_like(q)
    for _ in range(10):
        h.kv_store(0, q, k, v, w, w, pos, slots, qo, kc, vc)
    torch.cuda.synchronize(device)
    h.check_device("kv_store warmup")
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(20_000_000)
    a.record()
    for _ in range(50):
        h.kv_store(0, q, k, v, w, w, pos, slots, qo, kc, vc)
    b.record()
    torch.cuda.synchronize(device)
    h.check_device("kv_store")
    h.close()
    return kv_store_roofline(T, hq, hkv, a.elapsed_time(b) / 50, q_out_bytes=4)


def bench_sample(args, world, rank, device):
    """Token sampling over the headline batch: 256 rows of Qwen3's 151936
    logits (f32, N(0, 4^2)), temperature 0.8 and repetition penalty 1.2 (the
    reference's example settings), each sequence's history its decode
    context length of uniform random ids (1k-32k ids, 2.7 M in all).  Two
    logits buffers alternate (311 MB > L2).  Reports the call's device time
    (history count, logits pass and finish kernels), the same rows greedy
    without history (the bare logits pass), GB/s of the call's algorithmic
    bytes, and on one GPU the oracle's restatement of the reference's Sample
    on a bounded sample of rows, timed on one host core as the reference
    runs it."""
    import torch
    import nvattn
    V, temp, pen = 151936, 0.8, 1.2
    lens, _, _ = workload()
    B = lens.shape[0]
    rng = np.random.default_rng(SEED + 5)
    off_np = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    hist_np = rng.integers(0, V, int(off_np[-1])).astype(np.int32)
    cfg = nvattn.qwen3_config(n_layer=1, n_q_heads=8, n_kv_heads=8, num_blocks=1, max_seqs=B,
                              max_context=BS, device=device.index)
    h = nvattn.Handle(cfg)
    gen = torch.Generator(device=device)
    gen.manual_seed(5000 + rank)
    xs = [4.0 * torch.randn((B, V), generator=gen, device=device) for _ in range(2)]
    t = torch.full((B,), temp, device=device)
    t0 = torch.zeros(B, device=device)
    p = torch.full((B,), pen, device=device)
    u = torch.rand(B, generator=gen, device=device)
    hist = torch.from_numpy(hist_np).to(device)
    off = torch.from_numpy(off_np).to(device)
    tok = torch.empty(B, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    steps = 50

    def timed(fn):
        for i in range(5):
            fn(xs[i % 2])
        torch.cuda.synchronize(device)
        evs = []
        for i in range(steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn(xs[i % 2])
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize(device)
        return sum(a.elapsed_time(b) for a, b in evs) / steps

    full_ms = timed(lambda x: h.sample(x, t, p, u, tok, hist, off, stream=stream))
    greedy_ms = timed(lambda x: h.sample(x, t0, p, u, tok, None, None, stream=stream))
    temp_ms = timed(lambda x: h.sample(x, t, p, u, tok, None, None, stream=stream))
    greedy_pen_ms = timed(lambda x: h.sample(x, t0, p, u, tok, hist, off, stream=stream))
    h.check_device("sample")
    tv = torch.tensor([full_ms, greedy_ms, temp_ms, greedy_pen_ms], dtype=torch.float64,
                      device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(tv, op=dist.ReduceOp.MAX)
    full_ms, greedy_ms, temp_ms, greedy_pen_ms = tv.tolist()
    hbm_peak, _, kind = peaks()
    logit_bytes = B * V * 4
    # logits once, history ids once, per-row scalars and offsets, tokens
    alg = logit_bytes + int(off_np[-1]) * 4 + B * (4 * 3 + 8 + 4)
    res = {"workload": "sample_qwen3_vocab151936_256seq_t0.8_penalty1.2",
           "n_seqs": B, "vocab": V, "history_ids": int(off_np[-1]), "steps": steps,
           "sample_us": full_ms * 1e3, "greedy_no_history_us": greedy_ms * 1e3,
           "temperature_no_history_us": temp_ms * 1e3, "greedy_penalty_us": greedy_pen_ms * 1e3,
           "roofline": {"bound": "hbm", "kernel": "sample (count + pass + finish)",
                        "achieved": alg / (full_ms / 1e3) / 1e9, "peak": hbm_peak,
                        "unit": "GB/s", "frac": alg / (full_ms / 1e3) / 1e9 / hbm_peak,
                        "peak_source": kind, "algorithmic_bytes": alg,
                        "greedy_pass_gbs": logit_bytes / (greedy_ms / 1e3) / 1e9}}
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        n_cpu = 8
        xh = xs[0][:n_cpu].cpu().numpy()
        uh = u[:n_cpu].cpu().numpy()
        t_begin = time.perf_counter()
        O.sample(xh, np.full(n_cpu, temp, np.float32), np.full(n_cpu, pen, np.float32), uh,
                 hist_np[:off_np[n_cpu]], off_np[:n_cpu + 1])
        dt = time.perf_counter() - t_begin
        res["cpu"] = {"cores": 1, "kind": "port", "us_per_row": dt / n_cpu * 1e6,
                      "batch_us_projected": dt / n_cpu * B * 1e6,
                      "sample": f"first {n_cpu} of the {B} rows, one host thread (the "
                                "reference's Sample loop is sequential)"}
    h.close()
    del xs
    torch.cuda.empty_cache()
    return res


def run_prefills(args, world, rank, device):
    """Times every selected prefill workload; returns JSON-ready dicts (the
    per-step times are the max over ranks)."""
    import torch
    kinds = [k for k in args.prefill.split(",") if k and k != "none"]
    _, tflops_peak, peak_kind = peaks()
    results = []
    for kind in kinds:
        fields, pre_ms, step_ms = bench_prefill(kind, args, world, rank, device)
        t = torch.tensor([pre_ms, step_ms], dtype=torch.float64, device=device)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pre_ms, step_ms = t.tolist()
        job_tflops = fields["flops_per_step"] / (pre_ms / 1e3) / 1e12
        achieved = job_tflops / world  # per GPU, against one GPU's peak
        fields.update({
            "tokens_per_s": fields["new_tokens"] / (step_ms / 1e3), "ms_per_step": step_ms,
            "tflops": job_tflops,
            "roofline": {"bound": "tensor", "kernel": "paged_prefill (tcgen05)",
                         "achieved": achieved, "peak": tflops_peak, "unit": "TFLOP/s",
                         "frac": achieved / tflops_peak, "peak_source": peak_kind,
                         "prefill_ms": pre_ms, "frac_of_2250_nominal": achieved / 2250.0},
        })
        # tensor-pipe utilisation from an ncu capture of this kernel
        # (sm__pipe_tensor_cycles_active, fraction of elapsed cycles) on the
        # chunk shape or the prefix-hit workload; null for other shapes
        wl = fields["workload"]
        fields["roofline"]["ncu_tensor_pipe_active"] = (
            NCU_PREFILL_TENSOR_ACTIVE if wl.startswith("chunked_prefill")
            else NCU_PREFIX_HIT_TENSOR_ACTIVE if wl.startswith("prefill_prefix_hit") else None)
        # the dense BF16 tensor rate at the SM clock sampled during the run
        # (148 SMs x 8192 FLOP per cycle; 2.25 PFLOP/s is this at ~1.86 GHz)
        mhz = (fields.get("clocks") or {}).get("sm_mhz")
        if mhz:
            at_clock = 148 * 8192 * mhz * 1e6 / 1e12
            fields["roofline"]["peak_at_sampled_clock"] = at_clock
            fields["roofline"]["frac_of_peak_at_sampled_clock"] = achieved / at_clock
        fields["kind"] = kind
        fields["roofline"]["flops_per_step"] = fields["flops_per_step"]
        results.append(fields)
    return results


def allgather_loop(args, world, rank, local_rank, step, out, stream, B, hq, lens, bt_np, kc,
                   vc, normed_q):
    """Second timed loop at N > 1: every step is the decode step followed by
    NCCL's all-gather of the [B][Hq/N][128] head outputs into
    [N][B][Hq/N][128] (the head-concatenated attention output o_proj needs).
    Then rank 0 checks the gathered output of the two shortest sequences
    against the oracle (exact math over all heads): every rank hands over
    those sequences' cache rows and normed q for its heads (normed_q() runs
    the step's KV store, which writes them), and rank 0 reassembles them.
    Every rank runs the same collectives in the same order."""
    import torch
    import torch.distributed as dist
    gathered = torch.empty((world * B, hq, D), device=device_of(out))
    ev = []

    def gstep():
        step()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        dist.all_gather_into_tensor(gathered, out)
        b.record(stream)
        ev.append((a, b))

    for _ in range(3):
        gstep()
    dist.barrier(device_ids=[local_rank])
    torch.cuda.synchronize()
    ev.clear()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        gstep()
    t1.record(stream)
    torch.cuda.synchronize()
    dist.barrier(device_ids=[local_rank])
    tv = torch.tensor([t0.elapsed_time(t1) / 1e3,
                       sum(a.elapsed_time(b) for a, b in ev) / len(ev)],
                      dtype=torch.float64, device=device_of(out))
    dist.all_reduce(tv, op=dist.ReduceOp.MAX)
    elapsed, ag_ms = tv.tolist()

    # sharded parity: the gathered output holds the last step's attention
    full = gathered.view(world, B, hq, D).permute(1, 0, 2, 3).reshape(B, world * hq, D)
    sel = np.argsort(lens, kind="stable")[:2]
    need = (lens[sel] + BS - 1) // BS
    ids = np.concatenate([bt_np[s, :need[i]] for i, s in enumerate(sel)])
    rows = (torch.from_numpy(ids.astype(np.int64)).to(kc.device)[:, None] * BS
            + torch.arange(BS, device=kc.device)[None]).reshape(-1)
    # bf16 on the wire (NCCL gathers no int16), bit patterns on the host
    mine = torch.cat([kc.index_select(0, rows), vc.index_select(0, rows)], 0).contiguous()
    theirs = torch.empty((world,) + tuple(mine.shape), dtype=mine.dtype, device=mine.device)
    dist.all_gather_into_tensor(theirs, mine)
    q = normed_q()
    qs = q[torch.from_numpy(sel).to(q.device)].contiguous()
    q_all = torch.empty((world,) + tuple(qs.shape), dtype=qs.dtype, device=qs.device)
    dist.all_gather_into_tensor(q_all, qs)
    res = {"allgather_ms": ag_ms, "steps": args.steps, "ms_per_step": 1e3 * elapsed / args.steps,
           "e2e_with_gather": {"value": B * args.steps / elapsed, "unit": "tokens/s"},
           "bytes_per_rank": B * hq * D * 4, "_gathered": gathered}
    if rank == 0:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        k_full, v_full, q_full, btc = reassemble_shards(
            theirs.view(torch.int16).cpu().numpy().view(np.uint16), q_all.cpu().numpy(), need)
        p = O.params(n_q_heads=world * hq, n_kv_heads=k_full.shape[2],
                     n_slots=k_full.shape[1], n_threads=0)
        ref = O.paged_decode(p, O.MODE_TRUTH, 0, q_full, k_full, v_full, btc,
                             lens[sel].astype(np.int32))
        got = full[torch.from_numpy(sel).to(full.device)].cpu().numpy()
        mx, mr = O.err_stats(got, ref)
        res["sharded_parity"] = {"seqs": [int(s) for s in sel], "max_abs": mx, "mean_rel": mr,
                                 "ok": bool(mx <= 2e-2 and mr <= 1e-3),
                                 "against": "oracle TRUTH over all heads"}
    return res


def peer_gather_loop(args, world, rank, local_rank, h, peer_step, stream, B, hq, nccl_gathered):
    """Third timed loop at N > 1: the decode step with the gather fused over
    peer memory (nvattn_paged_decode_step_gather): each rank's decode stores
    its output rows into every rank's gathered buffer as it finishes them,
    and the launch's last CTA to write final rows releases them to every
    rank and waits for the other ranks' -- one launch for the step and its
    gather (two where the step's grid takes the store launch first).
    The rows of the last step are compared with the NCCL all-gather's (the
    same step's outputs: equal bit for bit).  The IPC handles travel by an
    NCCL all-gather.  Every rank runs the same collectives in the same order
    whether or not its own part failed: a failure (no IPC mapping between the
    ranks, a release/wait that ran out of time) is reported in the returned
    dict as "error" instead of ending the run."""
    import nvattn
    import torch
    import torch.distributed as dist
    device = device_of(nccl_gathered)
    err = None

    def agree(ok):
        flag = torch.tensor([int(ok)], dtype=torch.int32, device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        return bool(flag.item())

    try:
        blob = h.gather_init(world, rank)
    except Exception as e:  # reported; the other ranks learn of it below
        err, blob = f"gather_init: {e}", bytes(nvattn.IPC_HANDLE_BYTES)
    mine = torch.tensor(list(blob), dtype=torch.uint8, device=device)
    handles = torch.empty((world, mine.numel()), dtype=torch.uint8, device=device)
    dist.all_gather_into_tensor(handles, mine)
    if err is None:
        hb = handles.cpu().numpy()
        try:
            h.gather_connect([hb[p].tobytes() for p in range(world)])
        except Exception as e:
            err = f"gather_connect: {e}"
    if not agree(err is None):
        return {"error": err or "another rank could not map the gathered buffers"}
    dist.barrier(device_ids=[local_rank])
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        for _ in range(3):
            peer_step()
        torch.cuda.synchronize()
        h.check_device("peer gather warm-up")
    except Exception as e:
        err = str(e)
    if agree(err is None):
        dist.barrier(device_ids=[local_rank])
        try:
            t0.record(stream)
            for _ in range(args.steps):
                peer_step()
            t1.record(stream)
            torch.cuda.synchronize()
            h.check_device("peer gather")
        except Exception as e:
            err = str(e)
    if not agree(err is None):
        return {"error": err or "the release/wait failed on another rank"}
    tv = torch.tensor([t0.elapsed_time(t1) / 1e3], dtype=torch.float64, device=device)
    dist.all_reduce(tv, op=dist.ReduceOp.MAX)
    elapsed = tv.item()
    got = torch.empty((world, B, hq, D), device=device)
    h.gather_read(3 + args.steps - 1, B, got, stream=stream)
    torch.cuda.synchronize()
    same = torch.tensor([int(torch.equal(got.view(-1), nccl_gathered.view(-1)))], device=device)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    return {"ms_per_step": 1e3 * elapsed / args.steps,
            "e2e_with_gather": {"value": B * args.steps / elapsed, "unit": "tokens/s"},
            "identical_to_nccl_gather": bool(same.item()),
            "note": "decode step whose output rows are stored into every rank's gathered "
                    "buffer over NVLink; its last final-row CTA releases them and waits for "
                    "the other ranks' (bounded); no NCCL on the data path"}


def reassemble_shards(kv_ranks, q_ranks, need):
    """Rebuilds all heads from per-rank pieces (rank r owns kv heads
    [r*Hkv/N, (r+1)*Hkv/N) and their q heads, consecutively): kv_ranks
    [N][2n][Hkv/N][D] = each rank's K rows then V rows of the sampled
    sequences' blocks (n rows, blocks in sequence order), q_ranks
    [N][S][Hq/N][D].  Returns a one-layer K and V cache [1][n][Hkv][D], the
    queries [S][Hq][D] and a block table numbering the blocks in order."""
    world = kv_ranks.shape[0]
    n = kv_ranks.shape[1] // 2
    k_full = np.concatenate([kv_ranks[r, :n] for r in range(world)], axis=1)[None]
    v_full = np.concatenate([kv_ranks[r, n:] for r in range(world)], axis=1)[None]
    q_full = np.concatenate([q_ranks[r] for r in range(world)], axis=1)
    btc = np.full((len(need), int(max(need))), -1, np.int32)
    off = 0
    for i, nb in enumerate(need):
        btc[i, :nb] = np.arange(off, off + nb)
        off += int(nb)
    return (np.ascontiguousarray(k_full), np.ascontiguousarray(v_full),
            np.ascontiguousarray(q_full), btc)


def device_of(t):
    return t.device


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def mark(self):
        return len(self.rows)

    def stop(self, since=0):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()
        rows = self.rows[since:] or self.rows[-3:]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def cpu_sample(lens, bt, k_host_fn, n_target_s=12.0):
    """Times the oracle's GGML-mode paged decode (the reference's dtype chain)
    on all host cores over the first sequences of the workload; returns
    (tokens/s, n_seqs, seconds, cores)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    results = []
    n = 2
    while True:
        kc, vc, btc, lc, q = k_host_fn(n)
        p = O.params(n_q_heads=HQ, n_kv_heads=HKV, n_slots=kc.shape[1], n_threads=cores)
        t0 = time.perf_counter()
        O.paged_decode(p, O.MODE_GGML, 0, q, kc, vc, btc, lc)
        dt = time.perf_counter() - t0
        results.append((n, dt))
        if dt >= n_target_s or n >= len(lens):
            break
        n = min(len(lens), max(n + 1, int(n * min(8.0, n_target_s / max(dt, 1e-3)))))
    n, dt = results[-1]
    return n / dt, n, dt, cores


def headline_config(world, ways, n_seqs, lens, allgather):
    """The headline workload's `config` object, shared by both arms so that
    they describe the same job (the reference arm: the same N, its own
    sample of it timed on the host)."""
    kv_bytes = int(lens.sum()) * (HKV // ways) * D * 2 * 2
    return {"workload": WORKLOAD if n_seqs == N_SEQS else f"{WORKLOAD}[first {n_seqs}]",
            "n_seqs": n_seqs, "q_heads": HQ, "kv_heads": HKV,
            "head_dim": D, "block_size": BS, "sum_context": int(lens.sum()),
            "kv_gb_per_gpu": round(kv_bytes / 1e9, 3),
            "parallelism": (f"kv-head shard x{world}" if ways == world else
                            f"rank 0's kv-head shard of x{ways} on one GPU"),
            "l2": "inputs larger than L2 (KV cache >> 126 MB), no flush",
            "allgather": allgather}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    lens, bt, _ = workload()
    rng = np.random.default_rng(SEED + 1)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    # A pool of 128 physical blocks of N(0,1) bf16 K/V; the sample's block
    # tables walk it cyclically (physical blocks may be shared, as prefix
    # caching does), which keeps host set-up time independent of the sample.
    POOL = 128
    kpool = O.f32_to_bf16(rng.standard_normal((1, POOL * BS, HKV, D), dtype=np.float32))
    vpool = O.f32_to_bf16(rng.standard_normal((1, POOL * BS, HKV, D), dtype=np.float32))

    def host_case(n):
        need = (lens[:n] + BS - 1) // BS
        btc = np.full((n, bt.shape[1]), -1, np.int32)
        o = 0
        for s in range(n):
            btc[s, :need[s]] = np.arange(o, o + need[s]) % POOL
            o += int(need[s])
        q = rng.standard_normal((n, HQ, D), dtype=np.float32)
        return kpool, vpool, btc, lens[:n].astype(np.int32), q

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    # size one step so that warmup + steps take about two minutes in all
    per_step = min(2.0, 120.0 / max(1, args.steps + args.warmup))
    tps, n, dt, cores = cpu_sample(lens, bt, host_case, n_target_s=per_step)
    kc, vc, btc, lc, q = host_case(n)
    p = O.params(n_q_heads=HQ, n_kv_heads=HKV, n_slots=kc.shape[1], n_threads=cores)
    for _ in range(args.warmup):
        O.paged_decode(p, O.MODE_GGML, 0, q, kc, vc, btc, lc)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.paged_decode(p, O.MODE_GGML, 0, q, kc, vc, btc, lc)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = n * args.steps / total
    sample = (f"first {n} of the {N_SEQS} sequences (sum L = {int(lc.sum())} tokens) per step; "
              "oracle GGML mode: f16 Q/K/V, f32 online softmax, f16 V accumulator, paged form "
              "(the reference's concat-all form is O(B*sum L))")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16/f32 (ggml chain)",
            "data": "synthetic",
            "config": headline_config(args.gpus, args.gpus, N_SEQS, lens,
                                      args.gpus > 1 and not args.no_allgather),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-allgather", action="store_true",
                    help="with N > 1 GPUs, skip the second timed loop that all-gathers the "
                         "head-sharded outputs every step (NCCL) and checks them")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seqs", type=int, default=N_SEQS,
                    help="use the first SEQS sequences only (smaller case for profiling)")
    ap.add_argument("--prefill", default="prefix_hit,chunk",
                    help="comma list of prefill workloads to time (prefix_hit, chunk) or none")
    ap.add_argument("--prefill-steps", type=int, default=5)
    ap.add_argument("--no-decode-long", action="store_true",
                    help="skip the secondary decode workloads (32B-shape long context, "
                         "4-sequence small batch)")
    ap.add_argument("--no-chunked", dest="chunked", action="store_false",
                    help="skip the chunked-prefill workload")
    ap.add_argument("--no-model-step", action="store_true",
                    help="skip the full-model (28-layer) decode step workload")
    ap.add_argument("--no-sample", action="store_true",
                    help="skip the token-sampling workload")
    ap.add_argument("--only-sample", action="store_true",
                    help="run only the token-sampling workload (one JSON line)")
    ap.add_argument("--only-kv-store", action="store_true",
                    help="run only the decode step's KV store, back to back (one JSON line)")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="profiling on one GPU: time rank 0's kv-head shard of an N-way split "
                         "(the per-GPU work of an N-GPU run)")
    ap.add_argument("--only-prefill", action="store_true",
                    help="skip the decode workload (for profiling the prefill kernel)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist
    import nvattn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"note: WORLD_SIZE={world} but --gpus={args.gpus}; using WORLD_SIZE")
    assert HKV % world == 0, "kv heads must divide across ranks"
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=120))

    if args.only_prefill:
        res = run_prefills(args, world, rank, device)
        chunked = bench_prefill_chunked(args, world, rank, device) if args.chunked else None
        if rank == 0:
            first = res[0] if res else {}
            print(json.dumps({"metric": METRIC, "value": first.get("tokens_per_s"),
                              "unit": "tokens/s", "n_gpus": world, "prefill": res,
                              "prefill_chunked": chunked}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0

    if args.only_kv_store:
        res = bench_kv_store(args, world, rank, device)
        if rank == 0:
            print(json.dumps({"n_gpus": world, "kv_store": res}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0

    if args.only_sample:
        res = bench_sample(args, world, rank, device)
        if rank == 0:
            print(json.dumps({"n_gpus": world, "sample": res}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0

    ways = world if world > 1 else max(1, args.shard_of)
    assert HKV % ways == 0, "kv heads must divide across the shards"
    hkv, hq = HKV // ways, HQ // ways
    B = args.seqs
    lens, bt_np, num_blocks = workload(n_seqs=B)
    max_ctx = int(lens.max())
    cfg = nvattn.qwen3_config(n_layer=1, n_q_heads=hq, n_kv_heads=hkv, num_blocks=num_blocks,
                              max_seqs=B, max_context=max_ctx, max_position=max_ctx,
                              device=local_rank)
    h = nvattn.Handle(cfg)

    # KV cache shard, generated on the device (N(0,1) -> bf16) in chunks.
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    n_slots = num_blocks * BS
    kc = torch.empty((n_slots, hkv, D), dtype=torch.bfloat16, device=device)
    vc = torch.empty_like(kc)
    chunk = 1 << 16
    for t in (kc, vc):
        for i in range(0, n_slots, chunk):
            t[i:i + chunk].copy_(torch.randn((min(chunk, n_slots - i), hkv, D), generator=gen,
                                             device=device))
    bt = torch.from_numpy(bt_np).to(device)
    cl, pos_np, slot_np = nvattn.plan_decode(lens, bt_np)
    ctx = torch.from_numpy(cl).to(device)
    pos = torch.from_numpy(pos_np).to(device)
    slots = torch.from_numpy(slot_np).to(device)
    q0 = torch.randn((B, hq, D), generator=gen, device=device)
    k_new = torch.randn((B, hkv, D), generator=gen, device=device)
    v_new = torch.randn((B, hkv, D), generator=gen, device=device)
    w = (1 + 0.02 * torch.randn(D, generator=gen, device=device)).to(torch.bfloat16)
    q = torch.empty_like(q0)
    out = torch.empty((B, hq, D), device=device)
    stream = torch.cuda.current_stream(device)
    kc16, vc16, w16 = kc.view(torch.int16), vc.view(torch.int16), w.view(torch.int16)

    # nvattn_paged_decode_step: the new token's q/k RMSNorm + RoPE and K/V
    # row store, then the split-KV decode, reading the step's raw q (q0) --
    # one fused launch, or the store and decode launches for grids past 32
    # CTAs per SM (this workload's full grid and its 2- and 4-way shards; the
    # 8-way shard fuses)
    step_launches = h.decode_step_launches(B, max_ctx)

    def step():
        ev_z.record(stream)
        h.decode_step(0, q0, k_new, v_new, w16, w16, pos, slots, kc16, vc16, bt, ctx, max_ctx,
                      out, stream=stream)
        ev_b.record(stream)

    def two_call_step(z, a, b):
        # the same step as two launches: the KV store writes the normed,
        # rotated q (q) that the decode then reads
        z.record(stream)
        h.kv_store(0, q0, k_new, v_new, w16, w16, pos, slots, q, kc16, vc16, stream=stream)
        a.record(stream)
        h.decode(0, q, kc16, vc16, bt, ctx, max_ctx, out, stream=stream)
        b.record(stream)

    def normed_q():
        # the normed, rotated q of this step (what the decode attends with),
        # for the sharded parity check; the store rewrites the same K/V bits
        two_call_step(*(torch.cuda.Event() for _ in range(3)))
        return q

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(device)

    ev_z = torch.cuda.Event(enable_timing=True)
    ev_b = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local_rank)
    clocks.start()
    for _ in range(max(args.warmup, 3)):
        step()
    h.check_device("warmup")
    barrier()
    mark = clocks.mark()

    # ---- timed region: device-resident inputs ----
    dec_ms = 0.0
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    pairs = []
    t0.record(stream)
    for _ in range(args.steps):
        ev_z = torch.cuda.Event(enable_timing=True)
        ev_b = torch.cuda.Event(enable_timing=True)
        step()
        pairs.append((ev_z, ev_b))
    t1.record(stream)
    barrier()
    clk = clocks.stop(mark)
    elapsed = t0.elapsed_time(t1) / 1e3
    dec_ms = sum(z.elapsed_time(b) for z, b in pairs) / len(pairs)
    h.check_device("timed region")

    # ---- the same step as two launches (KV store, then decode) ----
    # reported beside the headline, timed the same way (events around the
    # whole loop, per-launch events inside it)
    tri = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(23)]
    for z, a, b in tri[:3]:
        two_call_step(z, a, b)
    tc0, tc1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tc0.record(stream)
    for z, a, b in tri[3:]:
        two_call_step(z, a, b)
    tc1.record(stream)
    torch.cuda.synchronize(device)
    two_ms = tc0.elapsed_time(tc1) / len(tri[3:])
    store_ms = sum(z.elapsed_time(a) for z, a, _ in tri[3:]) / len(tri[3:])
    two_dec_ms = sum(a.elapsed_time(b) for _, a, b in tri[3:]) / len(tri[3:])
    h.check_device("two-call step")

    # ---- e2e: the same step through the C ABI with pinned host buffers ----
    # Every step uploads its inputs (q, new k/v, block tables, context
    # lengths, positions, slots) from pinned host memory and reads its output
    # back, as a serving loop does; uploads run on one copy stream and
    # read-backs on another, double-buffered, so step i+1's upload and step
    # i-1's read-back overlap step i's kernels.
    hq0 = q0.cpu().pin_memory()
    hk = k_new.cpu().pin_memory()
    hv = v_new.cpu().pin_memory()
    hbt = bt.cpu().pin_memory()
    hctx = ctx.cpu().pin_memory()
    hpos = pos.cpu().pin_memory()
    hslot = slots.cpu().pin_memory()
    h2d = sum(x.numel() * x.element_size() for x in (hq0, hk, hv, hbt, hctx, hpos, hslot))
    bufs = []
    for _ in range(2):
        bufs.append({
            "q": torch.empty_like(q), "k": torch.empty_like(k_new), "v": torch.empty_like(v_new),
            "bt": torch.empty_like(bt), "ctx": torch.empty_like(ctx), "pos": torch.empty_like(pos),
            "slot": torch.empty_like(slots), "out": torch.empty_like(out),
            "hout": torch.empty((B, hq, D), dtype=torch.float32).pin_memory(),
            "up": torch.cuda.Event(), "done": torch.cuda.Event(), "down": torch.cuda.Event(),
        })
    d2h = bufs[0]["hout"].numel() * bufs[0]["hout"].element_size()
    up_stream = torch.cuda.Stream(device=device)
    down_stream = torch.cuda.Stream(device=device)

    def e2e_step(i):
        bb = bufs[i & 1]
        with torch.cuda.stream(up_stream):
            if i >= 2:
                up_stream.wait_event(bb["done"])  # step i-2's kernels are done with bb
            for name, src in (("q", hq0), ("k", hk), ("v", hv), ("bt", hbt), ("ctx", hctx),
                              ("pos", hpos), ("slot", hslot)):
                bb[name].copy_(src, non_blocking=True)
            bb["up"].record(up_stream)
        stream.wait_event(bb["up"])
        if i >= 2:
            stream.wait_event(bb["down"])  # step i-2's output has been read back
        h.decode_step(0, bb["q"], bb["k"], bb["v"], w16, w16, bb["pos"], bb["slot"], kc16, vc16,
                      bb["bt"], bb["ctx"], max_ctx, bb["out"], stream=stream)
        bb["done"].record(stream)
        with torch.cuda.stream(down_stream):
            down_stream.wait_event(bb["done"])
            bb["hout"].copy_(bb["out"], non_blocking=True)
            bb["down"].record(down_stream)

    def e2e_drain():
        stream.wait_stream(up_stream)
        stream.wait_stream(down_stream)

    for i in range(3):
        e2e_step(i)
    e2e_drain()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up_stream.wait_event(e0)
    down_stream.wait_event(e0)
    for i in range(args.steps):
        e2e_step(i)
    e2e_drain()
    e1.record(stream)
    barrier()
    e2e_elapsed = e0.elapsed_time(e1) / 1e3
    h.check_device("e2e region")
    # the read-back holds the last step's attention output
    assert torch.isfinite(bufs[(args.steps - 1) & 1]["hout"]).all()

    times = torch.tensor([elapsed, e2e_elapsed, dec_ms, two_ms, store_ms, two_dec_ms],
                         dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed, e2e_elapsed, dec_ms, two_ms, store_ms, two_dec_ms = times.tolist()

    # ---- N > 1: the step plus the all-gather of the head-sharded outputs ----
    allgather = None
    if world > 1 and not args.no_allgather:
        allgather = allgather_loop(args, world, rank, local_rank, step, out, stream, B, hq,
                                   lens, bt_np, kc, vc, normed_q)

        def peer_step():
            h.decode_step_gather(0, q0, k_new, v_new, w16, w16, pos, slots, kc16, vc16, bt, ctx,
                                 max_ctx, out, stream=stream)

        allgather["peer_gather"] = peer_gather_loop(args, world, rank, local_rank, h, peer_step,
                                                    stream, B, hq, allgather.pop("_gathered"))

    # CPU baseline (rank 0, one GPU): the oracle's ggml-chain decode on the
    # host cores over the workload's first sequences, with this run's K/V.
    cpu_base = None
    if world == 1 and ways == 1 and rank == 0 and not args.no_cpu_baseline:
        def host_case(n):
            need = (lens[:n] + BS - 1) // BS
            ids = np.concatenate([bt_np[s, :need[s]] for s in range(n)])
            idx = torch.from_numpy(ids.astype(np.int64)).to(device)
            rows = (idx[:, None] * BS + torch.arange(BS, device=device)[None]).reshape(-1)
            kh = kc.index_select(0, rows).view(torch.int16).cpu().numpy().view(np.uint16)
            vh = vc.index_select(0, rows).view(torch.int16).cpu().numpy().view(np.uint16)
            btc = np.full((n, bt_np.shape[1]), -1, np.int32)
            o = 0
            for s in range(n):
                btc[s, :need[s]] = np.arange(o, o + need[s])
                o += int(need[s])
            return (kh[None], vh[None], btc, lens[:n].astype(np.int32),
                    q.cpu().numpy()[:n].copy())
        tps, n, dt, cores = cpu_sample(lens, bt_np, host_case)
        cpu_base = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                    "sample": f"oracle GGML-mode paged decode of the first {n} sequences "
                              f"({dt:.1f} s on {cores} threads)"}

    # release the decode cache before the prefill workloads allocate theirs
    del kc, vc, kc16, vc16
    torch.cuda.empty_cache()
    prefill_results = run_prefills(args, world, rank, device)
    decode_long = None if args.no_decode_long else bench_decode_long(args, world, rank, device)
    decode_small = None if args.no_decode_long else bench_decode_small(args, world, rank, device)
    model_step = (bench_model_step(args, world, rank, device)
                  if world == 1 and not args.no_model_step else None)
    sample = None if args.no_sample else bench_sample(args, world, rank, device)
    prefill_chunked = bench_prefill_chunked(args, world, rank, device) if args.chunked else None

    if rank == 0:
        hbm_peak, _, peak_kind = peaks()
        n_tok = B * args.steps
        kv_bytes = int(lens.sum()) * hkv * D * 2 * 2
        # decode: cache rows read, q read + out written, block-table entries,
        # lengths; the store of the new token: its k and v read (f32), its
        # RoPE row read, its K/V rows written (bf16), position and slot
        dec_bytes = (kv_bytes + B * hq * D * 4 * 2 + int(((lens + BS - 1) // BS).sum()) * 4
                     + B * 4)
        alg_bytes = dec_bytes + B * (2 * hkv * D * 4 + D * 4 + 2 * hkv * D * 2 + 8)
        achieved = alg_bytes / (dec_ms / 1e3) / 1e9
        two_dec_gbs = dec_bytes / (two_dec_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": n_tok / elapsed, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * elapsed / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16 KV, fp32 accumulate",
            "data": "synthetic (seeded N(0,1) Q/K/V, log-uniform context lengths)",
            "config": headline_config(world, ways, B, lens, allgather is not None),
            "roofline": {"bound": "hbm",
                         "kernel": ("paged_decode_step: q/k norm + RoPE and K/V row store, "
                                    "split-KV decode merged in-kernel by the last split "
                                    + ("(one fused launch)" if step_launches == 1 else
                                       "(store launch + decode launch; the step's device "
                                       "time)")),
                         "step_launches": step_launches,
                         "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_source": peak_kind,
                         "traffic": NCU_TRAFFIC_BYTES_N1 if world == 1 else None,
                         "algorithmic_bytes": alg_bytes, "decode_ms": dec_ms,
                         "frac_of_8tbs": achieved / 8000.0},
            "e2e": {"value": n_tok / e2e_elapsed, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            # the kernel launches nvattn_paged_decode_step makes per step (1 or 2)
            "gpu_launches": args.steps * step_launches,
            "clocks": clk,
            "decode_long": decode_long,
            "decode_small": decode_small,
            "model_step": model_step,
            "sample": sample,
            "prefill_chunked": prefill_chunked,
            "kv_store": kv_store_roofline(B, hq, hkv, store_ms, q_out_bytes=4),
            "two_call_step": {"ms_per_step": two_ms, "decode_ms": two_dec_ms,
                              "decode_gbs": two_dec_gbs, "store_ms": store_ms,
                              "note": "the same step as two launches (nvattn_kv_store_qk_"
                                      "norm_rope, then nvattn_paged_decode), device time"},
        }
        for res in prefill_results:
            line["prefill_" + res["kind"]] = res
        if allgather is not None:
            line["allgather"] = allgather
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
        print(json.dumps(line), flush=True)
    h.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
