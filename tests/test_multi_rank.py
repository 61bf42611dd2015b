"""World-size-2 tests of the KV-head-sharded path on CPU (gloo).

Each rank keeps the cache shard of its kv heads (same layout, fewer heads),
computes its q heads, and the optional all-gather reassembles the full head
dimension.  The per-rank compute here is the oracle standing in for the
device kernel; what is under test is the host logic: shard ranges, cache /
query slicing and the reassembly.  A rank that fails before the collective
is detected by the survivor through the process group's timeout, on the
host, without any GPU involvement.
"""
import multiprocessing as mp
import os
import socket
import traceback
from datetime import timedelta

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    try:
        import sys
        here = os.path.dirname(os.path.abspath(__file__))
        root = os.path.dirname(here)
        for p in (os.path.join(root, "oracle"), os.path.join(root, "nano-vllm.cpp_b200", "python"),
                  here):
            sys.path.insert(0, p)
        import torch
        import torch.distributed as dist

        import cases
        import nvattn
        import oracle as O
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=5 if mode == "fail" else 60))
        Hq, Hkv = 32, 8
        c = cases.decode_case(90, Hq, Hkv, [700, 33, 1500])
        kv0, kv1, q0, q1 = nvattn.kv_head_shard(Hq, Hkv, world, rank)
        kc = np.ascontiguousarray(c.cache.k[:, :, kv0:kv1])
        vc = np.ascontiguousarray(c.cache.v[:, :, kv0:kv1])
        qs = np.ascontiguousarray(c.q[:, q0:q1])
        p = O.params(n_q_heads=q1 - q0, n_kv_heads=kv1 - kv0, n_slots=c.cache.n_slots,
                     n_threads=2)
        mine = O.paged_decode(p, O.MODE_TRUTH, 0, qs, kc, vc, c.block_tables, c.lens)
        if mode == "fail" and rank == 1:
            raise SystemExit(0)  # leaves before the collective, between steps
        out = [torch.empty_like(torch.from_numpy(mine)) for _ in range(world)]
        dist.all_gather(out, torch.from_numpy(mine))
        full = nvattn.gather_heads([t.numpy() for t in out])
        pf = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=c.cache.n_slots, n_threads=2)
        ref = O.paged_decode(pf, O.MODE_TRUTH, 0, c.q, c.cache.k, c.cache.v, c.block_tables,
                             c.lens)
        q.put((rank, "ok", bool(np.array_equal(full, ref))))
        dist.destroy_process_group()
    except SystemExit:
        q.put((rank, "exited", None))
    except Exception as e:  # reported to the parent
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()[-400:]}"))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, status, val = q.get(timeout=120)
        res[r] = (status, val)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return res


def test_shard_ranges():
    import nvattn
    assert nvattn.kv_head_shard(32, 8, 2, 1) == (4, 8, 16, 32)
    assert nvattn.kv_head_shard(64, 8, 8, 3) == (3, 4, 24, 32)
    assert nvattn.kv_head_shard(16, 8, 1, 0) == (0, 8, 0, 16)
    with pytest.raises(ValueError):
        nvattn.kv_head_shard(32, 8, 3, 0)


def test_two_rank_kv_head_sharding_reassembles_exactly():
    res = _run("ok")
    assert res[0] == ("ok", True), res
    assert res[1] == ("ok", True), res


def test_rank_failure_is_detected_by_the_survivor():
    res = _run("fail")
    assert res[1][0] == "exited"
    assert res[0][0] == "error", res  # the collective ends with an error, no hang


def test_bench_reassembles_sharded_cache_rows_and_queries():
    """bench.py's sharded parity check rebuilds every head from the ranks'
    pieces; on a sharded copy of a case that must give the original cache
    rows and queries back, and the oracle over them the unsharded output."""
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import bench
    import cases
    import nvattn
    import oracle as O
    Hq, Hkv, world = 32, 8, 4
    c = cases.decode_case(91, Hq, Hkv, [300, 900])
    need = (c.lens + 255) // 256
    ids = np.concatenate([c.block_tables[s, :need[s]] for s in range(2)])
    rows = (ids[:, None] * 256 + np.arange(256)[None]).reshape(-1)
    kv_ranks, q_ranks = [], []
    for r in range(world):
        kv0, kv1, q0, q1 = nvattn.kv_head_shard(Hq, Hkv, world, r)
        kv_ranks.append(np.concatenate([c.cache.k[0, rows, kv0:kv1], c.cache.v[0, rows, kv0:kv1]]))
        q_ranks.append(c.q[:, q0:q1])
    k_full, v_full, q_full, btc = bench.reassemble_shards(np.stack(kv_ranks), np.stack(q_ranks),
                                                          need)
    assert np.array_equal(k_full[0], c.cache.k[0, rows])
    assert np.array_equal(v_full[0], c.cache.v[0, rows])
    assert np.array_equal(q_full, c.q)
    p = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=k_full.shape[1], n_threads=2)
    got = O.paged_decode(p, O.MODE_TRUTH, 0, q_full, k_full, v_full, btc, c.lens)
    pf = O.params(n_q_heads=Hq, n_kv_heads=Hkv, n_slots=c.cache.n_slots, n_threads=2)
    want = O.paged_decode(pf, O.MODE_TRUTH, 0, c.q, c.cache.k, c.cache.v, c.block_tables, c.lens)
    assert np.array_equal(got, want)
