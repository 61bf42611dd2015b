"""The decode step with the all-gather fused over peer memory
(nvattn_paged_decode_step_gather), on two GPUs: bench.py under torchrun runs
the NCCL all-gather loop and then the peer-memory loop on the same step, and
the peer-gathered rows must equal NCCL's bit for bit (skipped on one GPU)."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_peer_gather_equals_nccl_all_gather():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29517", os.path.join(ROOT, "bench.py"), "--gpus", "2", "--seqs", "64",
           "--steps", "5", "--warmup", "3", "--prefill", "none", "--no-chunked", "--no-sample",
           "--no-decode-long", "--no-cpu-baseline", "--no-model-step"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=700, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")][-1]
    d = json.loads(line)
    ag = d["allgather"]
    assert ag["sharded_parity"]["ok"]
    pg = ag["peer_gather"]
    assert "error" not in pg, pg["error"]
    assert pg["identical_to_nccl_gather"] is True
    assert pg["ms_per_step"] > 0
