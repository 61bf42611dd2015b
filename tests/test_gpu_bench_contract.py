"""bench.py's own JSON line on a GPU: one line with every key of the output
contract (metric, value, unit, roofline, e2e, gpu_launches, clocks, ...),
from a short run of the headline decode workload."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_bench_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--steps", "3",
                        "--warmup", "3", "--no-decode-long", "--no-sample", "--no-chunked",
                        "--prefill", "none", "--no-cpu-baseline"],
                       capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "roofline", "e2e", "gpu_launches", "clocks"):
        assert key in d, key
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert "workload" in d["config"]
    roof = d["roofline"]
    for key in ("bound", "achieved", "peak", "unit", "frac", "traffic"):
        assert key in roof, key
    assert roof["bound"] == "hbm" and roof["unit"] == "GB/s"
    assert abs(roof["frac"] - roof["achieved"] / roof["peak"]) < 1e-9
    e2e = d["e2e"]
    assert e2e["value"] > 0 and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] > 0 and e2e["d2h_bytes_per_step"] > 0
    # nvattn_paged_decode_step per step: one fused launch, or the store and
    # decode launches for the full 256-sequence grid; the explicit two calls
    # are timed beside it
    assert d["roofline"]["step_launches"] in (1, 2)
    assert d["gpu_launches"] == d["steps"] * d["roofline"]["step_launches"]
    two = d["two_call_step"]
    assert two["ms_per_step"] > 0 and two["store_ms"] > 0 and two["decode_ms"] > 0
    for key in ("sm_mhz", "sm_max_mhz", "reasons"):
        assert key in d["clocks"], key
