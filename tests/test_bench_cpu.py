"""bench.py's contract, as far as it runs without a GPU.

The reference arm (``--impl reference``) times the CPU restatement of the
reference's fp32 dequantize-then-matmul on the host cores, so it runs here:
its JSON line must carry the keys the driver reads.  Ranks other than 0 print
nothing and exit 0.  The headline metric name must be BASELINE.json's, and
every line carries its provenance (``meta``) without failing when a source of
it is missing.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def _bench(*args: str, env: dict | None = None) -> subprocess.CompletedProcess:
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, str(REPO / "bench.py"), *args], cwd=REPO, env=e,
                          capture_output=True, text=True, timeout=300)


def test_headline_metric_is_the_baseline_metric():
    sys.path.insert(0, str(REPO))
    import bench

    want = json.loads((REPO / "BASELINE.json").read_text())["metric"]
    assert bench.metric_name(4096, 4096, 1) == want


def test_reference_arm_line_on_host_cores():
    r = _bench("--impl", "reference", "--m", "512", "--k", "1024", "--steps", "2", "--warmup", "3",
               "--no-reference-cuda")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["config"]["workload"] == "512x1024 W4A16 GEMV B=1"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    meta = d["meta"]
    assert meta["torch"] and meta["host_threads"] >= 1 and meta["timestamp"].endswith("Z")


def test_reference_arm_other_ranks_exit_quietly():
    r = _bench("--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3",
               "--no-reference-cuda", env={"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def test_run_meta_never_raises_without_a_gpu():
    sys.path.insert(0, str(REPO))
    import bench

    for gpu in (None, 0):
        meta = bench.run_meta(gpu)
        json.dumps(meta)
        assert set(meta) >= {"timestamp", "host_threads", "torch", "cuda", "gpu", "driver", "git"}
