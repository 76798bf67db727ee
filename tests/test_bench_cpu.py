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
    # The same workload dict this library's arm reports (bench.workload_config).
    sys.path.insert(0, str(REPO))
    import bench

    assert d["config"] == bench.workload_config(512, 1024, 1, 64, 1)
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


def test_kernel_path_follows_the_dispatch():
    sys.path.insert(0, str(REPO))
    import bench

    assert bench.kernel_path(4096, 4096, 1).startswith("k_stream (v5, 1 n-tile")
    assert bench.kernel_path(4096, 4096, 16).startswith("k_stream (v5, 2 n-tiles")
    assert bench.kernel_path(4096, 4096, 32).startswith("k_stream (v5, 4 n-tiles")
    assert bench.kernel_path(28672, 8192, 32) == "k_batch (tcgen05)"


def test_fp16_reference_bytes_are_the_references():
    # The cross-precision cuBLAS points count fp16 W + x + y, as the
    # reference's bytes_moved_fp16 does; the W4 metric counts packed W and
    # scales instead.
    sys.path.insert(0, str(REPO))
    import bench

    assert bench.fp16_bytes(4096, 4096, 1) == 4096 * 4096 * 2 + 4096 * 2 + 4096 * 2
    assert bench.fp16_bytes(11008, 4096, 8) == 11008 * 4096 * 2 + 8 * 4096 * 2 + 8 * 11008 * 2
    assert (4096, 4096, 1) in bench.FP16_SHAPES  # (M, K, B)


def test_run_meta_never_raises_without_a_gpu():
    sys.path.insert(0, str(REPO))
    import bench

    for gpu in (None, 0):
        meta = bench.run_meta(gpu)
        json.dumps(meta)
        assert set(meta) >= {"timestamp", "host_threads", "torch", "cuda", "gpu", "driver", "git"}


def test_marlin_peer_without_a_gpu_prints_unavailable():
    r = _bench("--impl", "marlin", "--steps", "1", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(ln) for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert lines == [{"impl": "marlin (vLLM)", "unavailable": "no CUDA device"}]


_MARLIN_HOST_CHECK = """
import sys
import torch
try:
    from vllm.model_executor.layers.quantization.utils.marlin_utils import (
        apply_gptq_marlin_linear, marlin_make_empty_g_idx, marlin_make_workspace_new,
        marlin_permute_scales)
    from vllm.scalar_type import scalar_types
except Exception as e:
    print("SKIP", type(e).__name__, e)
    sys.exit(0)
from decode_kernel.gptq import to_gptq
from decode_kernel.quantize import quantize_and_pack

M, K = 256, 512
packed, scales = quantize_and_pack(torch.randn(M, K) * 0.02)
g = to_gptq(packed, scales)
s = marlin_permute_scales(g.scales, size_k=K, size_n=M, group_size=128)
assert tuple(s.shape) == (K // 128, M) and s.dtype == torch.float16
assert torch.equal(s.flatten().sort().values, g.scales.flatten().sort().values)
assert scalar_types.uint4b8.size_bits == 4
print("OK")
"""


def test_marlin_peer_host_steps_accept_the_gptq_tensors():
    # The host-side half of the peer's weight loading, on the CPU and in a
    # child process (importing vLLM changes process-wide state): the names
    # bench.py imports from vLLM exist, and vLLM's scale permutation takes the
    # scales that to_gptq produces (a permutation of the same values).  The
    # repack and the GEMM are GPU ops.
    import pytest

    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(REPO / "decode-kernel_b200"), str(REPO),
                                         env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", _MARLIN_HOST_CHECK], cwd=REPO, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = r.stdout.strip().splitlines()[-1]
    if out.startswith("SKIP"):
        pytest.skip(out)
    assert out == "OK"
