#!/usr/bin/env python
"""bench.py -- W4A16 decode GEMV throughput on B200 (the BASELINE metric).

Metric: achieved HBM read GB/s (and % of the measured B200 read roof) and
µs per GEMV, 4096x4096, batch 1.

A *step* is one decode-style pass over a stack of ``sets`` distinct
4096x4096 int4 weight matrices (64 by default, 555 MB in total, > 4x the
126 MB L2), one batch-1 GEMV per matrix.  Every byte of every matrix is read
from HBM once per step -- no L2 flush is needed because no matrix is touched
again until 63 others have streamed through L2.

value   device-resident throughput: the step is captured once in a CUDA
        graph (GEMVs launched through the C ABI with programmatic dependent
        launch, so each kernel's weight stream overlaps its predecessor's
        tail) and replayed K times between CUDA events.
e2e     the same metric through the public Python API (decode_kernel.gemv_out,
        the reference's operator surface writing into a preallocated output),
        one call per GEMV, captured once with torch.cuda.graph and replayed:
        per step, the step's activations come from pinned host memory and the
        outputs go back to the host.  e2e.eager is the same with the calls
        launched eagerly from Python (host-bound: ~7 µs per call).
cpu_baseline / --impl reference
        the reference's CPU path (fp32 dequantize-then-matmul,
        python/decode_kernel/reference.py:17-26) restated in numpy
        (oracle/oracle.py: linear_fp32_np), timed on the host cores.

baseline_configs (one GPU)
        the other BASELINE configurations under the same two protocols
        (chain and isolated): the Llama-7B MLP shapes 11008x4096 and
        4096x11008, the 70B-shaped 28672x8192 and 8192x28672 at B = 1 and 8,
        and the 4096^2 batch sweep B in {1, 2, 4, 8, 16, 32}; each with µs,
        GB/s, the fraction of the measured roof and an oracle spot check.
strong_scaling
        the 70B-shaped decoder layers' projections (8 layers, B = 1) in the
        tensor-parallel layout over every rank of the run -- the same command
        at N = 1 -- with the fused NVLink exchange; rank 0 checks layer 0
        against the unsharded layer before timing.

Multi-GPU (torchrun, one rank per GPU): for ``value`` each rank streams its
own weight stack (weak scaling, no data-path collective); time = max over
ranks.  ``strong_scaling`` shards one model over the ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (str(REPO), str(REPO / "decode-kernel_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

def metric_name(m: int, k: int, b: int) -> str:
    return ("achieved HBM read GB/s (% of measured B200 read roof) and µs/GEMV, "
            f"{m}x{k} B={b}")
L2_BYTES = 126 * 1024 * 1024


def gemv_bytes(m: int, k: int, b: int) -> int:
    """Algorithmic bytes of one GEMV: packed W + scales + x + y
    (bench/common.py:111-117 of the reference)."""
    return m * (k // 2) + m * (k // 128) * 2 + b * k * 2 + b * m * 2


def workload_config(m: int, k: int, b: int, sets: int, ws: int) -> dict:
    """The workload, as both arms report it under ``config`` -- the same dict
    from this library's arm and from the reference arm, so the two lines say
    that they measured the same thing.  How each arm runs it goes under
    ``arm``."""
    per = gemv_bytes(m, k, b)
    return {"workload": f"{m}x{k} W4A16 GEMV B={b}", "M": m, "K": k, "global_batch": b * ws,
            "gemvs_per_step": sets,
            "l2": f"inputs larger than L2: {sets} distinct weight sets "
                  f"({sets * per / 2**20:.0f} MiB) cycled, no flush",
            "parallelism": f"x{ws}: independent weight stacks per GPU (weak scaling), "
                           f"no collective"}


# --------------------------------------------------------------------------
# helpers
# --------------------------------------------------------------------------

def dist_info():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def ncu_traffic_per_launch(m: int, k: int, b: int):
    """dram read+write bytes per launch of the dominant kernel, from the
    committed ncu summary of this workload (profiles/), or None."""
    p = REPO / "profiles" / f"k_stream_{m}x{k}_b{b}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except Exception:
                return None
    return None


def run_meta(gpu_index=None) -> dict:
    """Provenance of a result line, as the reference's bench JSON records it
    (bench/common.py:18-52): GPU, driver, torch and CUDA versions, source
    revision, host threads, UTC time.  Best effort: a field whose source is
    missing (no GPU, no nvidia-smi, no git checkout) is None, and nothing
    here raises."""
    meta = {"timestamp": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
            "host_threads": os.cpu_count(), "torch": None, "cuda": None, "gpu": None,
            "driver": None, "git": None}
    try:
        import torch

        meta["torch"], meta["cuda"] = torch.__version__, torch.version.cuda
        if gpu_index is not None and torch.cuda.is_available():
            prop = torch.cuda.get_device_properties(gpu_index)
            meta["gpu"] = {"name": prop.name, "sm_count": prop.multi_processor_count,
                           "cc": f"{prop.major}.{prop.minor}",
                           "memory_gib": round(prop.total_memory / 2**30, 1)}
    except Exception:
        pass
    for key, cmd in (("driver", ["nvidia-smi", "--query-gpu=driver_version",
                                 "--format=csv,noheader"]),
                     ("git", ["git", "rev-parse", "--short", "HEAD"])):
        try:
            out = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=10)
            text = out.stdout.strip()
            if out.returncode == 0 and text:
                meta[key] = text.splitlines()[0].strip()
        except Exception:
            pass
    return meta


class ClockSampler:
    """nvidia-smi samples during the timed region (recipe's clocks line)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = None

    def __enter__(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.tmp, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.tmp is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.tmp.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((float(parts[1]), float(parts[2]), parts[3], parts[4:]))
                except ValueError:
                    continue
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        reasons = set()
        for r in rows:
            for name, val in zip(names[1:], r[3][1:]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(rows),
                "reasons": sorted(reasons)}


def read_roof_gbs(torch, capi, nbytes=512 << 20, iters=20) -> float:
    """This library's sm_100a stream_read over 512 MiB: the read-only HBM
    roof the BASELINE metric is quoted against (median of ``iters``)."""
    src = torch.ones(nbytes // 4, dtype=torch.float32, device="cuda")
    blocks = capi.load().dk_stream_recommended_blocks(-1)
    part = torch.empty(blocks, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for i in range(iters + 3):
        e0.record()
        capi.check(capi.load().dk_stream_read(src.data_ptr(), part.data_ptr(), nbytes, blocks,
                                              stream), "dk_stream_read")
        e1.record()
        torch.cuda.synchronize()
        if i >= 3:
            ts.append(e0.elapsed_time(e1) / 1e3)
    del src, part
    return nbytes / statistics.median(ts) / 1e9


# --------------------------------------------------------------------------
# CPU reference path (oracle port) -- reference arm and cpu_baseline
# --------------------------------------------------------------------------

def cpu_problem(M, K, B, seed=0):
    import numpy as np

    from oracle import oracle as O

    rng = np.random.default_rng(seed)
    w = rng.standard_normal((M, K), dtype=np.float32) * np.float32(0.02)
    x = rng.standard_normal((B, K), dtype=np.float32).astype(np.float16)
    packed, scales = O.quantize_and_pack_np(w)
    return packed, scales, x


def time_cpu_reference(M, K, B, budget_s, seed=0):
    """Times the restated reference CPU path on row samples; returns
    (GB/s, seconds per sample, rows per sample, samples)."""
    from oracle import oracle as O

    packed, scales, x = cpu_problem(M, K, B, seed)
    t0 = time.perf_counter()
    O.linear_fp32_np(x, packed, scales)
    t_full = time.perf_counter() - t0
    n = max(3, min(200, int(budget_s / max(t_full, 1e-3))))
    ts = []
    for _ in range(n):
        t0 = time.perf_counter()
        O.linear_fp32_np(x, packed, scales)
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    return gemv_bytes(M, K, B) / t / 1e9, t, M, n


FLUSH_BYTES = 512 << 20  # the L2 flush of the BASELINE protocol


def time_isolated(torch, call, iters=200, warmup=20) -> float:
    """The reference's own timing protocol (bench/common.py:64-108 of the
    reference, with BASELINE's 512 MiB flush): fill a 512 MiB buffer, record
    an event, make one call, record an event, synchronize; median µs."""
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for i in range(warmup + iters):
        flush.fill_(1.0)
        e0.record()
        call()
        e1.record()
        torch.cuda.synchronize()
        if i >= warmup:
            ts.append(e0.elapsed_time(e1) * 1e3)
    del flush
    return statistics.median(ts)


def time_reference_cuda(M, K, B, sets=64, chain_steps=20):
    """The reference's own CUDA kernels on this GPU: csrc/gemv_w4a16.cu of the
    reference, compiled unmodified for sm_100a (oracle/_ref, built from the
    checkout by oracle/Makefile), called through its host entry point
    w4a16_gemv (gemv_w4a16.cu:568-591: stamp reset copy + launch).  Its best
    kernel (v1), its default (v5) and, for B > 1, its weight-reuse batch path,
    each (a) isolated under the reference's
    protocol and (b) over the same 64-matrix chain as this library's
    ``value``, launched back to back.  None when there is no GPU or the
    reference was not built."""
    import torch

    from oracle import ref_cuda

    if not torch.cuda.is_available() or not ref_cuda.available():
        return None
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    # Timing inputs only: random packed words and small positive scales.
    packed = [torch.randint(-2**31, 2**31 - 1, (M, K // 8), generator=g, device=dev,
                            dtype=torch.int32) for _ in range(sets)]
    scales = [(torch.rand(M, K // 128, generator=g, device=dev) * 0.01).half()
              for _ in range(sets)]
    x = torch.randn(B, K, generator=g, device=dev).half()
    y = torch.empty(B, M, dtype=torch.float16, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = {"build": "reference csrc/gemv_w4a16.cu, unmodified, nvcc -O3 --use_fast_math "
                    "for sm_100a (its setup.py flags)",
           "per_gemv_bytes": gemv_bytes(M, K, B)}
    kernels = [("v1", 1, False), ("v5", 5, False)]
    if B > 1:
        kernels.append(("reuse", 5, True))  # its batch path (gemv_w4a16.cu:364-413)
    for name, ver, reuse in kernels:
        iso = time_isolated(torch, lambda: ref_cuda.gemv(packed[0], scales[0], x, y, version=ver,
                                                         reuse_weights=reuse))
        for _ in range(3):
            for s in range(sets):
                ref_cuda.gemv(packed[s], scales[s], x, y, version=ver, reuse_weights=reuse)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(chain_steps):
            for s in range(sets):
                ref_cuda.gemv(packed[s], scales[s], x, y, version=ver, reuse_weights=reuse)
        e1.record()
        torch.cuda.synchronize()
        chain = e0.elapsed_time(e1) * 1e3 / (chain_steps * sets)
        out[name] = {"isolated_us": iso, "isolated_GBps": gemv_bytes(M, K, B) / iso / 1e3,
                     "chain_us_per_gemv": chain, "chain_GBps": gemv_bytes(M, K, B) / chain / 1e3}
    del packed, scales
    torch.cuda.empty_cache()
    return out


def run_reference(args) -> None:
    ws, rank, _ = dist_info()
    if rank != 0:
        return
    import numpy as np

    from oracle import oracle as O

    M, K, B = args.m, args.k, args.batch
    packed, scales, x = cpu_problem(M, K, B)
    # Size each step's row sample so warm-up + K steps take about 90 s.
    t0 = time.perf_counter()
    O.linear_fp32_np(x, packed, scales)
    t_full = time.perf_counter() - t0
    budget = 90.0 / max(1, args.steps + args.warmup)
    rows = int(min(M, max(64, (M * budget / t_full) // 64 * 64)))
    p_s, s_s = np.ascontiguousarray(packed[:rows]), np.ascontiguousarray(scales[:rows])
    for _ in range(args.warmup):
        O.linear_fp32_np(x, p_s, s_s)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.linear_fp32_np(x, p_s, s_s)
    dt = time.perf_counter() - t0
    gbs = args.steps * gemv_bytes(rows, K, B) / dt / 1e9
    cores = O.cpu_threads()
    line = {
        "impl": "reference",
        "metric": metric_name(M, K, B),
        "value": gbs,
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(M, K, B, args.sets, ws),
        "arm": {"runs_on": f"host cores of rank 0 ({cores} threads); other ranks exit",
                "step": f"a bounded sample of the workload: rows [0, {rows}) of one {M}x{K} "
                        f"matrix per step"},
        "cpu_baseline": {
            "value": gbs, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"each step: rows [0, {rows}) of the {M}x{K} matrix, x [{B},{K}]; "
                      f"fp32 dequantize then fp32 BLAS matmul (numpy restatement of "
                      f"reference.py:17-26), {cores} BLAS threads"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_reference_cuda:
        rc = time_reference_cuda(M, K, B)
        if rc is not None:
            line["reference_cuda_same_gpu"] = rc
    line["meta"] = run_meta(None)
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# Same-precision peer: Marlin (as vLLM ships it) on the same GPU
# --------------------------------------------------------------------------

def run_marlin_peer(args) -> None:
    """Marlin's W4A16 GEMM, the same-precision peer the reference never ran,
    on this GPU and on the workload of ``value``.

    This library's weights become GPTQ tensors (``decode_kernel.gptq.to_gptq``,
    exact), then go through vLLM's own loading steps for a symmetric uint4b8
    checkpoint without act-order (vllm/model_executor/kernels/linear/
    mixed_precision/marlin.py: ``gptq_marlin_repack``, ``marlin_permute_scales``,
    empty g_idx and zero points, ``marlin_make_workspace_new``), and run with
    vLLM's ``apply_gptq_marlin_linear``.  One full output is checked against
    the CPU oracle (max abs < 1e-2) before anything is timed.  Timed like
    ``value`` (S distinct matrices per step, a CUDA graph of one step when it
    captures, else eager launches) and like ``isolated``.  Rank 0 only.
    Prints one JSON line with "impl": "marlin (vLLM ...)", or an
    "unavailable" line when there is no GPU or vLLM lacks its Marlin ops."""
    ws, rank, local = dist_info()
    if rank != 0:
        return
    import torch

    name = "marlin (vLLM)"
    if not torch.cuda.is_available():
        print(json.dumps({"impl": name, "unavailable": "no CUDA device"}), flush=True)
        return
    try:
        import vllm
        from vllm import _custom_ops as ops
        from vllm.model_executor.layers.quantization.utils.marlin_utils import (
            apply_gptq_marlin_linear, marlin_make_empty_g_idx, marlin_make_workspace_new,
            marlin_permute_scales)
        from vllm.scalar_type import scalar_types

        if not hasattr(torch.ops._C, "marlin_gemm"):
            raise ImportError("this vLLM build has no marlin_gemm")
        name = f"marlin (vLLM {vllm.__version__})"
    except Exception as e:  # noqa: BLE001 -- any import failure means no peer
        print(json.dumps({"impl": name, "unavailable": f"{type(e).__name__}: {e}"[:300]}),
              flush=True)
        return
    import numpy as np

    from decode_kernel.gptq import to_gptq
    from decode_kernel.quantize import quantize_and_pack_cuda
    from oracle import oracle as O

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    M, K, B, S = args.m, args.k, args.batch, args.sets
    per_gemv = gemv_bytes(M, K, B)
    empty = marlin_make_empty_g_idx(dev)
    workspace = marlin_make_workspace_new(dev)
    mats, xs, first = [], [], None
    for s in range(S):
        g = torch.Generator(device=dev).manual_seed(s)
        w = torch.randn(M, K, generator=g, device=dev) * 0.02
        p, sc = quantize_and_pack_cuda(w)
        del w
        if first is None:
            first = (p.cpu().numpy(), sc.cpu().view(torch.int16).numpy().view(np.uint16))
        t = to_gptq(p, sc)
        try:
            wq = ops.gptq_marlin_repack(t.qweight, perm=empty, size_k=K, size_n=M, num_bits=4)
        except RuntimeError as e:  # e.g. no kernel image for this GPU
            print(json.dumps({"impl": name, "unavailable": f"gptq_marlin_repack: {e}"[:300]}),
                  flush=True)
            return
        wsc = marlin_permute_scales(t.scales, size_k=K, size_n=M, group_size=128)
        mats.append((wq, wsc))
        xs.append(torch.randn(B, K, generator=g, device=dev).half())
        del p, sc, t
    torch.cuda.synchronize()

    def call(s):
        return apply_gptq_marlin_linear(
            input=xs[s], weight=mats[s][0], weight_scale=mats[s][1], weight_zp=empty,
            g_idx=empty, g_idx_sort_indices=empty, workspace=workspace,
            wtype=scalar_types.uint4b8, output_size_per_partition=M,
            input_size_per_partition=K, is_k_full=True)

    # Parity before timing: the whole first output against the CPU oracle.
    try:
        y0 = call(0)
        torch.cuda.synchronize()
    except RuntimeError as e:  # e.g. no Marlin kernel image for this GPU
        print(json.dumps({"impl": name, "unavailable": f"marlin_gemm: {e}"[:300]}), flush=True)
        return
    ref = O.linear_fp32(xs[0].cpu().view(torch.int16).numpy().view(np.uint16), *first)
    err = float(np.abs(y0.float().cpu().numpy() - ref).max())
    line = {"impl": name, "metric": metric_name(M, K, B), "unit": "GB/s", "n_gpus": 1,
            "higher_is_better": True, "dtype": "int4*f16 (uint4b8, group 128)",
            "data": "synthetic", "parity_max_abs_err": err,
            "config": {"workload": f"{M}x{K} W4A16 GEMV B={B}", "M": M, "K": K,
                       "global_batch": B, "gemvs_per_step": S}}
    if not err < 1e-2:
        line.update(value=None, error="Marlin output differs from the oracle by more than 1e-2")
        print(json.dumps(line), flush=True)
        return

    def step():
        for s in range(S):
            call(s)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    graph, launch = None, "CUDA graph of one step, replayed"
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001 -- capture refused: time eager launches
        graph, launch = None, f"eager launches (graph capture failed: {type(e).__name__})"
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record()
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    us = ms * 1e3 / (args.steps * S)
    iso = time_isolated(torch, lambda: call(0))
    del graph
    line.update(value=per_gemv / (us * 1e-6) / 1e9, steps=args.steps, warmup=args.warmup,
                ms_per_step=ms / args.steps, us_per_gemv=us, clocks=clocks.summary(),
                isolated={"us_per_gemv": iso, "GBps": per_gemv / (iso * 1e-6) / 1e9,
                          "protocol": "512 MiB fill flush, CUDA events around one call, "
                                      "median of 200 after 20 warm-up"})
    line["config"]["launch"] = launch
    line["meta"] = run_meta(local)
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# GPU path
# --------------------------------------------------------------------------

def kernel_path(m: int, k: int, b: int) -> str:
    """Which kernel dk_w4a16_gemv's default dispatch (version 5) runs for a
    pass of ``b`` <= 32 rows (the host dispatch in dk_gemv.cu)."""
    if b <= 8:
        return "k_stream (v5, 1 n-tile)"
    if b > 16 and m >= 16384 and k % 128 == 0:
        return "k_batch (tcgen05)"
    return f"k_stream (v5, {2 if b <= 16 else 4} n-tiles)"


def make_stack(torch, quantize, dev, m: int, k: int, b: int, sets: int, seed0: int):
    """``sets`` distinct seeded W ~ N(0, 0.02) [m, k], quantized on the GPU
    (bit-exact with the CPU quantizer), each with its own x ~ N(0, 1) [b, k]
    and output [b, m]."""
    packed, scales, xs, ys = [], [], [], []
    for s in range(sets):
        g = torch.Generator(device=dev).manual_seed(seed0 + s)
        w = torch.randn(m, k, generator=g, device=dev) * 0.02
        p, sc = quantize(w)
        del w
        packed.append(p)
        scales.append(sc)
        xs.append(torch.randn(b, k, generator=g, device=dev).half())
        ys.append(torch.empty(b, m, dtype=torch.float16, device=dev))
    torch.cuda.synchronize()
    return packed, scales, xs, ys


def time_chain_us(torch, capi, packed, scales, xs, ys, m, k, b, cfg, steps: int) -> float:
    """µs per GEMV over ``steps`` replays of a CUDA graph that runs one C-ABI
    GEMV per weight set, back to back (PDL when ``cfg`` asks for it) -- the
    protocol of ``value``."""
    nsets = len(packed)

    def step(stream):
        for i in range(nsets):
            st = capi.gemv(packed[i].data_ptr(), scales[i].data_ptr(), xs[i].data_ptr(),
                           ys[i].data_ptr(), m, k, b, cfg, 0, 0, stream)
            if st:
                capi.check(st, "dk_w4a16_gemv")

    for _ in range(3):
        step(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) * 1e3 / (steps * nsets)


def spot_check(torch, packed, scales, x, y, rows: int = 64) -> float:
    """Max abs error of the first ``rows`` outputs against the CPU oracle
    (outside every timed region)."""
    import numpy as np

    from oracle import oracle as O

    pk = packed[:rows].cpu().numpy()
    sc = scales[:rows].cpu().view(torch.int16).numpy().view(np.uint16)
    xx = x.cpu().view(torch.int16).numpy().view(np.uint16)
    ref = O.linear_fp32(xx, pk, sc)
    return float(np.abs(y[:, :rows].float().cpu().numpy() - ref).max())


# The other BASELINE configurations, each timed under the headline's two
# protocols: the Llama-7B MLP shapes (config 2), the 70B-shaped layers on one
# GPU at B = 1 and 8 (config 5's per-GPU shapes) and the 4096^2 batch sweep
# (config 3).
SWEEP_SHAPES = [(11008, 4096, 1), (4096, 11008, 1), (28672, 8192, 1), (8192, 28672, 1),
                (28672, 8192, 8), (8192, 28672, 8)]
SWEEP_BATCHES = [1, 2, 4, 8, 16, 32]


# The reference's cross-precision reference points (bench/bench.py:106-155 of
# the reference): an fp16 weight matrix through cuBLAS -- torch.mv at B = 1
# (a GEMV), torch.mm above -- and through F.linear.  Not a peer (4x the weight
# bytes): it shows where a dense fp16 GEMV sits on this GPU.
FP16_SHAPES = [(4096, 4096, 1), (4096, 4096, 8), (4096, 4096, 32), (11008, 4096, 1),
               (4096, 11008, 1)]


def fp16_bytes(m: int, k: int, b: int) -> int:
    """Bytes an fp16 GEMV moves: W + x + y (bench/common.py:120-121 of the
    reference)."""
    return m * k * 2 + b * k * 2 + b * m * 2


def run_fp16_reference(args, torch, dev, peak: float) -> dict:
    """µs per call of cuBLAS fp16 (torch.mv / torch.mm) and F.linear over a
    chain of distinct fp16 weights (> 3x L2, CUDA graph, back to back) and
    isolated (512 MiB flush, one call), per FP16_SHAPES entry.  A failure
    here is reported in the key and does not end the run."""
    import torch.nn.functional as F

    steps = max(20, min(args.steps, 500))
    out = []
    try:
        for m, k, b in FP16_SHAPES:
            per = fp16_bytes(m, k, b)
            nsets = max(4, -(-3 * L2_BYTES // per))
            g = torch.Generator(device=dev).manual_seed(40000 + m + k + b)
            ws = [(torch.randn(m, k, generator=g, device=dev) * 0.02).half()
                  for _ in range(nsets)]
            xs = [torch.randn(b, k, generator=g, device=dev).half() for _ in range(nsets)]
            row = {"M": m, "K": k, "B": b, "sets": nsets, "bytes": per}
            impls = {
                ("cublas_fp16_gemv" if b == 1 else "cublas_fp16_gemm"):
                    (lambda w, x: torch.mv(w, x[0])) if b == 1 else
                    (lambda w, x: torch.mm(x, w.t())),
                "pytorch_linear_fp16": lambda w, x: F.linear(x, w),
            }
            for name, fn in impls.items():
                def step():
                    for w, x in zip(ws, xs):
                        fn(w, x)

                step()
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    step()
                for _ in range(3):
                    graph.replay()
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(steps):
                    graph.replay()
                e1.record()
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (steps * nsets)
                del graph
                iso = time_isolated(torch, lambda: fn(ws[0], xs[0]), iters=100, warmup=10)
                row[name] = {"us": us, "GBps": per / us / 1e3, "frac": per / us / 1e3 / peak,
                             "isolated_us": iso}
            out.append(row)
            del ws, xs
            torch.cuda.empty_cache()
    except Exception as e:  # a reference point only: keep the run's line
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        return {"error": f"{type(e).__name__}: {e}"[:300], "shapes": out}
    return {"protocol": f"fp16 weights (not W4): chain of {steps} replays of a CUDA graph of one "
                        f"call per distinct weight (> 3x L2); isolated: 512 MiB fill flush, one "
                        f"call, median of 100; bytes = fp16 W + x + y",
            "shapes": out}


def run_sweeps(args, torch, capi, quantize, dev, packed, scales, peak: float) -> dict:
    """Per-shape and per-batch lines for the BASELINE configs besides the
    headline: µs per GEMV in the chain (``value``'s protocol) and isolated
    (the reference's), GB/s and the fraction of the measured roof; each
    checked against the CPU oracle on its first 64 rows before timing."""
    cfg = capi.default_config(flags=0 if args.no_pdl else capi.DK_FLAG_PDL)
    plain = capi.default_config()
    steps = max(args.steps, 20)

    def entry(m, k, b, pk, sc, xs, ys):
        err = spot_check(torch, pk[0], sc[0], xs[0], ys[0])
        assert err < 1e-2, f"sweep spot check {m}x{k} B={b}: {err}"
        us = time_chain_us(torch, capi, pk, sc, xs, ys, m, k, b, cfg, steps)
        st = torch.cuda.current_stream().cuda_stream
        iso = time_isolated(torch, lambda: capi.check(
            capi.gemv(pk[0].data_ptr(), sc[0].data_ptr(), xs[0].data_ptr(), ys[0].data_ptr(),
                      m, k, b, plain, 0, 0, st), "dk_w4a16_gemv"), iters=100, warmup=10)
        nbytes = gemv_bytes(m, k, b)
        return {"M": m, "K": k, "B": b, "kernel": kernel_path(m, k, b), "sets": len(pk),
                "us_per_gemv": us, "GBps": nbytes / us / 1e3, "frac": nbytes / us / 1e3 / peak,
                "isolated_us": iso, "isolated_GBps": nbytes / iso / 1e3,
                "spot_check_max_abs": err}

    shapes = []
    for m, k, b in SWEEP_SHAPES:
        per = gemv_bytes(m, k, b)
        nsets = max(4, -(-3 * L2_BYTES // per))  # > 3x L2 of distinct weights
        pk, sc, xs, ys = make_stack(torch, quantize, dev, m, k, b, nsets, 20000 + m + k)
        # first call of each set, so the check below reads computed outputs
        for i in range(nsets):
            capi.check(capi.gemv(pk[i].data_ptr(), sc[i].data_ptr(), xs[i].data_ptr(),
                                 ys[i].data_ptr(), m, k, b, plain, 0, 0,
                                 torch.cuda.current_stream().cuda_stream), "dk_w4a16_gemv")
        torch.cuda.synchronize()
        shapes.append(entry(m, k, b, pk, sc, xs, ys))
        del pk, sc, xs, ys
        torch.cuda.empty_cache()
    batches = []
    m, k = packed[0].shape[0], packed[0].shape[1] * 8
    for b in SWEEP_BATCHES:
        g = torch.Generator(device=dev).manual_seed(30000 + b)
        xs = [torch.randn(b, k, generator=g, device=dev).half() for _ in packed]
        ys = [torch.empty(b, m, dtype=torch.float16, device=dev) for _ in packed]
        capi.check(capi.gemv(packed[0].data_ptr(), scales[0].data_ptr(), xs[0].data_ptr(),
                             ys[0].data_ptr(), m, k, b, plain, 0, 0,
                             torch.cuda.current_stream().cuda_stream), "dk_w4a16_gemv")
        torch.cuda.synchronize()
        batches.append(entry(m, k, b, packed, scales, xs, ys))
        del xs, ys
    return {"protocol": f"chain: {steps} replays of a CUDA graph of one GEMV per distinct weight "
                        f"set (> 3x L2 of weights, PDL); isolated: 512 MiB fill flush, events "
                        f"around one plain C-ABI call, median of 100",
            "shapes": shapes, "batch_sweep_4096x4096": batches,
            "cublas_fp16": run_fp16_reference(args, torch, dev, peak)}


def tp_leg(args, workload: str, ws: int, rank: int, dev, dist, steps: int,
           check: bool = True) -> dict:
    """One decode step of ``layers`` decoder layers' projections in the
    tensor-parallel layout over the ranks (q/k/v and gate/up+SiLU-mul split
    by output rows with no exchange; o and down K-parallel with the fused
    reduction: two exchanges per layer), captured in a CUDA graph and
    replayed ``steps`` times; time = max over ranks.  Every rank takes the
    same collective steps.  Before timing, rank 0 checks layer 0's outputs:
    bit for bit against the rank-ordered fp32 sum of the K-slice partials
    computed on one GPU (the exchange's contract), and within 1e-2 of the
    unsharded single-GPU GEMVs."""
    import torch

    import decode_kernel as dk
    from decode_kernel import capi
    from decode_kernel.quantize import quantize_and_pack_cuda
    from decode_kernel.sharded import (PeerBuffers, TensorParallelAttentionProj,
                                       TensorParallelMLP, split_dim)

    B = args.batch
    layers = args.layers or (32 if workload == "llama7b-tp" else 8)
    H, Q, KV, I = tp_layer_shapes(workload)
    peers = PeerBuffers(8 * ws * B * H)

    def mat(m, k, seed):
        g = torch.Generator(device=dev).manual_seed(seed)  # same weights on every rank
        w = torch.randn(m, k, generator=g, device=dev) * 0.02
        out = quantize_and_pack_cuda(w)
        del w
        return out

    blocks, full0 = [], None
    for layer in range(layers):
        s0 = 9000 + 10 * layer
        mats = [mat(Q, H, s0), mat(KV, H, s0 + 1), mat(KV, H, s0 + 2), mat(H, Q, s0 + 3),
                mat(I, H, s0 + 4), mat(I, H, s0 + 5), mat(H, I, s0 + 6)]
        attn = TensorParallelAttentionProj(*mats[:4], peers, max_batch=B, exchange=args.exchange)
        mlp = TensorParallelMLP(*mats[4:], peers, max_batch=B, exchange=args.exchange)
        blocks.append((attn, mlp))
        if layer == 0 and check and rank == 0:
            full0 = mats
        del mats
        torch.cuda.empty_cache()
    x = torch.randn(B, H, generator=torch.Generator(device=dev).manual_seed(1), device=dev).half()
    # This rank's algorithmic bytes per layer: its weight slices, x per kernel,
    # the local outputs, and the partials it exchanges.
    _, nq = split_dim(Q, ws, rank)
    _, nkv = split_dim(KV, ws, rank)
    _, ni = split_dim(I, ws, rank)
    per_layer = (gemv_bytes(nq + 2 * nkv, H, B) + gemv_bytes(H, nq, B) + gemv_bytes(2 * ni, H, B)
                 - B * ni * 2 + gemv_bytes(H, ni, B))
    if ws > 1 and args.exchange == "fused":
        per_layer += 2 * (ws - 1) * B * H * 4
    shard_bytes = per_layer * layers
    pdl = not args.no_pdl and args.exchange == "fused"
    # this library's kernels per layer: q/k/v, o (+ sum), gate/up, down (+ sum)
    launches = layers * (4 + (2 if ws > 1 and args.exchange == "fused" else 0))

    def step():
        for attn, mlp in blocks:
            attn(x, pdl=pdl)
            mlp(x, pdl=pdl)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    parity = None
    if check:
        attn0, mlp0 = blocks[0]
        ya = attn0(x).clone()
        ym = mlp0(x).clone()
        torch.cuda.synchronize()
        if rank == 0:
            (pq, sq), _, _, (po, so), (pg, sg), (pu, su), (pd, sd) = full0
            f32 = capi.default_config(version=5, flags=capi.DK_FLAG_F32_OUT)
            st = torch.cuda.current_stream().cuda_stream

            def rank_ordered(pw, sw, inp):
                n = inp.shape[1]
                acc = torch.zeros((B, pw.shape[0]), dtype=torch.float32, device=dev)
                for r in range(ws):
                    k0, kn = split_dim(n, ws, r)
                    p_r = pw[:, k0 // 8:(k0 + kn) // 8].contiguous()
                    s_r = sw[:, k0 // 128:(k0 + kn) // 128].contiguous()
                    x_r = inp[:, k0:k0 + kn].contiguous()
                    part = torch.empty_like(acc)
                    capi.check(capi.gemv(p_r.data_ptr(), s_r.data_ptr(), x_r.data_ptr(),
                                         part.data_ptr(), pw.shape[0], kn, B, f32, 0, 0, st),
                               "dk_w4a16_gemv")
                    acc = acc + part
                return acc.half()

            q = dk.gemv(pq, sq, x)
            h = dk.gemv_silu_mul((pg, sg), (pu, su), x)
            want_a, want_m = rank_ordered(po, so, q), rank_ordered(pd, sd, h)
            parity = {
                "bitwise_o": bool(torch.equal(ya, want_a)),
                "bitwise_down": bool(torch.equal(ym, want_m)),
                "max_abs_vs_unsharded_o": float((ya.float() - dk.gemv(po, so, q).float())
                                                .abs().max()),
                "max_abs_vs_unsharded_down": float((ym.float() - dk.gemv(pd, sd, h).float())
                                                   .abs().max()),
                "contract": "bit for bit the rank-ordered fp32 sum of the K-slice partials "
                            "computed on one GPU; within 1e-2 of the unsharded GEMV"}
            full0 = None
    # Every rank learns whether rank 0's check passed before anything is timed.
    ok = torch.tensor([1.0 if parity is None or (
        parity["bitwise_o"] and parity["bitwise_down"] and
        parity["max_abs_vs_unsharded_o"] < 1e-2 and parity["max_abs_vs_unsharded_down"] < 1e-2)
        else 0.0], device=dev)
    if dist:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if ok.item() != 1.0:
        raise AssertionError(f"tensor-parallel parity check failed: {parity}")

    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clocks:
        e0.record()
        for _ in range(steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    total = torch.tensor([float(shard_bytes)], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(total)
    err = capi.load().dk_device_error(-1, 0)
    del graph
    torch.cuda.synchronize()
    peers.close()
    ms_max = float(t[0].item())
    return {"workload": f"{workload} x{layers} layers (hidden {H}, q {Q}, k/v {KV}, "
                        f"intermediate {I}), B={B}; attention not run",
            "n_gpus": ws, "steps": steps, "us_per_step": ms_max * 1e3 / steps,
            "aggregate_GBps": float(total.item()) * steps / (ms_max / 1e3) / 1e9,
            "exchange": args.exchange, "pdl": pdl,
            "parallelism": f"tensor-parallel x{ws}: 2 exchanges per layer",
            "gpu_launches": launches * steps, "device_error": err, "parity": parity,
            "clocks": clocks.summary(), "layers": layers, "H": H, "Q": Q, "KV": KV, "I": I}


def run_ours(args) -> None:
    import numpy as np
    import torch

    import decode_kernel as dk
    from decode_kernel import capi
    from decode_kernel.quantize import quantize_and_pack_cuda

    ws, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        # The exchange is plain peer stores; NCCL carries only barriers and the
        # max-over-ranks of the timings, with NVLink SHARP (NVLS) off.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        pg = dist

    M, K, B, S = args.m, args.k, args.batch, args.sets
    per_gemv = gemv_bytes(M, K, B)
    assert S * M * K // 2 > 2 * L2_BYTES, "weight stack must exceed 2x L2"

    # Seeded synthetic weights, quantized on the GPU (bit-exact with the CPU
    # quantizer), distinct per set and per rank.
    packed, scales, xs, ys = [], [], [], []
    for s in range(S):
        g = torch.Generator(device=dev).manual_seed(1000 * rank + s)
        w = torch.randn(M, K, generator=g, device=dev) * 0.02
        p, sc = quantize_and_pack_cuda(w)
        packed.append(p)
        scales.append(sc)
        xs.append(torch.randn(B, K, generator=g, device=dev).half())
        ys.append(torch.empty(B, M, dtype=torch.float16, device=dev))
        del w
    torch.cuda.synchronize()

    cfg = capi.default_config(flags=0 if args.no_pdl else capi.DK_FLAG_PDL)
    lib = capi.load()

    def step(stream):
        for s in range(S):
            st = capi.gemv(packed[s].data_ptr(), scales[s].data_ptr(), xs[s].data_ptr(),
                           ys[s].data_ptr(), M, K, B, cfg, 0, 0, stream)
            if st:
                capi.check(st, "dk_w4a16_gemv")

    # Warm-up (eager), then capture one step in a CUDA graph.
    cur = torch.cuda.current_stream().cuda_stream
    for _ in range(max(args.warmup, 3)):
        step(cur)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()

    # Correctness spot check of the measured configuration (first set, 64 rows).
    if rank == 0:
        from oracle import oracle as O

        pk = packed[0][:64].cpu().numpy()
        sc = scales[0][:64].cpu().view(torch.int16).numpy().view(np.uint16)
        xx = xs[0].cpu().view(torch.int16).numpy().view(np.uint16)
        ref = O.linear_fp32(xx, pk, sc)
        err = float(np.abs(ys[0][:, :64].float().cpu().numpy() - ref).max())
        assert err < 1e-2, f"bench spot check failed: {err}"

    # ---- timed region: K graph replays ----
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.nvtx.range_push("dk_timed")  # lets ncu --nvtx-include select it
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t_local = torch.tensor([ms], dtype=torch.float64, device=dev)
    if pg:
        pg.all_reduce(t_local, op=pg.ReduceOp.MAX)
    ms_max = float(t_local.item())
    launches = args.steps * S
    value = ws * launches * per_gemv / (ms_max / 1e3) / 1e9
    us_per_gemv_local = ms * 1e3 / launches
    achieved = per_gemv / (us_per_gemv_local / 1e6) / 1e9
    assert lib.dk_device_error(-1, 0) == 0, "a bounded device wait timed out"
    del graph

    # ---- e2e through the public API with host buffers ----
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    hx = torch.empty((S, B, K), dtype=torch.float16).pin_memory()
    hx.copy_(torch.stack([x.cpu() for x in xs]))
    hy = torch.empty((S, B, M), dtype=torch.float16).pin_memory()
    dx = torch.empty((S, B, K), dtype=torch.float16, device=dev)
    dy = torch.empty((S, B, M), dtype=torch.float16, device=dev)

    # Eager public-API calls, one per GEMV, into the step's output buffer (no
    # allocation per call), launched with PDL like the device-timed chain.
    pdl = not args.no_pdl

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        for s in range(S):
            dk.gemv_out(packed[s], scales[s], dx[s], dy[s], pdl=pdl)
        hy.copy_(dy, non_blocking=True)

    # The same public-API calls captured once in a CUDA graph (how a decode
    # loop runs them), replayed per step between the host copies.
    gemv_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gemv_graph):
        for s in range(S):
            dk.gemv_out(packed[s], scales[s], dx[s], dy[s], pdl=pdl)

    def e2e_graph_step():
        dx.copy_(hx, non_blocking=True)
        gemv_graph.replay()
        hy.copy_(dy, non_blocking=True)

    def time_e2e(fn) -> float:
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(e2e_steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if pg:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return ws * e2e_steps * S * per_gemv / (float(t.item()) / 1e3) / 1e9

    e2e_eager = time_e2e(e2e_step)
    eager_y = hy.clone()
    e2e_value = time_e2e(e2e_graph_step)
    # The replayed calls return the eager calls' bits.
    assert torch.equal(hy, eager_y), "graph-replayed e2e outputs differ from the eager calls"
    del gemv_graph

    roof = read_roof_gbs(torch, capi) if rank == 0 else None

    # One call at a time under the reference's own protocol (512 MiB flush,
    # events around a single plain launch): the number the reference's
    # published table is made of.
    isolated = None
    if rank == 0 and not args.no_isolated:
        cfg_plain = capi.default_config()

        def one_call():
            capi.check(capi.gemv(packed[0].data_ptr(), scales[0].data_ptr(), xs[0].data_ptr(),
                                 ys[0].data_ptr(), M, K, B, cfg_plain, 0, 0,
                                 torch.cuda.current_stream().cuda_stream), "dk_w4a16_gemv")

        iso_us = time_isolated(torch, one_call)
        isolated = {"us_per_gemv": iso_us, "GBps": per_gemv / iso_us / 1e3,
                    "protocol": "512 MiB fill flush, CUDA events around one C-ABI call "
                                "(no PDL), median of 200 after 20 warm-up "
                                "(reference bench/common.py:64-108)"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O

        gbs, t, rows, n = time_cpu_reference(M, K, B, budget_s=args.cpu_budget)
        cpu = {"value": gbs, "unit": "GB/s", "cores": O.cpu_threads(), "kind": "port",
               "sample": f"{n} full {M}x{K} B={B} GEMVs (median {t * 1e3:.1f} ms each); fp32 "
                         f"dequantize then fp32 BLAS matmul (numpy restatement of "
                         f"reference.py:17-26)"}

    peak, peak_kind = measured_peaks()
    # The other BASELINE configurations (one GPU, rank 0): extra keys.
    sweeps = None
    if rank == 0 and ws == 1 and not args.no_sweeps:
        del hx, hy, dx, dy
        sweeps = run_sweeps(args, torch, capi, quantize_and_pack_cuda, dev, packed, scales, peak)
    # Strong scaling: the 70B-shaped layers sharded over every rank of this
    # run (the same command at N = 1), with the exchange between the GPUs
    # and an in-run parity check against the unsharded layer.
    strong = None
    if not args.no_strong:
        del packed, scales, xs, ys
        torch.cuda.empty_cache()
        strong = tp_leg(args, "llama70b-tp", ws, rank, dev, pg, max(args.steps, 100))

    if pg:
        pg.barrier()
        pg.destroy_process_group()
    if rank != 0:
        return
    traffic = ncu_traffic_per_launch(M, K, B)
    clk = clocks.summary()
    line = {
        "metric": metric_name(M, K, B),
        "value": value,
        "unit": "GB/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps,
        "us_per_gemv": ms_max * 1e3 / launches,
        "pct_of_read_roof": (100.0 * value / ws / roof) if roof else None,
        "read_roof_gbs": roof,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int4*f16->f32",
        "data": "synthetic",
        "config": workload_config(M, K, B, S, ws),
        "arm": {"kernel": kernel_path(M, K, B) + (", PDL" if not args.no_pdl else ""),
                "launch": "CUDA graph of one step (one C-ABI call per weight set), replayed",
                "weight_stack_bytes": S * M * K // 2},
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy)" if peak_kind ==
            "measured" else "fallback 6650 GB/s",
            "traffic": traffic,
            "bytes_per_launch": per_gemv,
        },
        "e2e": {"value": e2e_value, "unit": "GB/s",
                "h2d_bytes_per_step": S * B * K * 2, "d2h_bytes_per_step": S * B * M * 2,
                "steps": e2e_steps,
                "path": "decode_kernel.gemv_out per GEMV (torch extension -> C ABI, PDL), "
                        "the step's calls captured once with torch.cuda.graph and replayed; "
                        "every step: one pinned-host H2D of its x, the replay, one D2H of its y",
                "eager": {"value": e2e_eager, "unit": "GB/s",
                          "path": "the same calls launched eagerly, one Python call per GEMV"}},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if isolated is not None:
        line["isolated"] = isolated
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if sweeps is not None:
        line["baseline_configs"] = sweeps
    if strong is not None:
        line["strong_scaling"] = strong
    line["meta"] = run_meta(local)
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# Sharded model shapes (row- / K-parallel across the ranks, strong scaling)
# --------------------------------------------------------------------------

def model_gemvs(workload: str, layers: int):
    """(M, K, layout) of every GEMV in one decode step of the model shapes:
    Llama-2-7B (q/k/v/o 4096x4096, gate/up 11008x4096, down 4096x11008; all
    row-parallel -- 86 groups of K in down do not divide by 4 or 8),
    Llama-3-8B (q/o 4096x4096, k/v 1024x4096 -- 8 kv heads of 128 --,
    gate/up 14336x4096 row-parallel, down 4096x14336 K-parallel) and
    Llama-70B-shaped layers (q/o 8192x8192 and gate/up 28672x8192
    row-parallel, down 8192x28672 K-parallel)."""
    if workload == "llama7b":
        one = [(4096, 4096, "row")] * 4 + [(11008, 4096, "row")] * 2 + [(4096, 11008, "row")]
    elif workload == "llama8b":
        one = ([(4096, 4096, "row"), (1024, 4096, "row"), (1024, 4096, "row"), (4096, 4096, "row")]
               + [(14336, 4096, "row")] * 2 + [(4096, 14336, "k")])
    else:
        one = [(8192, 8192, "row"), (8192, 8192, "row"), (28672, 8192, "row"),
               (28672, 8192, "row"), (8192, 28672, "k")]
    return one * layers


def run_sharded(args) -> None:
    import datetime

    import torch

    from decode_kernel.quantize import quantize_and_pack_cuda
    from decode_kernel.sharded import (KParallelW4A16, PeerBuffers, RowParallelW4A16, k_range,
                                       row_range)

    ws, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if ws > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    B = args.batch
    layers = args.layers or (32 if args.workload in ("llama7b", "llama8b") else 8)
    shapes = model_gemvs(args.workload, layers)
    maxm = max(m for m, _, _ in shapes)
    peers = PeerBuffers(max(2 * B * maxm, 8 * ws * B * maxm))
    xs = {}
    mods, shard_bytes = [], 0
    for i, (M, K, layout) in enumerate(shapes):
        g = torch.Generator(device=dev).manual_seed(7000 + i)  # same weights on every rank
        w = torch.randn(M, K, generator=g, device=dev) * 0.02
        p, s = quantize_and_pack_cuda(w)
        del w
        cls = RowParallelW4A16 if layout == "row" else KParallelW4A16
        mods.append(cls(p, s, peers, max_batch=B, exchange=args.exchange))
        del p, s
        if K not in xs:
            gx = torch.Generator(device=dev).manual_seed(K)
            xs[K] = torch.randn(B, K, generator=gx, device=dev).half()
        if layout == "row":
            _, rows = row_range(M, ws, rank)
            shard_bytes += gemv_bytes(rows, K, B) + B * (M - rows) * 2
        else:
            _, kn = k_range(K, ws, rank)
            shard_bytes += gemv_bytes(M, kn, B) + B * M * 2 * (ws - 1)
    torch.cuda.synchronize()
    pdl = not args.no_pdl and args.exchange == "fused"
    # this library's kernels per step: GEMV + wait (+ the K-parallel sum)
    launches = sum((2 if lay == "row" else 3) if args.exchange == "fused" else 1
                   for _, _, lay in shapes)

    def step():
        for mod, (M, K, _) in zip(mods, shapes):
            mod(xs[K], pdl=pdl)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms, float(shard_bytes)], dtype=torch.float64, device=dev)
    total = torch.tensor([float(shard_bytes)], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(total)
    from decode_kernel import capi

    err = capi.load().dk_device_error(-1, 0)
    del graph
    torch.cuda.synchronize()
    peers.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    ms_max = float(t[0].item())
    value = float(total.item()) * args.steps / (ms_max / 1e3) / 1e9
    line = {
        "metric": f"aggregate HBM read GB/s, {args.workload} decode-step GEMV stack",
        "value": value, "unit": "GB/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "us_per_token": ms_max * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int4*f16->f32", "data": "synthetic",
        "config": {"workload": f"{args.workload} x{layers} layers, {len(shapes)} GEMVs, B={B}",
                   "global_batch": B, "exchange": args.exchange, "pdl": pdl,
                   "parallelism": f"row/K-parallel x{ws}",
                   "l2": "inputs larger than L2 (the step streams every layer's weights)"},
        "device_error": err, "gpu_launches": launches * args.steps, "clocks": clocks.summary(),
    }
    line["meta"] = run_meta(local)
    print(json.dumps(line), flush=True)


def tp_layer_shapes(workload: str):
    """(hidden, q rows, k/v rows, intermediate) of one decoder layer: Llama-2-7B
    (MHA, 32 heads of 128) and the Llama-70B shapes (GQA: 64 query and 8 kv
    heads of 128)."""
    return (4096, 4096, 4096, 11008) if workload == "llama7b-tp" else (8192, 8192, 1024, 28672)


def run_tensor_parallel(args) -> None:
    """A decoder layer's projections in the tensor-parallel layout: q/k/v and
    gate/up (with the SiLU-mul epilogue) split by output rows with no
    exchange, o and down K-parallel over the same split with the fused
    reduction -- two exchanges per layer.  Attention itself is not run: o
    reads the rank's q slice (the shape of its heads' attention output)."""
    import datetime

    import torch

    ws, rank, local = dist_info()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if ws > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    leg = tp_leg(args, args.workload, ws, rank, dev, dist, args.steps)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": f"aggregate HBM read GB/s, {args.workload} decode-step projections",
        "value": leg["aggregate_GBps"], "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": leg["us_per_step"] / 1e3,
        "us_per_token": leg["us_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int4*f16->f32", "data": "synthetic",
        "config": {"workload": leg["workload"], "global_batch": args.batch,
                   "exchange": args.exchange, "pdl": leg["pdl"],
                   "parallelism": leg["parallelism"],
                   "l2": "inputs larger than L2 (the step streams every layer's weights)"},
        "device_error": leg["device_error"], "parity": leg["parity"],
        "gpu_launches": leg["gpu_launches"], "clocks": leg["clocks"],
    }
    line["meta"] = run_meta(local)
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "marlin"], default="ours",
                    help="marlin: the same-precision peer (vLLM's Marlin) on this GPU")
    ap.add_argument("--m", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--sets", type=int, default=64)
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-cuda", action="store_true",
                    help="reference arm: skip timing the reference's own CUDA kernels")
    ap.add_argument("--no-isolated", action="store_true",
                    help="skip the isolated-call timing under the reference's protocol")
    ap.add_argument("--workload",
                    choices=["gemv", "llama7b", "llama8b", "llama70b", "llama7b-tp",
                             "llama70b-tp"],
                    default="gemv",
                    help="gemv: the BASELINE metric; llama7b / llama8b / llama70b: the sharded model "
                         "decode-step GEMV stacks, every GEMV gathered (strong scaling over "
                         "the ranks); llama7b-tp / llama70b-tp: the same layers in the "
                         "tensor-parallel layout, two exchanges per layer")
    ap.add_argument("--exchange", choices=["fused", "nccl"], default="fused")
    ap.add_argument("--no-sweeps", action="store_true",
                    help="skip the other BASELINE configs (shapes, batch sweep)")
    ap.add_argument("--no-strong", action="store_true",
                    help="skip the strong-scaling leg (70B-shaped tensor-parallel layers)")
    ap.add_argument("--layers", type=int, default=0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "marlin":
        run_marlin_peer(args)
    elif args.workload.endswith("-tp"):
        run_tensor_parallel(args)
    elif args.workload != "gemv":
        run_sharded(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
