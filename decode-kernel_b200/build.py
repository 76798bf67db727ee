"""Build the library in-tree.

1. ``libdk_b200.so`` -- every CUDA source under csrc/ compiled by nvcc for
   sm_100a only (``-gencode arch=compute_100a,code=sm_100a``), CUDA runtime
   linked statically, C ABI per include/dk_w4a16.h.
2. ``decode_kernel/_cuda*.so`` -- the torch extension (csrc/bindings.cpp),
   linked against libdk_b200.so with an $ORIGIN rpath.

Both land in decode-kernel_b200/decode_kernel/ so they travel with the source
tree.  Rebuilds are incremental (mtime based).

    python decode-kernel_b200/build.py [--ptxas-v] [--force]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
PKG = HERE / "decode_kernel"
BUILD = HERE / "_build"
INCLUDE = REPO / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB_SOURCES = ["dk_abi.cu", "dk_gemv.cu", "dk_stream.cu", "dk_quant.cu", "dk_shard.cu"]
COMMON_DEPS = [CSRC / "dk_device.cuh", CSRC / "dk_host.h", CSRC / "dk_batch.cuh", INCLUDE / "dk_w4a16.h"]
LIB = PKG / "libdk_b200.so"


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME") or "/usr/local/cuda"
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def nvcc_flags(ptxas_verbose: bool = False) -> list[str]:
    flags = ARCH + [
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden",
        "-Xcompiler", "-Wall",
        f"-I{INCLUDE}",
        f"-I{CSRC}",
    ]
    if ptxas_verbose:
        flags += ["-Xptxas", "-v"]
    return flags


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], cwd: Path | None = None, quiet: bool = False) -> str:
    proc = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    if not quiet and proc.stderr.strip():
        sys.stderr.write(proc.stderr)
    return proc.stdout + proc.stderr


def build_lib(force: bool = False, ptxas_verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    objs = []
    for src in LIB_SOURCES:
        s = CSRC / src
        obj = BUILD / (src + ".o")
        objs.append(obj)
        if force or ptxas_verbose or _stale(obj, [s] + COMMON_DEPS):
            out = _run([nvcc(), *nvcc_flags(ptxas_verbose), "-c", str(s), "-o", str(obj)],
                       quiet=not ptxas_verbose)
            if ptxas_verbose:
                sys.stdout.write(out)
    if force or _stale(LIB, objs):
        _run([nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs)])
    return LIB


def ext_path() -> Path:
    return PKG / ("_cuda" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_ext(force: bool = False) -> Path:
    out = ext_path()
    deps = [CSRC / "bindings.cpp", INCLUDE / "dk_w4a16.h", LIB, HERE / "setup.py"]
    if force or _stale(out, deps):
        _run([sys.executable, "setup.py", "build_ext", "--inplace",
              "--build-temp", str(BUILD / "ext")], cwd=HERE, quiet=True)
    return out


def build_all(force: bool = False, ptxas_verbose: bool = False) -> None:
    build_lib(force=force, ptxas_verbose=ptxas_verbose)
    build_ext(force=force)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print registers/smem/spills")
    ap.add_argument("--lib-only", action="store_true")
    a = ap.parse_args()
    if a.lib_only:
        build_lib(force=a.force, ptxas_verbose=a.ptxas_v)
    else:
        build_all(force=a.force, ptxas_verbose=a.ptxas_v)
    print(LIB)
    if not a.lib_only:
        print(ext_path())


if __name__ == "__main__":
    main()
