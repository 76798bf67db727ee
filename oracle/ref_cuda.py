"""The reference's own CUDA kernels on this GPU -- TEST INFRASTRUCTURE ONLY.

``oracle/_ref/libdkref.so`` is RohanDisa/decode-kernel's csrc/gemv_w4a16.cu,
compiled unmodified from the reference checkout for sm_100a with the
reference's nvcc flags (oracle/Makefile ``ref``), behind the C shim
oracle/ref_shim.cu.  It exists only where the checkout was present at build
time; the built library travels with the tree to the GPU box.

Used by the GPU parity tests (this library against the reference's kernels on
the same device buffers) and by bench.py's reference arm (the reference's
kernels timed on the same B200 under the reference's own protocol).  Never by
the library.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "_ref" / "libdkref.so"
# The reference checkout: DK_REFERENCE, as for tests/golden/make_golden.py, else
# a checkout named "reference" beside this repository.
REF_CHECKOUT = Path(os.environ.get("DK_REFERENCE") or (_HERE.parent.parent / "reference"))
_lib = None


def build() -> Path | None:
    """Compile the reference's kernels where the checkout is present."""
    if not (REF_CHECKOUT / "csrc" / "gemv_w4a16.cu").exists():
        return LIB_PATH if LIB_PATH.exists() else None
    subprocess.run(["make", "-s", "-C", str(_HERE), "ref", f"REF={REF_CHECKOUT}"], check=True)
    return LIB_PATH


def available() -> bool:
    return LIB_PATH.exists()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} not built (needs the reference checkout at build time)")
        L = ctypes.CDLL(str(LIB_PATH))
        p, i = ctypes.c_void_p, ctypes.c_int
        L.dkref_gemv.argtypes = [p, p, p, p, i, i, i, i, i, i, i, p, p]
        L.dkref_gemv.restype = i
        L.dkref_last_kernel_stamp.argtypes = []
        L.dkref_last_kernel_stamp.restype = i
        _lib = L
    return _lib


def gemv(packed, scales, x, y, version=5, split_k=4, reuse_weights=False, warps_per_row=1,
         workspace=None, stream=None) -> int:
    """The reference's ``w4a16_gemv`` on torch CUDA tensors (packed int32 [M, K/8],
    scales fp16 [M, K/128], x fp16 [B, K], y fp16 [B, M]).  ``workspace``: a
    zero-filled fp32 [B, M] tensor, needed by version 4 (bindings.cpp:63-68)."""
    import torch

    M, K, B = packed.shape[0], packed.shape[1] * 8, x.shape[0]
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    ws = workspace.data_ptr() if workspace is not None else None
    return lib().dkref_gemv(packed.data_ptr(), scales.data_ptr(), x.data_ptr(), y.data_ptr(),
                            M, K, B, int(version), int(split_k), int(bool(reuse_weights)),
                            int(warps_per_row), ws, stream)
