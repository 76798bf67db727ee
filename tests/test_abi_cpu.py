"""The C-ABI library and the torch extension load on a machine without a GPU,
export every entry point include/dk_w4a16.h declares, and reject bad
arguments before touching the device."""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "dk_w4a16.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^DK_API [^()]*?\b(dk_\w+)\(", text, flags=re.M)))


def test_header_declares_the_abi():
    names = declared_functions()
    for must in ("dk_w4a16_gemv", "dk_w4a16_workspace_bytes", "dk_stream_read",
                 "dk_stream_write", "dk_d2d_copy", "dk_stream_recommended_blocks",
                 "dk_last_kernel_stamp", "dk_quantize_pack", "dk_status_string"):
        assert must in names


def test_library_exports_exactly_the_header():
    from decode_kernel import capi

    lib = capi.LIB_PATH
    assert lib.exists(), "build the library first (__graft_entry__.build())"
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted({ln.split()[-1] for ln in out.splitlines() if " T " in ln})
    assert exported == declared_functions()
    # The ctypes binding knows every declared symbol too.
    assert sorted(capi.SIGNATURES) == declared_functions()


def test_library_loads_and_reports():
    from decode_kernel import capi

    lib = capi.load()
    assert b"sm_100a" in lib.dk_version()
    assert lib.dk_status_string(capi.DK_OK) == b"ok"
    for st in range(7):
        assert lib.dk_status_string(st)
    cfg = capi.default_config()
    assert (cfg.version, cfg.split_k, cfg.reuse_weights, cfg.warps_per_row, cfg.flags) == \
        (5, 4, 0, 1, 0)


def test_workspace_sizes():
    from decode_kernel import capi

    assert capi.workspace_bytes(4096, 4096, 1) == 0  # v5 needs none
    v4 = capi.default_config(version=4, split_k=4)
    ws = capi.workspace_bytes(4096, 4096, 1, v4)
    assert ws >= 4 * 4096 * 4 and ws % 4 == 0
    assert capi.workspace_bytes(4096, 4096, 1, capi.default_config(version=4, split_k=1)) == 0
    # Batches go through in passes of 32 rows, so the workspace stops growing.
    assert capi.workspace_bytes(64, 256, 64, v4) == capi.workspace_bytes(64, 256, 32, v4)


@pytest.mark.parametrize("kw,shape", [
    (dict(version=6), (64, 256, 1)),
    (dict(version=-1), (64, 256, 1)),
    (dict(split_k=0), (64, 256, 1)),
    (dict(split_k=33), (64, 256, 1)),
    (dict(warps_per_row=9), (64, 256, 1)),
    (dict(warps_per_row=2, version=5), (64, 256, 1)),
    (dict(warps_per_row=2, version=1, reuse_weights=1), (64, 256, 1)),
    (dict(flags=0x80), (64, 256, 1)),
    (dict(), (64, 200, 1)),
    (dict(), (-1, 256, 1)),
])
def test_invalid_arguments_rejected_without_a_device(kw, shape):
    from decode_kernel import capi

    M, K, B = shape
    st = capi.gemv(16, 16, 16, 16, M, K, B, capi.default_config(**kw))
    assert st == capi.DK_ERR_INVALID_ARG


def test_empty_problem_is_a_noop():
    from decode_kernel import capi

    assert capi.gemv(0, 0, 0, 0, 0, 256, 1) == capi.DK_OK
    assert capi.gemv(0, 0, 0, 0, 64, 256, 0) == capi.DK_OK


def test_misaligned_pointers_rejected():
    from decode_kernel import capi

    assert capi.gemv(8, 16, 16, 16, 64, 256, 1) == capi.DK_ERR_INVALID_ARG
    assert capi.gemv(16, 16, 24, 16, 64, 256, 1) == capi.DK_ERR_INVALID_ARG


def test_quantize_abi_rejects_bad_k():
    from decode_kernel import capi

    lib = capi.load()
    assert lib.dk_quantize_pack(16, 4, 100, 16, 16, 0, None) == capi.DK_ERR_INVALID_ARG
    assert lib.dk_quantize_pack(16, 4, 128, 16, 16, 0x8, None) == capi.DK_ERR_INVALID_ARG


def test_torch_extension_surface():
    from decode_kernel import _cuda

    for name in ("w4a16_gemv", "d2d_copy", "stream_read", "stream_write",
                 "stream_recommended_blocks", "last_kernel_stamp"):
        assert callable(getattr(_cuda, name))
    assert "sm_100a" in _cuda.version()
