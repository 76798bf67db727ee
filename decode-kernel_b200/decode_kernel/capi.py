"""ctypes binding of the C ABI (include/dk_w4a16.h) in libdk_b200.so.

This is the binding a non-torch caller would write; the tests use it to drive
the kernels through the exact extern "C" entry points.  Device memory is passed
as raw addresses (e.g. ``tensor.data_ptr()``).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdk_b200.so"

DK_OK = 0
DK_ERR_INVALID_ARG = 1
DK_ERR_UNSUPPORTED = 2
DK_ERR_LAUNCH = 3
DK_ERR_TIMEOUT = 4
DK_ERR_CUDA = 5
DK_ERR_WORKSPACE = 6

DK_FLAG_PDL = 0x1
DK_FLAG_F32_OUT = 0x2
DK_FLAG_SHARD_WAIT = 0x4
DK_QUANT_TORCH_CUDA_SCALE = 0x1
DK_NOALLOC_SCRATCH_BYTES = 8 << 20
DK_MAX_SHARDS = 8
DK_MAX_SEGMENTS = 4
DK_SHARD_SLOTS = 256
DK_PEER_HANDLE_BYTES = 64


class GemvConfig(ctypes.Structure):
    """struct dk_gemv_config (gemv_w4a16.h:22-27 GemvLaunchConfig + flags)."""

    _fields_ = [
        ("version", ctypes.c_int),
        ("split_k", ctypes.c_int),
        ("reuse_weights", ctypes.c_int),
        ("warps_per_row", ctypes.c_int),
        ("flags", ctypes.c_uint),
    ]


class ShardGroup(ctypes.Structure):
    """struct dk_shard_group: this rank, the world size, every rank's result
    buffer and arrival-slot array as mapped in this process, and this rank's
    own [calls completed, CTAs per rank] pair."""

    _fields_ = [
        ("rank", ctypes.c_int),
        ("world", ctypes.c_int),
        ("bufs", ctypes.c_void_p * DK_MAX_SHARDS),
        ("slots", ctypes.c_void_p * DK_MAX_SHARDS),
        ("seq", ctypes.c_void_p),
    ]


# name -> (restype, argtypes); every symbol include/dk_w4a16.h declares.
_P, _I, _U, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint, ctypes.c_size_t
SIGNATURES = {
    "dk_gemv_config_init": (None, [ctypes.POINTER(GemvConfig)]),
    "dk_w4a16_workspace_bytes": (_SZ, [_I, _I, _I, ctypes.POINTER(GemvConfig)]),
    "dk_w4a16_gemv": (_I, [_P, _P, _P, _P, _I, _I, _I, ctypes.POINTER(GemvConfig), _P, _SZ, _P]),
    "dk_w4a16_gemv_splitk_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "dk_w4a16_gemv_multi": (_I, [_I, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_I),
                                 ctypes.POINTER(_P), _P, _I, _I, ctypes.POINTER(GemvConfig), _P]),
    "dk_w4a16_gemv_silu_mul": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I,
                                    ctypes.POINTER(GemvConfig), _P]),
    "dk_w4a16_gemv_rowshard": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, ctypes.POINTER(ShardGroup),
                                    ctypes.POINTER(GemvConfig), _P]),
    "dk_w4a16_gemv_kshard": (_I, [_P, _P, _P, _I, _I, _I, _I, ctypes.POINTER(ShardGroup),
                                  ctypes.POINTER(GemvConfig), _P]),
    "dk_shard_wait": (_I, [ctypes.POINTER(ShardGroup), _P]),
    "dk_w4a16_gemv_rowshard_gather": (_I, [_P, _P, _P, _I, _I, _I, _I, _I,
                                           ctypes.POINTER(ShardGroup), _P,
                                           ctypes.POINTER(GemvConfig), _P]),
    "dk_w4a16_gemv_kshard_sum": (_I, [_P, _P, _P, _I, _I, _I, _I, ctypes.POINTER(ShardGroup),
                                      _P, ctypes.POINTER(GemvConfig), _P]),
    "dk_shard_reduce": (_I, [ctypes.POINTER(ShardGroup), _I, _I, _P, _I, _P]),
    "dk_peer_alloc": (_I, [_SZ, ctypes.POINTER(ctypes.c_void_p)]),
    "dk_peer_free": (_I, [_P]),
    "dk_peer_export": (_I, [_P, ctypes.c_char_p]),
    "dk_peer_import": (_I, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "dk_peer_close": (_I, [_P]),
    "dk_d2d_copy": (_I, [_P, _P, _SZ, _P]),
    "dk_stream_read": (_I, [_P, _P, _SZ, _I, _P]),
    "dk_stream_write": (_I, [_P, _SZ, _I, _P]),
    "dk_stream_recommended_blocks": (_I, [_I]),
    "dk_last_kernel_stamp": (_I, [_I]),
    "dk_device_error": (_I, [_I, _I]),
    "dk_quantize_pack": (_I, [_P, _I, _I, _P, _P, _U, _P]),
    "dk_unpack_to_int": (_I, [_P, _I, _I, _P, _P]),
    "dk_dequantize": (_I, [_P, _P, _I, _I, _P, _P]),
    "dk_status_string": (ctypes.c_char_p, [_I]),
    "dk_last_cuda_error": (ctypes.c_char_p, []),
    "dk_version": (ctypes.c_char_p, []),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load libdk_b200.so and attach the declared signatures.  Raises when the
    library has not been built -- there is nothing to fall back to."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build()")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def default_config(**kw) -> GemvConfig:
    cfg = GemvConfig()
    load().dk_gemv_config_init(ctypes.byref(cfg))
    for k, v in kw.items():
        setattr(cfg, k, int(v))
    return cfg


class DkError(RuntimeError):
    def __init__(self, status: int, what: str):
        lib = load()
        msg = f"{what}: {lib.dk_status_string(status).decode()}"
        if status in (DK_ERR_LAUNCH, DK_ERR_CUDA):
            msg += f" [{lib.dk_last_cuda_error().decode()}]"
        super().__init__(msg)
        self.status = status


def check(status: int, what: str) -> None:
    if status != DK_OK:
        raise DkError(status, what)


def gemv(packed_ptr: int, scales_ptr: int, x_ptr: int, y_ptr: int, M: int, K: int, B: int,
         cfg: GemvConfig | None = None, workspace_ptr: int = 0, workspace_bytes: int = 0,
         stream: int = 0) -> int:
    """dk_w4a16_gemv; returns the status (0 = DK_OK)."""
    return load().dk_w4a16_gemv(packed_ptr, scales_ptr, x_ptr, y_ptr, M, K, B,
                                ctypes.byref(cfg) if cfg is not None else None,
                                workspace_ptr or None, workspace_bytes, stream or None)


def workspace_bytes(M: int, K: int, B: int, cfg: GemvConfig | None = None) -> int:
    return int(load().dk_w4a16_workspace_bytes(M, K, B,
                                               ctypes.byref(cfg) if cfg is not None else None))


def gemv_silu_mul(packed_gate: int, scales_gate: int, packed_up: int, scales_up: int,
                  x_ptr: int, h_ptr: int, M: int, K: int, B: int,
                  cfg: GemvConfig | None = None, stream: int = 0) -> int:
    """dk_w4a16_gemv_silu_mul over device addresses; returns the status."""
    return load().dk_w4a16_gemv_silu_mul(packed_gate, scales_gate, packed_up, scales_up, x_ptr,
                                         h_ptr, M, K, B,
                                         ctypes.byref(cfg) if cfg is not None else None,
                                         stream or None)


def gemv_multi(packed_ptrs, scales_ptrs, Ms, y_ptrs, x_ptr: int, K: int, B: int,
               cfg: GemvConfig | None = None, stream: int = 0) -> int:
    """dk_w4a16_gemv_multi over lists of device addresses; returns the status."""
    n = len(packed_ptrs)
    P = (ctypes.c_void_p * n)(*packed_ptrs)
    S = (ctypes.c_void_p * n)(*scales_ptrs)
    Mv = (ctypes.c_int * n)(*Ms)
    Y = (ctypes.c_void_p * n)(*y_ptrs)
    return load().dk_w4a16_gemv_multi(n, P, S, Mv, Y, x_ptr, K, B,
                                      ctypes.byref(cfg) if cfg is not None else None,
                                      stream or None)
