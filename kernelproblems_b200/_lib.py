"""ctypes binding of libfrag.so (the C ABI declared in include/frag.h).

There is no fallback: if the library is missing or cannot be loaded, every op
raises.  Build it with ``python -m kernelproblems_b200._build``.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfrag.so"

FRAG_OK = 0
STATUS_NAMES = {
    0: "FRAG_OK",
    1: "FRAG_ERR_INVALID_ARG",
    2: "FRAG_ERR_SHAPE",
    3: "FRAG_ERR_ALIGN",
    4: "FRAG_ERR_WORKSPACE",
    5: "FRAG_ERR_CUDA",
    6: "FRAG_ERR_NO_DEVICE",
    7: "FRAG_ERR_SCRATCH_LIMIT",
}
FRAG_DEVFLAG_INDEX_OOB = 1
FRAG_DEVFLAG_WAIT_TIMEOUT = 2
FRAG_ROPE_OUT_BF16 = 0
FRAG_ROPE_OUT_F32 = 1
FRAG_DT_BF16 = 0
FRAG_DT_F32 = 1
FRAG_ROPE_IN_BF16 = 0
FRAG_ROPE_IN_F32 = 1
FRAG_ROPE_NEOX = 0
FRAG_ROPE_INTERLEAVED = 1
FRAG_POS_NONE = 0
FRAG_POS_I32 = 1
FRAG_POS_I64 = 2

_vp = C.c_void_p
_i64 = C.c_int64
_f32 = C.c_float
_int = C.c_int
_sz = C.c_size_t


class FragError(RuntimeError):
    """A libfrag entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{fn} failed: {name}{(': ' + detail) if detail else ''}")


class RopeTensor(C.Structure):
    _fields_ = [
        ("x", _vp),
        ("out", _vp),
        ("H", _i64),
        ("x_stride_b", _i64),
        ("x_stride_s", _i64),
        ("x_stride_h", _i64),
        ("out_stride_b", _i64),
        ("out_stride_s", _i64),
        ("out_stride_h", _i64),
        ("out_dtype", C.c_int32),  # FRAG_ROPE_OUT_BF16 / FRAG_ROPE_OUT_F32
        ("in_dtype", C.c_int32),   # FRAG_ROPE_IN_BF16 / FRAG_ROPE_IN_F32
    ]


FRAG_COPY_MAX_SEGMENTS = 16
FRAG_PEER_MAX_RANKS = 8
FRAG_IPC_HANDLE_BYTES = 64


class CopySegment(C.Structure):
    _fields_ = [
        ("src", _vp),
        ("dst", _vp),
        ("src_stride", _i64),
        ("dst_stride", _i64),
        ("rows", _i64),
        ("row_bytes", _i64),
    ]


# name -> (restype, argtypes); mirrors include/frag.h one to one.
SIGNATURES: dict[str, tuple] = {
    "frag_version": (C.c_char_p, []),
    "frag_status_string": (C.c_char_p, [_int]),
    "frag_last_cuda_error": (_int, []),
    "frag_device_sm_count": (_int, []),
    "frag_device_errors": (_int, [_int]),
    "frag_rmsnorm_fwd": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "frag_add_rmsnorm_fwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "frag_rmsnorm_bwd_workspace_bytes": (_sz, [_i64, _i64]),
    "frag_rmsnorm_bwd": (
        _int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp, _sz, _vp],
    ),
    "frag_rmsnorm_bwd_noalloc": (
        _int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "frag_rmsnorm_bwd3": (
        _int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp, _sz, _vp]),
    "frag_rmsnorm_fwd_bwd": (
        _int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp,
               _sz, _vp]),
    "frag_rmsnorm_bwd_num_blocks": (_i64, [_i64, _i64]),
    "frag_rmsnorm_bwd_plan_blocks": (_i64, [_i64, _i64, _int]),
    "frag_dw_reduce": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "frag_embedding_fwd": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "frag_peer_alloc": (_int, [_sz, C.POINTER(_vp), _vp]),
    "frag_peer_open": (_int, [_vp, C.POINTER(_vp)]),
    "frag_peer_close": (_int, [_vp]),
    "frag_peer_free": (_int, [_vp]),
    "frag_dw_exchange_peer": (
        _int, [_vp, _i64, C.POINTER(_vp), C.POINTER(_vp), _vp, _int, _int, _vp, _vp]),
    "frag_embedding_fwd_vp_peer": (
        _int, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, C.POINTER(_vp), C.POINTER(_vp), _vp, _int, _int,
               _vp, _vp]),
    "frag_embedding_rmsnorm_fwd": (
        _int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _f32, _vp, _vp]),
    "frag_embedding_bwd_workspace_bytes": (_sz, [_i64, _i64]),
    "frag_copy_rows": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _vp]),
    "frag_copy_rows_grouped": (_int, [C.POINTER(CopySegment), C.c_int32, _vp]),
    "frag_convert_rows": (_int, [_vp, C.c_int32, _i64, _vp, _vp, C.c_int32, _i64, _i64, _i64, _vp]),
    "frag_selftest_bounded_wait": (_int, [_i64, _vp]),
    "frag_rmsnorm_embedding_bwd_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "frag_rmsnorm_embedding_bwd": (
        _int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
         _i64, _i64, _i64, _i64, _i64, _i64, _f32, _vp, _sz, _vp, _vp],
    ),
    "frag_embedding_bwd": (
        _int,
        [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _vp, _vp],
    ),
    "frag_rope": (
        _int,
        [C.POINTER(RopeTensor), _int, _i64, _i64, _i64, _vp, _int, _i64, _i64, _vp, _i64, _i64,
         _f32, _int, _int, _vp],
    ),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Load libfrag.so once (raises FileNotFoundError / OSError if unusable)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("FRAG_LIBRARY", LIB_PATH))
        if not path.exists():
            raise FileNotFoundError(
                f"{path} is missing: build it with `python -m kernelproblems_b200._build` "
                "(there is no CPU fallback)"
            )
        lib = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise FragError on failure."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != FRAG_OK:
        detail = ""
        if st == 5:
            detail = f"cudaError {lib.frag_last_cuda_error()}"
        raise FragError(name, st, detail)


def version() -> str:
    return load().frag_version().decode()
