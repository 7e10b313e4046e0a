"""ctypes binding of libmfcuda.so (the C ABI declared in include/mfcuda.h).

The library is built in-tree (python -m manifesto_b200.build).  There is no
fallback: if the shared library is missing or fails to load, importing this
module raises, so nothing silently runs on the CPU.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

from .errors import raise_for_status

LIB_PATH = Path(__file__).resolve().parent / "libmfcuda.so"


class ChunkDesc(ctypes.Structure):
    """mf_chunk_desc: one contiguous chunk of one tensor owned by this rank."""

    _fields_ = [
        ("src", ctypes.c_void_p),
        ("dst", ctypes.c_void_p),
        ("n", ctypes.c_int64),
        ("tensor", ctypes.c_int32),
        ("src_dtype", ctypes.c_int32),
    ]


class FusedProgram(ctypes.Structure):
    """mf_fused_program: a FusionAST in postfix order."""

    _fields_ = [
        ("n_nodes", ctypes.c_int32),
        ("op", ctypes.POINTER(ctypes.c_int32)),
        ("arg", ctypes.POINTER(ctypes.c_int32)),
        ("n_consts", ctypes.c_int32),
        ("consts", ctypes.POINTER(ctypes.c_double)),
        ("n_inputs", ctypes.c_int32),
        ("in_dtype", ctypes.POINTER(ctypes.c_int32)),
        ("in_bcast", ctypes.POINTER(ctypes.c_int64)),
        ("out_dtype", ctypes.c_int32),
    ]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> argtypes (every function returns int status except where noted)
SIGNATURES: dict[str, list] = {
    "mf_abi_version": [],
    "mf_device_count": [ctypes.POINTER(_int)],
    "mf_init": [_int],
    "mf_shutdown": [],
    "mf_last_error_copy": [ctypes.c_char_p, _sz],
    "mf_device_status": [ctypes.POINTER(_int)],
    "mf_wait_flag": [_vp, _int, _i64, _vp],
    "mf_device_info": [ctypes.POINTER(_int), ctypes.POINTER(_int), ctypes.POINTER(_int), ctypes.POINTER(_sz)],
    "mf_alloc": [ctypes.POINTER(_vp), _sz],
    "mf_free": [_vp],
    "mf_host_alloc": [ctypes.POINTER(_vp), _sz],
    "mf_host_free": [_vp],
    "mf_memcpy_h2d_async": [_vp, _vp, _sz, _vp],
    "mf_memcpy_d2h_async": [_vp, _vp, _sz, _vp],
    "mf_memcpy_d2d_async": [_vp, _vp, _sz, _vp],
    "mf_memset_async": [_vp, _int, _sz, _vp],
    "mf_stream_create": [ctypes.POINTER(_vp)],
    "mf_stream_destroy": [_vp],
    "mf_stream_sync": [_vp],
    "mf_event_create": [ctypes.POINTER(_vp), _int],
    "mf_event_destroy": [_vp],
    "mf_event_record": [_vp, _vp],
    "mf_stream_wait_event": [_vp, _vp],
    "mf_event_sync": [_vp],
    "mf_event_elapsed_ms": [_vp, _vp, ctypes.POINTER(_f32)],
    "mf_device_sync": [],
    "mf_convert": [_int, _int, _vp, _vp, _i64, _int, _vp],
    "mf_int4_dequant_grouped": [_vp, _vp, _int, _vp, _int, _i64, _i64, _i64, _vp],
    "mf_axpy": [_vp, _vp, _i64, _f32, _int, _int, _vp],
    "mf_scalar_broadcast": [_vp, _int, _vp, _int, _i64, _f32, _int, _vp],
    "mf_linspace": [_f32, _f32, _i64, _int, _vp, _int, _vp],
    "mf_fused_compile": [ctypes.POINTER(FusedProgram), ctypes.POINTER(_vp)],
    "mf_fused_destroy": [_vp],
    "mf_fused_is_specialised": [_vp, ctypes.POINTER(_int)],
    "mf_fused_launch": [_vp, ctypes.POINTER(_vp), _vp, _i64, _vp, _vp],
    "mf_amax": [_vp, _int, _i64, _vp, _vp],
    "mf_fp8_scaled_cast": [_vp, _int, _vp, _int, _vp, _vp, _i64, _int, _vp],
    "mf_fp8_quantize": [_vp, _int, _vp, _int, _vp, _vp, _i64, _int, _vp],
    "mf_fused_fp8": [_vp, ctypes.POINTER(_vp), _vp, _vp, _int, _vp, _vp, _i64, _int, _vp],
    "mf_ckpt_partition": [ctypes.POINTER(_i64), _i32, _i32, _i32, ctypes.POINTER(_i64), ctypes.POINTER(_i64)],
    "mf_comm_unique_id": [_vp],
    "mf_comm_init": [ctypes.POINTER(_vp), _i32, _i32, _vp],
    "mf_comm_destroy": [_vp],
    "mf_comm_allreduce_max_f32": [_vp, _vp, _i64, _vp],
    "mf_ckpt_amax_pass": [ctypes.POINTER(ChunkDesc), _i32, _i32, _vp, _vp],
    "mf_ckpt_cast_pass": [ctypes.POINTER(ChunkDesc), _i32, _i32, _vp, _vp, _int, _int, _vp],
    "mf_ckpt_quant_fp8": [ctypes.POINTER(ChunkDesc), _i32, _i32, _vp, _vp, _int, _int, _vp, _vp],
    "mf_ckpt_quant_fp8_noalloc": [ctypes.POINTER(ChunkDesc), _i32, _i32, _vp, _int, _int, _vp, _vp],
    "mf_bw_probe": [_vp, _int, _vp, _int, _i64, _vp],
    "mf_ckpt_plan_create": [ctypes.POINTER(ChunkDesc), _i32, _i32, ctypes.POINTER(_i64), _i64, _i32, _i32, _int, _int,
                            ctypes.POINTER(_vp), _vp],
    "mf_ckpt_plan_connect": [_vp, _vp],
    "mf_ckpt_plan_run": [_vp, _vp, _vp, _vp],
    "mf_ckpt_plan_run_passes": [_vp, _int, _vp, _vp, _vp],
    "mf_ckpt_plan_info": [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i64)],
    "mf_ckpt_plan_destroy": [_vp],
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load libmfcuda.so once; raises ImportError if it is absent."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build the CUDA library with `python -m manifesto_b200.build` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _int
        L.mf_last_error.argtypes = []
        L.mf_last_error.restype = ctypes.c_char_p
        _lib = L
    return _lib


def last_error() -> str:
    msg = lib().mf_last_error()
    return msg.decode() if msg else ""


def call(name: str, *args) -> None:
    """Call an mf_* entry point and raise the mapped exception on failure.

    Only entry points with a declared signature may be called: without
    argtypes ctypes would pass 64-bit pointers and stream handles as 32-bit
    ints.
    """
    if name not in SIGNATURES:
        raise KeyError(f"{name} has no declared ctypes signature in manifesto_b200._abi.SIGNATURES")
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise_for_status(rc, f"{name}: {last_error()}")
