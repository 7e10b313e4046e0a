"""ctypes binding of the C oracle (oracle/libmfref.so) with numpy helpers.

TEST INFRASTRUCTURE (see oracle/__init__.py).  The C functions restate
manifesto's Go scalar code; this module only marshals numpy arrays and can
split element ranges over threads (ctypes releases the GIL during each call,
so the chunks run in parallel on the host cores).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libmfref.so"

# dtype wire codes, manifesto dtype/dtype.go:29-49
F64, F32, F16, BF16, E4M3, E5M2 = 1, 2, 3, 4, 5, 6
I64, I32, I16, I8, I4, U64, U32, U16, U8 = 7, 8, 9, 10, 11, 12, 13, 14, 15

ITEMSIZE = {F64: 8, F32: 4, F16: 2, BF16: 2, E4M3: 1, E5M2: 1, I64: 8, I32: 4, I16: 2, I8: 1,
            U64: 8, U32: 4, U16: 2, U8: 1}

_lib = None


def build() -> Path:
    """Compile libmfref.so with the committed Makefile (gcc, no FMA contraction)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        u8, u16, u32, i32, i64 = ctypes.c_uint8, ctypes.c_uint16, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int64
        vp = ctypes.c_void_p
        for name, res, args in [
            ("ref_e4m3_decode", u32, [u8]), ("ref_e4m3_encode", u8, [u32]), ("ref_e4m3_encode_ocp", u8, [u32]),
            ("ref_e5m2_decode", u32, [u8]), ("ref_e5m2_encode", u8, [u32]), ("ref_e5m2_encode_ocp", u8, [u32]),
            ("ref_bf16_encode", u16, [u32]), ("ref_bf16_decode", u32, [u16]),
            ("ref_f16_encode", u16, [u32]), ("ref_f16_decode", u32, [u16]),
            ("ref_int4_lo", ctypes.c_int8, [u8]), ("ref_int4_hi", ctypes.c_int8, [u8]),
            ("ref_int4_pair", u8, [ctypes.c_int8, ctypes.c_int8]),
            ("ref_decode_f32", ctypes.c_int, [ctypes.c_int, vp, vp, i64, i64]),
            ("ref_encode_f32", ctypes.c_int, [ctypes.c_int, vp, vp, i64, i64, ctypes.c_int]),
            ("ref_convert", ctypes.c_int, [ctypes.c_int, ctypes.c_int, vp, vp, i64, i64, ctypes.c_int]),
            ("ref_int4_dequant_grouped", ctypes.c_int, [vp, vp, ctypes.c_int, vp, ctypes.c_int, i64, i64, i64, i64, i64]),
            ("ref_axpy", ctypes.c_int, [vp, vp, i64, i64, ctypes.c_float, ctypes.c_int, ctypes.c_int]),
            ("ref_scalar_broadcast", ctypes.c_int, [vp, ctypes.c_int, vp, ctypes.c_int, i64, i64, ctypes.c_float, ctypes.c_int]),
            ("ref_linspace", ctypes.c_int, [ctypes.c_float, ctypes.c_float, i64, ctypes.c_int, vp, ctypes.c_int, i64, i64]),
            ("ref_fused_eval", ctypes.c_int, [ctypes.c_int, vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int, vp, vp, vp,
                                              vp, ctypes.c_int, i64, i64]),
            ("ref_amax", u32, [vp, ctypes.c_int, i64, i64]),
            ("ref_fp8_scale", ctypes.c_float, [ctypes.c_float, ctypes.c_int]),
            ("ref_scaled_cast", ctypes.c_int, [vp, ctypes.c_int, vp, ctypes.c_int, ctypes.c_float, i64, i64, ctypes.c_int]),
        ]:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def default_threads() -> int:
    return os.cpu_count() or 1


def _ranges(n: int, threads: int, align: int = 1):
    threads = max(1, min(threads, (n + align - 1) // align or 1))
    per = (n // threads) // align * align or align
    out, b = [], 0
    for t in range(threads):
        e = n if t == threads - 1 else min(n, b + per)
        if e > b:
            out.append((b, e - b))
        b = e
    return out


def _parallel(fn, n: int, threads: int, align: int = 1, work: int | None = None):
    """Split [0, n) over threads; `work` (default n) is the element count the small-job cutoff compares,
    for callers that split rows rather than elements."""
    rcs = []
    if threads <= 1 or (n if work is None else work) < 1 << 16:
        rcs.append(fn(0, n))
    else:
        with ThreadPoolExecutor(threads) as ex:
            rcs = list(ex.map(lambda r: fn(*r), _ranges(n, threads, align)))
    for rc in rcs:
        if rc != 0:
            raise RuntimeError(f"oracle call failed with status {rc}")


def raw_bytes(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint8).reshape(-1)


def convert(src: np.ndarray, src_dtype: int, dst_dtype: int, n: int | None = None, compat: int = 0,
            threads: int = 1) -> np.ndarray:
    """convert.BytesTo<dst>(src_dtype, bytes) element loop; returns raw codes."""
    src = np.ascontiguousarray(src)
    if n is None:
        n = src.nbytes * 2 if src_dtype == I4 else src.nbytes // ITEMSIZE[src_dtype]
    out = np.empty(n * ITEMSIZE[dst_dtype], dtype=np.uint8)
    L = lib()
    _parallel(lambda b, c: L.ref_convert(src_dtype, dst_dtype, _ptr(src), _ptr(out), b, c, compat), n, threads,
              align=2)
    return out.view({1: np.uint8, 2: np.uint16, 4: np.uint32}[ITEMSIZE[dst_dtype]])


def int4_dequant(q: np.ndarray, scales: np.ndarray, scale_dtype: int, out_dtype: int, rows: int, cols: int,
                 group: int, threads: int = 1) -> np.ndarray:
    q = np.ascontiguousarray(q)
    scales = np.ascontiguousarray(scales)
    out = np.empty(rows * cols * ITEMSIZE[out_dtype], dtype=np.uint8)
    L = lib()
    _parallel(lambda b, c: L.ref_int4_dequant_grouped(_ptr(q), _ptr(scales), scale_dtype, _ptr(out), out_dtype,
                                                      rows, cols, group, b, b + c), rows, threads,
              work=rows * cols)
    return out.view({2: np.uint16, 4: np.uint32}[ITEMSIZE[out_dtype]])


def axpy(y: np.ndarray, x: np.ndarray, alpha: float, dtype: int, fused: int = 0, threads: int = 1) -> np.ndarray:
    """Returns the updated copy of y (raw codes)."""
    y = np.array(y, copy=True)
    x = np.ascontiguousarray(x)
    n = y.size
    L = lib()
    _parallel(lambda b, c: L.ref_axpy(_ptr(y), _ptr(x), b, c, alpha, dtype, fused), n, threads)
    return y


def scalar_broadcast(src: np.ndarray, src_dtype: int, dst_dtype: int, scalar: float, op: int,
                     n: int | None = None, threads: int = 1) -> np.ndarray:
    src = np.ascontiguousarray(src)
    if n is None:
        n = src.nbytes * 2 if src_dtype == I4 else src.nbytes // ITEMSIZE[src_dtype]
    out = np.empty(n * ITEMSIZE[dst_dtype], dtype=np.uint8)
    L = lib()
    _parallel(lambda b, c: L.ref_scalar_broadcast(_ptr(src), src_dtype, _ptr(out), dst_dtype, b, c, scalar, op), n,
              threads, align=2)
    return out.view({2: np.uint16, 4: np.uint32}[ITEMSIZE[dst_dtype]])


def linspace(start: float, stop: float, count: int, endpoint: bool = True, dst_dtype: int = F32,
             threads: int = 1) -> np.ndarray:
    """runLinspace (runtime/executor_math.go:57-108) stored as dst_dtype; returns raw codes."""
    out = np.empty(count * ITEMSIZE[dst_dtype], dtype=np.uint8)
    L = lib()
    _parallel(lambda b, c: L.ref_linspace(start, stop, count, 1 if endpoint else 0, _ptr(out), dst_dtype, b, c),
              count, threads)
    return out


def fused_eval(tree: dict, inputs: list[np.ndarray], in_dtypes: list[int], in_bcast: list[int], out_dtype: int,
               n: int, threads: int = 1) -> np.ndarray:
    """evalCPU over a node table {type, value, input, child0, child1, root}."""
    t = np.ascontiguousarray(tree["type"], dtype=np.int32)
    v = np.ascontiguousarray(tree["value"], dtype=np.float64)
    inp = np.ascontiguousarray(tree["input"], dtype=np.int32)
    c0 = np.ascontiguousarray(tree["child0"], dtype=np.int32)
    c1 = np.ascontiguousarray(tree["child1"], dtype=np.int32)
    ins = [np.ascontiguousarray(a) for a in inputs]
    ptrs = (ctypes.c_void_p * max(1, len(ins)))(*[_ptr(a) for a in ins])
    dts = np.ascontiguousarray(in_dtypes, dtype=np.int32)
    bc = np.ascontiguousarray(in_bcast, dtype=np.int64)
    out = np.empty(n * ITEMSIZE[out_dtype], dtype=np.uint8)
    L = lib()
    _parallel(lambda b, c: L.ref_fused_eval(len(t), _ptr(t), _ptr(v), _ptr(inp), _ptr(c0), _ptr(c1), int(tree["root"]),
                                            len(ins), ctypes.cast(ptrs, ctypes.c_void_p), _ptr(dts), _ptr(bc),
                                            _ptr(out), out_dtype, b, c), n, threads)
    return out.view({2: np.uint16, 4: np.uint32}[ITEMSIZE[out_dtype]])


def amax(src: np.ndarray, src_dtype: int, threads: int = 1) -> float:
    src = np.ascontiguousarray(src)
    n = src.nbytes // ITEMSIZE[src_dtype]
    L = lib()
    ranges = _ranges(n, threads) if threads > 1 and n >= 1 << 16 else [(0, n)]
    if len(ranges) > 1:
        with ThreadPoolExecutor(len(ranges)) as ex:
            parts = list(ex.map(lambda r: L.ref_amax(_ptr(src), src_dtype, r[0], r[1]), ranges))
    else:
        parts = [L.ref_amax(_ptr(src), src_dtype, 0, n)]
    vals = np.array(parts, dtype=np.uint32).view(np.float32)
    return float(vals.max()) if len(vals) else 0.0


def fp8_scale(amax_value: float, fp8_dtype: int) -> float:
    return float(lib().ref_fp8_scale(amax_value, fp8_dtype))


def fp8_scale_inv(amax_value: float, fp8_dtype: int) -> float:
    """amax / fp8_max in float32 (1 when amax is 0 or not finite)."""
    a = np.float32(amax_value)
    if not (a > 0) or np.isinf(a):
        return 1.0
    fmax = np.float32(57344.0 if fp8_dtype == E5M2 else 448.0)
    return float(a / fmax)


def scaled_cast(src: np.ndarray, src_dtype: int, fp8_dtype: int, amax_value: float, compat: int = 0,
                threads: int = 1) -> np.ndarray:
    src = np.ascontiguousarray(src)
    n = src.nbytes // ITEMSIZE[src_dtype]
    out = np.empty(n, dtype=np.uint8)
    L = lib()
    _parallel(lambda b, c: L.ref_scaled_cast(_ptr(src), src_dtype, _ptr(out), fp8_dtype, amax_value, b, c, compat), n,
              threads)
    return out


# scalar helpers (vectorised with np.vectorize-free loops over small sets)
def e4m3_encode_all(bits: np.ndarray, compat: int = 0) -> np.ndarray:
    return convert(np.ascontiguousarray(bits, dtype=np.uint32), F32, E4M3, compat=compat)


def e5m2_encode_all(bits: np.ndarray, compat: int = 0) -> np.ndarray:
    return convert(np.ascontiguousarray(bits, dtype=np.uint32), F32, E5M2, compat=compat)
