"""Helpers for the GPU tests: numpy <-> device buffers through the C ABI."""
from __future__ import annotations

import numpy as np

from manifesto_b200 import DeviceBuffer, sync_device
from manifesto_b200._abi import call


def to_device(a: np.ndarray, pad: int = 0) -> DeviceBuffer:
    """Upload a copy of `a` (raw bytes); `pad` extra bytes are zero-filled."""
    raw = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
    buf = DeviceBuffer(max(1, raw.nbytes + pad))
    if pad:
        buf.memset(0)
    if raw.nbytes:
        buf.upload(raw)
    return buf


def empty(nbytes: int, fill: int | None = 0xA5) -> DeviceBuffer:
    buf = DeviceBuffer(max(1, nbytes))
    if fill is not None:
        buf.memset(fill)
    return buf


def fetch(buf: DeviceBuffer, nbytes: int, dtype=np.uint8, offset: int = 0) -> np.ndarray:
    sync_device()
    return buf.download(nbytes, offset=offset).view(dtype)


def convert(src: np.ndarray, src_dt: int, dst_dt: int, n: int, compat: int = 0, src_off: int = 0,
            dst_off: int = 0) -> np.ndarray:
    """Run mf_convert on device copies (optionally at byte offsets) and return the codes."""
    from oracle.ref import ITEMSIZE
    s = to_device(np.concatenate([np.zeros(src_off, np.uint8), np.ascontiguousarray(src).view(np.uint8).reshape(-1)]))
    osz = ITEMSIZE[dst_dt]
    d = empty(dst_off + n * osz + 64)
    call("mf_convert", src_dt, dst_dt, s.ptr + src_off, d.ptr + dst_off, n, compat, None)
    out = fetch(d, dst_off + n * osz + 64)
    # bytes past the output must be untouched (canary 0xA5)
    assert (out[dst_off + n * osz:] == 0xA5).all(), "kernel wrote past the end of its output"
    assert (out[:dst_off] == 0xA5).all(), "kernel wrote before the start of its output"
    s.free()
    d.free()
    return out[dst_off:dst_off + n * osz].view({1: np.uint8, 2: np.uint16, 4: np.uint32}[osz])


def bits_equal(a: np.ndarray, b: np.ndarray) -> None:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    bad = np.nonzero(a != b)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:8].tolist()}: got {a[bad[:8]].tolist()} " \
                          f"want {b[bad[:8]].tolist()}"
