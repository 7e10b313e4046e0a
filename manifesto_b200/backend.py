"""CUDA backend for manifesto's hot path, mirroring its Go interfaces.

* ``CUDABackend`` mirrors ``tensor.Backend`` (tensor/backend.go:18-68) for
  ``Location() == "cuda"`` plus the ``axpyDevice.Axpy`` capability
  (runtime/axpy.go:13-15) and the device halves of the dtype conversions.
* ``DeviceTensor`` mirrors ``tensor.Tensor`` (tensor/tensor.go:53-130) as a
  device-resident tensor: its native host views raise ``DTypeMismatch`` (like
  the reference's ``rawDeviceTensor`` test double, runtime/executor_test.go:713-758),
  ``raw_bytes`` materialises through a device-to-host copy, and
  ``dispatch_pointer`` returns the device address (runtime/axpy.go:17-20).

Every call goes through the C ABI of libmfcuda.so; nothing falls back to the
CPU.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Iterable, Sequence

import numpy as np

from . import _abi
from ._abi import call
from .dtype import DECODE_SOURCES, DType
from .errors import (DTypeMismatch, DTypeUnsupported, InvalidArgument, LayoutUnsupported, ShapeInvalid,
                     ShapeMismatch, TensorClosed)

LOCATION_CUDA = "cuda"
COMPAT_REFERENCE = 0
COMPAT_OCP = 1

# scalar-broadcast op names of math.scalar_broadcast (runtime/executor_math.go:202-233)
SCALAR_OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3}


# ----------------------------------------------------------------- plumbing

def device_count() -> int:
    c = ctypes.c_int(0)
    call("mf_device_count", ctypes.byref(c))
    return c.value


class Stream:
    """A CUDA stream (ir.Node.StreamID maps onto one of these)."""

    def __init__(self, handle: int | None = None, owned: bool = True):
        if handle is None:
            h = ctypes.c_void_p()
            call("mf_stream_create", ctypes.byref(h))
            handle, owned = h.value, True
        self.handle = handle
        self._owned = owned

    def sync(self) -> None:
        call("mf_stream_sync", self.handle)

    def wait(self, event: "Event") -> None:
        """SyncEvent{Wait: true} (ir/sync_event.go:14-26)."""
        call("mf_stream_wait_event", self.handle, event.handle)

    def close(self) -> None:
        if self._owned and self.handle:
            call("mf_stream_destroy", self.handle)
        self.handle = None


def stream_handle(stream: "Stream | int | None") -> int | None:
    if stream is None:
        return None
    if isinstance(stream, Stream):
        return stream.handle
    return int(stream)


class Event:
    """A CUDA event; record() is SyncEvent{Wait: false}."""

    def __init__(self, timing: bool = False):
        h = ctypes.c_void_p()
        call("mf_event_create", ctypes.byref(h), 1 if timing else 0)
        self.handle = h.value

    def record(self, stream: "Stream | int | None" = None) -> None:
        call("mf_event_record", self.handle, stream_handle(stream))

    def sync(self) -> None:
        call("mf_event_sync", self.handle)

    def elapsed_ms(self, end: "Event") -> float:
        ms = ctypes.c_float()
        call("mf_event_elapsed_ms", self.handle, end.handle, ctypes.byref(ms))
        return ms.value

    def close(self) -> None:
        if self.handle:
            call("mf_event_destroy", self.handle)
        self.handle = None


class DeviceBuffer:
    """A device allocation (256-byte aligned)."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        call("mf_alloc", ctypes.byref(p), int(nbytes))
        self.ptr = p.value or 0
        self.nbytes = int(nbytes)

    def free(self) -> None:
        if self.ptr:
            call("mf_free", self.ptr)
        self.ptr = 0

    def upload(self, host: np.ndarray, stream=None, offset: int = 0) -> None:
        host = np.ascontiguousarray(host)
        if host.nbytes + offset > self.nbytes:
            raise ShapeMismatch(f"upload of {host.nbytes} bytes at {offset} into a {self.nbytes}-byte buffer")
        call("mf_memcpy_h2d_async", self.ptr + offset, host.ctypes.data, host.nbytes, stream_handle(stream))
        if stream is None:
            call("mf_stream_sync", None)

    def download(self, nbytes: int | None = None, stream=None, offset: int = 0) -> np.ndarray:
        nbytes = self.nbytes - offset if nbytes is None else nbytes
        out = np.empty(nbytes, dtype=np.uint8)
        call("mf_memcpy_d2h_async", out.ctypes.data, self.ptr + offset, nbytes, stream_handle(stream))
        call("mf_stream_sync", stream_handle(stream))
        return out

    def memset(self, value: int = 0, stream=None) -> None:
        call("mf_memset_async", self.ptr, value, self.nbytes, stream_handle(stream))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.free()


class DeviceView(DeviceBuffer):
    """`nbytes` at `ptr` inside an allocation someone else owns (a slot of a graph's
    workspace): a tensor over it never frees it."""

    def __init__(self, ptr: int, nbytes: int):
        self.ptr = int(ptr)
        self.nbytes = int(nbytes)

    def free(self) -> None:
        self.ptr = 0


class PinnedBuffer:
    """Page-locked host memory viewed as a numpy byte array."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        call("mf_host_alloc", ctypes.byref(p), int(nbytes))
        self.ptr = p.value or 0
        self.nbytes = int(nbytes)
        self.array = (np.ctypeslib.as_array((ctypes.c_uint8 * self.nbytes).from_address(self.ptr))
                      if self.nbytes else np.empty(0, np.uint8))

    def free(self) -> None:
        if self.ptr:
            call("mf_host_free", self.ptr)
        self.ptr = 0
        self.array = None


# ------------------------------------------------------------------ tensors

@dataclass(frozen=True)
class Capabilities:
    """tensor.Capabilities (tensor/backend.go:82-110)."""

    max_bytes: int
    supports_async: bool
    supports_sparse: bool
    supports_autograd: bool
    native_alignment: int
    numa_nodes: int


def _shape_elements(shape: Sequence[int]) -> int:
    dims = tuple(int(d) for d in shape)
    if any(d < 0 for d in dims):
        raise ShapeInvalid(f"tensor: invalid shape {dims}")
    return math.prod(dims) if dims else 1


class DeviceTensor:
    """A dense tensor resident on the CUDA device."""

    def __init__(self, backend: "CUDABackend", shape: Sequence[int], dtype: DType, buffer: DeviceBuffer,
                 event: Event | None = None):
        self.backend = backend
        self._shape = tuple(int(d) for d in shape)
        self._dtype = DType(dtype)
        self._buffer = buffer
        self._event = event  # pending upload, if any
        self._closed = False

    def shape(self) -> tuple[int, ...]:
        return self._shape

    def dtype(self) -> DType:
        return self._dtype

    def layout(self) -> str:
        return "dense"

    def location(self) -> str:
        return LOCATION_CUDA

    def __len__(self) -> int:
        return _shape_elements(self._shape)

    def nbytes(self) -> int:
        return self._dtype.bytes_for(len(self))

    def _check_open(self) -> None:
        if self._closed:
            raise TensorClosed("tensor: closed")

    def dispatch_pointer(self) -> int:
        """Device address of the storage (the reference's DispatchPointer)."""
        self._check_open()
        return self._buffer.ptr

    def state(self) -> str:
        if self._closed:
            return "closed"
        return "pending" if self._event is not None else "ready"

    def ready(self) -> bool:
        return self.state() == "ready"

    def sync(self) -> None:
        """Wait for a pending upload and surface sticky device errors."""
        self._check_open()
        if self._event is not None:
            self._event.sync()
            self._event.close()
            self._event = None
        call("mf_device_status", None)

    def raw_bytes(self) -> bytes:
        self._check_open()
        self.sync()
        return self._buffer.download(self.nbytes()).tobytes()

    def float32_native(self):
        """Host views are not available for device tensors."""
        raise DTypeMismatch("tensor: dtype mismatch (device tensor has no host view)")

    bfloat16_native = float16_native = float32_native

    def close(self) -> None:
        if not self._closed:
            if self._event is not None:
                self._event.sync()
                self._event.close()
                self._event = None
            self._buffer.free()
            self._closed = True


class CUDABackend:
    """tensor.Backend for Location CUDA, plus the hot-path device operations."""

    _SUPPORTED = (DType.FLOAT32, DType.FLOAT16, DType.BFLOAT16, DType.FLOAT8_E4M3, DType.FLOAT8_E5M2, DType.INT4,
                  DType.INT32, DType.INT8, DType.UINT8, DType.INT64, DType.FLOAT64)

    def __init__(self, device: int = 0):
        call("mf_init", int(device))
        self.device = int(device)
        self._closed = False

    # -- tensor.Backend ---------------------------------------------------
    def location(self) -> str:
        return LOCATION_CUDA

    def supported_dtypes(self) -> list[DType]:
        return list(self._SUPPORTED)

    def supported_layouts(self) -> list[str]:
        return ["dense"]

    def capabilities(self) -> Capabilities:
        total = ctypes.c_size_t()
        call("mf_device_info", None, None, None, ctypes.byref(total))
        return Capabilities(max_bytes=total.value, supports_async=True, supports_sparse=False,
                            supports_autograd=False, native_alignment=128, numa_nodes=1)

    def _check(self) -> None:
        if self._closed:
            from .errors import BackendClosed
            raise BackendClosed("tensor: backend closed")

    def _host_bytes(self, shape, src_dtype: DType, data) -> np.ndarray:
        src_dtype = DType(src_dtype)
        if src_dtype not in self._SUPPORTED:
            raise DTypeUnsupported(f"tensor: dtype {src_dtype.name} not supported by backend")
        raw = np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray, memoryview)) else \
            np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        want = src_dtype.bytes_for(_shape_elements(shape))
        if raw.nbytes != want:
            raise ShapeMismatch(f"tensor: shape {tuple(shape)} x {src_dtype.name} needs {want} bytes, got {raw.nbytes}")
        return raw

    def upload(self, shape: Sequence[int], src_dtype: DType, data) -> DeviceTensor:
        """Copy host bytes to a new device tensor (the caller keeps `data`)."""
        self._check()
        raw = self._host_bytes(shape, src_dtype, data)
        buf = DeviceBuffer(max(raw.nbytes, 1))
        if raw.nbytes:
            buf.upload(raw)
        return DeviceTensor(self, shape, DType(src_dtype), buf)

    def upload_async(self, shape: Sequence[int], src_dtype: DType, data, stream=None) -> DeviceTensor:
        """Non-blocking upload; the tensor is pending until its event fires.

        ``data`` must stay alive and unmodified until the tensor is synced.
        """
        self._check()
        raw = self._host_bytes(shape, src_dtype, data)
        buf = DeviceBuffer(max(raw.nbytes, 1))
        ev = Event()
        if raw.nbytes:
            call("mf_memcpy_h2d_async", buf.ptr, raw.ctypes.data, raw.nbytes, stream_handle(stream))
        ev.record(stream)
        t = DeviceTensor(self, shape, DType(src_dtype), buf, event=ev)
        t._host_ref = raw  # keep the source alive until sync
        return t

    def upload_sparse(self, *args, **kwargs):
        raise LayoutUnsupported("tensor: layout not supported")

    def zeros(self, shape: Sequence[int], dtype: DType, stream=None) -> DeviceTensor:
        """Upload(shape, dtype, make([]byte, n)) without the host buffer: a device memset."""
        self._check()
        t = self.empty(shape, dtype)
        t._buffer.memset(0, stream)
        if stream is None:
            call("mf_stream_sync", None)
        return t

    def linspace(self, start: float, stop: float, count: int, endpoint: bool = True,
                 dtype: DType = DType.FLOAT32, stream=None) -> DeviceTensor:
        """math.linspace generated on the device in its storage dtype (F32, BF16 or F16)."""
        self._check()
        out = self.empty([int(count)], dtype)
        try:
            call("mf_linspace", float(start), float(stop), int(count), 1 if endpoint else 0, out.dispatch_pointer(),
                 int(dtype), stream_handle(stream))
        except BaseException:
            out.close()
            raise
        return out

    def upload_float32_as(self, shape: Sequence[int], dtype: DType, values, stream=None) -> DeviceTensor:
        """Upload(shape, dtype, Float32AsDTypeBytes(values, dtype)) with the encode on the device.

        Float32AsDTypeBytes (runtime/session.go:431-452) encodes BF16 and F16 and
        passes every other dtype through as float32 bytes; here the float32 values
        cross PCIe once and mf_convert encodes them with the same rounding.  Like
        the reference, a dtype that is none of F32/BF16/F16 gets float32 bytes and
        so fails Upload's byte-count check (ShapeMismatch)."""
        self._check()
        dtype = DType(dtype)
        vals = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        if dtype not in (DType.FLOAT32, DType.BFLOAT16, DType.FLOAT16):
            want = dtype.bytes_for(_shape_elements(shape))
            raise ShapeMismatch(f"tensor: shape {tuple(shape)} x {dtype.name} needs {want} bytes, got {vals.nbytes}")
        if vals.size != _shape_elements(shape):
            raise ShapeMismatch(f"tensor: shape {tuple(shape)} x {dtype.name} needs "
                                f"{dtype.bytes_for(_shape_elements(shape))} bytes, got "
                                f"{dtype.bytes_for(vals.size)}")
        if dtype == DType.FLOAT32:
            return self.upload(shape, dtype, vals)
        staged = self.upload(shape, DType.FLOAT32, vals)
        try:
            out = self.convert(staged, dtype, stream=stream)
            call("mf_stream_sync", stream_handle(stream))  # the staging copy is freed next
        finally:
            staged.close()
        return out

    def download(self, t: DeviceTensor) -> tuple[DType, bytes]:
        """Materialise a fresh host copy owned by the caller."""
        self._check()
        return t.dtype(), t.raw_bytes()

    def empty(self, shape: Sequence[int], dtype: DType) -> DeviceTensor:
        self._check()
        nbytes = DType(dtype).bytes_for(_shape_elements(shape))
        return DeviceTensor(self, shape, DType(dtype), DeviceBuffer(max(nbytes, 1)))

    def close(self) -> None:
        if not self._closed:
            call("mf_shutdown")
            self._closed = True

    # -- device operations ---------------------------------------------------
    def axpy(self, y: int, x: int, count: int, alpha: float, fmt: DType, stream=None, fused_fma: bool = False) -> None:
        """axpyDevice.Axpy(y, x, count, alpha, format): y += alpha * x in place.

        Like the Go interface it returns nothing; launch failures are raised
        here, device-side failures surface on the next DeviceTensor.sync().
        """
        call("mf_axpy", int(y), int(x), int(count), float(alpha), int(fmt), 1 if fused_fma else 0,
             stream_handle(stream))

    def convert(self, src: DeviceTensor, dst_dtype: DType, compat: int = COMPAT_REFERENCE,
                stream=None) -> DeviceTensor:
        """convert.BytesTo<dst>(src) on the device: a new tensor of dst_dtype."""
        if src.dtype() not in DECODE_SOURCES:
            raise DTypeUnsupported(f"convert: unsupported source dtype {src.dtype().name}")
        out = self.empty(src.shape(), dst_dtype)
        convert_raw(src.dtype(), dst_dtype, src.dispatch_pointer(), out.dispatch_pointer(), len(src), compat, stream)
        return out

    def scalar_broadcast(self, src: DeviceTensor, scalar: float, op: str, dst_dtype: DType | None = None,
                         stream=None) -> DeviceTensor:
        """math.scalar_broadcast (runtime/executor_math.go:195-234) on the device."""
        if op not in SCALAR_OPS:
            raise InvalidArgument(f"math.scalar_broadcast: unsupported op {op!r}")
        dst_dtype = DType(dst_dtype if dst_dtype is not None else
                          (src.dtype() if src.dtype() in (DType.FLOAT32, DType.FLOAT16, DType.BFLOAT16)
                           else DType.FLOAT32))
        out = self.empty(src.shape(), dst_dtype)
        call("mf_scalar_broadcast", src.dispatch_pointer(), int(src.dtype()), out.dispatch_pointer(), int(dst_dtype),
             len(src), float(scalar), SCALAR_OPS[op], stream_handle(stream))
        return out

    def int4_dequant(self, q: DeviceTensor, scales: DeviceTensor, group: int, out_dtype: DType = DType.BFLOAT16,
                     stream=None) -> DeviceTensor:
        rows, cols = q.shape()
        out = self.empty((rows, cols), out_dtype)
        call("mf_int4_dequant_grouped", q.dispatch_pointer(), scales.dispatch_pointer(), int(scales.dtype()),
             out.dispatch_pointer(), int(out_dtype), rows, cols, int(group), stream_handle(stream))
        return out


# ------------------------------------------------------------ raw wrappers

def convert_raw(src_dtype: DType, dst_dtype: DType, src: int, dst: int, n: int, compat: int = COMPAT_REFERENCE,
                stream=None) -> None:
    call("mf_convert", int(src_dtype), int(dst_dtype), int(src), int(dst), int(n), int(compat), stream_handle(stream))


def sync_device() -> None:
    call("mf_device_sync")


def supported_pairs() -> Iterable[tuple[DType, DType]]:
    from .dtype import ENCODE_TARGETS
    for s in DECODE_SOURCES:
        for d in ENCODE_TARGETS:
            yield s, d
