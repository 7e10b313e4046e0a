"""manifesto_b200: a B200 (sm_100a) backend for manifesto's data-parallel hot path.

The path: dtype conversion (FP8 E4M3/E5M2, BF16, FP16, packed Int4 with group
scales, to and from FP32/BF16), the fused elementwise chains manifesto's
optimizer builds, the runtime's axpy / scalar-broadcast vector loops, and
per-tensor amax-scaled FP8 quantisation of whole checkpoints across the GPUs
of one node.  All arithmetic runs in libmfcuda.so (hand-written CUDA for
sm_100a behind a C ABI, include/mfcuda.h); this package is the host side
that mirrors manifesto's Go interfaces (tensor.Backend, tensor.Tensor,
axpyDevice, codegen targets) over that ABI.
"""
from . import _abi
from .backend import (COMPAT_OCP, COMPAT_REFERENCE, CUDABackend, DeviceBuffer, DeviceTensor, Event, PinnedBuffer,
                      Stream, convert_raw, device_count, sync_device)
from .dtype import DType
from .errors import MFError

__all__ = [
    "COMPAT_OCP", "COMPAT_REFERENCE", "CUDABackend", "DeviceBuffer", "DeviceTensor", "DType", "Event", "MFError",
    "PinnedBuffer", "Stream", "convert_raw", "device_count", "sync_device", "library_path", "abi_version",
]


def library_path() -> str:
    return str(_abi.LIB_PATH)


def abi_version() -> int:
    return _abi.lib().mf_abi_version()
