"""Exceptions for C-ABI status codes.

Each class mirrors one sentinel of manifesto's tensor/errors.go:10-72, so
host code can branch on intent the same way the Go code uses errors.Is.
"""
from __future__ import annotations


class MFError(RuntimeError):
    """Base class: carries the C-ABI status code."""

    code = -1

    def __init__(self, message: str, code: int | None = None):
        super().__init__(message)
        if code is not None:
            self.code = code


class InvalidArgument(MFError, ValueError):
    code = -1


class DTypeMismatch(MFError):
    """tensor.ErrDTypeMismatch (tensor/errors.go:13)."""

    code = -2


class DTypeUnsupported(MFError):
    """tensor.ErrDTypeUnsupported (tensor/errors.go:18)."""

    code = -3


class LayoutUnsupported(MFError):
    """tensor.ErrLayoutUnsupported (tensor/errors.go:23)."""

    code = -4


class ShapeMismatch(MFError):
    """tensor.ErrShapeMismatch (tensor/errors.go:28)."""

    code = -5


class BackendClosed(MFError):
    """tensor.ErrBackendClosed (tensor/errors.go:46)."""

    code = -6


class ShapeInvalid(MFError):
    """tensor.ErrShapeInvalid (tensor/errors.go:50)."""

    code = -7


class NeedsPlatformSetup(MFError):
    """tensor.ErrNeedsPlatformSetup (tensor/errors.go:64)."""

    code = -8


class AllocatorExhausted(MFError, MemoryError):
    """tensor.ErrAllocatorExhausted (tensor/errors.go:71)."""

    code = -9


class CudaError(MFError):
    code = -10


class NcclError(MFError):
    code = -11


class DeviceStickyError(MFError):
    code = -12


class TensorClosed(MFError):
    """tensor.ErrTensorClosed (tensor/errors.go:42); host-side only."""

    code = -100


_BY_CODE = {c.code: c for c in (InvalidArgument, DTypeMismatch, DTypeUnsupported, LayoutUnsupported, ShapeMismatch,
                                BackendClosed, ShapeInvalid, NeedsPlatformSetup, AllocatorExhausted, CudaError,
                                NcclError, DeviceStickyError)}


def raise_for_status(code: int, message: str) -> None:
    cls = _BY_CODE.get(code, MFError)
    raise cls(message, code)
