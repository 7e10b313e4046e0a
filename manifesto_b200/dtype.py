"""Storage dtypes with manifesto's wire values (dtype/dtype.go:29-49).

Sizes, byte counts and element counts follow DType.Size / BytesFor /
LogicalElements (dtype/dtype.go:57-134): Int4 packs two elements per byte.
"""
from __future__ import annotations

import enum

import numpy as np


class DType(enum.IntEnum):
    INVALID = 0
    FLOAT64 = 1
    FLOAT32 = 2
    FLOAT16 = 3
    BFLOAT16 = 4
    FLOAT8_E4M3 = 5
    FLOAT8_E5M2 = 6
    INT64 = 7
    INT32 = 8
    INT16 = 9
    INT8 = 10
    INT4 = 11
    UINT64 = 12
    UINT32 = 13
    UINT16 = 14
    UINT8 = 15
    BOOL = 16
    COMPLEX64 = 17
    COMPLEX128 = 18

    @property
    def size(self) -> int:
        """DType.Size: bytes per element, 0 for the packed Int4 and Bool."""
        return _SIZE[self]

    def bytes_for(self, elements: int) -> int:
        """DType.BytesFor (dtype/dtype.go:81-100)."""
        if elements < 0:
            raise ValueError(f"dtype: negative element count {elements}")
        if self == DType.INT4:
            return (elements + 1) // 2
        if self == DType.BOOL:
            return (elements + 7) // 8
        if self.size == 0:
            raise ValueError(f"dtype: unsupported dtype {int(self)}")
        return elements * self.size

    def logical_elements(self, nbytes: int) -> int:
        """DType.LogicalElements (dtype/dtype.go:108-134)."""
        if nbytes < 0:
            raise ValueError(f"dtype: negative byte count {nbytes}")
        if self == DType.INT4:
            return nbytes * 2
        if self == DType.BOOL:
            return nbytes * 8
        if nbytes % self.size:
            raise ValueError(f"dtype: byte count {nbytes} is not a multiple of dtype size {self.size}")
        return nbytes // self.size

    @property
    def storage_numpy(self) -> np.dtype:
        """numpy dtype holding the raw storage codes of one element."""
        return _NP[self]

    def wire_name(self) -> str:
        """DType.String (dtype/dtype.go:185-232): the uppercase serialised identifier."""
        return _WIRE.get(self, f"DTYPE({int(self)})")


def parse(name: str) -> DType:
    """dtype.Parse (dtype/dtype.go:234-290): SafeTensors-style uppercase names, the
    lowercase forms and the aliases, ignoring case, '_' and '-' ("F8_E4M3" is
    FLOAT8_E4M3).  Raises ValueError for an unknown name."""
    key = name.strip().upper().replace("_", "").replace("-", "")
    for dt, names in _PARSE.items():
        if key in names:
            return dt
    raise ValueError(f'dtype: unknown dtype name "{name}"')


_SIZE = {
    DType.INVALID: 0, DType.FLOAT64: 8, DType.FLOAT32: 4, DType.FLOAT16: 2, DType.BFLOAT16: 2,
    DType.FLOAT8_E4M3: 1, DType.FLOAT8_E5M2: 1, DType.INT64: 8, DType.INT32: 4, DType.INT16: 2, DType.INT8: 1,
    DType.INT4: 0, DType.UINT64: 8, DType.UINT32: 4, DType.UINT16: 2, DType.UINT8: 1, DType.BOOL: 0,
    DType.COMPLEX64: 8, DType.COMPLEX128: 16,
}

_NP = {
    DType.FLOAT64: np.dtype(np.float64), DType.FLOAT32: np.dtype(np.uint32), DType.FLOAT16: np.dtype(np.uint16),
    DType.BFLOAT16: np.dtype(np.uint16), DType.FLOAT8_E4M3: np.dtype(np.uint8), DType.FLOAT8_E5M2: np.dtype(np.uint8),
    DType.INT64: np.dtype(np.int64), DType.INT32: np.dtype(np.int32), DType.INT16: np.dtype(np.int16),
    DType.INT8: np.dtype(np.int8), DType.INT4: np.dtype(np.uint8), DType.UINT64: np.dtype(np.uint64),
    DType.UINT32: np.dtype(np.uint32), DType.UINT16: np.dtype(np.uint16), DType.UINT8: np.dtype(np.uint8),
}

_WIRE = {
    DType.FLOAT64: "F64", DType.FLOAT32: "F32", DType.FLOAT16: "F16", DType.BFLOAT16: "BF16",
    DType.FLOAT8_E4M3: "F8E4M3", DType.FLOAT8_E5M2: "F8E5M2", DType.INT64: "I64", DType.INT32: "I32",
    DType.INT16: "I16", DType.INT8: "I8", DType.INT4: "I4", DType.UINT64: "U64", DType.UINT32: "U32",
    DType.UINT16: "U16", DType.UINT8: "U8", DType.BOOL: "BOOL", DType.COMPLEX64: "C64", DType.COMPLEX128: "C128",
    DType.INVALID: "INVALID",
}

_PARSE = {
    DType.FLOAT64: ("F64", "FLOAT64", "DOUBLE"), DType.FLOAT32: ("F32", "FLOAT32", "FLOAT", "SINGLE"),
    DType.FLOAT16: ("F16", "FLOAT16", "HALF"), DType.BFLOAT16: ("BF16", "BFLOAT16", "BRAINFLOAT16"),
    DType.FLOAT8_E4M3: ("F8E4M3", "FP8E4M3", "FLOAT8E4M3"), DType.FLOAT8_E5M2: ("F8E5M2", "FP8E5M2", "FLOAT8E5M2"),
    DType.INT64: ("I64", "INT64", "LONG"), DType.INT32: ("I32", "INT32", "INT"), DType.INT16: ("I16", "INT16", "SHORT"),
    DType.INT8: ("I8", "INT8", "BYTE"), DType.INT4: ("I4", "INT4"), DType.UINT64: ("U64", "UINT64", "ULONG"),
    DType.UINT32: ("U32", "UINT32", "UINT"), DType.UINT16: ("U16", "UINT16", "USHORT"),
    DType.UINT8: ("U8", "UINT8", "UBYTE"), DType.BOOL: ("BOOL", "BOOLEAN", "B1"),
    DType.COMPLEX64: ("C64", "COMPLEX64"), DType.COMPLEX128: ("C128", "COMPLEX128"),
}

# Formats the conversion kernels encode to (dtype/convert/convert.go:148-228)
ENCODE_TARGETS = (DType.FLOAT32, DType.FLOAT16, DType.BFLOAT16, DType.FLOAT8_E4M3, DType.FLOAT8_E5M2)
# Formats the conversion kernels decode from (convert.BytesToFloat32, convert.go:85-146)
DECODE_SOURCES = tuple(d for d in DType if d not in (DType.INVALID, DType.BOOL, DType.COMPLEX64, DType.COMPLEX128))
