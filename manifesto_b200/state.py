"""Runtime state on the device: MaterializeStateTensors and the float32 store path.

manifesto keeps graph state (tensors, paged tensors, page tables) in a StateStore and,
when the session has a tensor backend, makes it resident before the first graph call
(MaterializeStateTensors, runtime/session.go:160-205) and writes float32 vector results
of host ops back as resident tensors (writeFloat32VectorOutput,
runtime/executor_math.go:254-292).  Both encode the float32 values on the host first
(Float32AsDTypeBytes, runtime/session.go:431-452) and upload the result; page tables
and paged tensors upload host buffers of zeros.

Here the same steps run on the device: float32 values cross PCIe once and the
conversion kernel encodes them (CUDABackend.upload_float32_as, bit-identical to the
host encoders), and zero-filled storage is a device memset (CUDABackend.zeros).  The
checks, their order and their messages follow the reference.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Sequence

import numpy as np

from .backend import DeviceTensor
from .dtype import DType, parse

FLOAT_DTYPES = (DType.FLOAT64, DType.FLOAT32, DType.FLOAT16, DType.BFLOAT16, DType.FLOAT8_E4M3, DType.FLOAT8_E5M2)


class StateError(ValueError):
    """A state declaration or value the session cannot materialise."""


@dataclass
class StateDeclaration:
    """ast.StateDeclaration: the fields materialisation reads."""
    name: str
    type: str
    shape: list = field(default_factory=list)
    config: dict[str, Any] = field(default_factory=dict)


@dataclass
class PageTableState:
    """runtime.PageTableState: Storage becomes an Int32 [capacity] device tensor."""
    capacity: int
    storage: Any = None


@dataclass
class PagedTensorState:
    """runtime.PagedTensorState: Storage becomes a zeroed device tensor of Shape."""
    shape: list[int]
    storage: Any = None


class StateStore:
    """The name -> value map of runtime.StateStore (Get / Set)."""

    def __init__(self, values: dict[str, Any] | None = None):
        self._values = dict(values or {})

    def get(self, name: str) -> tuple[Any, bool]:
        if name in self._values:
            return self._values[name], True
        return None, False

    def set(self, name: str, value: Any) -> None:
        self._values[name] = value


def _go_type(v: Any) -> str:
    return type(v).__name__


def state_tensor_shape(decl: StateDeclaration) -> list[int]:
    """StateTensorShape (runtime/session.go:405-425): int, int64 and float64 dimensions."""
    dims = []
    for d in decl.shape:
        if isinstance(d, bool) or not isinstance(d, (int, float, np.integer, np.floating)):
            raise StateError(f"runtime session: unsupported state dimension {_go_type(d)}")
        dims.append(int(d))
    if any(d < 0 for d in dims):
        raise StateError(f"tensor: invalid shape {dims}")
    return dims


def state_storage_dtype(decl: StateDeclaration, fallback: DType) -> DType:
    """stateStorageDType (runtime/session.go:207-224)."""
    raw = decl.config.get("dtype")
    if not isinstance(raw, str) or raw == "":
        return fallback
    try:
        parsed = parse(raw)
    except ValueError:
        raise StateError(f'runtime session: state "{decl.name}" has invalid config dtype "{raw}"') from None
    if parsed in FLOAT_DTYPES or parsed == DType.INT32:
        return parsed
    raise StateError(f'runtime session: state "{decl.name}" has unsupported config dtype "{raw}"')


def _is_tensor(v: Any) -> bool:
    return isinstance(v, DeviceTensor) or (hasattr(v, "dispatch_pointer") and hasattr(v, "dtype"))


def materialize_state_tensors(store: StateStore | None, declarations: Sequence[StateDeclaration], memory,
                              storage_dtype: DType) -> None:
    """MaterializeStateTensors (runtime/session.go:160-205) with device-side encode and zero fill."""
    if store is None:
        raise StateError("runtime session: state store is required")
    if memory is None:
        raise StateError("runtime session: tensor backend is required")
    if DType(storage_dtype) not in FLOAT_DTYPES:
        raise StateError("runtime session: execution dtype is required for state materialization")
    for decl in declarations:
        if decl.type not in ("tensor", "paged_tensor", "page_table"):
            continue
        dt = state_storage_dtype(decl, DType(storage_dtype))
        if decl.type == "paged_tensor":
            _materialize_paged(store, decl, memory, dt)
        elif decl.type == "page_table":
            _materialize_page_table(store, decl, memory)
        else:
            _materialize_tensor(store, decl, memory, dt)


def _materialize_tensor(store: StateStore, decl: StateDeclaration, memory, dt: DType) -> None:
    value, ok = store.get(decl.name)
    if not ok or value is None or _is_tensor(value):
        return
    if isinstance(value, np.ndarray) and value.dtype == np.float32:
        values = value
    elif isinstance(value, list) and all(isinstance(v, float) for v in value):
        values = np.asarray(value, np.float32)
    else:
        raise StateError(f'runtime session: state "{decl.name}" is {_go_type(value)}, expected []float32')
    shape = state_tensor_shape(decl)
    if dt == DType.INT32:
        # the reference uploads len(values) * 4 zero bytes for the declared shape
        if len(values) != int(np.prod(shape, dtype=np.int64)):
            memory.upload(shape, DType.INT32, bytes(4 * len(values)))  # raises its shape mismatch
        store.set(decl.name, memory.zeros(shape, DType.INT32))
        return
    store.set(decl.name, memory.upload_float32_as(shape, dt, values))


def _materialize_page_table(store: StateStore, decl: StateDeclaration, memory) -> None:
    value, ok = store.get(decl.name)
    if not ok:
        return
    if not isinstance(value, PageTableState):
        raise StateError(f'runtime session: state "{decl.name}" is {_go_type(value)}, expected *PageTableState')
    if _is_tensor(value.storage):
        return
    value.storage = memory.zeros([max(int(value.capacity), 1)], DType.INT32)
    store.set(decl.name, value)


def _materialize_paged(store: StateStore, decl: StateDeclaration, memory, dt: DType) -> None:
    value, ok = store.get(decl.name)
    if not ok:
        return
    if not isinstance(value, PagedTensorState):
        raise StateError(f'runtime session: state "{decl.name}" is {_go_type(value)}, expected *PagedTensorState')
    if _is_tensor(value.storage):
        return
    shape = [int(d) for d in value.shape]
    if any(d < 0 for d in shape):
        raise StateError(f"tensor: invalid shape {shape}")
    value.storage = memory.zeros(shape, dt)
    store.set(decl.name, value)


@dataclass
class Float32VectorOutput:
    """runtime.float32VectorOutput: a host op's float32 result, its shape and storage format."""
    values: np.ndarray
    shape: list[int]
    format: DType


def write_float32_vector_output(values: dict[str, Any], reference: str, payload: Float32VectorOutput,
                                state: StateStore | None, state_memory) -> None:
    """writeFloat32VectorOutput (runtime/executor_math.go:254-292): a plain value stays a host
    copy; a "state.*" reference becomes a resident tensor encoded on the device."""
    copied = np.array(payload.values, dtype=np.float32, copy=True)
    if not reference.startswith("state."):
        values[reference] = copied
        return
    if state is None:
        raise StateError(f'state output "{reference}" requires a state store')
    output: Any = copied
    if state_memory is not None:
        output = state_memory.upload_float32_as(payload.shape, payload.format, copied)
    try:
        state.set(reference[len("state."):], output)
    except Exception:
        if _is_tensor(output):
            output.close()
        raise


# ------------------------------------------------------------- math.linspace

def _required_float32(config: dict[str, Any], key: str) -> float:
    """requiredFloat32FromConfig (runtime/executor_math.go:445-480)."""
    if key not in config:
        raise StateError(f"{key} is required")
    raw = config[key]
    if isinstance(raw, bool) or not isinstance(raw, (int, float, str, np.floating, np.integer)):
        raise StateError(f"{key} must be numeric, got {_go_type(raw)}")
    try:
        return float(np.float32(float(raw)))
    except ValueError as e:
        raise StateError(str(e)) from None


def _required_int(config: dict[str, Any], key: str) -> int:
    """requiredIntFromConfig / requiredIntFromAny (runtime/executor_math.go:387-443)."""
    if key not in config:
        raise StateError(f"{key} is required")
    raw = config[key]
    if isinstance(raw, bool) or not isinstance(raw, (int, float, str, np.integer)):
        raise StateError(f"expected integer, got {_go_type(raw)}")
    if isinstance(raw, str):
        # strconv.Atoi: an optional sign and decimal digits, nothing else
        body = raw[1:] if raw[:1] in "+-" else raw
        if not body.isascii() or not body.isdigit():
            raise StateError(f'strconv.Atoi: parsing "{raw}": invalid syntax')
        return int(raw)
    return int(raw)


def _float_dtype_from_config(config: dict[str, Any], fallback: DType) -> DType:
    """floatDTypeFromConfig (runtime/executor_math.go:361-385)."""
    if "dtype" not in config:
        return fallback
    raw = config["dtype"]
    if not isinstance(raw, str):
        raise StateError("dtype must be a string")
    try:
        fmt = parse(raw)
    except ValueError as e:
        raise StateError(str(e)) from None
    if fmt not in FLOAT_DTYPES:
        raise StateError(f"dtype {fmt.wire_name()} is not floating point")
    return fmt


def run_linspace(config: dict[str, Any], outputs: dict[str, str], values: dict[str, Any],
                 state: StateStore | None, state_memory) -> None:
    """runLinspace (runtime/executor_math.go:57-134) with the vector made on the device.

    A "state.*" output becomes a resident tensor generated straight into its storage
    dtype (no float32 host vector, no upload); any other output is the float32 host
    copy the reference keeps (generated on the device and read back when device
    memory is given).  Checks and messages follow the reference."""
    def wrap(fn, *args):
        try:
            return fn(*args)
        except StateError as e:
            raise StateError(f"math.linspace: {e}") from None
    start = wrap(_required_float32, config, "start")
    stop = wrap(_required_float32, config, "stop")
    count = wrap(_required_int, config, "count")
    if count <= 0:
        raise StateError("math.linspace: count must be positive")
    endpoint = config.get("endpoint")
    endpoint = endpoint if isinstance(endpoint, bool) else True
    fmt = wrap(_float_dtype_from_config, config, DType.FLOAT32)
    if not outputs:
        raise StateError("runtime vector output requires at least one target")
    host = None
    for reference in outputs.values():
        if reference.startswith("state.") and state is not None and state_memory is not None:
            if fmt not in (DType.FLOAT32, DType.BFLOAT16, DType.FLOAT16):
                # Float32AsDTypeBytes hands Upload float32 bytes for any other format
                from .errors import ShapeMismatch
                raise ShapeMismatch(f"tensor: shape ({count},) x {fmt.name} needs {fmt.bytes_for(count)} bytes, "
                                    f"got {4 * count}")
            t = state_memory.linspace(start, stop, count, endpoint, fmt)
            try:
                state.set(reference[len("state."):], t)
            except Exception:
                t.close()
                raise
            continue
        if reference.startswith("state.") and state is None:
            raise StateError(f'state output "{reference}" requires a state store')
        if host is None:
            if state_memory is not None:
                t = state_memory.linspace(start, stop, count, endpoint, DType.FLOAT32)
                host = np.frombuffer(t.raw_bytes(), np.float32).copy()
                t.close()
            else:
                raise StateError("math.linspace: a device backend is required")
        if reference.startswith("state."):
            state.set(reference[len("state."):], host.copy())
        else:
            values[reference] = host.copy()
