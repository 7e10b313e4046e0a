"""State materialisation and the float32 store path (runtime/session.go, executor_math.go) on the CPU."""
import numpy as np
import pytest

from manifesto_b200 import state
from manifesto_b200.dtype import DType


class FakeTensor:
    def __init__(self, shape, dtype, how):
        self.shape_, self.dtype_, self.how, self.closed = tuple(shape), DType(dtype), how, False

    def dispatch_pointer(self):
        return 1

    def dtype(self):
        return self.dtype_

    def close(self):
        self.closed = True


class FakeMemory:
    def __init__(self):
        self.calls = []

    def zeros(self, shape, dtype, stream=None):
        self.calls.append(("zeros", tuple(shape), DType(dtype)))
        return FakeTensor(shape, dtype, "zeros")

    def upload_float32_as(self, shape, dtype, values, stream=None):
        self.calls.append(("encode", tuple(shape), DType(dtype), len(values)))
        return FakeTensor(shape, dtype, "encode")

    def upload(self, shape, dtype, data):
        raise ValueError("shape mismatch")


def decl(name, typ="tensor", shape=(2, 3), **config):
    return state.StateDeclaration(name, typ, list(shape), config)


def test_materialize_tensor_state_per_declaration_dtype():
    mem = FakeMemory()
    st = state.StateStore({"a": np.zeros(6, np.float32), "b": [0.5] * 6, "i": np.ones(6, np.float32),
                           "skip_none": None, "already": FakeTensor((1,), DType.FLOAT32, "x"),
                           "pt": state.PageTableState(0), "pg": state.PagedTensorState([4, 8])})
    decls = [decl("a"), decl("b", dtype="f16"), decl("i", dtype="I32"), decl("skip_none"), decl("already"),
             decl("absent"), decl("pt", "page_table"), decl("pg", "paged_tensor", dtype="F32"),
             decl("other", "scalar")]
    state.materialize_state_tensors(st, decls, mem, DType.BFLOAT16)
    assert mem.calls == [("encode", (2, 3), DType.BFLOAT16, 6), ("encode", (2, 3), DType.FLOAT16, 6),
                         ("zeros", (2, 3), DType.INT32), ("zeros", (1,), DType.INT32),
                         ("zeros", (4, 8), DType.FLOAT32)]
    assert st.get("a")[0].how == "encode" and st.get("i")[0].dtype() == DType.INT32
    assert st.get("pt")[0].storage.how == "zeros" and st.get("pg")[0].storage.shape_ == (4, 8)
    state.materialize_state_tensors(st, decls, mem, DType.BFLOAT16)  # everything resident: no new work
    assert len(mem.calls) == 5


def test_materialize_errors_follow_the_reference():
    mem, st = FakeMemory(), state.StateStore({"x": "text", "p": 3, "q": np.zeros(6, np.float32)})
    with pytest.raises(state.StateError, match="state store is required"):
        state.materialize_state_tensors(None, [], mem, DType.FLOAT32)
    with pytest.raises(state.StateError, match="tensor backend is required"):
        state.materialize_state_tensors(st, [], None, DType.FLOAT32)
    with pytest.raises(state.StateError, match="execution dtype is required"):
        state.materialize_state_tensors(st, [], mem, DType.INT32)
    with pytest.raises(state.StateError, match=r'state "x" is str, expected \[\]float32'):
        state.materialize_state_tensors(st, [decl("x")], mem, DType.FLOAT32)
    with pytest.raises(state.StateError, match=r'state "p" is int, expected \*PageTableState'):
        state.materialize_state_tensors(st, [decl("p", "page_table")], mem, DType.FLOAT32)
    with pytest.raises(state.StateError, match='state "q" has invalid config dtype "F7"'):
        state.materialize_state_tensors(st, [decl("q", dtype="F7")], mem, DType.FLOAT32)
    with pytest.raises(state.StateError, match='state "q" has unsupported config dtype "I64"'):
        state.materialize_state_tensors(st, [decl("q", dtype="I64")], mem, DType.FLOAT32)
    with pytest.raises(state.StateError, match="unsupported state dimension str"):
        state.materialize_state_tensors(st, [decl("q", shape=("T", 3))], mem, DType.FLOAT32)


def test_state_shape_accepts_ints_and_floats():
    assert state.state_tensor_shape(decl("s", shape=(2, np.int64(3), 4.0))) == [2, 3, 4]


def test_write_float32_vector_output():
    mem, st, values = FakeMemory(), state.StateStore(), {}
    payload = state.Float32VectorOutput(np.arange(4, dtype=np.float32), [2, 2], DType.BFLOAT16)
    state.write_float32_vector_output(values, "h", payload, st, mem)
    assert np.array_equal(values["h"], payload.values) and values["h"] is not payload.values
    state.write_float32_vector_output(values, "state.h", payload, st, mem)
    assert st.get("h")[0].how == "encode" and mem.calls[-1] == ("encode", (2, 2), DType.BFLOAT16, 4)
    state.write_float32_vector_output(values, "state.k", payload, st, None)  # no resident memory: host copy
    assert isinstance(st.get("k")[0], np.ndarray)
    with pytest.raises(state.StateError, match='state output "state.h" requires a state store'):
        state.write_float32_vector_output(values, "state.h", payload, None, mem)


class FakeLinspaceMemory(FakeMemory):
    def linspace(self, start, stop, count, endpoint=True, dtype=DType.FLOAT32, stream=None):
        self.calls.append(("linspace", start, stop, count, endpoint, DType(dtype)))
        t = FakeTensor((count,), dtype, "linspace")
        t.raw_bytes = lambda: np.arange(count, dtype=np.float32).tobytes()
        return t


def test_run_linspace_routes_outputs_and_parses_config():
    mem, st, values = FakeLinspaceMemory(), state.StateStore(), {}
    cfg = {"start": "0.5", "stop": 2, "count": 4.0, "endpoint": False, "dtype": "bf16"}
    state.run_linspace(cfg, {"a": "state.grid", "b": "plain"}, values, st, mem)
    assert mem.calls[0] == ("linspace", 0.5, 2.0, 4, False, DType.BFLOAT16)
    assert st.get("grid")[0].how == "linspace"
    assert mem.calls[1][5] == DType.FLOAT32 and values["plain"].tolist() == [0.0, 1.0, 2.0, 3.0]
    state.run_linspace({"start": 1, "stop": 3, "count": "3"}, {"x": "v"}, values, st, mem)  # defaults: endpoint, F32
    assert mem.calls[-1][1:] == (1.0, 3.0, 3, True, DType.FLOAT32)


@pytest.mark.parametrize("cfg,msg", [
    ({"stop": 1, "count": 2}, "math.linspace: start is required"),
    ({"start": [1], "stop": 1, "count": 2}, "math.linspace: start must be numeric, got list"),
    ({"start": 0, "stop": 1}, "math.linspace: count is required"),
    ({"start": 0, "stop": 1, "count": " 5"}, 'math.linspace: strconv.Atoi: parsing " 5": invalid syntax'),
    ({"start": 0, "stop": 1, "count": 0}, "math.linspace: count must be positive"),
    ({"start": 0, "stop": 1, "count": 3, "dtype": 5}, "math.linspace: dtype must be a string"),
    ({"start": 0, "stop": 1, "count": 3, "dtype": "i32"}, "math.linspace: dtype I32 is not floating point"),
])
def test_run_linspace_errors(cfg, msg):
    with pytest.raises(state.StateError, match="^" + msg.replace("(", r"\(").replace(")", r"\)") + "$"):
        state.run_linspace(cfg, {"o": "v"}, {}, state.StateStore(), FakeLinspaceMemory())


def test_run_linspace_needs_a_target():
    with pytest.raises(state.StateError, match="requires at least one target"):
        state.run_linspace({"start": 0, "stop": 1, "count": 3}, {}, {}, state.StateStore(), FakeLinspaceMemory())
