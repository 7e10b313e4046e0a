"""State materialisation on the device: encodes bit-identical to Float32AsDTypeBytes, zero fills."""
import numpy as np
import pytest

from manifesto_b200 import state, synthetic
from manifesto_b200.dtype import DType
from manifesto_b200.errors import ShapeMismatch
from oracle.ref import BF16, F16, F32

pytestmark = pytest.mark.gpu


def special_f32(n, seed):
    v = synthetic.normal_f32(seed, n, 0.0, 100.0)
    bits = v.view(np.uint32)
    bits[:8] = [0x7FC00000, 0xFFC00001, 0x7F800000, 0xFF800000, 0x00000001, 0x807FFFFF, 0x7F7FFFFF, 0x33800000]
    return v


@pytest.mark.parametrize("dt,oracle_dt", [(DType.BFLOAT16, BF16), (DType.FLOAT16, F16), (DType.FLOAT32, F32)])
def test_materialized_state_is_bit_exact(backend, ref, dt, oracle_dt):
    n = 3 * 1001
    vals = special_f32(n, 11)
    st = state.StateStore({"kv": vals, "table": state.PageTableState(16), "pages": state.PagedTensorState([5, 7])})
    decls = [state.StateDeclaration("kv", "tensor", [3, 1001]),
             state.StateDeclaration("table", "page_table"),
             state.StateDeclaration("pages", "paged_tensor", [], {"dtype": "bf16"})]
    state.materialize_state_tensors(st, decls, backend, dt)
    kv = st.get("kv")[0]
    assert kv.shape() == (3, 1001) and kv.dtype() == dt
    want = ref.convert(vals, F32, oracle_dt)
    assert backend.download(kv)[1] == want.tobytes()
    table = st.get("table")[0].storage
    assert table.dtype() == DType.INT32 and backend.download(table)[1] == bytes(64)
    pages = st.get("pages")[0].storage
    assert pages.dtype() == DType.BFLOAT16 and backend.download(pages)[1] == bytes(70)
    for t in (kv, table, pages):
        t.close()


def test_store_path_and_reference_byte_count_failure(backend, ref):
    st, values = state.StateStore(), {}
    v = special_f32(4096, 12)
    state.write_float32_vector_output(values, "state.h", state.Float32VectorOutput(v, [64, 64], DType.BFLOAT16),
                                      st, backend)
    h = st.get("h")[0]
    assert backend.download(h)[1] == ref.convert(v, F32, BF16).tobytes()
    h.close()
    # Float32AsDTypeBytes passes FP8 through as float32 bytes, which Upload rejects
    with pytest.raises(ShapeMismatch):
        backend.upload_float32_as([64, 64], DType.FLOAT8_E4M3, v)


@pytest.mark.parametrize("start,stop,count,endpoint", [
    (0.0, 1.0, 1, True), (0.0, 1.0, 2, True), (0.0, 1.0, 5, False), (-3.25, 17.5, 100003, True),
    (1e30, -1e30, 4097, False), (0.0, 1.0, (1 << 24) + 17, True), (float("nan"), 2.0, 33, True),
    (1.0, float("inf"), 9, True), (5.0, 5.0, 1000, False)])
@pytest.mark.parametrize("dt,oracle_dt", [(DType.FLOAT32, F32), (DType.BFLOAT16, BF16), (DType.FLOAT16, F16)])
def test_linspace_bit_exact(backend, ref, start, stop, count, endpoint, dt, oracle_dt):
    t = backend.linspace(start, stop, count, endpoint, dt)
    assert t.shape() == (count,) and t.dtype() == dt
    want = ref.linspace(start, stop, count, endpoint, oracle_dt, threads=4)
    assert backend.download(t)[1] == want.tobytes()
    t.close()


def test_run_linspace_on_the_device(backend, ref):
    st, values = state.StateStore(), {}
    state.run_linspace({"start": -1, "stop": 1, "count": 257, "dtype": "f16"},
                       {"grid": "state.grid", "copy": "grid_host"}, values, st, backend)
    g = st.get("grid")[0]
    assert g.dtype() == DType.FLOAT16 and backend.download(g)[1] == ref.linspace(-1.0, 1.0, 257, True, F16).tobytes()
    assert values["grid_host"].tobytes() == ref.linspace(-1.0, 1.0, 257, True, F32).tobytes()
    g.close()
    with pytest.raises(ShapeMismatch):  # Float32AsDTypeBytes passes FP8 through as float32 bytes
        state.run_linspace({"start": 0, "stop": 1, "count": 8, "dtype": "F8_E4M3"}, {"q": "state.q"}, values, st,
                           backend)
