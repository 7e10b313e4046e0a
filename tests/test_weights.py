"""SafeTensors reader/writer (weights/reader.go) and dtype name parsing (dtype/dtype.go), on the CPU."""
import json
import struct

import numpy as np
import pytest

from manifesto_b200 import weights
from manifesto_b200.dtype import DType, parse


# dtype.Parse's accepted spellings (dtype/dtype.go:234-290) and DType.String (:185-232)
PARSE_CASES = {
    DType.FLOAT64: ["F64", "float64", "DOUBLE"], DType.FLOAT32: ["F32", "f32", "FLOAT", "single"],
    DType.FLOAT16: ["F16", "half"], DType.BFLOAT16: ["BF16", "bf16", "BFloat16", "brain_float16"],
    DType.FLOAT8_E4M3: ["F8_E4M3", "FP8_E4M3", "f8e4m3", "float8-e4m3"], DType.FLOAT8_E5M2: ["F8_E5M2", "fp8e5m2"],
    DType.INT64: ["I64", "long"], DType.INT32: ["I32", "int"], DType.INT16: ["short"], DType.INT8: ["I8", "byte"],
    DType.INT4: ["I4", "int4"], DType.UINT64: ["U64"], DType.UINT32: ["uint"], DType.UINT16: ["ushort"],
    DType.UINT8: ["U8", "ubyte"], DType.BOOL: ["BOOL", "b1"], DType.COMPLEX64: ["C64"], DType.COMPLEX128: ["complex128"],
}


@pytest.mark.parametrize("dt", list(PARSE_CASES))
def test_dtype_parse_aliases(dt):
    for name in PARSE_CASES[dt]:
        assert parse(name) == dt
        assert parse(f"  {name} ") == dt
    assert parse(dt.wire_name()) == dt


def test_dtype_parse_unknown_and_wire_names():
    with pytest.raises(ValueError, match='dtype: unknown dtype name "F7"'):
        parse("F7")
    assert DType.FLOAT8_E4M3.wire_name() == "F8E4M3" and DType.BFLOAT16.wire_name() == "BF16"
    assert DType.INVALID.wire_name() == "INVALID"


def sample_tensors():
    rng = np.random.default_rng(5)
    a = rng.standard_normal((3, 5)).astype(np.float32)
    b = rng.integers(-9, 9, (7,)).astype(np.int64)
    c = rng.integers(0, 255, (2, 2, 3)).astype(np.uint8)
    return [("layer.a", "F32", a.shape, a.tobytes()), ("layer.b", "I64", b.shape, b.tobytes()),
            ("c", "U8", c.shape, c.tobytes()), ("empty", "F32", (0, 4), b"")]


def test_write_then_index_and_read(tmp_path):
    p = tmp_path / "x.safetensors"
    ts = sample_tensors()
    weights.write_file(p, ts, meta={"format": "pt"})
    index, base = weights.index_file(p)
    assert set(index) == {t[0] for t in ts}
    (hlen,) = struct.unpack("<Q", p.read_bytes()[:8])
    assert base == hlen + 8 and base % 8 == 0
    off = 0
    for name, dt, shape, data in ts:
        m = index[name]
        assert (m.dtype, m.shape, m.data_offsets) == (dt, tuple(shape), (off, off + len(data)))
        got, meta = weights.read_tensor(p, name)
        assert got == data and meta == m
        off += len(data)
    assert weights.metadata(p) == {"format": "pt"}
    with open(p, "rb") as f:
        assert weights.index_reader(f) == (index, base)


def test_written_file_loads_in_safetensors(tmp_path):
    safetensors = pytest.importorskip("safetensors")
    torch = pytest.importorskip("torch")
    p = tmp_path / "y.safetensors"
    bf = torch.randn(4, 6).to(torch.bfloat16)
    f8 = torch.randn(16).to(torch.float8_e4m3fn)
    ts = [("w", "BF16", (4, 6), bf.view(torch.uint16).numpy().tobytes()),
          ("q", "F8_E4M3", (16,), f8.view(torch.uint8).numpy().tobytes())] + sample_tensors()[:3]
    weights.write_file(p, ts)
    with safetensors.safe_open(str(p), framework="pt") as f:
        assert torch.equal(f.get_tensor("w"), bf)
        assert torch.equal(f.get_tensor("q").view(torch.uint8), f8.view(torch.uint8))
        assert np.array_equal(f.get_tensor("layer.b").numpy(), np.frombuffer(ts[3][3], np.int64))


def test_reads_files_written_by_safetensors(tmp_path):
    st_torch = pytest.importorskip("safetensors.torch")
    torch = pytest.importorskip("torch")
    p = tmp_path / "z.safetensors"
    tensors = {"model.w": torch.randn(8, 3).to(torch.bfloat16), "model.n": torch.randn(3),
               "model.f8": torch.randn(5, 2).to(torch.float8_e5m2)}
    st_torch.save_file(tensors, str(p), metadata={"k": "v"})
    index, _ = weights.index_file(p)
    assert {n: parse(m.dtype) for n, m in index.items()} == {
        "model.w": DType.BFLOAT16, "model.n": DType.FLOAT32, "model.f8": DType.FLOAT8_E5M2}
    for n, t in tensors.items():
        data, meta = weights.read_tensor(p, n)
        assert meta.shape == tuple(t.shape)
        assert data == t.contiguous().view(torch.uint8).numpy().tobytes()
    assert weights.metadata(p) == {"k": "v"}


def _raw_file(tmp_path, header_obj=None, header_bytes=None, data=b"", length=None):
    hb = header_bytes if header_bytes is not None else json.dumps(header_obj).encode()
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", len(hb) if length is None else length) + hb + data)
    return p


def test_reader_errors_carry_the_reference_messages(tmp_path):
    empty = tmp_path / "e.safetensors"
    empty.write_bytes(b"")
    with pytest.raises(weights.SafeTensorsError, match="^safetensors index: EOF$"):
        weights.index_file(empty)
    short = tmp_path / "s.safetensors"
    short.write_bytes(b"\x01\x02\x03")
    with pytest.raises(weights.SafeTensorsError, match="^safetensors index: unexpected EOF$"):
        weights.index_file(short)
    with pytest.raises(weights.SafeTensorsError, match="^safetensors index: unexpected EOF$"):
        weights.index_file(_raw_file(tmp_path, {"a": {}}, length=1000))
    with pytest.raises(weights.SafeTensorsError, match="^safetensors index: "):
        weights.index_file(_raw_file(tmp_path, header_bytes=b"{not json"))
    with pytest.raises(weights.SafeTensorsError, match='^safetensors tensor "t": '):
        weights.index_file(_raw_file(tmp_path, {"t": [1, 2]}))
    p = _raw_file(tmp_path, {"__metadata__": {"a": "b"}, "t": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]}},
                  data=b"\x01\x02")
    index, _ = weights.index_file(p)
    assert list(index) == ["t"]  # __metadata__ is skipped
    with pytest.raises(weights.SafeTensorsError, match='^safetensors: missing tensor "u"$'):
        weights.read_tensor(p, "u")
    with pytest.raises(weights.SafeTensorsError, match='^safetensors read "t": '):
        weights.read_tensor(p, "t")  # 4 bytes promised, 2 present


def test_default_selection():
    m = lambda dt, shape: weights.TensorMeta(dt, tuple(shape), (0, 0))
    assert weights.default_select("w", m("BF16", [4, 4]))
    assert weights.default_select("w", m("F32", [2, 3, 4]))
    assert not weights.default_select("n", m("BF16", [4]))      # vectors stay
    assert not weights.default_select("i", m("I64", [4, 4]))    # not floating
    assert not weights.default_select("q", m("F8_E4M3", [4, 4]))
    assert not weights.default_select("z", m("BF16", [0, 4]))
    assert not weights.default_select("x", m("WEIRD", [4, 4]))
