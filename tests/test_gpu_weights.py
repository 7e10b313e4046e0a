"""SafeTensors checkpoint -> FP8 SafeTensors checkpoint through the GPU (weights.quantize_file)."""
import numpy as np
import pytest

from manifesto_b200 import synthetic, weights
from manifesto_b200.dtype import DType, parse
from oracle.ref import BF16, E4M3, E5M2, F16, F32

from .conftest import host_threads

pytestmark = pytest.mark.gpu

WIRE = {BF16: "BF16", F16: "F16", F32: "F32"}


def make_checkpoint(path):
    """(name, oracle dtype or None for pass-through, shape, raw array) in file order."""
    rng = np.random.default_rng(17)

    def bf16(shape, sigma=0.02):
        return synthetic.f32_to_bf16_bits((rng.standard_normal(shape) * sigma).astype(np.float32))

    nan = bf16((8, 8), 1.0)
    nan[0, 0], nan[3, 5], nan[7, 7] = 0x7FC0, 0xFFC1, 0x7F80  # NaN, -NaN, +Inf
    ts = [
        ("embed.weight", BF16, (1000, 64), bf16((1000, 64))),          # larger than a batch
        ("layers.0.q.weight", BF16, (64, 64), bf16((64, 64))),
        ("layers.0.norm.weight", None, (64,), bf16((64,), 1.0)),        # a vector: copied through
        ("layers.0.up.weight", F16, (96, 64), (rng.standard_normal((96, 64)) * 3).astype(np.float16).view(np.uint16)),
        ("layers.0.down.weight", F32, (64, 96), (rng.standard_normal((64, 96)) * 1e-3).astype(np.float32).view(np.uint32)),
        ("ragged.weight", BF16, (7, 13), bf16((7, 13), 5.0)),          # 91 elements
        ("zeros.weight", BF16, (16, 16), np.zeros((16, 16), np.uint16)),
        ("nan.weight", BF16, (8, 8), nan),
        ("step", None, (1,), np.array([12345], np.int64)),
    ]
    wire = lambda dt, a: WIRE[dt] if dt is not None else ("BF16" if a.dtype == np.uint16 else "I64")
    weights.write_file(path, [(n, wire(dt, a), shp, a.tobytes()) for n, dt, shp, a in ts], meta={"src": "test"})
    return ts


@pytest.mark.parametrize("fp8,compat", [(E4M3, 0), (E5M2, 0), (E4M3, 1)])
def test_quantize_file_bit_exact(backend, ref, tmp_path, fp8, compat):
    src, dst = tmp_path / "in.safetensors", tmp_path / "out.safetensors"
    ts = make_checkpoint(src)
    rep = weights.quantize_file(src, dst, DType(fp8), compat=compat, batch_bytes=40_000)
    quantised = [t for t in ts if t[1] is not None]
    assert rep.quantized == len(quantised) and rep.tensors == len(ts) and rep.batches >= 3
    assert rep.params == sum(a.size for _, _, _, a in quantised)
    index, _ = weights.index_file(dst)
    assert set(index) == {t[0] for t in ts} | {t[0] + "_scale_inv" for t in quantised}
    assert weights.metadata(dst)["src"] == "test"
    for name, dt, shape, a in ts:
        data, meta = weights.read_tensor(dst, name)
        if dt is None:
            assert data == a.tobytes() and meta.shape == shape
            continue
        assert parse(meta.dtype) == DType(fp8) and meta.shape == shape
        amax = ref.amax(a.reshape(-1), dt)
        want = ref.scaled_cast(a.reshape(-1), dt, fp8, amax, compat, threads=host_threads())
        assert np.array_equal(np.frombuffer(data, np.uint8), want), name
        sinv_bytes, smeta = weights.read_tensor(dst, name + "_scale_inv")
        assert smeta.dtype == "F32" and smeta.shape == ()
        sinv = float(np.frombuffer(sinv_bytes, np.float32)[0])
        assert sinv == ref.fp8_scale_inv(amax, fp8) == rep.scale_inv[name], name
    assert rep.scale_inv["zeros.weight"] == 1.0


def test_quantized_file_loads_in_safetensors(backend, tmp_path):
    """The output opens with the safetensors package as float8_e4m3fn + float32 scales.  With OCP
    rounding (compat=1) q * scale_inv is within E4M3 precision of the source; in reference mode
    every |v * scale| >= 248 saturates to 0x7e (448), so the top of the range reads back as +-amax."""
    safetensors = pytest.importorskip("safetensors")
    torch = pytest.importorskip("torch")
    src = tmp_path / "in.safetensors"
    make_checkpoint(src)
    w, _ = weights.read_tensor(src, "layers.0.q.weight")
    w = torch.frombuffer(bytearray(w), dtype=torch.bfloat16).float().reshape(64, 64)
    amax = float(w.abs().max())
    for compat in (1, 0):
        dst = tmp_path / f"out{compat}.safetensors"
        weights.quantize_file(src, dst, compat=compat)
        with safetensors.safe_open(str(dst), framework="pt") as f:
            q = f.get_tensor("layers.0.q.weight")
            s = f.get_tensor("layers.0.q.weight_scale_inv")
            assert q.dtype == torch.float8_e4m3fn and tuple(q.shape) == (64, 64) and s.dtype == torch.float32
            assert f.get_tensor("layers.0.norm.weight").dtype == torch.bfloat16
        deq = q.float() * s
        assert float(s) == pytest.approx(amax / 448.0, rel=1e-6)
        if compat:
            assert torch.allclose(deq, w, rtol=0.07, atol=float(s) * 2)
        else:
            top = w.abs() * (448.0 / amax) >= 248.0
            assert top.any()
            assert torch.equal(deq[top].abs(), torch.full_like(deq[top], 448.0 * float(s)))
            assert torch.allclose(deq[~top], w[~top], rtol=0.07, atol=float(s) * 8)


def test_quantize_file_rejects(backend, tmp_path):
    src = tmp_path / "in.safetensors"
    weights.write_file(src, [("w", "BF16", (2, 2), b"\0" * 8), ("w_scale_inv", "F32", (), b"\0" * 4)])
    with pytest.raises(weights.SafeTensorsError, match="name taken"):
        weights.quantize_file(src, tmp_path / "o.safetensors")
    with pytest.raises(ValueError, match="not an FP8 dtype"):
        weights.quantize_file(src, tmp_path / "o.safetensors", DType.BFLOAT16)
    bad = tmp_path / "bad.safetensors"
    weights.write_file(bad, [("w", "BF16", (4, 4), b"\0" * 8)])  # 8 bytes for 16 BF16 elements
    with pytest.raises(weights.SafeTensorsError, match="8 bytes for shape"):
        weights.quantize_file(bad, tmp_path / "o.safetensors")
