"""K4 Int4 group dequant, K5 axpy and K6 scalar broadcast on the GPU (bit-exact)."""
import numpy as np
import pytest

from manifesto_b200 import synthetic
from manifesto_b200._abi import call, lib
from oracle.ref import BF16, E4M3, F16, F32, I4, I8, ITEMSIZE

from .conftest import host_threads
from .gpu_util import bits_equal, empty, fetch, to_device

pytestmark = pytest.mark.gpu


def run_int4(q, s, sdt, odt, rows, cols, group):
    dq, ds = to_device(q), to_device(s)
    nbytes = rows * cols * ITEMSIZE[odt]
    d = empty(nbytes + 64)
    call("mf_int4_dequant_grouped", dq.ptr, ds.ptr, sdt, d.ptr, odt, rows, cols, group, None)
    out = fetch(d, nbytes + 64)
    assert (out[nbytes:] == 0xA5).all()
    for b in (dq, ds, d):
        b.free()
    return out[:nbytes].view({2: np.uint16, 4: np.uint32}[ITEMSIZE[odt]])


def test_int4_config2_full_shape(backend, ref):
    """Config 2: 4096 x 14336 packed nibbles, BF16 scale per 128 along K, BF16 out."""
    rows, cols, group = 4096, 14336, 128
    q = synthetic.uniform_bytes(synthetic.CONFIG_SEED + 2, rows * cols // 2)
    s = synthetic.abs_normal_bf16(synthetic.CONFIG_SEED + 3, rows * (cols // group), 0.02)
    got = run_int4(q, s, BF16, BF16, rows, cols, group)
    bits_equal(got, ref.int4_dequant(q, s, BF16, BF16, rows, cols, group, threads=host_threads()))


@pytest.mark.parametrize("rows,cols,group", [(1, 32, 32), (3, 64, 32), (7, 256, 128), (5, 96, 48), (2, 10, 4),
                                             (4, 130, 128), (1, 2, 1), (3, 136, 64), (300, 2048, 256)])
@pytest.mark.parametrize("sdt,odt", [(BF16, BF16), (F16, F32), (F32, F16), (F32, BF16)])
def test_int4_shapes_and_dtypes(backend, ref, rows, cols, group, sdt, odt):
    q = synthetic.uniform_bytes(rows * 1000 + cols, rows * cols // 2)
    ng = (cols + group - 1) // group
    if sdt == BF16:
        s = synthetic.abs_normal_bf16(7, rows * ng, 0.02)
    elif sdt == F16:
        s = np.abs(synthetic.normal_f32(7, rows * ng, 0, 0.02)).astype(np.float16).view(np.uint16)
    else:
        s = synthetic.normal_f32(7, rows * ng, 0, 3.0)
    bits_equal(run_int4(q, s, sdt, odt, rows, cols, group), ref.int4_dequant(q, s, sdt, odt, rows, cols, group))


def test_int4_golden_hash(backend, golden):
    import hashlib
    q = synthetic.uniform_bytes(synthetic.CONFIG_SEED + 2, 64 * 128)
    s = synthetic.abs_normal_bf16(synthetic.CONFIG_SEED + 3, 64 * 2, 0.02)
    got = run_int4(q, s, BF16, BF16, 64, 256, 128)
    assert hashlib.sha256(got.tobytes()).hexdigest() == golden["oracle"]["int4_64x256_g128_sha256"]


def test_int4_nonfinite_scales(backend, ref):
    rows, cols, group = 2, 256, 128
    q = synthetic.uniform_bytes(3, rows * cols // 2)
    s = np.array([0x7F80, 0xFFC1, 0x0001, 0x8000], dtype=np.uint16)  # inf, NaN, subnormal, -0
    bits_equal(run_int4(q, s, BF16, BF16, rows, cols, group), ref.int4_dequant(q, s, BF16, BF16, rows, cols, group))


def test_int4_rejects_bad_shapes(backend):
    L = lib()
    assert L.mf_int4_dequant_grouped(1, 1, BF16, 1, BF16, 4, 7, 2, None) == -7  # odd cols
    assert L.mf_int4_dequant_grouped(1, 1, BF16, 1, BF16, 4, 8, 0, None) == -1
    assert L.mf_int4_dequant_grouped(1, 1, I8, 1, BF16, 4, 8, 2, None) == -3


# ------------------------------------------------------------------ axpy

def run_axpy(y, x, alpha, dt, fused=0):
    dy, dx = to_device(y), to_device(x)
    call("mf_axpy", dy.ptr, dx.ptr, y.size, alpha, dt, fused, None)
    out = fetch(dy, y.nbytes, y.dtype)
    dy.free()
    dx.free()
    return out


def test_axpy_known_answers(backend, golden):
    case = golden["known_answers"]["axpy_f32"]
    y = np.array(case["y"], np.float32)
    x = np.array(case["x"], np.float32)
    assert run_axpy(y, x, case["alpha"], F32).tolist() == case["out"]
    case = golden["known_answers"]["axpy_bf16"]
    yb = synthetic.f32_to_bf16_bits(np.array(case["y"], np.float32))
    xb = synthetic.f32_to_bf16_bits(np.array(case["x"], np.float32))
    out = run_axpy(yb, xb, case["alpha"], BF16)
    assert (out.astype(np.uint32) << 16).view(np.float32).tolist() == case["out"]


def test_axpy_golden_hash(backend, golden):
    import hashlib
    x = synthetic.normal_f32(synthetic.CONFIG_SEED + 4, 4099)
    y = synthetic.normal_f32(synthetic.CONFIG_SEED + 5, 4099)
    h = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    assert h(run_axpy(y.view(np.uint32), x.view(np.uint32), 0.75, F32)) == golden["oracle"]["axpy_f32_4099_sha256"]
    xb, yb = synthetic.f32_to_bf16_bits(x), synthetic.f32_to_bf16_bits(y)
    assert h(run_axpy(yb, xb, 0.75, BF16)) == golden["oracle"]["axpy_bf16_4099_sha256"]


@pytest.mark.parametrize("dt", [F32, BF16, F16])
@pytest.mark.parametrize("n", [1, 17, 65536 + 5])
@pytest.mark.parametrize("fused", [0, 1])
def test_axpy_matches_oracle(backend, ref, dt, n, fused):
    x = synthetic.normal_f32(n, n)
    y = synthetic.normal_f32(n + 1, n)
    if dt == BF16:
        x, y = synthetic.f32_to_bf16_bits(x), synthetic.f32_to_bf16_bits(y)
    elif dt == F16:
        x, y = x.astype(np.float16).view(np.uint16), y.astype(np.float16).view(np.uint16)
    else:
        x, y = x.view(np.uint32), y.view(np.uint32)
    bits_equal(run_axpy(y, x, 0.75, dt, fused), ref.axpy(y, x, 0.75, dt, fused))


@pytest.mark.parametrize("dt", [F32, BF16])
@pytest.mark.parametrize("fused", [0, 1])
def test_axpy_special_values(backend, ref, dt, fused):
    """NaN payloads, infinities, zeros and huge values: the amd64 NaN rule, bit-exact."""
    specials = np.array([0x7FC01234, 0xFF812345, 0x7F800000, 0xFF800000, 0x00000000, 0x80000000, 0x7F7FFFFF,
                         0x00000001, 0x3F800000, 0xBF800000], dtype=np.uint32)
    x = np.repeat(specials, specials.size)
    y = np.tile(specials, specials.size)
    if dt == BF16:
        x, y = (x >> 16).astype(np.uint16), (y >> 16).astype(np.uint16)
    for alpha in (0.75, 0.0, float("inf"), float("nan")):
        bits_equal(run_axpy(y, x, alpha, dt, fused), ref.axpy(y, x, alpha, dt, fused))


def test_axpy_unfused_differs_from_fma_somewhere(backend, ref):
    """Both rounding modes are real: on random data they disagree on some elements."""
    n = 1 << 16
    x = synthetic.normal_f32(1, n).view(np.uint32)
    y = synthetic.normal_f32(2, n).view(np.uint32)
    a = run_axpy(y, x, 0.1, F32, 0)
    b = run_axpy(y, x, 0.1, F32, 1)
    assert (a != b).any()


def test_axpy_config3_f32_full_size(backend, ref):
    """Config 3: y = 0.75 x + y over 2^28 float32, bit-exact, then the BF16 variant."""
    n = 1 << 28
    x = synthetic.normal_f32(synthetic.CONFIG_SEED + 30, n)
    y = synthetic.normal_f32(synthetic.CONFIG_SEED + 31, n)
    got = run_axpy(y.view(np.uint32), x.view(np.uint32), 0.75, F32)
    bits_equal(got, ref.axpy(y.view(np.uint32), x.view(np.uint32), 0.75, F32, threads=host_threads()))
    xb, yb = synthetic.f32_to_bf16_bits(x), synthetic.f32_to_bf16_bits(y)
    del x, y, got
    bits_equal(run_axpy(yb, xb, 0.75, BF16), ref.axpy(yb, xb, 0.75, BF16, threads=host_threads()))


def test_axpy_rejects(backend):
    L = lib()
    assert L.mf_axpy(1, 1, 4, 1.0, E4M3, 0, None) == -3
    assert L.mf_axpy(1, 1, -4, 1.0, F32, 0, None) == -7
    assert L.mf_axpy(None, None, 0, 1.0, F32, 0, None) == 0


# ------------------------------------------------------- scalar broadcast

@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("src,dst", [(F32, F32), (BF16, BF16), (F16, F16), (E4M3, F32), (I8, BF16), (I4, F32)])
def test_scalar_broadcast(backend, ref, op, src, dst):
    n = 10007
    raw = synthetic.uniform_bytes(op * 10 + src, (n + 1) // 2 if src == I4 else n * ITEMSIZE[src])
    ds = to_device(raw)
    d = empty(n * ITEMSIZE[dst])
    # random bytes hold NaN and infinity codes; the scalars add inf * 0, inf - inf and NaN operands
    for sc in (-1.375, float("inf"), float("-inf"), float("nan"), 0.0):
        if op == 3 and sc == 0.0:
            continue
        call("mf_scalar_broadcast", ds.ptr, src, d.ptr, dst, n, sc, op, None)
        got = fetch(d, n * ITEMSIZE[dst]).view({2: np.uint16, 4: np.uint32}[ITEMSIZE[dst]])
        bits_equal(got, ref.scalar_broadcast(raw, src, dst, sc, op, n=n))
    ds.free()
    d.free()


def test_scalar_broadcast_div_by_zero(backend):
    from manifesto_b200._abi import last_error
    rc = lib().mf_scalar_broadcast(1, F32, 1, F32, 4, 0.0, 3, None)
    assert rc == -1 and "divisor must be nonzero" in last_error()
    assert lib().mf_scalar_broadcast(1, F32, 1, F32, 4, 1.0, 9, None) == -1
