"""K1-K3 dtype conversion on the GPU against the CPU oracle (bit-exact)."""
import numpy as np
import pytest

from manifesto_b200 import synthetic
from oracle.ref import BF16, E4M3, E5M2, F16, F32, F64, I4, I8, I16, I32, I64, ITEMSIZE, U8, U16, U32, U64

from .conftest import host_threads
from .gpu_util import bits_equal, convert

pytestmark = pytest.mark.gpu

FLOATS = [F32, F16, BF16, E4M3, E5M2]
DSTS = [F32, F16, BF16, E4M3, E5M2]


@pytest.mark.parametrize("src", [E4M3, E5M2])
@pytest.mark.parametrize("dst", DSTS)
def test_all_fp8_codes(backend, ref, src, dst):
    codes = np.arange(256, dtype=np.uint8)
    for compat in (0, 1):
        bits_equal(convert(codes, src, dst, 256, compat), ref.convert(codes, src, dst, compat=compat))


@pytest.mark.parametrize("src", [F16, BF16])
@pytest.mark.parametrize("dst", DSTS)
def test_all_16bit_codes(backend, ref, src, dst):
    codes = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    for compat in (0, 1):
        bits_equal(convert(codes, src, dst, 65536, compat), ref.convert(codes, src, dst, compat=compat))


@pytest.mark.parametrize("dst", DSTS)
def test_random_f32_patterns(backend, ref, dst):
    b = synthetic.splitmix64(synthetic.CONFIG_SEED + 100, 1 << 22).astype(np.uint32)
    for compat in (0, 1):
        bits_equal(convert(b, F32, dst, b.size, compat), ref.convert(b, F32, dst, compat=compat,
                                                                     threads=host_threads()))


def test_golden_fixture_hashes(backend, golden):
    import hashlib
    h = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    o = golden["oracle"]
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    assert h(convert(allh, BF16, E4M3, 65536)) == o["bf16_to_e4m3_sha256"]
    assert h(convert(allh, BF16, E5M2, 65536)) == o["bf16_to_e5m2_sha256"]
    assert h(convert(allh, F16, E4M3, 65536)) == o["f16_to_e4m3_sha256"]
    assert h(convert(allh, F16, F32, 65536)) == o["f16_to_f32_sha256"]
    bits = synthetic.splitmix64(o["f32_random_seed"], 1 << 16).astype(np.uint32)
    for name, dt in (("bf16", BF16), ("f16", F16), ("e4m3", E4M3), ("e5m2", E5M2)):
        assert h(convert(bits, F32, dt, bits.size)) == o[f"f32_random_to_{name}_sha256"], name
    codes = np.arange(256, dtype=np.uint8)
    assert convert(codes, E4M3, F32, 256).tolist() == o["e4m3_decode_f32"]


@pytest.mark.parametrize("dst", [E4M3, E5M2, F16, BF16])
def test_quirk_bands_dense(backend, ref, dst):
    """Every float32 pattern with exponent in the E4M3/E5M2 subnormal bands and near the top, strided."""
    parts = []
    for e in list(range(105, 125)) + list(range(133, 144)):
        parts.append(((e << 23) | np.arange(0, 1 << 23, 61, dtype=np.uint32)).astype(np.uint32))
    b = np.concatenate(parts)
    b = np.concatenate([b, b | np.uint32(0x80000000)])
    for compat in (0, 1):
        bits_equal(convert(b, F32, dst, b.size, compat), ref.convert(b, F32, dst, compat=compat,
                                                                     threads=host_threads()))


def test_fp8_encode_edge_values(backend, ref, golden):
    """Band edges, the 2^-10 tie, saturation edges, NaN/Inf, in every lane position of a quad."""
    f32 = lambda x: int(np.array([x], np.float32).view(np.uint32)[0])
    base = [2.0 ** -10, 2.0 ** -11, 2.0 ** -9, 2.0 ** -7, 2.0 ** -6, 1.5 * 2 ** -10, 248.0, 247.99998, 256.0, 448.0,
            449.0, 464.0, 57344.0, 57345.0, 61440.0, 2.0 ** -14, 2.0 ** -16, 2.0 ** -17, 1.0, 0.0]
    vals = [f32(v) for v in base] + [f32(-v) for v in base]
    vals += [v + d for v in vals for d in (1, 0xFFFFFFFF)]  # one ulp either side (wraps harmlessly)
    vals += [0x7FC00000, 0xFFC00000, 0x7F800001, 0x7F800000, 0xFF800000, 0x00000001, 0x80000001]
    vals += [int(c["in"]) for c in golden["known_answers"]["e4m3_encode"]]
    v = np.array([x & 0xFFFFFFFF for x in vals], np.uint32)
    # every value in every quad lane, next to band / ordinary / zero neighbours
    fill = np.array([f32(1.0), f32(2.0 ** -8), 0, f32(300.0)], np.uint32)
    rows = []
    for x in v:
        for lane in range(4):
            for f in fill:
                q = np.full(4, f, np.uint32)
                q[lane] = x
                rows.append(q)
    b = np.concatenate(rows)
    for dst in (E4M3, E5M2):
        for compat in (0, 1):
            bits_equal(convert(b, F32, dst, b.size, compat), ref.convert(b, F32, dst, compat=compat))


@pytest.mark.parametrize("n", [0, 1, 15, 16, 17, 4095, (1 << 20) + 3])
@pytest.mark.parametrize("pair", [(E4M3, F32), (BF16, E4M3), (F32, BF16), (F16, F32)])
def test_ragged_sizes(backend, ref, n, pair):
    src, dst = pair
    raw = synthetic.uniform_bytes(n + 7, n * ITEMSIZE[src])
    got = convert(raw, src, dst, n)
    bits_equal(got, ref.convert(raw, src, dst, n=n))


@pytest.mark.parametrize("pair", [(E4M3, F32), (BF16, E4M3), (F32, F16), (F16, BF16)])
def test_unaligned_pointers(backend, ref, pair):
    src, dst = pair
    n = 1000
    raw = synthetic.uniform_bytes(99, n * ITEMSIZE[src])
    want = ref.convert(raw, src, dst, n=n)
    bits_equal(convert(raw, src, dst, n, src_off=ITEMSIZE[src], dst_off=ITEMSIZE[dst]), want)


@pytest.mark.parametrize("src", [F64, I64, I32, I16, I8, U64, U32, U16, U8])
@pytest.mark.parametrize("dst", [F32, BF16, E4M3])
def test_wide_and_integer_sources(backend, ref, src, dst):
    n = 70001
    raw = synthetic.uniform_bytes(src * 31 + dst, n * ITEMSIZE[src])
    if src == F64:
        # a mix of ordinary values, NaN payloads and extremes
        v = raw.view(np.float64).copy()
        v[: n // 2] = synthetic.normal_f32(5, n // 2).astype(np.float64) * 1e3
        raw = v.view(np.uint8)
    bits_equal(convert(raw, src, dst, n), ref.convert(raw, src, dst, n=n))


@pytest.mark.parametrize("n", [1, 2, 3, 4096, 100001])
def test_int4_source(backend, ref, n):
    raw = synthetic.uniform_bytes(n, (n + 1) // 2)
    for dst in (F32, BF16, F16):
        bits_equal(convert(raw, I4, dst, n), ref.convert(raw, I4, dst, n=n))


def test_config1_fp8_to_f32_full_size(backend, ref):
    """Config 1: E4M3 -> FP32 over 2^26 uniform bytes, bit-exact."""
    n = 1 << 26
    raw = synthetic.uniform_bytes(synthetic.CONFIG_SEED + 1, n)
    got = convert(raw, E4M3, F32, n)
    bits_equal(got, ref.convert(raw, E4M3, F32, threads=host_threads()))


def test_invalid_arguments(backend):
    from manifesto_b200._abi import lib
    L = lib()
    assert L.mf_convert(F32, I32, 1, 1, 4, 0, None) == -3  # unsupported destination
    assert L.mf_convert(99, F32, 1, 1, 4, 0, None) == -3
    assert L.mf_convert(F32, BF16, 1, 1, -1, 0, None) == -7
    assert L.mf_convert(F32, BF16, None, None, 4, 0, None) == -1
    assert L.mf_convert(F32, E4M3, 1, 1, 4, 7, None) == -1
    assert L.mf_convert(F32, BF16, None, None, 0, 0, None) == 0
