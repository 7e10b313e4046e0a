"""The CPU oracle against the reference's own known answers (CPU only).

Every case in tests/golden/reference_vectors.json["known_answers"] comes from
a manifesto Go test (file:line recorded beside it) or from the Go encoders'
code read by hand; the oracle must reproduce all of them before it is used
to check the GPU kernels.  Independent cross-checks against numpy and
ml_dtypes cover the ranges where the reference follows IEEE / OCP rules.
"""
import math
import struct

import numpy as np
import pytest

from manifesto_b200 import synthetic


def f32(bits: int) -> float:
    return struct.unpack("<f", struct.pack("<I", bits))[0]


def bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", v))[0]


def test_e4m3_encode_known_answers(ref, golden):
    L = ref.lib()
    for case in golden["known_answers"]["e4m3_encode"]:
        assert L.ref_e4m3_encode(case["in"]) == case["out"], case


def test_e5m2_encode_known_answers(ref, golden):
    L = ref.lib()
    for case in golden["known_answers"]["e5m2_encode"]:
        assert L.ref_e5m2_encode(case["in"]) == case["out"], case


@pytest.mark.parametrize("name,enc,dec", [("e4m3_roundtrip", "ref_e4m3_encode", "ref_e4m3_decode"),
                                          ("e5m2_roundtrip", "ref_e5m2_encode", "ref_e5m2_decode")])
def test_fp8_roundtrips(ref, golden, name, enc, dec):
    L = ref.lib()
    case = golden["known_answers"][name]
    for v in case["values"]:
        got = f32(getattr(L, dec)(getattr(L, enc)(bits(v))))
        assert abs(got - v) <= case["tol"], (v, got)


def test_fp8_overflow_decode(ref):
    L = ref.lib()
    # dtype/fp8_test.go:24-32 and :68-76
    assert f32(L.ref_e4m3_decode(L.ref_e4m3_encode(bits(1e9)))) == 448.0
    assert f32(L.ref_e4m3_decode(L.ref_e4m3_encode(bits(-1e9)))) == -448.0
    assert math.isinf(f32(L.ref_e5m2_decode(L.ref_e5m2_encode(bits(1e9)))))
    assert f32(L.ref_e5m2_decode(L.ref_e5m2_encode(bits(-1e9)))) == -math.inf
    assert math.isnan(f32(L.ref_e4m3_decode(0x7F)))
    assert math.isnan(f32(L.ref_e5m2_decode(L.ref_e5m2_encode(0x7FC00000))))


def test_bf16_known_answers(ref, golden):
    L = ref.lib()
    for case in golden["known_answers"]["bf16_encode"]:
        assert L.ref_bf16_encode(case["in"]) == case["out"], case
    h = L.ref_bf16_encode(golden["known_answers"]["bf16_nan_stays_nan"]["in"])
    assert math.isnan(f32(L.ref_bf16_decode(h)))
    case = golden["known_answers"]["bf16_decode_le_bytes"]
    raw = np.array(case["bytes"], dtype=np.uint8)
    out = ref.convert(raw, ref.BF16, ref.F32).view(np.float32)
    assert out.tolist() == case["values"]


def test_f16_known_answers(ref, golden):
    L = ref.lib()
    for case in golden["known_answers"]["f16_encode"]:
        assert L.ref_f16_encode(case["in"]) == case["out"], case
    for case in golden["known_answers"]["f16_decode"]:
        assert L.ref_f16_decode(case["in"]) == case["out"], case
    # dtype/float16_test.go:77,129: NaN() = 0x7e01 is a NaN
    assert math.isnan(f32(L.ref_f16_decode(0x7E01)))
    assert L.ref_f16_decode(0x7C00) == 0x7F800000 and L.ref_f16_decode(0xFC00) == 0xFF800000


def test_int4_known_answers(ref, golden):
    L = ref.lib()
    for case in golden["known_answers"]["int4_pairs"]:
        p = L.ref_int4_pair(case["lo"], case["hi"])
        assert (L.ref_int4_lo(p), L.ref_int4_hi(p)) == (case["byte_lo"], case["byte_hi"]), case
    for case in golden["known_answers"]["int4_decode"]:
        raw = np.array([L.ref_int4_pair(lo, hi) for lo, hi in case["pairs"]], dtype=np.uint8)
        out = ref.convert(raw, ref.I4, ref.F32).view(np.float32)
        assert out.tolist() == case["values"], case


def test_int8_and_f32_decode(ref, golden):
    case = golden["known_answers"]["int8_decode"]
    out = ref.convert(np.array(case["bytes"], np.uint8), ref.I8, ref.F32).view(np.float32)
    assert out.tolist() == case["values"]
    case = golden["known_answers"]["f32_roundtrip"]
    v = np.array(case["values"], np.float32)
    assert ref.convert(v.view(np.uint32), ref.F32, ref.F32).view(np.float32).tolist() == case["values"]


def _relu_add_tree():
    # ReLU(Add(In0, In1)) as a node table (codegen/codegen_test.go:13-50)
    return {"type": np.array([1, 1, 3, 14], np.int32), "value": np.zeros(4),
            "input": np.array([0, 1, 0, 0], np.int32), "child0": np.array([-1, -1, 0, 2], np.int32),
            "child1": np.array([-1, -1, 1, -1], np.int32), "root": 3}


def test_fused_known_answers(ref, golden):
    case = golden["known_answers"]["fused_relu_add"]
    x = np.array(case["x"], np.float32)
    y = np.array(case["y"], np.float32)
    out = ref.fused_eval(_relu_add_tree(), [x, y], [ref.F32, ref.F32], [0, 0], ref.F32, 4)
    assert out.view(np.float32).tolist() == case["out"]


@pytest.mark.parametrize("op,fn", [(15, lambda v: 1.0 / (1.0 + math.exp(-v))), (16, math.tanh),
                                   (18, lambda v: 0.5 * v * (1 + math.tanh(math.sqrt(2 / math.pi) *
                                                                          (v + 0.044715 * v ** 3))))])
def test_fused_activation_tolerance(ref, golden, op, fn):
    case = golden["known_answers"]["fused_activation_tol"]
    x = np.array(case["inputs"], np.float32)
    tree = {"type": np.array([1, op], np.int32), "value": np.zeros(2), "input": np.zeros(2, np.int32),
            "child0": np.array([-1, 0], np.int32), "child1": np.array([-1, -1], np.int32), "root": 1}
    out = ref.fused_eval(tree, [x], [ref.F32], [0], ref.F32, len(x)).view(np.float32)
    for v, o in zip(x.tolist(), out.tolist()):
        assert abs(o - fn(v)) <= case["tol"]


def test_axpy_known_answers(ref, golden):
    case = golden["known_answers"]["axpy_f32"]
    y = np.array(case["y"], np.float32).view(np.uint32)
    x = np.array(case["x"], np.float32).view(np.uint32)
    assert ref.axpy(y, x, case["alpha"], ref.F32).view(np.float32).tolist() == case["out"]
    case = golden["known_answers"]["axpy_bf16"]
    yb = synthetic.f32_to_bf16_bits(np.array(case["y"], np.float32))
    xb = synthetic.f32_to_bf16_bits(np.array(case["x"], np.float32))
    out = ref.axpy(yb, xb, case["alpha"], ref.BF16)
    assert ref.convert(out, ref.BF16, ref.F32).view(np.float32).tolist() == case["out"]


def test_oracle_frozen_vectors(ref, golden):
    """The oracle still produces the committed fixture hashes."""
    import hashlib
    o = golden["oracle"]
    codes = np.arange(256, dtype=np.uint8)
    assert ref.convert(codes, ref.E4M3, ref.F32).tolist() == o["e4m3_decode_f32"]
    assert ref.convert(codes, ref.E5M2, ref.F32).tolist() == o["e5m2_decode_f32"]
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    h = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    assert h(ref.convert(allh, ref.BF16, ref.E4M3)) == o["bf16_to_e4m3_sha256"]
    assert h(ref.convert(allh, ref.F16, ref.F32)) == o["f16_to_f32_sha256"]


def test_bf16_f16_encoders_match_ieee_rne(ref):
    """Outside NaN lanes the reference BF16/F16 encoders are IEEE RNE (numpy / ml_dtypes)."""
    ml_dtypes = pytest.importorskip("ml_dtypes")
    b = synthetic.splitmix64(11, 1 << 20).astype(np.uint32)
    f = b.view(np.float32)
    nan = np.isnan(f)
    with np.errstate(all="ignore"):
        assert (ref.convert(b, ref.F32, ref.F16)[~nan] == f[~nan].astype(np.float16).view(np.uint16)).all()
        assert (ref.convert(b, ref.F32, ref.BF16)[~nan] ==
                f[~nan].astype(ml_dtypes.bfloat16).view(np.uint16)).all()
    # NaN rules: BF16 keeps the high half and sets bit 6; F16 sets the quiet bit
    assert ref.lib().ref_bf16_encode(0x7F800001) == 0x7FC0
    assert ref.lib().ref_f16_encode(0xFF800001 | (0x155 << 13)) == (0xFC00 | 0x0200 | 0x155)


def test_fp8_decoders_match_ocp(ref):
    ml_dtypes = pytest.importorskip("ml_dtypes")
    codes = np.arange(256, dtype=np.uint8)
    for dt, md in ((ref.E4M3, ml_dtypes.float8_e4m3fn), (ref.E5M2, ml_dtypes.float8_e5m2)):
        mine = ref.convert(codes, dt, ref.F32).view(np.float32)
        theirs = codes.view(md).astype(np.float32)
        assert ((mine == theirs) | (np.isnan(mine) & np.isnan(theirs))).all()


def test_fp8_encoders_quirk_bands(ref):
    """Reference E4M3/E5M2 encoders differ from OCP only inside the documented bands."""
    ml_dtypes = pytest.importorskip("ml_dtypes")
    b = synthetic.splitmix64(12, 1 << 21).astype(np.uint32)
    f = b.view(np.float32)
    a = np.abs(f)
    fin = np.isfinite(f)
    r4 = ref.convert(b, ref.F32, ref.E4M3)
    o4 = ref.convert(b, ref.F32, ref.E4M3, compat=1)
    in_range = fin & (a <= 448)
    with np.errstate(all="ignore"):
        assert (o4[in_range] == f[in_range].astype(ml_dtypes.float8_e4m3fn).view(np.uint8)).all()
    differ = (r4 != o4) & fin
    band = ((a >= 2.0 ** -10) & (a < 2.0 ** -6)) | ((a >= 248) & (a <= 448))
    assert not (differ & ~band).any()
    r5 = ref.convert(b, ref.F32, ref.E5M2)
    o5 = ref.convert(b, ref.F32, ref.E5M2, compat=1)
    d5 = (r5 != o5) & fin
    band5 = ((a >= 2.0 ** -17) & (a < 2.0 ** -14)) | (a > 57344)
    assert not (d5 & ~band5).any()


def test_int_sources_round_through_float64(ref):
    # int64 -> float64 -> float32 rounds twice (convert.go:135-145)
    v = np.array([2 ** 53 + 1, (2 ** 24 + 1) * 2 ** 29 + 2 ** 28 + 1, -(2 ** 62) - 1], dtype=np.int64)
    got = ref.convert(v, ref.I64, ref.F32).view(np.float32)
    want = v.astype(np.float64).astype(np.float32)
    assert got.tolist() == want.tolist()


def test_f64_nan_payload(ref):
    d = np.array([np.nan], np.float64).view(np.uint64) | np.uint64(0x0000_1234_5678_9ABC)
    got = int(ref.convert(d.view(np.float64), ref.F64, ref.F32)[0])
    assert got == (0x7FC00000 | ((int(d[0]) >> 29) & 0x7FFFFF))


def test_scaled_cast_rule(ref):
    x = synthetic.normal_bf16(13, 4096)
    amax = ref.amax(x, ref.BF16)
    assert amax == float(np.abs(synthetic.normal_f32(13, 4096)).astype(np.float32).max()) or amax > 0
    s = ref.fp8_scale(amax, ref.E4M3)
    assert s == np.float32(448.0) / np.float32(amax)
    assert ref.fp8_scale(0.0, ref.E4M3) == 1.0
    assert ref.fp8_scale(float("inf"), ref.E4M3) == 1.0
    q = ref.scaled_cast(x, ref.BF16, ref.E4M3, amax)
    # the element equal to amax scales to exactly 448 -> code 0x7e
    xf = ref.convert(x, ref.BF16, ref.F32).view(np.float32)
    assert q[np.argmax(np.abs(xf))] & 0x7F == 0x7E


def _np_linspace(start, stop, count, endpoint=True):
    """runLinspace restated with numpy float32 scalars (IEEE, no contraction)."""
    f = np.float32
    if count == 1:
        return np.array([start], np.float32)
    intervals = count - 1 if endpoint else count
    step = (f(stop) - f(start)) / f(intervals)
    idx = np.arange(count, dtype=np.int64).astype(np.float32)
    out = (f(start) + idx * step).astype(np.float32)
    if endpoint:
        out[0], out[-1] = f(start), f(stop)
    return out


def test_linspace_known_answers(ref):
    assert ref.linspace(0.0, 1.0, 5).view(np.float32).tolist() == [0.0, 0.25, 0.5, 0.75, 1.0]
    got = ref.linspace(0.0, 1.0, 5, endpoint=False).view(np.float32)
    assert got.tolist() == [np.float32(i) * np.float32(0.2) for i in range(5)]
    assert ref.linspace(3.5, -7.0, 1).view(np.float32).tolist() == [3.5]
    # the endpoint is stop exactly even where start + (n-1)*step rounds elsewhere
    g = ref.linspace(0.1, 0.7, 7).view(np.float32)
    assert g[-1] == np.float32(0.7) and g[0] == np.float32(0.1)


@pytest.mark.parametrize("start,stop,count,endpoint", [
    (0.0, 1.0, 1001, True), (-3.25, 17.5, 4097, False), (1e30, -1e30, 77, True),
    (0.0, 1.0, (1 << 24) + 5, True), (5.0, 5.0, 10, True)])
def test_linspace_matches_float32_restatement(ref, start, stop, count, endpoint):
    got = ref.linspace(start, stop, count, endpoint, threads=4).view(np.float32)
    assert np.array_equal(got, _np_linspace(start, stop, count, endpoint))


def test_linspace_nan_and_encoders(ref):
    v = ref.linspace(float("nan"), 1.0, 9).view(np.uint32)
    assert (v[:-1] == 0x7FC00000).all() and v[-1] == np.float32(1.0).view(np.uint32)
    for dt in (ref.BF16, ref.F16):
        f32 = ref.linspace(-2.0, 3.0, 1000)
        assert ref.linspace(-2.0, 3.0, 1000, dst_dtype=dt).tobytes() == ref.convert(f32, ref.F32, dt).tobytes()
