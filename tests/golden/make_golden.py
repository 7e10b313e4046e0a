"""Write tests/golden/reference_vectors.json.

Two kinds of vectors:

1. ``known_answers``: the known-answer checks of manifesto's own Go tests for
   this path, transcribed case by case with the file:line each comes from,
   plus the extra E4M3/E5M2 known answers derived by hand from
   dtype/fp8.go:77-136 and :190-249 (the rounding quirks those tests do not
   exercise).  These pin the oracle.
2. ``oracle``: oracle outputs on small seeded inputs (every FP8 code decoded,
   every BF16 code encoded to E4M3/E5M2, a seeded fused chain, Int4 dequant,
   axpy).  They freeze the oracle's behaviour so a change to it shows up as a
   fixture diff, and give the GPU tests expected values that do not depend
   on rebuilding the oracle.

Run: python tests/golden/make_golden.py   (needs oracle/libmfref.so; builds it)
"""
from __future__ import annotations

import hashlib
import json
import struct
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from manifesto_b200 import synthetic  # noqa: E402
from oracle import ref  # noqa: E402


def f32bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", v))[0]


NAN = 0x7FC00000
NEG_NAN = 0xFFC00000
INF = 0x7F800000
NEG_INF = 0xFF800000
NEG_ZERO = 0x80000000

KNOWN_ANSWERS = {
    # E4M3 encode: exact codes (the Go tests check ±448 decode and NaN/zero codes)
    "e4m3_encode": [
        {"in": f32bits(1e9), "out": 0x7E, "src": "dtype/fp8_test.go:26,30"},
        {"in": f32bits(-1e9), "out": 0xFE, "src": "dtype/fp8_test.go:27,31"},
        {"in": NAN, "out": 0x7F, "src": "dtype/fp8_test.go:36-38"},
        {"in": 0, "out": 0x00, "src": "dtype/fp8_test.go:45,48"},
        {"in": NEG_ZERO, "out": 0x80, "src": "dtype/fp8_test.go:46,49"},
        # hand-derived from dtype/fp8.go:77-136 (subnormal shift 20-exponent, exponent-15 saturation)
        {"in": f32bits(2.0 ** -9), "out": 0x02, "src": "dtype/fp8.go:101-115"},
        {"in": f32bits(2.0 ** -10), "out": 0x01, "src": "dtype/fp8.go:101-115"},
        {"in": f32bits(2.0 ** -7), "out": 0x08, "src": "dtype/fp8.go:110-111"},
        {"in": f32bits(0.01171875), "out": 0x08, "src": "dtype/fp8.go:110-111"},
        {"in": f32bits(249.0), "out": 0x7E, "src": "dtype/fp8.go:117-118"},
        {"in": f32bits(256.0), "out": 0x7E, "src": "dtype/fp8.go:117-118"},
        {"in": f32bits(400.0), "out": 0x7E, "src": "dtype/fp8.go:117-118"},
        {"in": f32bits(247.0), "out": 0x77, "src": "dtype/fp8.go:121-135"},
        {"in": f32bits(1.0625), "out": 0x38, "src": "dtype/fp8.go:263-284 (tie to even)"},
        {"in": f32bits(1.1875), "out": 0x3A, "src": "dtype/fp8.go:263-284"},
        {"in": NEG_NAN, "out": 0x7F, "src": "dtype/fp8.go:78-79"},
        {"in": INF, "out": 0x7E, "src": "dtype/fp8.go:89-90"},
    ],
    # E4M3 round trips within 1e-2 (dtype/fp8_test.go:12-20)
    "e4m3_roundtrip": {"values": [0, 1, -1, 2, 0.5, -0.5, 448, -448, 0.015625], "tol": 1e-2,
                       "src": "dtype/fp8_test.go:12-20"},
    "e5m2_encode": [
        {"in": f32bits(1e9), "out": 0x7C, "src": "dtype/fp8_test.go:70,74"},
        {"in": f32bits(-1e9), "out": 0xFC, "src": "dtype/fp8_test.go:71,75"},
        {"in": INF, "out": 0x7C, "src": "dtype/fp8_test.go:80-82"},
        {"in": f32bits(2.0 ** -16), "out": 0x02, "src": "dtype/fp8.go:214-228"},
        {"in": f32bits(2e-5), "out": 0x03, "src": "dtype/fp8.go:214-228"},
        {"in": f32bits(1e-5), "out": 0x00, "src": "dtype/fp8.go:215-216"},
        {"in": f32bits(60000.0), "out": 0x7C, "src": "dtype/fp8.go:202-203"},
        {"in": NAN, "out": 0x7F, "src": "dtype/fp8.go:191-192 (decodes to NaN, dtype/fp8_test.go:88-91)"},
    ],
    "e5m2_roundtrip": {"values": [0, 1, -1, 2, 0.5, -0.5, 57344, -57344], "tol": 1e-2,
                       "src": "dtype/fp8_test.go:56-64"},
    "bf16_encode": [
        {"in": f32bits(1.0), "out": 0x3F80, "src": "dtype/bfloat16_test.go:11-16"},
        {"in": 0x3F808000, "out": 0x3F80, "src": "dtype/bfloat16_test.go:29-31"},
        {"in": 0x3F808001, "out": 0x3F81, "src": "dtype/bfloat16_test.go:35-37"},
        {"in": 0x3F818000, "out": 0x3F82, "src": "dtype/bfloat16_test.go:46-48"},
        {"in": INF, "out": 0x7F80, "src": "dtype/bfloat16_test.go:52-53"},
        {"in": NEG_INF, "out": 0xFF80, "src": "dtype/bfloat16_test.go:55-56"},
        {"in": f32bits(2.0), "out": 0x4000, "src": "dtype/bfloat16_test.go:130-134"},
    ],
    "bf16_nan_stays_nan": {"in": NAN, "src": "dtype/bfloat16_test.go:58-59"},
    "bf16_decode_le_bytes": {"bytes": [0x80, 0x3F, 0x00, 0x40], "values": [1.0, 2.0],
                             "src": "dtype/bfloat16_test.go:122-126"},
    "f16_encode": [
        {"in": f32bits(1.0), "out": 0x3C00, "src": "dtype/float16_test.go:41-46"},
        {"in": f32bits(-2.0), "out": 0xC000, "src": "dtype/float16_test.go:109-114"},
        {"in": f32bits(1.5), "out": 0x3E00, "src": "dtype/float16_test.go:181-186 (formats as 1.5)"},
    ],
    "f16_decode": [
        {"in": 0x3C00, "out": f32bits(1.0), "src": "dtype/float16_test.go:31-35"},
        {"in": 0x4200, "out": f32bits(3.0), "src": "dtype/float16_test.go:100-104"},
    ],
    "int4_pairs": [
        {"lo": -3, "hi": 5, "byte_lo": -3, "byte_hi": 5, "src": "dtype/int4_test.go:11-16"},
        {"lo": -8, "hi": 7, "byte_lo": -8, "byte_hi": 7, "src": "dtype/int4_test.go:20-25"},
        {"lo": -100, "hi": 100, "byte_lo": -8, "byte_hi": 7, "src": "dtype/int4_test.go:29-36 (clamped)"},
        {"lo": -5, "hi": 6, "byte_lo": -5, "byte_hi": 6, "src": "dtype/int4_test.go:59-65"},
    ],
    "int4_decode": [
        {"pairs": [[1, -2], [-8, 7]], "values": [1, -2, -8, 7], "src": "dtype/convert/convert_test.go:56-66"},
        {"pairs": [[-8, -1], [0, 7]], "values": [-8, -1, 0, 7], "src": "dtype/convert/convert_test.go:136-146"},
        {"pairs": [[3, -4]], "values": [3, -4], "src": "dtype/convert/convert_test.go:117-131 (odd output length)"},
    ],
    "int8_decode": {"bytes": [0, 1, 255, 128], "values": [0, 1, -1, -128],
                    "src": "dtype/convert/convert_test.go:46-53"},
    "f32_roundtrip": {"values": [1.0, -2.5, 0.125, 1024.5], "src": "dtype/convert/convert_test.go:78-87"},
    "fused_relu_add": {"x": [1, -3, 5, -2], "y": [2, 1, -4, 1], "out": [3, 0, 1, 0],
                       "src": "codegen/codegen_test.go:13-50"},
    "fused_activation_tol": {"inputs": [0.0, 1.0, -1.0, 2.0], "tol": 1e-5, "ops": ["Sigmoid", "Tanh", "Gelu"],
                             "src": "codegen/codegen_test.go:60-100"},
    "axpy_f32": {"y": [1, 2, 3], "x": [4, 5, 6], "alpha": 0.5, "out": [3, 4.5, 6],
                 "src": "runtime/axpy_test.go:14-23"},
    "axpy_bf16": {"y": [1, 2, 3], "x": [4, 5, 6], "alpha": 0.5, "out": [3, 4.5, 6],
                  "src": "runtime/axpy_test.go:25-52"},
}


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def oracle_vectors() -> dict:
    codes = np.arange(256, dtype=np.uint8)
    bf16_all = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    out = {
        "e4m3_decode_f32": ref.convert(codes, ref.E4M3, ref.F32).tolist(),
        "e5m2_decode_f32": ref.convert(codes, ref.E5M2, ref.F32).tolist(),
        "bf16_to_e4m3_sha256": digest(ref.convert(bf16_all, ref.BF16, ref.E4M3)),
        "bf16_to_e5m2_sha256": digest(ref.convert(bf16_all, ref.BF16, ref.E5M2)),
        "f16_to_e4m3_sha256": digest(ref.convert(bf16_all, ref.F16, ref.E4M3)),
        "f16_to_f32_sha256": digest(ref.convert(bf16_all, ref.F16, ref.F32)),
    }
    # seeded f32 bit patterns through every encoder
    bits = synthetic.splitmix64(synthetic.CONFIG_SEED + 100, 1 << 16).astype(np.uint32)
    for name, dt in (("bf16", ref.BF16), ("f16", ref.F16), ("e4m3", ref.E4M3), ("e5m2", ref.E5M2)):
        out[f"f32_random_to_{name}_sha256"] = digest(ref.convert(bits, ref.F32, dt))
    out["f32_random_seed"] = synthetic.CONFIG_SEED + 100
    # Int4 group dequant, 64 x 256, group 128
    q = synthetic.uniform_bytes(synthetic.CONFIG_SEED + 2, 64 * 128)
    s = synthetic.abs_normal_bf16(synthetic.CONFIG_SEED + 3, 64 * 2, 0.02)
    out["int4_64x256_g128_sha256"] = digest(ref.int4_dequant(q, s, ref.BF16, ref.BF16, 64, 256, 128))
    # axpy f32 / bf16 on 4099 seeded values
    x = synthetic.normal_f32(synthetic.CONFIG_SEED + 4, 4099)
    y = synthetic.normal_f32(synthetic.CONFIG_SEED + 5, 4099)
    out["axpy_f32_4099_sha256"] = digest(ref.axpy(y.view(np.uint32), x.view(np.uint32), 0.75, ref.F32))
    xb, yb = synthetic.f32_to_bf16_bits(x), synthetic.f32_to_bf16_bits(y)
    out["axpy_bf16_4099_sha256"] = digest(ref.axpy(yb, xb, 0.75, ref.BF16))
    return out


def main() -> None:
    ref.build()
    data = {"known_answers": KNOWN_ANSWERS, "oracle": oracle_vectors()}
    path = Path(__file__).resolve().parent / "reference_vectors.json"
    path.write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")
    print(path)


if __name__ == "__main__":
    main()
