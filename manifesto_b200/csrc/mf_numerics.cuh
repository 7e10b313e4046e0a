// mf_numerics.cuh -- device codecs for manifesto's storage formats.
//
// Every function reproduces the manifesto Go scalar codec it names bit for
// bit (paths inside the manifesto Go module), but is written for the GPU:
// integer and select arithmetic on the float32 bit pattern, no loops, no
// divergent branches on the common path.  The CPU oracle (oracle/mfref.c)
// restates the same Go code independently and the tests compare the two.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/mfcuda.h"

namespace mf {

// ------------------------------------------------------------------ FP8

// Small unsigned integer m (< 2^23) times 2^k, exactly, without I2F:
// (2^23 + m) * 2^k - 2^(23+k) is exact, so one FFMA on the bit pattern
// 0x4B000000 | m gives m * 2^k.
__device__ __forceinline__ float small_uint_scaled(uint32_t m, float two_k, float two_23k) {
    return __fmaf_rn(__uint_as_float(0x4B000000u | m), two_k, -two_23k);
}

// E4M3 -> f32 bits, dtype/fp8.go:39-70.  Normal codes widen by re-biasing
// the exponent (+120); subnormal codes are m * 2^-9 (exact in float32);
// S.1111.111 is NaN and widens to sign | 0x7fc00000.
__device__ __forceinline__ uint32_t e4m3_to_f32bits(uint32_t code) {
    const uint32_t sign = (code & 0x80u) << 24;
    const uint32_t mag = code & 0x7fu;
    const uint32_t normal = (mag << 20) + (120u << 23);
    const uint32_t sub = __float_as_uint(small_uint_scaled(mag & 7u, 0.001953125f, 16384.0f));
    uint32_t r = (mag >> 3) ? normal : sub;
    r = (mag == 0x7fu) ? 0x7fc00000u : r;
    return sign | r;
}

// E5M2 -> f32 bits, dtype/fp8.go:149-183.  Exponent 31 with mantissa 0 is
// Inf; with mantissa m != 0 it is sign | 0x7fc00000 | m << 21.
__device__ __forceinline__ uint32_t e5m2_to_f32bits(uint32_t code) {
    const uint32_t sign = (code & 0x80u) << 24;
    const uint32_t mag = code & 0x7fu;
    const uint32_t normal = (mag << 21) + (112u << 23);
    const uint32_t sub = __float_as_uint(small_uint_scaled(mag & 3u, 1.52587890625e-05f, 128.0f));
    uint32_t r = (mag >> 2) ? normal : sub;
    const uint32_t special = (mag & 3u) ? (0x7fc00000u | ((mag & 3u) << 21)) : 0x7f800000u;
    r = ((mag >> 2) == 31u) ? special : r;
    return sign | r;
}

// Round-to-nearest-even of the low `shift` bits of `full` (1..23 bits),
// the rule of roundToNearestEven (dtype/fp8.go:263-284).
__device__ __forceinline__ uint32_t rne_shift(uint32_t full, uint32_t shift) {
    const uint32_t t = full >> shift;
    const uint32_t dropped = full & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    return t + ((dropped > half) | ((dropped == half) & (t & 1u)));
}

// f32 bits -> E4M3 with the reference's rules, dtype/fp8.go:77-136:
//   NaN -> 0x7f (either sign)                              (:78-79)
//   |v| > 448 or Inf -> sign|0x7e                           (:89-90)
//   |v| >= 248: the rounded exponent reaches 15 -> sign|0x7e (:117,:128)
//   2^-6 <= |v| < 248: RNE on the top 3 mantissa bits      (:121-135)
//   |v| < 2^-6: subnormal path with shift 20-exponent      (:101-115)
__device__ __forceinline__ uint32_t f32bits_to_e4m3_ref(uint32_t u) {
    const uint32_t sign = (u >> 24) & 0x80u;
    const uint32_t a = u & 0x7fffffffu;
    if (a >= 0x3c800000u) {                      // 2^-6 and above (incl. Inf/NaN)
        uint32_t code = ((a + 0x7ffffu + ((a >> 20) & 1u)) >> 20) - 960u;
        code = (a >= 0x43780000u) ? 0x7eu : code;  // 248 and above saturate
        code = (a > 0x7f800000u) ? 0x7fu : (code | sign);
        return code;
    }
    const uint32_t e = a >> 23;                  // biased float32 exponent
    if (e < 117u) return sign;                   // exponent field < -3 flushes to +-0
    const uint32_t shift = 140u - e;             // 20 - (e - 120), 20..23
    uint32_t r = rne_shift((a & 0x7fffffu) | 0x800000u, shift);
    r = r > 8u ? 8u : r;
    return sign | r;
}

// f32 bits -> E5M2 with the reference's rules, dtype/fp8.go:190-249:
//   NaN -> 0x7f; |v| > 57344 or Inf -> sign|0x7c (Inf)       (:191-204)
//   2^-14 <= |v| <= 57344: RNE on the top 2 mantissa bits    (:230-248)
//   |v| < 2^-14: exponent field < -1 -> 0, else shift 21-exponent (:214-228)
__device__ __forceinline__ uint32_t f32bits_to_e5m2_ref(uint32_t u) {
    const uint32_t sign = (u >> 24) & 0x80u;
    const uint32_t a = u & 0x7fffffffu;
    if (a >= 0x38800000u) {
        uint32_t code = ((a + 0xfffffu + ((a >> 21) & 1u)) >> 21) - 448u;
        code = (a > 0x47600000u) ? 0x7cu : code;
        code = (a > 0x7f800000u) ? 0x7fu : (code | sign);
        return code;
    }
    const uint32_t e = a >> 23;
    if (e < 111u) return sign;
    const uint32_t shift = 133u - e;             // 21 - (e - 112), 21..22
    uint32_t r = rne_shift((a & 0x7fffffu) | 0x800000u, shift);
    r = r > 4u ? 4u : r;
    return sign | r;
}

// OCP FP8 encode with .satfinite (RNE, overflow and Inf -> +-max finite);
// NaN -> 0x7f regardless of sign, as in the reference's encoders.
__device__ __forceinline__ uint32_t f32_to_e4m3_ocp(float v) {
    uint16_t pair;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(pair) : "f"(0.0f), "f"(v));
    const uint32_t code = pair & 0xffu;
    return (v != v) ? 0x7fu : code;
}
__device__ __forceinline__ uint32_t f32_to_e5m2_ocp(float v) {
    uint16_t pair;
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(pair) : "f"(0.0f), "f"(v));
    const uint32_t code = pair & 0xffu;
    return (v != v) ? 0x7fu : code;
}

// ----------------------------------------------------------------- BF16

// NewBfloat16FromFloat32, dtype/bfloat16.go:41-55: NaN keeps its high half
// and sets bit 6; everything else rounds to nearest even by adding
// 0x7fff + lsb (overflow rolls into Inf).
__device__ __forceinline__ uint32_t f32bits_to_bf16(uint32_t u) {
    const uint32_t rounded = (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
    return ((u & 0x7fffffffu) > 0x7f800000u) ? ((u >> 16) | 0x40u) : rounded;
}

// Two float32 -> packed BF16x2 (lo in bits 0..15).  The hardware cvt rounds
// to nearest even exactly like the reference for every non-NaN input; NaN
// lanes are replaced by the reference's NaN rule.
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    if ((lo != lo) | (hi != hi)) {
        r = f32bits_to_bf16(__float_as_uint(lo)) | (f32bits_to_bf16(__float_as_uint(hi)) << 16);
    }
    return r;
}

// ----------------------------------------------------------------- F16

// Fromfloat32 -> f32bitsToF16bits, dtype/float16.go:261-297: IEEE binary16
// round to nearest even; NaN -> sign|0x7c00|0x0200|coef>>13.
__device__ __forceinline__ uint32_t f32bits_to_f16(uint32_t u) {
    const uint32_t sign = (u >> 16) & 0x8000u;
    const uint32_t a = u & 0x7fffffffu;
    if (a >= 0x38800000u) {                      // binary16 normal range and above
        if (a >= 0x7f800000u) {
            return sign | 0x7c00u | ((a > 0x7f800000u) ? (0x0200u | ((a & 0x7fffffu) >> 13)) : 0u);
        }
        uint32_t h = ((a + 0xfffu + ((a >> 13) & 1u)) >> 13) - (112u << 10);
        h = (a >= 0x477ff000u) ? 0x7c00u : h;    // rounds to >= 65520: Inf
        return sign | h;
    }
    const uint32_t e = a >> 23;
    if (e < 102u) return sign;                   // below 2^-25: +-0
    const uint32_t shift = 126u - e;             // 14 - (e - 112), 14..24
    return sign | rne_shift((a & 0x7fffffu) | 0x800000u, shift);
}

// float32 x2 -> packed IEEE binary16 x2 (lo in bits 0..15): the hardware cvt
// rounds like the reference for every non-NaN input; NaN lanes take the
// reference's NaN rule.
__device__ __forceinline__ uint32_t f32x2_to_f16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    if ((lo != lo) | (hi != hi)) {
        r = f32bits_to_f16(__float_as_uint(lo)) | (f32bits_to_f16(__float_as_uint(hi)) << 16);
    }
    return r;
}

// f16bitsToF32bits, dtype/float16.go:222-255: exact widening with
// NaN -> sign | 0x7fc00000 | coef << 13.
__device__ __forceinline__ uint32_t f16_to_f32bits(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t mag = h & 0x7fffu;
    const uint32_t normal = (mag << 13) + (112u << 23);
    const uint32_t sub = __float_as_uint(small_uint_scaled(mag & 0x3ffu, 5.9604644775390625e-08f, 0.5f));
    uint32_t r = (mag >> 10) ? normal : sub;
    const uint32_t special = (mag & 0x3ffu) ? (0x7fc00000u | ((mag & 0x3ffu) << 13)) : 0x7f800000u;
    r = ((mag >> 10) == 31u) ? special : r;
    return sign | r;
}

// ------------------------------------------- amd64 NaN rule for f32 ops

// The GPU returns the canonical NaN 0x7FFFFFFF for any NaN result; the
// reference's Go code runs on amd64, where SSE propagates a NaN operand
// (quieted; the first operand as written when both are NaN) and produces
// the default NaN 0xFFC00000 for invalid operations on non-NaN operands.
// These wrappers keep the IEEE result and only rewrite NaN results, so
// they cost one compare on the common path.
__device__ __forceinline__ float x86_nan2(float a, float b) {
    if (a != a) return __uint_as_float(__float_as_uint(a) | 0x400000u);
    if (b != b) return __uint_as_float(__float_as_uint(b) | 0x400000u);
    return __uint_as_float(0xffc00000u);
}
__device__ __forceinline__ float x86_add(float a, float b) { const float r = __fadd_rn(a, b); return r != r ? x86_nan2(a, b) : r; }
__device__ __forceinline__ float x86_sub(float a, float b) { const float r = __fsub_rn(a, b); return r != r ? x86_nan2(a, b) : r; }
__device__ __forceinline__ float x86_mul(float a, float b) { const float r = __fmul_rn(a, b); return r != r ? x86_nan2(a, b) : r; }
__device__ __forceinline__ float x86_div(float a, float b) { const float r = __fdiv_rn(a, b); return r != r ? x86_nan2(a, b) : r; }
__device__ __forceinline__ float x86_fma(float a, float b, float c) {
    const float r = __fmaf_rn(a, b, c);
    if (r == r) return r;
    if ((a != a) | (b != b)) return x86_nan2(a, b);
    if (c != c) return __uint_as_float(__float_as_uint(c) | 0x400000u);
    return __uint_as_float(0xffc00000u);
}

// ----------------------------------------------------- float64 -> f32

// float32(float64) as the amd64 Go conversion does it: RNE, and a NaN
// keeps its sign and top 23 payload bits with the quiet bit set.
__device__ __forceinline__ float f64_to_f32(double d) {
    if (d != d) {
        const unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(d));
        return __uint_as_float(static_cast<uint32_t>(b >> 32 & 0x80000000ull) | 0x7fc00000u |
                               static_cast<uint32_t>((b >> 29) & 0x7fffffull));
    }
    return __double2float_rn(d);
}

// ------------------------------------------------------ generic codecs

__host__ __device__ constexpr int dtype_bytes(int dt) {
    return (dt == MF_DT_F64 || dt == MF_DT_I64 || dt == MF_DT_U64) ? 8
         : (dt == MF_DT_F32 || dt == MF_DT_I32 || dt == MF_DT_U32) ? 4
         : (dt == MF_DT_F16 || dt == MF_DT_BF16 || dt == MF_DT_I16 || dt == MF_DT_U16) ? 2
         : (dt == MF_DT_I4) ? 0 : 1;
}

// Element i of a buffer of dtype DT decoded to float32 with
// convert.BytesToFloat32 semantics (dtype/convert/convert.go:85-146).
// Integer sources go through float64, as the Go path does (:135-145).
template <int DT>
__device__ __forceinline__ float load_as_f32(const void* p, int64_t i) {
    if constexpr (DT == MF_DT_F32) return static_cast<const float*>(p)[i];
    else if constexpr (DT == MF_DT_BF16) return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(p)[i]) << 16);
    else if constexpr (DT == MF_DT_F16) return __uint_as_float(f16_to_f32bits(static_cast<const uint16_t*>(p)[i]));
    else if constexpr (DT == MF_DT_F8E4M3) return __uint_as_float(e4m3_to_f32bits(static_cast<const uint8_t*>(p)[i]));
    else if constexpr (DT == MF_DT_F8E5M2) return __uint_as_float(e5m2_to_f32bits(static_cast<const uint8_t*>(p)[i]));
    else if constexpr (DT == MF_DT_F64) return f64_to_f32(static_cast<const double*>(p)[i]);
    else if constexpr (DT == MF_DT_I64) return __double2float_rn(__ll2double_rn(static_cast<const long long*>(p)[i]));
    else if constexpr (DT == MF_DT_U64) return __double2float_rn(__ull2double_rn(static_cast<const unsigned long long*>(p)[i]));
    else if constexpr (DT == MF_DT_I32) return __double2float_rn(static_cast<double>(static_cast<const int32_t*>(p)[i]));
    else if constexpr (DT == MF_DT_U32) return __double2float_rn(static_cast<double>(static_cast<const uint32_t*>(p)[i]));
    else if constexpr (DT == MF_DT_I16) return static_cast<float>(static_cast<const int16_t*>(p)[i]);
    else if constexpr (DT == MF_DT_U16) return static_cast<float>(static_cast<const uint16_t*>(p)[i]);
    else if constexpr (DT == MF_DT_I8) return static_cast<float>(static_cast<const int8_t*>(p)[i]);
    else if constexpr (DT == MF_DT_U8) return static_cast<float>(static_cast<const uint8_t*>(p)[i]);
    else if constexpr (DT == MF_DT_I4) {
        const uint32_t b = static_cast<const uint8_t*>(p)[i >> 1];
        const int32_t s = static_cast<int32_t>(b << (24 + ((i & 1) ? 0 : 4))) >> 28;  // sign-extend nibble
        return static_cast<float>(s);
    } else return 0.0f;
}

// float32 -> storage code of DT (the store encoders of the reference).
template <int DT>
__device__ __forceinline__ uint32_t encode_f32(float v, int compat) {
    const uint32_t u = __float_as_uint(v);
    if constexpr (DT == MF_DT_F32) return u;
    else if constexpr (DT == MF_DT_BF16) return f32bits_to_bf16(u);
    else if constexpr (DT == MF_DT_F16) return f32bits_to_f16(u);
    else if constexpr (DT == MF_DT_F8E4M3) return compat ? f32_to_e4m3_ocp(v) : f32bits_to_e4m3_ref(u);
    else if constexpr (DT == MF_DT_F8E5M2) return compat ? f32_to_e5m2_ocp(v) : f32bits_to_e5m2_ref(u);
    else return 0u;
}

template <int DT>
__device__ __forceinline__ void store_code(void* p, int64_t i, uint32_t code) {
    if constexpr (DT == MF_DT_F32) static_cast<uint32_t*>(p)[i] = code;
    else if constexpr (DT == MF_DT_BF16 || DT == MF_DT_F16) static_cast<uint16_t*>(p)[i] = static_cast<uint16_t>(code);
    else static_cast<uint8_t*>(p)[i] = static_cast<uint8_t>(code);
}

}  // namespace mf
