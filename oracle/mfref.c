/*
 * mfref.c -- CPU oracle (test infrastructure, never linked by the product).
 *
 * A scalar restatement of manifesto's Go hot-path code, one function per
 * Go function, each citing the file:line it follows (paths inside the
 * manifesto Go module).  Kept deliberately plain and branchy: it is the
 * checker, so it follows the Go control flow rather than the GPU kernels'
 * branch-free formulations.  Compile with -O2 -ffp-contract=off
 * -fno-fast-math (oracle/Makefile).
 */
#include "mfref.h"

#include <math.h>
#include <stddef.h>
#include <string.h>

/* dtype wire codes, dtype/dtype.go:29-49 */
enum {
    DT_F64 = 1, DT_F32 = 2, DT_F16 = 3, DT_BF16 = 4, DT_E4M3 = 5, DT_E5M2 = 6,
    DT_I64 = 7, DT_I32 = 8, DT_I16 = 9, DT_I8 = 10, DT_I4 = 11,
    DT_U64 = 12, DT_U32 = 13, DT_U16 = 14, DT_U8 = 15
};

#define ERR_INVALID (-1)
#define ERR_DTYPE_UNSUPPORTED (-3)

static inline float f_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t bits_from_f(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* float32 arithmetic with the amd64 (SSE) NaN rule, made explicit so the
 * result does not depend on which operand order a compiler picks: a NaN
 * operand propagates quieted (the first operand as written in the Go source
 * when both are NaN); an invalid operation on non-NaN operands (0 * inf,
 * inf - inf, 0 / 0) yields the x86 default NaN 0xFFC00000.  This is what
 * the reference's `y += alpha*x` (runtime/axpy.go:116) and
 * applyScalarBroadcast (runtime/executor_math.go:203-229) produce on amd64. */
static float nan2(float a, float b) {
    if (isnan(a)) return f_from_bits(bits_from_f(a) | 0x400000u);
    if (isnan(b)) return f_from_bits(bits_from_f(b) | 0x400000u);
    return f_from_bits(0xffc00000u);
}
static float x86_add(float a, float b) { float r = a + b; return isnan(r) ? nan2(a, b) : r; }
static float x86_sub(float a, float b) { float r = a - b; return isnan(r) ? nan2(a, b) : r; }
static float x86_mul(float a, float b) { float r = a * b; return isnan(r) ? nan2(a, b) : r; }
static float x86_div(float a, float b) { float r = a / b; return isnan(r) ? nan2(a, b) : r; }
static float x86_fma(float a, float b, float c) {
    float r = fmaf(a, b, c);
    if (!isnan(r)) return r;
    if (isnan(a) || isnan(b)) return nan2(a, b);
    if (isnan(c)) return f_from_bits(bits_from_f(c) | 0x400000u);
    return f_from_bits(0xffc00000u);
}

/* ---------------------------------------------------------------- FP8 */

/* roundToNearestEven, dtype/fp8.go:263-284 */
static uint32_t rne_dropped(uint32_t truncated, uint32_t full, uint32_t shift) {
    if (shift == 0) return truncated;
    uint32_t dropped = full & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (dropped < half) return truncated;
    if (dropped > half) return truncated + 1u;
    if (truncated & 1u) return truncated + 1u;
    return truncated;
}

/* F8E4M3.Float32, dtype/fp8.go:39-70 */
uint32_t ref_e4m3_decode(uint8_t code) {
    uint32_t sign = (uint32_t)(code >> 7) << 31;
    if ((code & 0x7f) == 0x7f) return sign | 0x7fc00000u;
    if ((code & 0x7f) == 0) return sign;
    uint32_t exponent = (code >> 3) & 0x0f;
    uint32_t mantissa = code & 0x07;
    int32_t e = (int32_t)exponent;
    if (exponent == 0) {
        uint32_t shift = 0;
        while ((mantissa & 0x08) == 0) { mantissa <<= 1; shift++; }
        mantissa &= 0x07;
        e = 1 - (int32_t)shift;
    }
    int32_t biased = e - 7 + 127;
    return sign | ((uint32_t)biased << 23) | (mantissa << 20);
}

/* NewF8E4M3FromFloat32, dtype/fp8.go:77-136 (including the reference's
 * subnormal shift 20-exponent at :106 and exponent>=15 saturation at
 * :117 and :128; NaN -> 0x7f regardless of sign at :78-79) */
uint8_t ref_e4m3_encode(uint32_t u) {
    float value = f_from_bits(u);
    if (isnan(value)) return 0x7f;
    uint8_t sign = 0;
    if (u >> 31) { sign = 0x80; value = -value; }
    if (isinf(value) || value > 448.0f) return sign | 0x7e;
    if (value == 0.0f) return sign;
    uint32_t bits = bits_from_f(value);
    int32_t exponent = (int32_t)((bits >> 23) & 0xff) - 127 + 7;
    uint32_t mantissa = bits & 0x7fffff;
    if (exponent <= 0) {
        if (exponent < -3) return sign;
        uint32_t shift = (uint32_t)(20 - exponent);
        uint32_t full = (mantissa | 0x800000u) >> shift;
        uint32_t rounded = rne_dropped(full, mantissa | 0x800000u, shift);
        if (rounded >= 0x08) return sign | 0x08;
        return sign | (uint8_t)rounded;
    }
    if (exponent >= 15) return sign | 0x7e;
    uint32_t mantissa8 = mantissa >> 20;
    uint32_t rounded = rne_dropped(mantissa8, mantissa, 20);
    if (rounded >= 0x08) {
        mantissa8 = 0;
        exponent++;
        if (exponent >= 15) return sign | 0x7e;
    } else {
        mantissa8 = rounded;
    }
    return sign | (uint8_t)((uint32_t)exponent << 3) | (uint8_t)mantissa8;
}

/* F8E5M2.Float32, dtype/fp8.go:149-183 (NaN keeps mantissa bits, :160) */
uint32_t ref_e5m2_decode(uint8_t code) {
    uint32_t sign = (uint32_t)(code >> 7) << 31;
    uint32_t exponent = (code >> 2) & 0x1f;
    uint32_t mantissa = code & 0x03;
    if (exponent == 0x1f) {
        if (mantissa == 0) return sign | 0x7f800000u;
        return sign | 0x7fc00000u | (mantissa << 21);
    }
    int32_t e = (int32_t)exponent;
    if (exponent == 0) {
        if (mantissa == 0) return sign;
        uint32_t shift = 0;
        while ((mantissa & 0x04) == 0) { mantissa <<= 1; shift++; }
        mantissa &= 0x03;
        e = 1 - (int32_t)shift;
    }
    int32_t biased = e - 15 + 127;
    return sign | ((uint32_t)biased << 23) | (mantissa << 21);
}

/* NewF8E5M2FromFloat32, dtype/fp8.go:190-249 (subnormal shift 21-exponent
 * at :219, flush below exponent -1 at :215, > 57344 -> inf at :202) */
uint8_t ref_e5m2_encode(uint32_t u) {
    float value = f_from_bits(u);
    if (isnan(value)) return 0x7f;
    uint8_t sign = 0;
    if (u >> 31) { sign = 0x80; value = -value; }
    if (isinf(value) || value > 57344.0f) return sign | 0x7c;
    if (value == 0.0f) return sign;
    uint32_t bits = bits_from_f(value);
    int32_t exponent = (int32_t)((bits >> 23) & 0xff) - 127 + 15;
    uint32_t mantissa = bits & 0x7fffff;
    if (exponent <= 0) {
        if (exponent < -1) return sign;
        uint32_t shift = (uint32_t)(21 - exponent);
        uint32_t full = (mantissa | 0x800000u) >> shift;
        uint32_t rounded = rne_dropped(full, mantissa | 0x800000u, shift);
        if (rounded >= 0x04) return sign | 0x04;
        return sign | (uint8_t)rounded;
    }
    if (exponent >= 0x1f) return sign | 0x7c;
    uint32_t mantissa8 = mantissa >> 21;
    uint32_t rounded = rne_dropped(mantissa8, mantissa, 21);
    if (rounded >= 0x04) {
        mantissa8 = 0;
        exponent++;
        if (exponent >= 0x1f) return sign | 0x7c;
    } else {
        mantissa8 = rounded;
    }
    return sign | (uint8_t)((uint32_t)exponent << 2) | (uint8_t)mantissa8;
}

/* OCP FP8 encode with saturation to the largest finite value (the
 * .satfinite rule): round to nearest even on the exact value, |v| beyond
 * the largest finite value and +-inf give +-max, NaN gives 0x7f.  Written
 * from the OCP 8-bit floating point specification (E4M3: bias 7, max 448,
 * subnormal quantum 2^-9; E5M2: bias 15, max 57344, quantum 2^-16). */
static uint8_t ocp_encode(uint32_t u, int mant_bits, int bias, float maxv, uint8_t maxcode) {
    float value = f_from_bits(u);
    if (isnan(value)) return 0x7f;
    uint8_t sign = (u >> 31) ? 0x80 : 0;
    float a = fabsf(value);
    if (!(a <= maxv)) return sign | maxcode; /* inf or beyond max */
    int min_normal_exp = 1 - bias; /* unbiased exponent of the smallest normal */
    float min_normal = ldexpf(1.0f, min_normal_exp);
    if (a < min_normal) {
        /* subnormal grid: multiples of 2^(min_normal_exp - mant_bits) */
        float q = nearbyintf(ldexpf(a, mant_bits - min_normal_exp));
        return sign | (uint8_t)q; /* q == 2^mant_bits encodes the smallest normal */
    }
    uint32_t ab = bits_from_f(a);
    int drop = 23 - mant_bits;
    uint32_t r = (ab + ((1u << (drop - 1)) - 1u) + ((ab >> drop) & 1u)) >> drop;
    uint32_t code = r - ((uint32_t)(127 - bias) << mant_bits);
    if (code > maxcode) code = maxcode;
    return sign | (uint8_t)code;
}

uint8_t ref_e4m3_encode_ocp(uint32_t u) { return ocp_encode(u, 3, 7, 448.0f, 0x7e); }
uint8_t ref_e5m2_encode_ocp(uint32_t u) { return ocp_encode(u, 2, 15, 57344.0f, 0x7b); }

/* --------------------------------------------------------------- BF16 */

/* NewBfloat16FromFloat32, dtype/bfloat16.go:41-55 */
uint16_t ref_bf16_encode(uint32_t bits) {
    if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x0040u);
    uint32_t rounded = bits + 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)(rounded >> 16);
}

/* BF16.Float32, dtype/bfloat16.go:82-84 */
uint32_t ref_bf16_decode(uint16_t h) { return (uint32_t)h << 16; }

/* ---------------------------------------------------------------- F16 */

/* Fromfloat32 -> f32bitsToF16bits, dtype/float16.go:109-111,261-297.
 * IEEE 754 binary16 round-to-nearest-even written from the format's
 * definition; NaN keeps the top payload bits and sets the quiet bit
 * (sign | 0x7c00 | 0x0200 | coef >> 13) and Inf maps to Inf, as the
 * reference does at :270-279. */
uint16_t ref_f16_encode(uint32_t u) {
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t e = (u >> 23) & 0xffu;
    uint32_t m = u & 0x7fffffu;
    if (e == 0xffu) {
        if (m == 0) return sign | 0x7c00u;
        return (uint16_t)(sign | 0x7c00u | 0x0200u | (m >> 13));
    }
    int32_t he = (int32_t)e - 127 + 15; /* binary16 biased exponent */
    if (he >= 0x1f) return sign | 0x7c00u;
    if (he <= 0) {
        /* result is a multiple of 2^-24: value / 2^-24 = sig >> (14 - he) */
        int32_t shift = 14 - he;
        if (shift > 24) return sign;
        uint32_t sig = m | 0x800000u;
        uint32_t q = rne_dropped(sig >> shift, sig, (uint32_t)shift);
        return (uint16_t)(sign | q); /* q may reach 0x400: the smallest normal */
    }
    uint32_t base = ((uint32_t)he << 10) | (m >> 13);
    uint32_t q = rne_dropped(base, m, 13); /* carry may roll into the exponent */
    return (uint16_t)(sign | q);          /* 0x7c00 on overflow to infinity */
}

/* F16.Float32 -> f16bitsToF32bits, dtype/float16.go:169-172,222-255:
 * exact widening; NaN -> sign | 0x7fc00000 | coef << 13. */
uint32_t ref_f16_decode(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t coef = (uint32_t)(h & 0x3ffu) << 13;
    if (e == 0x1f) {
        if (coef == 0) return sign | 0x7f800000u;
        return sign | 0x7fc00000u | coef;
    }
    if (e == 0) {
        if (coef == 0) return sign;
        float v = (float)(h & 0x3ffu) * 5.9604644775390625e-08f; /* 2^-24, exact */
        return sign | bits_from_f(v);
    }
    return sign | ((e + 127u - 15u) << 23) | coef;
}

/* --------------------------------------------------------------- Int4 */

/* int4Decode, dtype/int4.go:72-78 */
static int8_t int4_decode(uint8_t nibble) {
    if (nibble & 0x08) return (int8_t)((int)nibble - 16);
    return (int8_t)nibble;
}
/* Int4Pair.Lo / Hi, dtype/int4.go:28-37 */
int8_t ref_int4_lo(uint8_t pair) { return int4_decode(pair & 0x0f); }
int8_t ref_int4_hi(uint8_t pair) { return int4_decode((pair >> 4) & 0x0f); }
/* NewInt4Pair + int4Encode (clamping), dtype/int4.go:21-23,60-70 */
static uint8_t int4_encode(int8_t v) {
    if (v < -8) v = -8;
    if (v > 7) v = 7;
    return (uint8_t)v & 0x0f;
}
uint8_t ref_int4_pair(int8_t lo, int8_t hi) { return int4_encode(lo) | (uint8_t)(int4_encode(hi) << 4); }

/* -------------------------------------------------- slice conversions */

/* float32(float64): IEEE round to nearest even; a NaN keeps its sign and
 * top 23 payload bits with the quiet bit set, which is what the amd64
 * CVTSD2SS instruction behind Go's conversion produces. */
static float f64_to_f32(double d) {
    if (isnan(d)) {
        uint64_t b; memcpy(&b, &d, 8);
        uint32_t u = (uint32_t)(b >> 32) & 0x80000000u;
        u |= 0x7fc00000u | (uint32_t)((b >> 29) & 0x7fffffu);
        return f_from_bits(u);
    }
    return (float)d;
}

/* One element of convert.BytesToFloat32 (dtype/convert/convert.go:85-146);
 * integer sources go through float64 first (BytesToFloat64, :36-79 and
 * decoders.go:126-289), so int64/uint64 round twice like the Go path. */
static int decode_one(int dt, const void* src, int64_t i, float* out) {
    const uint8_t* b = (const uint8_t*)src;
    switch (dt) {
    case DT_F64: { double d; memcpy(&d, b + 8 * i, 8); *out = f64_to_f32(d); return 0; }
    case DT_F32: { uint32_t u; memcpy(&u, b + 4 * i, 4); *out = f_from_bits(u); return 0; }
    case DT_F16: { uint16_t h; memcpy(&h, b + 2 * i, 2); *out = f_from_bits(ref_f16_decode(h)); return 0; }
    case DT_BF16: { uint16_t h; memcpy(&h, b + 2 * i, 2); *out = f_from_bits(ref_bf16_decode(h)); return 0; }
    case DT_E4M3: *out = f_from_bits(ref_e4m3_decode(b[i])); return 0;
    case DT_E5M2: *out = f_from_bits(ref_e5m2_decode(b[i])); return 0;
    case DT_I64: { int64_t v; memcpy(&v, b + 8 * i, 8); *out = (float)(double)v; return 0; }
    case DT_I32: { int32_t v; memcpy(&v, b + 4 * i, 4); *out = (float)(double)v; return 0; }
    case DT_I16: { int16_t v; memcpy(&v, b + 2 * i, 2); *out = (float)(double)v; return 0; }
    case DT_I8: *out = (float)(double)(int8_t)b[i]; return 0;
    case DT_I4: {
        uint8_t packed = b[i >> 1];
        /* decodeInt4ToFloat64, decoders.go:281,284 */
        int8_t v = (i & 1) ? (int8_t)((int8_t)packed >> 4) : (int8_t)((int8_t)(uint8_t)(packed << 4) >> 4);
        *out = (float)(double)v;
        return 0;
    }
    case DT_U64: { uint64_t v; memcpy(&v, b + 8 * i, 8); *out = (float)(double)v; return 0; }
    case DT_U32: { uint32_t v; memcpy(&v, b + 4 * i, 4); *out = (float)(double)v; return 0; }
    case DT_U16: { uint16_t v; memcpy(&v, b + 2 * i, 2); *out = (float)(double)v; return 0; }
    case DT_U8: *out = (float)(double)b[i]; return 0;
    default: return ERR_DTYPE_UNSUPPORTED;
    }
}

/* One element of the narrowing drivers BytesToBFloat16 / BytesToFloat16 /
 * BytesToFloat8E4M3 / BytesToFloat8E5M2 (convert.go:155-228) and of the
 * store encoders Float32AsDTypeBytes (runtime/session.go:431-452). */
static int encode_one(int dt, float v, void* dst, int64_t i, int compat) {
    uint8_t* b = (uint8_t*)dst;
    uint32_t u = bits_from_f(v);
    switch (dt) {
    case DT_F32: memcpy(b + 4 * i, &u, 4); return 0;
    case DT_BF16: { uint16_t h = ref_bf16_encode(u); memcpy(b + 2 * i, &h, 2); return 0; }
    case DT_F16: { uint16_t h = ref_f16_encode(u); memcpy(b + 2 * i, &h, 2); return 0; }
    case DT_E4M3: b[i] = compat ? ref_e4m3_encode_ocp(u) : ref_e4m3_encode(u); return 0;
    case DT_E5M2: b[i] = compat ? ref_e5m2_encode_ocp(u) : ref_e5m2_encode(u); return 0;
    default: return ERR_DTYPE_UNSUPPORTED;
    }
}

int ref_decode_f32(int src_dtype, const void* src, float* dst, int64_t begin, int64_t n) {
    for (int64_t i = begin; i < begin + n; i++) {
        int rc = decode_one(src_dtype, src, i, &dst[i]);
        if (rc) return rc;
    }
    return 0;
}

int ref_encode_f32(int dst_dtype, const float* src, void* dst, int64_t begin, int64_t n, int compat) {
    for (int64_t i = begin; i < begin + n; i++) {
        int rc = encode_one(dst_dtype, src[i], dst, i, compat);
        if (rc) return rc;
    }
    return 0;
}

int ref_convert(int src_dtype, int dst_dtype, const void* src, void* dst,
                int64_t begin, int64_t n, int compat) {
    for (int64_t i = begin; i < begin + n; i++) {
        float v;
        int rc = decode_one(src_dtype, src, i, &v);
        if (rc) return rc;
        rc = encode_one(dst_dtype, v, dst, i, compat);
        if (rc) return rc;
    }
    return 0;
}

/* -------------------------------------------------- Int4 group dequant */

/* Builder-defined composition (no group scale exists in the reference):
 * nibble sign extension as decodeInt4ToFloat64 (decoders.go:262-289),
 * float32 product with the group's scale, store encode as
 * Float32AsDTypeBytes (runtime/session.go:431-452). */
int ref_int4_dequant_grouped(const uint8_t* q, const void* scales, int scale_dtype,
                             void* out, int out_dtype, int64_t rows, int64_t cols,
                             int64_t group, int64_t row_begin, int64_t row_end) {
    if (cols % 2 || group <= 0) return ERR_INVALID;
    int64_t ngroups = (cols + group - 1) / group;
    for (int64_t r = row_begin; r < row_end && r < rows; r++) {
        for (int64_t c = 0; c < cols; c++) {
            int64_t e = r * cols + c;
            uint8_t packed = q[e >> 1];
            int8_t nib = (e & 1) ? ref_int4_hi(packed) : ref_int4_lo(packed);
            float s;
            int rc = decode_one(scale_dtype, scales, r * ngroups + c / group, &s);
            if (rc) return rc;
            float v = x86_mul((float)nib, s);
            rc = encode_one(out_dtype, v, out, e, 0);
            if (rc) return rc;
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- axpy */

/* axpyOntoHost, runtime/axpy.go:95-165: y[i] += alpha * x[i] in float32
 * (two roundings on amd64), BF16/F16 targets decoded first and re-encoded
 * with float32VectorBytes (:171-194). */
int ref_axpy(void* y, const void* x, int64_t begin, int64_t n, float alpha, int dtype, int fused_fma) {
    if (dtype != DT_F32 && dtype != DT_BF16 && dtype != DT_F16) return ERR_DTYPE_UNSUPPORTED;
    for (int64_t i = begin; i < begin + n; i++) {
        float yv, xv;
        decode_one(dtype, y, i, &yv);
        decode_one(dtype, x, i, &xv);
        float r;
        if (fused_fma) {
            r = x86_fma(alpha, xv, yv);
        } else {
            float t = x86_mul(alpha, xv);
            r = x86_add(yv, t);
        }
        encode_one(dtype, r, y, i, 0);
    }
    return 0;
}

/* applyScalarBroadcast, runtime/executor_math.go:195-234, then the store
 * encode of writeFloat32VectorOutput (:254-292). */
int ref_scalar_broadcast(const void* src, int src_dtype, void* dst, int dst_dtype,
                         int64_t begin, int64_t n, float scalar, int op) {
    if (op == 3 && scalar == 0.0f) return ERR_INVALID;
    if (op < 0 || op > 3) return ERR_INVALID;
    for (int64_t i = begin; i < begin + n; i++) {
        float v;
        int rc = decode_one(src_dtype, src, i, &v);
        if (rc) return rc;
        float r;
        switch (op) {
        case 0: r = x86_add(v, scalar); break;
        case 1: r = x86_sub(v, scalar); break;
        case 2: r = x86_mul(v, scalar); break;
        default: r = x86_div(v, scalar); break;
        }
        rc = encode_one(dst_dtype, r, dst, i, 0);
        if (rc) return rc;
    }
    return 0;
}

/* runLinspace, runtime/executor_math.go:57-108: step = (stop - start) / float32(intervals)
 * with intervals = count - 1 (count when endpoint is false); output[i] = start +
 * float32(i) * step, each operation rounded to float32 (amd64: no contraction, the SSE
 * NaN rule); with the endpoint included output[0] = start and output[count-1] = stop;
 * count == 1 gives start.  Elements [begin, begin + n) are encoded with the store
 * encoder (Float32AsDTypeBytes, runtime/session.go:431-452). */
int ref_linspace(float start, float stop, int64_t count, int endpoint, void* dst, int dst_dtype,
                 int64_t begin, int64_t n) {
    if (count <= 0) return ERR_INVALID;
    const int64_t intervals = (endpoint || count == 1) ? count - 1 : count;
    const float step = count == 1 ? 0.0f : x86_div(x86_sub(stop, start), (float)intervals);
    for (int64_t i = begin; i < begin + n; i++) {
        float v;
        if (count == 1) {
            v = start;
        } else {
            v = x86_add(start, x86_mul((float)i, step));
            if (intervals == count - 1) {
                if (i == 0) v = start;
                if (i == count - 1) v = stop;
            }
        }
        int rc = encode_one(dst_dtype, v, dst, i, 0);
        if (rc) return rc;
    }
    return 0;
}

/* ------------------------------------------------------ fused evaluator */

/* optimizer.NodeType, optimizer/fusion_ast.go:32-65 */
enum {
    N_INVALID = 0, N_INPUT, N_CONSTANT, N_ADD, N_SUB, N_MUL, N_DIV, N_MAX, N_MIN,
    N_NEG, N_ABS, N_SQRT, N_EXP, N_LOG, N_RELU, N_SIGMOID, N_TANH, N_SILU, N_GELU, N_LEAKY
};

typedef struct {
    const int32_t* type;
    const double* value;
    const int32_t* input;
    const int32_t* child0;
    const int32_t* child1;
    const float* in_vals; /* decoded input values of the current element */
} fused_ctx;

/* evalCPU, codegen/cpu.go:126-212 */
static float eval_node(const fused_ctx* c, int k) {
    switch (c->type[k]) {
    case N_INPUT: return c->in_vals[c->input[k]];
    case N_CONSTANT: return f64_to_f32(c->value[k]);
    case N_ADD: return eval_node(c, c->child0[k]) + eval_node(c, c->child1[k]);
    case N_SUB: return eval_node(c, c->child0[k]) - eval_node(c, c->child1[k]);
    case N_MUL: return eval_node(c, c->child0[k]) * eval_node(c, c->child1[k]);
    case N_DIV: return eval_node(c, c->child0[k]) / eval_node(c, c->child1[k]);
    case N_MAX: {
        float l = eval_node(c, c->child0[k]), r = eval_node(c, c->child1[k]);
        return l > r ? l : r;
    }
    case N_MIN: {
        float l = eval_node(c, c->child0[k]), r = eval_node(c, c->child1[k]);
        return l < r ? l : r;
    }
    case N_NEG: return -eval_node(c, c->child0[k]);
    case N_ABS: { float v = eval_node(c, c->child0[k]); return v < 0 ? -v : v; }
    case N_SQRT: return f64_to_f32(sqrt((double)eval_node(c, c->child0[k])));
    case N_EXP: return f64_to_f32(exp((double)eval_node(c, c->child0[k])));
    case N_LOG: return f64_to_f32(log((double)eval_node(c, c->child0[k])));
    case N_RELU: { float v = eval_node(c, c->child0[k]); return v < 0 ? 0.0f : v; }
    case N_SIGMOID: {
        float v = eval_node(c, c->child0[k]);
        return f64_to_f32(1.0 / (1.0 + exp(-(double)v)));
    }
    case N_TANH: return f64_to_f32(tanh((double)eval_node(c, c->child0[k])));
    case N_SILU: {
        float v = eval_node(c, c->child0[k]);
        return f64_to_f32((double)v / (1.0 + exp(-(double)v)));
    }
    case N_GELU: {
        double v = (double)eval_node(c, c->child0[k]);
        /* math.Sqrt(2.0/math.Pi): Go folds 2/pi exactly, then one rounding */
        double inner = sqrt(0.63661977236758134307553505349005744813783858296182579499) *
                       (v + 0.044715 * v * v * v);
        return f64_to_f32(0.5 * v * (1.0 + tanh(inner)));
    }
    case N_LEAKY: {
        float v = eval_node(c, c->child0[k]);
        if (v >= 0) return v;
        return 0.01f * v;
    }
    default: return 0.0f;
    }
}

int ref_fused_eval(int n_nodes, const int32_t* type, const double* value, const int32_t* input,
                   const int32_t* child0, const int32_t* child1, int root,
                   int n_inputs, const void* const* inputs, const int32_t* in_dtype,
                   const int64_t* in_bcast, void* out, int out_dtype, int64_t begin, int64_t n) {
    if (root < 0 || root >= n_nodes || n_inputs > 64) return ERR_INVALID;
    float vals[64];
    fused_ctx c = {type, value, input, child0, child1, vals};
    for (int64_t i = begin; i < begin + n; i++) {
        for (int j = 0; j < n_inputs; j++) {
            int64_t idx = (in_bcast && in_bcast[j] > 0) ? i % in_bcast[j] : i;
            int rc = decode_one(in_dtype[j], inputs[j], idx, &vals[j]);
            if (rc) return rc;
        }
        float r = eval_node(&c, root);
        int rc = encode_one(out_dtype, r, out, i, 0);
        if (rc) return rc;
    }
    return 0;
}

/* ------------------------------------------------ amax-scaled FP8 cast */

/* Builder-defined (the reference has no amax / scale op): max |v| with
 * Go '>' semantics, so NaN never replaces the running maximum. */
uint32_t ref_amax(const void* src, int src_dtype, int64_t begin, int64_t n) {
    float m = 0.0f;
    for (int64_t i = begin; i < begin + n; i++) {
        float v;
        if (decode_one(src_dtype, src, i, &v)) return 0xffffffffu;
        float a = fabsf(v);
        if (a > m) m = a;
    }
    return bits_from_f(m);
}

float ref_fp8_scale(float amax, int fp8_dtype) {
    float fmax = (fp8_dtype == DT_E5M2) ? 57344.0f : 448.0f;
    if (!(amax > 0.0f) || isinf(amax)) return 1.0f;
    return fmax / amax;
}

int ref_scaled_cast(const void* src, int src_dtype, void* dst, int fp8_dtype, float amax,
                    int64_t begin, int64_t n, int compat) {
    if (fp8_dtype != DT_E4M3 && fp8_dtype != DT_E5M2) return ERR_DTYPE_UNSUPPORTED;
    float scale = ref_fp8_scale(amax, fp8_dtype);
    for (int64_t i = begin; i < begin + n; i++) {
        float v;
        int rc = decode_one(src_dtype, src, i, &v);
        if (rc) return rc;
        float s = v * scale;
        encode_one(fp8_dtype, s, dst, i, compat);
    }
    return 0;
}
