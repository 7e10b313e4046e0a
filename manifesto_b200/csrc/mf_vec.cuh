// mf_vec.cuh -- 128-bit streaming access to 16-element chunks.
//
// Every streaming kernel in this library moves data in chunks of 16
// logical elements: 16 B of an 8-bit format, 32 B of a 16-bit format, 64 B
// of float32.  A chunk is read with one to four 128-bit loads (LDG.128)
// and written with one to four 128-bit stores, so a warp touches whole
// 512 B..2 KB contiguous segments per access.  Inputs are read with the
// non-coherent path and the evict-first hint (each byte is read once);
// outputs are written with the streaming store hint.
#pragma once

#include "mf_numerics.cuh"

namespace mf {

constexpr int kChunk = 16;

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void st_stream(uint4* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

// Raw words of chunk c of a buffer whose elements are `Bytes` wide.
template <int Bytes>
struct RawChunk {
    uint32_t w[4 * Bytes];
};

template <int Bytes>
__device__ __forceinline__ void load_raw(const void* base, int64_t c, RawChunk<Bytes>& r) {
    const uint4* p = reinterpret_cast<const uint4*>(base) + c * Bytes;
#pragma unroll
    for (int k = 0; k < Bytes; ++k) {
        const uint4 v = ld_stream(p + k);
        r.w[4 * k + 0] = v.x;
        r.w[4 * k + 1] = v.y;
        r.w[4 * k + 2] = v.z;
        r.w[4 * k + 3] = v.w;
    }
}

template <int Bytes>
__device__ __forceinline__ void store_raw(void* base, int64_t c, const RawChunk<Bytes>& r) {
    uint4* p = reinterpret_cast<uint4*>(base) + c * Bytes;
#pragma unroll
    for (int k = 0; k < Bytes; ++k) st_stream(p + k, make_uint4(r.w[4 * k], r.w[4 * k + 1], r.w[4 * k + 2], r.w[4 * k + 3]));
}

// f16x2 bits -> two float32 (exact for every non-NaN value).
__device__ __forceinline__ void f16x2_to_f32x2(uint32_t h2, float& lo, float& hi) {
    asm("{\n\t.reg .f16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
        : "=f"(lo), "=f"(hi)
        : "r"(h2));
}

// Two E4M3 codes (bits 0..15) -> f16x2, exact (every E4M3 value is a normal f16).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two) {
    uint32_t r;
    const uint16_t x = static_cast<uint16_t>(two);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(x));
    return r;
}

// Decode 16 elements of a floating storage format to float32.
// E4M3, E5M2 and F16 widen through the hardware conversions (exact for
// every non-NaN code); a word holding a NaN code is redone with the integer
// codecs so NaN lanes get the reference's bit patterns
// (sign | 0x7fc00000 [| payload]).  The NaN tests are SWAR on the packed codes.
template <int DT>
__device__ __forceinline__ void decode16(const RawChunk<dtype_bytes(DT)>& r, float (&v)[kChunk]) {
    if constexpr (DT == MF_DT_F32) {
#pragma unroll
        for (int k = 0; k < kChunk; ++k) v[k] = __uint_as_float(r.w[k]);
    } else if constexpr (DT == MF_DT_BF16) {
#pragma unroll
        for (int k = 0; k < kChunk; ++k) {
            const uint32_t w = r.w[k >> 1];
            v[k] = __uint_as_float((k & 1) ? (w & 0xffff0000u) : (w << 16));
        }
    } else if constexpr (DT == MF_DT_F16) {
#pragma unroll
        for (int k = 0; k < kChunk / 2; ++k) {
            const uint32_t w = r.w[k];
            f16x2_to_f32x2(w, v[2 * k], v[2 * k + 1]);
            // half h is NaN iff (h & 0x7fff) + 0x3ff carries into bit 15
            if (((w & 0x7fff7fffu) + 0x03ff03ffu) & 0x80008000u) {
                v[2 * k] = __uint_as_float(f16_to_f32bits(w & 0xffffu));
                v[2 * k + 1] = __uint_as_float(f16_to_f32bits(w >> 16));
            }
        }
    } else if constexpr (DT == MF_DT_F8E4M3) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = r.w[k];
            f16x2_to_f32x2(e4m3x2_to_f16x2(w), v[4 * k], v[4 * k + 1]);
            f16x2_to_f32x2(e4m3x2_to_f16x2(w >> 16), v[4 * k + 2], v[4 * k + 3]);
            // byte b is NaN iff (b & 0x7f) == 0x7f: zero byte of x = ~w & 0x7f7f7f7f
            const uint32_t x = ~w & 0x7f7f7f7fu;
            if ((x - 0x01010101u) & ~x & 0x80808080u) {
#pragma unroll
                for (int j = 0; j < 4; ++j) v[4 * k + j] = __uint_as_float(e4m3_to_f32bits((w >> (8 * j)) & 0xffu));
            }
        }
    } else if constexpr (DT == MF_DT_F8E5M2) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t w = r.w[k];
            // an E5M2 code is the high byte of the binary16 with the same value
            f16x2_to_f32x2(__byte_perm(w, 0u, 0x1404u), v[4 * k], v[4 * k + 1]);
            f16x2_to_f32x2(__byte_perm(w, 0u, 0x3424u), v[4 * k + 2], v[4 * k + 3]);
            // byte b is NaN iff (b & 0x7f) > 0x7c, i.e. (b & 0x7f) + 3 sets bit 7
            if (((w & 0x7f7f7f7fu) + 0x03030303u) & 0x80808080u) {
#pragma unroll
                for (int j = 0; j < 4; ++j) v[4 * k + j] = __uint_as_float(e5m2_to_f32bits((w >> (8 * j)) & 0xffu));
            }
        }
    }
}

// float32 x2 -> packed IEEE binary16 x2 with the reference's NaN rule.
__device__ __forceinline__ uint32_t f32x2_to_f16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    if ((lo != lo) | (hi != hi)) {
        r = f32bits_to_f16(__float_as_uint(lo)) | (f32bits_to_f16(__float_as_uint(hi)) << 16);
    }
    return r;
}

// Four float32 -> four FP8 codes (byte k = v[k]) with the hardware
// round-to-nearest-even .satfinite conversion (OCP rule, largest finite on
// overflow and Inf).
template <int DT>
__device__ __forceinline__ uint32_t cvt4_fp8_satfinite(float v0, float v1, float v2, float v3) {
    uint16_t lo, hi;
    if constexpr (DT == MF_DT_F8E4M3) {
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(v1), "f"(v0));
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(v3), "f"(v2));
    } else {
        asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(v1), "f"(v0));
        asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(v3), "f"(v2));
    }
    return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// NaN lanes (magnitude 0x7f) -> 0x7f without sign, four bytes at a time.
__device__ __forceinline__ uint32_t fp8x4_canonical_nan(uint32_t w, uint32_t nan_mag4) {
    const uint32_t nan = __vcmpgeu4(w & 0x7f7f7f7fu, nan_mag4);
    return (w & ~nan) | (nan & 0x7f7f7f7fu);
}

// E4M3 encode of 16 values with the reference's rules (dtype/fp8.go:77-136),
// fast path: the hardware .satfinite conversion agrees with the reference
// everywhere except (a) |v| >= 248, where the reference saturates to 0x7e
// (exponent 15 is never produced), (b) NaN, always 0x7f, and (c) the
// subnormal band 2^-10 <= |v| < 2^-6, where the reference's shift differs.
// (a) and (b) are fixed on the packed codes with byte-SIMD compares; a chunk
// with any element in band (c) is re-encoded with the exact integer routine.
__device__ __forceinline__ void encode16_e4m3_ref(const float (&v)[kChunk], uint32_t (&w)[4]) {
    uint32_t band = 0;
#pragma unroll
    for (int k = 0; k < kChunk; ++k)
        band |= static_cast<uint32_t>(((__float_as_uint(v[k]) & 0x7fffffffu) - 0x3a800000u) < 0x02000000u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        uint32_t c = cvt4_fp8_satfinite<MF_DT_F8E4M3>(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        // .satfinite yields magnitude 0x7f (S.1111.111) only for NaN inputs
        const uint32_t m7 = c & 0x7f7f7f7fu;
        const uint32_t nan = __vcmpeq4(m7, 0x7f7f7f7fu);
        const uint32_t big = __vcmpgeu4(m7, 0x78787878u);  // |v| >= 248
        c = (c & ~big) | (big & ((c & 0x80808080u) | 0x7e7e7e7eu));
        w[k] = (c & ~nan) | (nan & 0x7f7f7f7fu);
    }
    if (band) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t c = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) c |= f32bits_to_e4m3_ref(__float_as_uint(v[4 * k + j])) << (8 * j);
            w[k] = c;
        }
    }
}

// E5M2 encode of 16 values with the reference's rules (dtype/fp8.go:190-249):
// the hardware result is kept unless the chunk holds a value in the
// reference's subnormal band 2^-17 <= |v| < 2^-14, a value above 57344
// (the reference returns Inf there) or a NaN; such chunks take the exact
// integer routine.
__device__ __forceinline__ void encode16_e5m2_ref(const float (&v)[kChunk], uint32_t (&w)[4]) {
    uint32_t slow = 0;
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
        const uint32_t a = __float_as_uint(v[k]) & 0x7fffffffu;
        slow |= static_cast<uint32_t>((a - 0x37000000u) < 0x01800000u) | static_cast<uint32_t>(a > 0x47600000u);
    }
    if (slow) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t c = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) c |= f32bits_to_e5m2_ref(__float_as_uint(v[4 * k + j])) << (8 * j);
            w[k] = c;
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k] = cvt4_fp8_satfinite<MF_DT_F8E5M2>(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    }
}

// OCP .satfinite encode of 16 values with NaN -> 0x7f.  .satfinite never
// produces Inf, so a code magnitude of 0x7f (E4M3) or >= 0x7d (E5M2) is NaN.
template <int DT>
__device__ __forceinline__ void encode16_fp8_ocp(const float (&v)[kChunk], uint32_t (&w)[4]) {
    constexpr uint32_t kNanMag = (DT == MF_DT_F8E4M3) ? 0x7f7f7f7fu : 0x7d7d7d7du;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        w[k] = fp8x4_canonical_nan(cvt4_fp8_satfinite<DT>(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]),
                                   kNanMag);
}

// Encode 16 float32 values to a storage format.
template <int DT>
__device__ __forceinline__ void encode16(const float (&v)[kChunk], RawChunk<dtype_bytes(DT)>& r, int compat) {
    if constexpr (DT == MF_DT_F32) {
#pragma unroll
        for (int k = 0; k < kChunk; ++k) r.w[k] = __float_as_uint(v[k]);
    } else if constexpr (DT == MF_DT_BF16) {
#pragma unroll
        for (int k = 0; k < kChunk / 2; ++k) r.w[k] = f32x2_to_bf16x2(v[2 * k], v[2 * k + 1]);
    } else if constexpr (DT == MF_DT_F16) {
#pragma unroll
        for (int k = 0; k < kChunk / 2; ++k) r.w[k] = f32x2_to_f16x2(v[2 * k], v[2 * k + 1]);
    } else if constexpr (DT == MF_DT_F8E4M3) {
        if (compat) encode16_fp8_ocp<DT>(v, r.w);
        else encode16_e4m3_ref(v, r.w);
    } else if constexpr (DT == MF_DT_F8E5M2) {
        if (compat) encode16_fp8_ocp<DT>(v, r.w);
        else encode16_e5m2_ref(v, r.w);
    }
}

}  // namespace mf
