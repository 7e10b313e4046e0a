// mf_vec.cuh -- vector access and packed codecs for the streaming kernels.
//
// Two granularities:
//   * chunks of 16 elements (16 B of an 8-bit format, 32 B of a 16-bit
//     format, 64 B of float32) read with one to four 128-bit loads, used by
//     the amax folds;
//   * quads of 4 elements, owned by consecutive lanes so every warp-wide
//     access is one contiguous span whatever the element widths, used by the
//     element-wise maps (the streaming engine's lane steps, axpy).
// Inputs are read with the non-coherent path and the evict-first hint (each
// byte is read once); outputs are written with the streaming store hint.
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

// Packed RNE conversions for inputs known not to be NaN (the hardware and the
// reference agree on every non-NaN value).
__device__ __forceinline__ uint32_t f32x2_to_bf16x2_nonan(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ uint32_t f32x2_to_f16x2_nonan(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
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

// NaN lanes -> 0x7f without sign, four bytes at a time.  A byte is NaN when
// its magnitude plus `add4`'s byte carries into bit 7: add 0x01 for E4M3
// (NaN magnitude 0x7f), 0x03 for E5M2 (NaN magnitudes 0x7d..0x7f).
__device__ __forceinline__ uint32_t fp8x4_canonical_nan(uint32_t w, uint32_t add4) {
    const uint32_t hi = ((w & 0x7f7f7f7fu) + add4) & 0x80808080u;
    const uint32_t nan = hi | (hi - (hi >> 7));
    return (w & ~nan) | (nan & 0x7f7f7f7fu);
}

// ------------------------------------------------------------ quads
//
// A quad is 4 consecutive elements owned by one lane; lane l of a warp owns
// quad q0 + l, so one warp-wide access covers 128 consecutive elements
// (128..512 contiguous bytes) and every vector load and store is fully
// coalesced whatever the element widths on the two sides.

// Byte-wise mask: 0xff in every byte whose bit 7 is set in `hi` (other bits 0).
__device__ __forceinline__ uint32_t bytes_from_bit7(uint32_t hi) { return hi | (hi - (hi >> 7)); }

// Four float32 -> four E4M3 codes with the reference's rules
// (dtype/fp8.go:77-136).  The hardware .satfinite conversion agrees with the
// reference except (a) |v| >= 248, which the reference saturates to 0x7e
// (hardware codes 0x78..0x7e, fixed with a byte mask), and (b) the
// reference's subnormal band 2^-10 <= |v| < 2^-6, (c) NaN -> 0x7f.  Band
// values get hardware codes 1..8, or 0 for exactly 2^-10; NaN gets 0x7f.
// A quad holding any of those is re-encoded with the exact integer routine.
//
// In the band the reference computes min(8, RNE(|v| * 2^10)) (its shift is
// one short), which is the hardware code of 2v clamped to 8.  So a quad with
// a band value is fixed with a second hardware conversion and byte masks;
// only a NaN or a value of exactly 2^-10 (the hardware rounds that tie to 0,
// the reference to 1) falls back to the scalar routine.
static __device__ __noinline__ uint32_t e4m3_ref_scalar4(float v0, float v1, float v2, float v3) {
    return f32bits_to_e4m3_ref(__float_as_uint(v0)) | (f32bits_to_e4m3_ref(__float_as_uint(v1)) << 8) |
           (f32bits_to_e4m3_ref(__float_as_uint(v2)) << 16) | (f32bits_to_e4m3_ref(__float_as_uint(v3)) << 24);
}

__device__ __forceinline__ uint32_t e4m3_ref_low(uint32_t res, uint32_t c, float v0, float v1, float v2, float v3) {
    const uint32_t c7 = c & 0x7f7f7f7fu;
    const bool nan = ((c7 + 0x01010101u) & 0x80808080u) != 0;
    const bool tie = (fabsf(v0) == 0.0009765625f) | (fabsf(v1) == 0.0009765625f) | (fabsf(v2) == 0.0009765625f) |
                     (fabsf(v3) == 0.0009765625f);
    if (nan | tie) return e4m3_ref_scalar4(v0, v1, v2, v3);
    // band lanes: hardware code in [1, 8] (y has a zero byte exactly there)
    const uint32_t y = ((c7 + 0x77777777u) ^ 0x78787878u) & 0xf8f8f8f8u;
    const uint32_t band = bytes_from_bit7(~(((y & 0x7f7f7f7fu) + 0x7f7f7f7fu) | y) & 0x80808080u);
    const uint32_t c2 = cvt4_fp8_satfinite<MF_DT_F8E4M3>(v0 + v0, v1 + v1, v2 + v2, v3 + v3) & 0x7f7f7f7fu;
    const uint32_t ge8 = bytes_from_bit7((c2 + 0x78787878u) & 0x80808080u);
    const uint32_t low = (c2 & ~ge8) | (0x08080808u & ge8) | (c & 0x80808080u);
    return (res & ~band) | (low & band);
}

__device__ __forceinline__ uint32_t encode4_e4m3_ref(float v0, float v1, float v2, float v3) {
    const uint32_t c = cvt4_fp8_satfinite<MF_DT_F8E4M3>(v0, v1, v2, v3);
    const uint32_t c7 = c & 0x7f7f7f7fu;
    const uint32_t big = bytes_from_bit7((c7 + 0x08080808u) & 0x80808080u);  // code >= 0x78
    const uint32_t res = (c & ~big) | (big & ((c & 0x80808080u) | 0x7e7e7e7eu));
    // any code in [0, 8] or 0x7f: (code + 1) mod 128 < 10
    const uint32_t t = ((c7 + 0x01010101u) & 0x7f7f7f7fu) + 0x76767676u;
    if (~t & 0x80808080u) return e4m3_ref_low(res, c, v0, v1, v2, v3);
    return res;
}

// Four float32 -> four E5M2 codes with the reference's rules
// (dtype/fp8.go:190-249): the hardware result unless a value lies in the
// reference's subnormal band 2^-17 <= |v| < 2^-14, above 57344 (the
// reference returns Inf) or is NaN; then the exact integer routine.
__device__ __forceinline__ bool e5m2_needs_exact(float v0, float v1, float v2, float v3) {
    const float a[4] = {fabsf(v0), fabsf(v1), fabsf(v2), fabsf(v3)};
    bool slow = false;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        slow |= ((a[j] >= 7.62939453125e-06f) & (a[j] < 6.103515625e-05f)) | !(a[j] <= 57344.0f);
    return slow;
}

__device__ __forceinline__ uint32_t encode4_e5m2_ref(float v0, float v1, float v2, float v3) {
    if (e5m2_needs_exact(v0, v1, v2, v3))
        return f32bits_to_e5m2_ref(__float_as_uint(v0)) | (f32bits_to_e5m2_ref(__float_as_uint(v1)) << 8) |
               (f32bits_to_e5m2_ref(__float_as_uint(v2)) << 16) | (f32bits_to_e5m2_ref(__float_as_uint(v3)) << 24);
    return cvt4_fp8_satfinite<MF_DT_F8E5M2>(v0, v1, v2, v3);
}

// 0xff in every byte of x whose bit 7 is set, 0x00 in the others: one byte
// permute with sign replication (selector nibble 8 + k copies the sign of
// byte k over all 8 bits of target byte k).
__device__ __forceinline__ uint32_t bytes_sign_mask(uint32_t x) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, 0xBA98;" : "=r"(r) : "r"(x));
    return r;
}

// The common case of the two encoders above, without their fix-up branch:
// returns the reference codes in `out` and a nonzero flag word when the quad
// needs encode4_e4m3_ref / encode4_e5m2_ref (then `out` is meaningless).
// Every byte sum below stays under 0x100 (codes have magnitude <= 0x7f), so no
// carry crosses a byte.
template <int DT>
__device__ __forceinline__ uint32_t encode4_fp8_fast(const float (&v)[4], uint32_t& out) {
    if constexpr (DT == MF_DT_F8E4M3) {
        const uint32_t c = cvt4_fp8_satfinite<MF_DT_F8E4M3>(v[0], v[1], v[2], v[3]);
        const uint32_t c7 = c & 0x7f7f7f7fu;
        const uint32_t big = bytes_sign_mask(c7 + 0x08080808u);  // code >= 0x78: the reference's 0x7e
        out = (c & ~big) | (big & ((c & 0x80808080u) | 0x7e7e7e7eu));
        // code <= 8 (c7 + 0x77 < 0x80) or NaN 0x7f (c7 + 0x01 == 0x80)
        return (~(c7 + 0x77777777u) | (c7 + 0x01010101u)) & 0x80808080u;
    } else {
        out = cvt4_fp8_satfinite<MF_DT_F8E5M2>(v[0], v[1], v[2], v[3]);
        return e5m2_needs_exact(v[0], v[1], v[2], v[3]) ? 1u : 0u;
    }
}

template <int DT>
__device__ __forceinline__ uint32_t encode4_fp8_ref(const float (&v)[4]) {
    if constexpr (DT == MF_DT_F8E4M3) return encode4_e4m3_ref(v[0], v[1], v[2], v[3]);
    else return encode4_e5m2_ref(v[0], v[1], v[2], v[3]);
}

// Decode one quad (raw words w[0 .. bytes-1]) of a floating storage format.
template <int DT>
__device__ __forceinline__ void decode4(const uint32_t* w, float (&v)[4]) {
    if constexpr (DT == MF_DT_F32) {
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = __uint_as_float(w[k]);
    } else if constexpr (DT == MF_DT_BF16) {
        v[0] = __uint_as_float(w[0] << 16);
        v[1] = __uint_as_float(w[0] & 0xffff0000u);
        v[2] = __uint_as_float(w[1] << 16);
        v[3] = __uint_as_float(w[1] & 0xffff0000u);
    } else if constexpr (DT == MF_DT_F16) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            f16x2_to_f32x2(w[k], v[2 * k], v[2 * k + 1]);
            if (((w[k] & 0x7fff7fffu) + 0x03ff03ffu) & 0x80008000u) {
                v[2 * k] = __uint_as_float(f16_to_f32bits(w[k] & 0xffffu));
                v[2 * k + 1] = __uint_as_float(f16_to_f32bits(w[k] >> 16));
            }
        }
    } else if constexpr (DT == MF_DT_F8E4M3) {
        f16x2_to_f32x2(e4m3x2_to_f16x2(w[0]), v[0], v[1]);
        f16x2_to_f32x2(e4m3x2_to_f16x2(w[0] >> 16), v[2], v[3]);
        const uint32_t x = ~w[0] & 0x7f7f7f7fu;
        if ((x - 0x01010101u) & ~x & 0x80808080u) {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = __uint_as_float(e4m3_to_f32bits((w[0] >> (8 * j)) & 0xffu));
        }
    } else if constexpr (DT == MF_DT_F8E5M2) {
        f16x2_to_f32x2(__byte_perm(w[0], 0u, 0x1404u), v[0], v[1]);
        f16x2_to_f32x2(__byte_perm(w[0], 0u, 0x3424u), v[2], v[3]);
        if (((w[0] & 0x7f7f7f7fu) + 0x03030303u) & 0x80808080u) {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = __uint_as_float(e5m2_to_f32bits((w[0] >> (8 * j)) & 0xffu));
        }
    }
}

// Encode one quad to raw words o[0 .. bytes-1].
template <int DT>
__device__ __forceinline__ void encode4(const float (&v)[4], uint32_t* o, int compat) {
    if constexpr (DT == MF_DT_F32) {
#pragma unroll
        for (int k = 0; k < 4; ++k) o[k] = __float_as_uint(v[k]);
    } else if constexpr (DT == MF_DT_BF16) {
        o[0] = f32x2_to_bf16x2(v[0], v[1]);
        o[1] = f32x2_to_bf16x2(v[2], v[3]);
    } else if constexpr (DT == MF_DT_F16) {
        o[0] = f32x2_to_f16x2(v[0], v[1]);
        o[1] = f32x2_to_f16x2(v[2], v[3]);
    } else if constexpr (DT == MF_DT_F8E4M3) {
        o[0] = compat ? fp8x4_canonical_nan(cvt4_fp8_satfinite<DT>(v[0], v[1], v[2], v[3]), 0x01010101u)
                      : encode4_e4m3_ref(v[0], v[1], v[2], v[3]);
    } else if constexpr (DT == MF_DT_F8E5M2) {
        o[0] = compat ? fp8x4_canonical_nan(cvt4_fp8_satfinite<DT>(v[0], v[1], v[2], v[3]), 0x03030303u)
                      : encode4_e5m2_ref(v[0], v[1], v[2], v[3]);
    }
}

// Quad-sized vector access: 4 elements of `Bytes` each.
template <int Bytes>
__device__ __forceinline__ void store4_stream(void* p, const uint32_t* w) {
    if constexpr (Bytes == 1) {
        asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(p), "r"(w[0]) : "memory");
    } else if constexpr (Bytes == 2) {
        asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(w[0]), "r"(w[1]) : "memory");
    } else {
        asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                     : "memory");
    }
}

// Coherent streaming load (evict-first), for buffers the kernel also writes
// (the in-place y of axpy): the non-coherent path requires read-only data.
template <int Bytes>
__device__ __forceinline__ void load4_cs(const void* p, uint32_t* w) {
    if constexpr (Bytes == 1) {
        asm volatile("ld.global.cs.u32 %0, [%1];" : "=r"(w[0]) : "l"(p));
    } else if constexpr (Bytes == 2) {
        asm volatile("ld.global.cs.v2.u32 {%0,%1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "l"(p));
    } else {
        asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                     : "l"(p));
    }
}

template <int Bytes>
__device__ __forceinline__ void load4_stream(const void* p, uint32_t* w) {
    if constexpr (Bytes == 1) {
        asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(w[0]) : "l"(p));
    } else if constexpr (Bytes == 2) {
        asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "l"(p));
    } else {
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                     : "l"(p));
    }
}

}  // namespace mf
