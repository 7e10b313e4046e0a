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

// Decode 16 elements of a floating storage format to float32.
template <int DT>
__device__ __forceinline__ void decode16(const RawChunk<dtype_bytes(DT)>& r, float (&v)[kChunk]) {
#pragma unroll
    for (int k = 0; k < kChunk; ++k) {
        if constexpr (DT == MF_DT_F32) {
            v[k] = __uint_as_float(r.w[k]);
        } else if constexpr (DT == MF_DT_BF16) {
            const uint32_t w = r.w[k >> 1];
            v[k] = __uint_as_float((k & 1) ? (w & 0xffff0000u) : (w << 16));
        } else if constexpr (DT == MF_DT_F16) {
            const uint32_t w = r.w[k >> 1];
            v[k] = __uint_as_float(f16_to_f32bits((k & 1) ? (w >> 16) : (w & 0xffffu)));
        } else if constexpr (DT == MF_DT_F8E4M3) {
            v[k] = __uint_as_float(e4m3_to_f32bits((r.w[k >> 2] >> (8 * (k & 3))) & 0xffu));
        } else if constexpr (DT == MF_DT_F8E5M2) {
            v[k] = __uint_as_float(e5m2_to_f32bits((r.w[k >> 2] >> (8 * (k & 3))) & 0xffu));
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
    } else if constexpr (DT == MF_DT_F8E4M3 || DT == MF_DT_F8E5M2) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            uint32_t w = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) w |= encode_f32<DT>(v[4 * k + j], compat) << (8 * j);
            r.w[k] = w;
        }
    }
}

}  // namespace mf
