// int4.cu -- K4: packed Int4 group dequantisation (mf_int4_dequant_grouped).
//
//   out[r, c] = encode( float32(q[r, c]) * float32(scale[r, c / group]) )
//
// q: row-major [rows, cols] signed nibbles, element 2i in the low nibble of
// byte i (dtype/int4.go:12-40, dtype/convert/decoders.go:262-289).
// scales: row-major [rows, ceil(cols / group)].  The product of a nibble
// in [-8, 7] and a BF16/F16 scale is exact in float32, so the only rounding
// is the final store encode (NewBfloat16FromFloat32, dtype/bfloat16.go:41-55).
//
// Paths, fastest first (all need 16-byte aligned q and out):
//   * flat words (cols % 8 == 0, cols % group == 0, group / 8 a power of two):
//     one grid-stride loop over the packed 32-bit words of the whole tensor,
//     the scale index a shift of the word index;
//   * row words (cols % 8 == 0, group % 8 == 0): the same per-word body on a
//     (row segment, row) grid;
//   * a per-element kernel for any even cols.
// Lane l of a warp owns word w0 + l: a warp reads 128 contiguous bytes of q
// and writes 512 contiguous bytes of BF16.  Nibble -> float uses the exponent
// trick: (n ^ 8) | 0x4B000000 is the float 2^23 + q + 8, so q = that -
// (2^23 + 8) exactly, with no I2F.
// Roofline: HBM, 0.5 B in + 2 B out per element + scales.
#include "mf_runtime.h"
#include "mf_vec.cuh"

namespace mf {
namespace {

constexpr int kThreads = 256;

template <int SDT>
__device__ __forceinline__ float load_scale(const void* s, int64_t i) {
    if constexpr (SDT == MF_DT_BF16) return __uint_as_float(static_cast<uint32_t>(__ldg(static_cast<const uint16_t*>(s) + i)) << 16);
    else if constexpr (SDT == MF_DT_F16) return __uint_as_float(f16_to_f32bits(__ldg(static_cast<const uint16_t*>(s) + i)));
    else return __ldg(static_cast<const float*>(s) + i);
}

// nibble k (0..7) of w as float32 (exact), via 2^23 + (q + 8) - (2^23 + 8)
__device__ __forceinline__ float nibble_f32(uint32_t w, int k) {
    const uint32_t bits = ((w >> (4 * k)) & 0xfu) ^ 0x4B000008u;
    return __fsub_rn(__uint_as_float(bits), 8388616.0f);
}

// One packed word (8 nibbles, elements e .. e+7) times its group scale,
// encoded and stored with 128-bit streaming stores.
template <int ODT>
__device__ __forceinline__ void dequant_word(uint32_t w, float s, void* __restrict__ out, int64_t e) {
    float v[8];
    uint32_t p[4];
    if (fabsf(s) <= 3.402823466e38f) {
        // Finite scale: the products are finite, so no NaN rule is needed.
        // Low nibbles (elements 0,2,4,6) and high nibbles (1,3,5,7), each
        // xor 8, land in the low byte of 0x4B0000nn = 2^23 + q + 8.
        const uint32_t lo = (w & 0x0f0f0f0fu) ^ 0x08080808u;
        const uint32_t hi = ((w >> 4) & 0x0f0f0f0fu) ^ 0x08080808u;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 m = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7650u + j)),
                                         __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7650u + j)));
            const float2 qv = __fadd2_rn(m, make_float2(-8388616.0f, -8388616.0f));  // exact q
            const float2 pr = __fmul2_rn(qv, make_float2(s, s));                      // exact q * s
            v[2 * j] = pr.x;
            v[2 * j + 1] = pr.y;
            if constexpr (ODT == MF_DT_BF16) p[j] = f32x2_to_bf16x2_nonan(pr.x, pr.y);
            else if constexpr (ODT == MF_DT_F16) p[j] = f32x2_to_f16x2_nonan(pr.x, pr.y);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = x86_mul(nibble_f32(w, j), s);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if constexpr (ODT == MF_DT_BF16) p[j] = f32x2_to_bf16x2(v[2 * j], v[2 * j + 1]);
            else if constexpr (ODT == MF_DT_F16) p[j] = f32x2_to_f16x2(v[2 * j], v[2 * j + 1]);
        }
    }
    if constexpr (ODT == MF_DT_F32) {
        uint4* o = reinterpret_cast<uint4*>(static_cast<float*>(out) + e);
        st_stream(o, make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                                __float_as_uint(v[3])));
        st_stream(o + 1, make_uint4(__float_as_uint(v[4]), __float_as_uint(v[5]), __float_as_uint(v[6]),
                                    __float_as_uint(v[7])));
    } else {
        st_stream(reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + e), make_uint4(p[0], p[1], p[2], p[3]));
    }
}

__device__ __forceinline__ uint32_t ld_word_once(const uint32_t* p) {
    uint32_t x;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(x) : "l"(p));
    return x;
}

// Word layout: a 32-bit word of q holds 8 consecutive nibbles (elements
// 8w .. 8w+7 of a row when cols % 8 == 0).  Lane l of a warp owns word w0 + l,
// so a warp reads 128 contiguous bytes of q and writes 32 x 8 outputs
// contiguously (512 B of BF16) per access.
//
// Flat form (also cols % group == 0 and group / 8 a power of two): the scale
// array [rows, cols / group] is then indexed by (flat word) >> log2(group / 8),
// so one grid-stride loop over all words of the tensor needs no row
// arithmetic; each thread keeps kFlatSteps words in flight (loads first, then
// the math and the stores).
// Compile-time tunable: 8 words in flight measured the same as 4 on config 2.
#ifndef MF_INT4_FLAT_STEPS
#define MF_INT4_FLAT_STEPS 4
#endif
constexpr int kFlatSteps = MF_INT4_FLAT_STEPS;

template <int SDT, int ODT>
__global__ void __launch_bounds__(kThreads) int4_dequant_flat_kernel(const uint32_t* __restrict__ q,
                                                                    const void* __restrict__ scales,
                                                                    void* __restrict__ out, int64_t nwords,
                                                                    int32_t gw_shift) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t w0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; w0 + (kFlatSteps - 1) * stride < nwords; w0 += kFlatSteps * stride) {
        uint32_t wv[kFlatSteps];
        float sv[kFlatSteps];
#pragma unroll
        for (int k = 0; k < kFlatSteps; ++k) {
            const int64_t w = w0 + k * stride;
            wv[k] = ld_word_once(q + w);
            sv[k] = load_scale<SDT>(scales, w >> gw_shift);
        }
#pragma unroll
        for (int k = 0; k < kFlatSteps; ++k) dequant_word<ODT>(wv[k], sv[k], out, (w0 + k * stride) * 8);
    }
    for (; w0 < nwords; w0 += stride) dequant_word<ODT>(ld_word_once(q + w0), load_scale<SDT>(scales, w0 >> gw_shift), out, w0 * 8);
}

// Row form for any group that is a multiple of 8 (a word never straddles a
// group): blockIdx.y walks rows, blockIdx.x covers a row in segments of
// kThreads * kWords words, each thread handling kWords words spaced by the
// block size.
constexpr int kWords = 4;

template <int SDT, int ODT>
__global__ void __launch_bounds__(kThreads) int4_dequant_words_kernel(const uint32_t* __restrict__ q,
                                                                     const void* __restrict__ scales,
                                                                     void* __restrict__ out, int64_t rows,
                                                                     uint32_t words_per_row, int32_t gw_shift,
                                                                     uint32_t group_words, int64_t ngroups) {
    const uint32_t seg = blockIdx.x;
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const uint32_t* qrow = q + r * words_per_row;
        uint32_t wv[kWords];
        float sv[kWords];
        uint32_t widx[kWords];
#pragma unroll
        for (int k = 0; k < kWords; ++k) {
            widx[k] = (seg * kWords + k) * kThreads + threadIdx.x;
            if (widx[k] < words_per_row) {
                wv[k] = ld_word_once(qrow + widx[k]);
                const uint32_t g = gw_shift >= 0 ? (widx[k] >> gw_shift) : (widx[k] / group_words);
                sv[k] = load_scale<SDT>(scales, r * ngroups + g);
            }
        }
#pragma unroll
        for (int k = 0; k < kWords; ++k)
            if (widx[k] < words_per_row) dequant_word<ODT>(wv[k], sv[k], out, (r * words_per_row + widx[k]) * 8);
    }
}

// Any shape with even cols: one element per thread-iteration.
template <int SDT, int ODT>
__global__ void __launch_bounds__(kThreads) int4_dequant_scalar_kernel(const uint8_t* __restrict__ q,
                                                                      const void* __restrict__ scales,
                                                                      void* __restrict__ out, int64_t rows,
                                                                      int64_t cols, int64_t group,
                                                                      int64_t ngroups) {
    const int64_t n = rows * cols;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += stride) {
        const int64_t r = e / cols;
        const int64_t col = e - r * cols;
        const float qv = load_as_f32<MF_DT_I4>(q, e);
        const float v = x86_mul(qv, load_scale<SDT>(scales, r * ngroups + col / group));
        store_code<ODT>(out, e, encode_f32<ODT>(v, 0));
    }
}

template <int SDT, int ODT>
int launch(const void* q, const void* scales, void* out, int64_t rows, int64_t cols, int64_t group,
           cudaStream_t s) {
    const int64_t ngroups = (cols + group - 1) / group;
    const bool words = (cols % 8 == 0) && (group % 8 == 0) && aligned16(q) && aligned16(out) &&
                       (cols / 8) < (int64_t(1) << 31);
    if (words) {
        const uint32_t words_per_row = static_cast<uint32_t>(cols / 8);
        const uint32_t group_words = static_cast<uint32_t>(group / 8);
        int32_t gw_shift = -1;
        if ((group_words & (group_words - 1)) == 0) {
            gw_shift = 0;
            while ((1u << gw_shift) < group_words) ++gw_shift;
        }
        if (gw_shift >= 0 && cols % group == 0) {
            const int64_t nwords = rows * words_per_row;
            const int64_t blocks = std::min<int64_t>(static_cast<int64_t>(state().sm_count) * (2048 / kThreads),
                                                     (nwords + kThreads - 1) / kThreads);
            int4_dequant_flat_kernel<SDT, ODT><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(
                static_cast<const uint32_t*>(q), scales, out, nwords, gw_shift);
        } else {
            const uint32_t per_block = kThreads * kWords;
            dim3 grid((words_per_row + per_block - 1) / per_block,
                      static_cast<unsigned>(std::min<int64_t>(rows, 65535)));
            int4_dequant_words_kernel<SDT, ODT><<<grid, kThreads, 0, s>>>(
                static_cast<const uint32_t*>(q), scales, out, rows, words_per_row, gw_shift, group_words, ngroups);
        }
    } else {
        const int64_t blocks = stream_grid(rows * cols, kThreads, 8);
        int4_dequant_scalar_kernel<SDT, ODT><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(
            static_cast<const uint8_t*>(q), scales, out, rows, cols, group, ngroups);
    }
    MF_LAUNCH_CHECK("mf_int4_dequant_grouped launch");
    return MF_OK;
}

template <int SDT>
int dispatch_out(int out_dtype, const void* q, const void* scales, void* out, int64_t rows, int64_t cols,
                 int64_t group, cudaStream_t s) {
    switch (out_dtype) {
    case MF_DT_BF16: return launch<SDT, MF_DT_BF16>(q, scales, out, rows, cols, group, s);
    case MF_DT_F16: return launch<SDT, MF_DT_F16>(q, scales, out, rows, cols, group, s);
    default: return launch<SDT, MF_DT_F32>(q, scales, out, rows, cols, group, s);
    }
}

}  // namespace
}  // namespace mf

using namespace mf;

extern "C" int mf_int4_dequant_grouped(const void* q, const void* scales, int scale_dtype, void* out,
                                       int out_dtype, int64_t rows, int64_t cols, int64_t group,
                                       mf_stream stream) {
    MF_ENTER();
    if (rows < 0 || cols < 0)
        return fail(MF_ERR_SHAPE_INVALID, "mf_int4_dequant_grouped: negative shape [%lld, %lld]",
                    (long long)rows, (long long)cols);
    if (cols % 2 != 0)
        return fail(MF_ERR_SHAPE_INVALID, "mf_int4_dequant_grouped: cols (%lld) must be even", (long long)cols);
    if (group <= 0)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_int4_dequant_grouped: group must be positive, got %lld",
                    (long long)group);
    if (scale_dtype != MF_DT_BF16 && scale_dtype != MF_DT_F16 && scale_dtype != MF_DT_F32)
        return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_int4_dequant_grouped: scale dtype %d unsupported", scale_dtype);
    if (!is_float_store_dtype(out_dtype))
        return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_int4_dequant_grouped: output dtype %d unsupported", out_dtype);
    if (rows == 0 || cols == 0) return MF_OK;
    if (!q || !scales || !out) return fail(MF_ERR_INVALID_ARGUMENT, "mf_int4_dequant_grouped: NULL buffer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (scale_dtype) {
    case MF_DT_BF16: return dispatch_out<MF_DT_BF16>(out_dtype, q, scales, out, rows, cols, group, s);
    case MF_DT_F16: return dispatch_out<MF_DT_F16>(out_dtype, q, scales, out, rows, cols, group, s);
    default: return dispatch_out<MF_DT_F32>(out_dtype, q, scales, out, rows, cols, group, s);
    }
}
