// axpy.cu -- K5 (mf_axpy) and K6 (mf_scalar_broadcast).
//
// mf_axpy replaces axpyDevice.Axpy (runtime/axpy.go:13-15, called at
// :84-90) and the host loops of axpyOntoHost (:115-117 and :145-147 with
// the BF16/F16 re-encode of float32VectorBytes, :171-194):
//   y[i] = encode( decode(y[i]) + alpha * decode(x[i]) )
// with the float32 multiply and add rounded separately (the amd64 Go
// build does not contract), or one fused rounding when fused_fma is set.
// mf_scalar_broadcast replaces applyScalarBroadcast
// (runtime/executor_math.go:195-234) plus its store encode.
// Both work on lane-contiguous quads (4 elements per lane per access).
// Roofline: HBM; axpy moves 3 * sizeof(dtype) bytes per element.
#include "mf_runtime.h"
#include "mf_vec.cuh"

namespace mf {
namespace {

constexpr int kThreads = 256;

// y + alpha * x with the amd64 NaN rule (Go source order: y += alpha*addend).
template <int FUSED>
__device__ __forceinline__ float axpy_op(float y, float x, float alpha) {
    if constexpr (FUSED) return x86_fma(alpha, x, y);
    else return x86_add(y, x86_mul(alpha, x));
}

// Lane-contiguous quads: lane l owns elements 4(q0 + l) .. +3, so every
// warp access is one contiguous span; each thread keeps kUnroll quads of y
// and of x in flight.
constexpr int kUnroll = 4;

template <int DT, int FUSED>
__device__ __forceinline__ void axpy_quad(void* y, const uint32_t* yw, const uint32_t* xw, int64_t q, float alpha) {
    constexpr int B = dtype_bytes(DT);
    float vy[4], vx[4];
    decode4<DT>(yw, vy);
    decode4<DT>(xw, vx);
#pragma unroll
    for (int k = 0; k < 4; ++k) vy[k] = axpy_op<FUSED>(vy[k], vx[k], alpha);
    uint32_t o[B];
    encode4<DT>(vy, o, 0);
    store4_stream<B>(static_cast<uint8_t*>(y) + q * 4 * B, o);
}

template <int DT, int FUSED>
__global__ void __launch_bounds__(kThreads) axpy_vec_kernel(void* y, const void* __restrict__ x,
                                                           int64_t n, float alpha) {
    constexpr int B = dtype_bytes(DT);
    const int64_t nq = n / 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const uint8_t* yb = static_cast<const uint8_t*>(y);
    const uint8_t* xb = static_cast<const uint8_t*>(x);
    int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; q + (kUnroll - 1) * stride < nq; q += kUnroll * stride) {
        uint32_t yw[kUnroll][B], xw[kUnroll][B];
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) {
            load4_cs<B>(yb + (q + j * stride) * 4 * B, yw[j]);
            load4_stream<B>(xb + (q + j * stride) * 4 * B, xw[j]);
        }
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) axpy_quad<DT, FUSED>(y, yw[j], xw[j], q + j * stride, alpha);
    }
    for (; q < nq; q += stride) {
        uint32_t yw[B], xw[B];
        load4_cs<B>(yb + q * 4 * B, yw);
        load4_stream<B>(xb + q * 4 * B, xw);
        axpy_quad<DT, FUSED>(y, yw, xw, q, alpha);
    }
    if (blockIdx.x == 0) {
        const int64_t i = nq * 4 + threadIdx.x;
        if (i < n) {
            const float r = axpy_op<FUSED>(load_as_f32<DT>(y, i), load_as_f32<DT>(x, i), alpha);
            store_code<DT>(y, i, encode_f32<DT>(r, 0));
        }
    }
}

template <int DT, int FUSED>
__global__ void __launch_bounds__(kThreads) axpy_scalar_kernel(void* __restrict__ y, const void* __restrict__ x,
                                                              int64_t n, float alpha) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float r = axpy_op<FUSED>(load_as_f32<DT>(y, i), load_as_f32<DT>(x, i), alpha);
        store_code<DT>(y, i, encode_f32<DT>(r, 0));
    }
}

template <int DT>
int launch_axpy(void* y, const void* x, int64_t n, float alpha, int fused, cudaStream_t s) {
    if (aligned16(y) && aligned16(x)) {
        const int64_t blocks = stream_grid(n / 4 / kUnroll + 1, kThreads, 8);
        if (fused) axpy_vec_kernel<DT, 1><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(y, x, n, alpha);
        else axpy_vec_kernel<DT, 0><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(y, x, n, alpha);
    } else {
        const int64_t blocks = stream_grid(n, kThreads, 8);
        if (fused) axpy_scalar_kernel<DT, 1><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(y, x, n, alpha);
        else axpy_scalar_kernel<DT, 0><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(y, x, n, alpha);
    }
    MF_LAUNCH_CHECK("mf_axpy launch");
    return MF_OK;
}

// ------------------------------------------------------ scalar broadcast

template <int OP>
__device__ __forceinline__ float scalar_op(float v, float s) {
    if constexpr (OP == MF_SCALAR_ADD) return x86_add(v, s);
    else if constexpr (OP == MF_SCALAR_SUB) return x86_sub(v, s);
    else if constexpr (OP == MF_SCALAR_MUL) return x86_mul(v, s);
    else return x86_div(v, s);
}

template <int SRC, int DST, int OP>
__global__ void __launch_bounds__(kThreads) scalar_vec_kernel(const void* __restrict__ src, void* __restrict__ dst,
                                                             int64_t n, float scalar) {
    constexpr int BI = dtype_bytes(SRC), BO = dtype_bytes(DST);
    const int64_t nq = n / 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const uint8_t* sb = static_cast<const uint8_t*>(src);
    int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; q + (kUnroll - 1) * stride < nq; q += kUnroll * stride) {
        uint32_t w[kUnroll][BI];
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) load4_cs<BI>(sb + (q + j * stride) * 4 * BI, w[j]);
#pragma unroll
        for (int j = 0; j < kUnroll; ++j) {
            float v[4];
            decode4<SRC>(w[j], v);
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = scalar_op<OP>(v[k], scalar);
            uint32_t o[BO];
            encode4<DST>(v, o, 0);
            store4_stream<BO>(static_cast<uint8_t*>(dst) + (q + j * stride) * 4 * BO, o);
        }
    }
    for (; q < nq; q += stride) {
        uint32_t w[BI];
        load4_cs<BI>(sb + q * 4 * BI, w);
        float v[4];
        decode4<SRC>(w, v);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = scalar_op<OP>(v[k], scalar);
        uint32_t o[BO];
        encode4<DST>(v, o, 0);
        store4_stream<BO>(static_cast<uint8_t*>(dst) + q * 4 * BO, o);
    }
    if (blockIdx.x == 0) {
        const int64_t i = nq * 4 + threadIdx.x;
        if (i < n) store_code<DST>(dst, i, encode_f32<DST>(scalar_op<OP>(load_as_f32<SRC>(src, i), scalar), 0));
    }
}

template <int SRC, int DST, int OP>
__global__ void __launch_bounds__(kThreads) scalar_elem_kernel(const void* __restrict__ src, void* __restrict__ dst,
                                                              int64_t n, float scalar) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        store_code<DST>(dst, i, encode_f32<DST>(scalar_op<OP>(load_as_f32<SRC>(src, i), scalar), 0));
}

template <int SRC, int DST, int OP>
void launch_scalar_op(const void* src, void* dst, int64_t n, float scalar, cudaStream_t s) {
    constexpr bool kVecSrc = SRC == MF_DT_F32 || SRC == MF_DT_F16 || SRC == MF_DT_BF16 || SRC == MF_DT_F8E4M3 ||
                             SRC == MF_DT_F8E5M2;
    if (kVecSrc && aligned16(src) && aligned16(dst)) {
        if constexpr (kVecSrc) {
            const int64_t blocks = stream_grid(n / 4 / kUnroll + 1, kThreads, 8);
            scalar_vec_kernel<SRC, DST, OP><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(src, dst, n, scalar);
        }
    } else {
        const int64_t blocks = stream_grid(n, kThreads, 8);
        scalar_elem_kernel<SRC, DST, OP><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(src, dst, n, scalar);
    }
}

template <int SRC, int DST>
void dispatch_op(int op, const void* src, void* dst, int64_t n, float scalar, cudaStream_t s) {
    switch (op) {
    case MF_SCALAR_ADD: launch_scalar_op<SRC, DST, MF_SCALAR_ADD>(src, dst, n, scalar, s); break;
    case MF_SCALAR_SUB: launch_scalar_op<SRC, DST, MF_SCALAR_SUB>(src, dst, n, scalar, s); break;
    case MF_SCALAR_MUL: launch_scalar_op<SRC, DST, MF_SCALAR_MUL>(src, dst, n, scalar, s); break;
    default: launch_scalar_op<SRC, DST, MF_SCALAR_DIV>(src, dst, n, scalar, s); break;
    }
}

template <int SRC>
void dispatch_scalar_dst(int dst_dt, int op, const void* src, void* dst, int64_t n, float scalar, cudaStream_t s) {
    switch (dst_dt) {
    case MF_DT_F32: dispatch_op<SRC, MF_DT_F32>(op, src, dst, n, scalar, s); break;
    case MF_DT_F16: dispatch_op<SRC, MF_DT_F16>(op, src, dst, n, scalar, s); break;
    default: dispatch_op<SRC, MF_DT_BF16>(op, src, dst, n, scalar, s); break;
    }
}

// math.linspace (runtime/executor_math.go:57-108): v[i] = start + float32(i) * step,
// every operation rounded to float32 and nothing contracted, the endpoints pinned when
// they are included, encoded with the store encoder.  With a finite start and step no
// NaN can arise, so plain operations are exact; otherwise the amd64 NaN rule applies.
template <int DT, bool SPECIAL>
__global__ void __launch_bounds__(256) linspace_kernel(float start, float stop, float step, int64_t count,
                                                       int pin_ends, void* __restrict__ dst) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
        const float fi = __ll2float_rn(i);
        float v = SPECIAL ? x86_add(start, x86_mul(fi, step)) : __fadd_rn(start, __fmul_rn(fi, step));
        if (count == 1 || (pin_ends && i == 0)) v = start;
        if (pin_ends && i == count - 1) v = stop;
        store_code<DT>(dst, i, encode_f32<DT>(v, 0));
    }
}

template <int DT>
void launch_linspace(float start, float stop, float step, int64_t count, int pin_ends, void* dst, cudaStream_t s) {
    const unsigned blocks = static_cast<unsigned>(stream_grid(count, 256, 8));
    const bool special = !(fabsf(start) <= 3.402823466e38f) || !(fabsf(step) <= 3.402823466e38f);
    if (special) linspace_kernel<DT, true><<<blocks, 256, 0, s>>>(start, stop, step, count, pin_ends, dst);
    else linspace_kernel<DT, false><<<blocks, 256, 0, s>>>(start, stop, step, count, pin_ends, dst);
}

}  // namespace
}  // namespace mf

using namespace mf;

extern "C" int mf_axpy(void* y, const void* x, int64_t n, float alpha, int dtype, int fused_fma,
                       mf_stream stream) {
    MF_ENTER();
    if (n < 0) return fail(MF_ERR_SHAPE_INVALID, "mf_axpy: negative element count %lld", (long long)n);
    if (!is_float_store_dtype(dtype))
        return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_axpy: dtype %d unsupported (F32, F16, BF16)", dtype);
    if (n == 0) return MF_OK;
    if (!y || !x) return fail(MF_ERR_INVALID_ARGUMENT, "mf_axpy: NULL buffer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (dtype) {
    case MF_DT_F32: return launch_axpy<MF_DT_F32>(y, x, n, alpha, fused_fma, s);
    case MF_DT_BF16: return launch_axpy<MF_DT_BF16>(y, x, n, alpha, fused_fma, s);
    default: return launch_axpy<MF_DT_F16>(y, x, n, alpha, fused_fma, s);
    }
}

extern "C" int mf_scalar_broadcast(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, float scalar,
                                   int op, mf_stream stream) {
    MF_ENTER();
    if (n < 0) return fail(MF_ERR_SHAPE_INVALID, "mf_scalar_broadcast: negative element count %lld", (long long)n);
    if (op < MF_SCALAR_ADD || op > MF_SCALAR_DIV)
        return fail(MF_ERR_INVALID_ARGUMENT, "math.scalar_broadcast: unsupported op %d", op);
    if (op == MF_SCALAR_DIV && scalar == 0.0f)
        return fail(MF_ERR_INVALID_ARGUMENT, "math.scalar_broadcast: scalar divisor must be nonzero");
    if (!is_decodable(src_dtype))
        return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_scalar_broadcast: source dtype %d unsupported", src_dtype);
    if (!is_float_store_dtype(dst_dtype))
        return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_scalar_broadcast: destination dtype %d unsupported", dst_dtype);
    if (n == 0) return MF_OK;
    if (!src || !dst) return fail(MF_ERR_INVALID_ARGUMENT, "mf_scalar_broadcast: NULL buffer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (src_dtype) {
    case MF_DT_F32: dispatch_scalar_dst<MF_DT_F32>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_F16: dispatch_scalar_dst<MF_DT_F16>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_BF16: dispatch_scalar_dst<MF_DT_BF16>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_F8E4M3: dispatch_scalar_dst<MF_DT_F8E4M3>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_F8E5M2: dispatch_scalar_dst<MF_DT_F8E5M2>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_F64: dispatch_scalar_dst<MF_DT_F64>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I64: dispatch_scalar_dst<MF_DT_I64>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I32: dispatch_scalar_dst<MF_DT_I32>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I16: dispatch_scalar_dst<MF_DT_I16>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I8: dispatch_scalar_dst<MF_DT_I8>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I4: dispatch_scalar_dst<MF_DT_I4>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_U64: dispatch_scalar_dst<MF_DT_U64>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_U32: dispatch_scalar_dst<MF_DT_U32>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_U16: dispatch_scalar_dst<MF_DT_U16>(dst_dtype, op, src, dst, n, scalar, s); break;
    default: dispatch_scalar_dst<MF_DT_U8>(dst_dtype, op, src, dst, n, scalar, s); break;
    }
    MF_LAUNCH_CHECK("mf_scalar_broadcast launch");
    return MF_OK;
}

extern "C" int mf_linspace(float start, float stop, int64_t count, int endpoint, void* dst, int dst_dtype,
                           mf_stream stream) {
    MF_ENTER();
    if (count <= 0) return fail(MF_ERR_INVALID_ARGUMENT, "math.linspace: count must be positive");
    if (dst_dtype != MF_DT_F32 && dst_dtype != MF_DT_BF16 && dst_dtype != MF_DT_F16)
        return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_linspace: output dtype %d unsupported (F32, BF16, F16)", dst_dtype);
    if (!dst) return fail(MF_ERR_INVALID_ARGUMENT, "mf_linspace: NULL buffer");
    // the step in float32 on the host, as the reference computes it (x86-64 SSE arithmetic:
    // the same rounding and NaN rule as Go on amd64)
    const int64_t intervals = (endpoint || count == 1) ? count - 1 : count;
    const float step = count == 1 ? 0.0f : (stop - start) / static_cast<float>(intervals);
    const int pin_ends = (count > 1 && intervals == count - 1) ? 1 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (dst_dtype) {
    case MF_DT_BF16: launch_linspace<MF_DT_BF16>(start, stop, step, count, pin_ends, dst, s); break;
    case MF_DT_F16: launch_linspace<MF_DT_F16>(start, stop, step, count, pin_ends, dst, s); break;
    default: launch_linspace<MF_DT_F32>(start, stop, step, count, pin_ends, dst, s); break;
    }
    MF_LAUNCH_CHECK("mf_linspace launch");
    return MF_OK;
}
