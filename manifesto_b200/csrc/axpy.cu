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
// With 16-byte aligned buffers both run on the bulk-copy streaming engine
// (mf_stream.cuh): axpy as a two-source op (y and x staged side by side in
// every stage, y written back in place), the scalar op as a one-source op;
// unaligned buffers take per-element kernels with the same arithmetic.
// Roofline: HBM; axpy moves 3 * sizeof(dtype) bytes per element, the scalar
// op src + dst bytes.
#include "mf_runtime.h"
#include "mf_stream.cuh"

namespace mf {
namespace {

constexpr int kThreads = 256;

// y + alpha * x with the amd64 NaN rule (Go source order: y += alpha*addend).
template <int FUSED>
__device__ __forceinline__ float axpy_op(float y, float x, float alpha) {
    if constexpr (FUSED) return x86_fma(alpha, x, y);
    else return x86_add(y, x86_mul(alpha, x));
}

// Four elements: the products alpha * x as packed float32 pairs (each half
// rounded like __fmul_rn), the sums as scalar __fadd_rn, which is never merged
// with the product into a fused multiply-add (the reference rounds both); a NaN
// result, whose payload follows the amd64 rule, is recomputed with the scalar
// operations.
template <int FUSED>
__device__ __forceinline__ void axpy_quad_f32(float (&vy)[4], const float (&vx)[4], float alpha) {
    if constexpr (FUSED) {
#pragma unroll
        for (int j = 0; j < 4; ++j) vy[j] = axpy_op<1>(vy[j], vx[j], alpha);
    } else {
        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
            const float2 p = __fmul2_rn(a2, make_float2(vx[j], vx[j + 1]));
            const float s0 = __fadd_rn(vy[j], p.x), s1 = __fadd_rn(vy[j + 1], p.y);
            const float r0 = (s0 != s0) ? axpy_op<0>(vy[j], vx[j], alpha) : s0;
            const float r1 = (s1 != s1) ? axpy_op<0>(vy[j + 1], vx[j + 1], alpha) : s1;
            vy[j] = r0;
            vy[j + 1] = r1;
        }
    }
}

// y = y + alpha * x on the streaming engine: y is source 1 (and the
// destination, written back in place), x source 2; a lane step is 8 BF16/F16
// or 4 float32 elements of each.
template <int DT, int FUSED>
struct AxpyOp {
    static constexpr int kIn = dtype_bytes(DT);
    static constexpr int kIn2 = kIn;
    static constexpr int kLane = lane_elems<kIn, kIn>();
    static constexpr int kQ = kLane / 4;
    static constexpr bool kDefers = false;
    static constexpr bool kPrologue = false;
    struct State {
        float alpha;
    };
    template <class A>
    __device__ static State setup(const A& a, const ChunkRec&) {
        return {a.scalar};
    }
    __device__ static void step2(const uint8_t* sy, const uint8_t* sx, const ChunkRec& ch, int64_t e, const State& st) {
        float vy[2][4], vx[2][4];
        load_decode_lane<DT, kQ>(sy, vy);
        load_decode_lane<DT, kQ>(sx, vx);
        uint32_t o[kQ * kIn];
#pragma unroll
        for (int k = 0; k < kQ; ++k) {
            axpy_quad_f32<FUSED>(vy[k], vx[k], st.alpha);
            encode4<DT>(vy[k], o + k * kIn, 0);
        }
        store_lane_stream<kLane * kIn>(static_cast<uint8_t*>(ch.dst) + e * kIn, o);
    }
    __device__ static void element(const ChunkRec& ch, int64_t i, const State& st) {
        const float r = axpy_op<FUSED>(load_as_f32<DT>(ch.dst, i), load_as_f32<DT>(ch.src2, i), st.alpha);
        store_code<DT>(ch.dst, i, encode_f32<DT>(r, 0));
    }
};

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
        StreamArgs<1> a{};
        single_chunk(a, y, y, n, true, StreamGeometry<AxpyOp<DT, 0>>::kTileElems);
        a.chunk[0].src2 = x;
        a.scalar = alpha;
        const cudaError_t e = fused ? launch_stream<AxpyOp<DT, 1>, 1>(a, state().sm_count, s)
                                    : launch_stream<AxpyOp<DT, 0>, 1>(a, state().sm_count, s);
        if (e != cudaSuccess) return cuda_fail(e, "mf_axpy launch");
        return MF_OK;
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

// out = src (op) scalar on the streaming engine (one source).
template <int SRC, int DST, int OP>
struct ScalarOp {
    static constexpr int kIn = dtype_bytes(SRC);
    static constexpr int kOut = dtype_bytes(DST);
    static constexpr int kIn2 = 0;
    static constexpr int kLane = lane_elems<kIn, kOut>();
    static constexpr int kQ = kLane / 4;
    static constexpr bool kDefers = false;
    static constexpr bool kPrologue = false;
    struct State {
        float s;
    };
    template <class A>
    __device__ static State setup(const A& a, const ChunkRec&) {
        return {a.scalar};
    }
    template <bool DEFER>
    __device__ static void step(const uint8_t* sp, const ChunkRec& ch, int64_t e, const State& st, FixQueue&) {
        float v[2][4];
        load_decode_lane<SRC, kQ>(sp, v);
        uint32_t o[kQ * kOut];
#pragma unroll
        for (int k = 0; k < kQ; ++k) {
#pragma unroll
            for (int j = 0; j < 4; ++j) v[k][j] = scalar_op<OP>(v[k][j], st.s);
            encode4<DST>(v[k], o + k * kOut, 0);
        }
        store_lane_stream<kLane * kOut>(static_cast<uint8_t*>(ch.dst) + e * kOut, o);
    }
    __device__ static void element(const ChunkRec& ch, int64_t i, const State& st) {
        store_code<DST>(ch.dst, i, encode_f32<DST>(scalar_op<OP>(load_as_f32<SRC>(ch.src, i), st.s), 0));
    }
};

template <int SRC, int DST, int OP>
__global__ void __launch_bounds__(kThreads) scalar_elem_kernel(const void* __restrict__ src, void* __restrict__ dst,
                                                              int64_t n, float scalar) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        store_code<DST>(dst, i, encode_f32<DST>(scalar_op<OP>(load_as_f32<SRC>(src, i), scalar), 0));
}

template <int SRC, int DST, int OP>
cudaError_t launch_scalar_op(const void* src, void* dst, int64_t n, float scalar, cudaStream_t s) {
    constexpr bool kVecSrc = SRC == MF_DT_F32 || SRC == MF_DT_F16 || SRC == MF_DT_BF16 || SRC == MF_DT_F8E4M3 ||
                             SRC == MF_DT_F8E5M2;
    if constexpr (kVecSrc) {
        if (aligned16(src) && aligned16(dst)) {
            StreamArgs<1> a{};
            single_chunk(a, src, dst, n, true, StreamGeometry<ScalarOp<SRC, DST, OP>>::kTileElems);
            a.scalar = scalar;
            return launch_stream<ScalarOp<SRC, DST, OP>, 1>(a, state().sm_count, s);
        }
    }
    const int64_t blocks = stream_grid(n, kThreads, 8);
    scalar_elem_kernel<SRC, DST, OP><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(src, dst, n, scalar);
    return cudaGetLastError();
}

template <int SRC, int DST>
cudaError_t dispatch_op(int op, const void* src, void* dst, int64_t n, float scalar, cudaStream_t s) {
    switch (op) {
    case MF_SCALAR_ADD: return launch_scalar_op<SRC, DST, MF_SCALAR_ADD>(src, dst, n, scalar, s);
    case MF_SCALAR_SUB: return launch_scalar_op<SRC, DST, MF_SCALAR_SUB>(src, dst, n, scalar, s);
    case MF_SCALAR_MUL: return launch_scalar_op<SRC, DST, MF_SCALAR_MUL>(src, dst, n, scalar, s);
    default: return launch_scalar_op<SRC, DST, MF_SCALAR_DIV>(src, dst, n, scalar, s);
    }
}

template <int SRC>
cudaError_t dispatch_scalar_dst(int dst_dt, int op, const void* src, void* dst, int64_t n, float scalar,
                                cudaStream_t s) {
    switch (dst_dt) {
    case MF_DT_F32: return dispatch_op<SRC, MF_DT_F32>(op, src, dst, n, scalar, s);
    case MF_DT_F16: return dispatch_op<SRC, MF_DT_F16>(op, src, dst, n, scalar, s);
    default: return dispatch_op<SRC, MF_DT_BF16>(op, src, dst, n, scalar, s);
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
    cudaError_t e;
    switch (src_dtype) {
    case MF_DT_F32: e = dispatch_scalar_dst<MF_DT_F32>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_F16: e = dispatch_scalar_dst<MF_DT_F16>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_BF16: e = dispatch_scalar_dst<MF_DT_BF16>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_F8E4M3: e = dispatch_scalar_dst<MF_DT_F8E4M3>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_F8E5M2: e = dispatch_scalar_dst<MF_DT_F8E5M2>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_F64: e = dispatch_scalar_dst<MF_DT_F64>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I64: e = dispatch_scalar_dst<MF_DT_I64>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I32: e = dispatch_scalar_dst<MF_DT_I32>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I16: e = dispatch_scalar_dst<MF_DT_I16>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I8: e = dispatch_scalar_dst<MF_DT_I8>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_I4: e = dispatch_scalar_dst<MF_DT_I4>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_U64: e = dispatch_scalar_dst<MF_DT_U64>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_U32: e = dispatch_scalar_dst<MF_DT_U32>(dst_dtype, op, src, dst, n, scalar, s); break;
    case MF_DT_U16: e = dispatch_scalar_dst<MF_DT_U16>(dst_dtype, op, src, dst, n, scalar, s); break;
    default: e = dispatch_scalar_dst<MF_DT_U8>(dst_dtype, op, src, dst, n, scalar, s); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "mf_scalar_broadcast launch");
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
