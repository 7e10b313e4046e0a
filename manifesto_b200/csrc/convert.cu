// convert.cu -- K1-K3: dtype conversion (mf_convert).
//
// Replaces the element loops of convert.BytesToFloat32 and the narrowing
// drivers BytesToBFloat16 / BytesToFloat16 / BytesToFloat8E4M3 /
// BytesToFloat8E5M2 (dtype/convert/convert.go:85-228): decode the source
// element to float32, then encode it with the destination's scalar encoder.
//
// Layout: flat arrays of n elements.  The floating formats {F32, F16, BF16,
// E4M3, E5M2} with 16-byte aligned buffers run on the bulk-copy streaming
// engine (mf_stream.cuh): the source is staged through shared memory by
// cp.async.bulk, decoded and re-encoded 16 elements at a time, and written
// with 128-bit stores.  Unaligned buffers and the integer / F64 / Int4
// sources use a scalar grid-stride kernel with the same codecs.
// Roofline: HBM, src_bytes + dst_bytes per element.
#include "mf_runtime.h"
#include "mf_stream.cuh"

namespace mf {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float decode_any(int dt, const void* p, int64_t i) {
    switch (dt) {
    case MF_DT_F64: return load_as_f32<MF_DT_F64>(p, i);
    case MF_DT_F32: return load_as_f32<MF_DT_F32>(p, i);
    case MF_DT_F16: return load_as_f32<MF_DT_F16>(p, i);
    case MF_DT_BF16: return load_as_f32<MF_DT_BF16>(p, i);
    case MF_DT_F8E4M3: return load_as_f32<MF_DT_F8E4M3>(p, i);
    case MF_DT_F8E5M2: return load_as_f32<MF_DT_F8E5M2>(p, i);
    case MF_DT_I64: return load_as_f32<MF_DT_I64>(p, i);
    case MF_DT_I32: return load_as_f32<MF_DT_I32>(p, i);
    case MF_DT_I16: return load_as_f32<MF_DT_I16>(p, i);
    case MF_DT_I8: return load_as_f32<MF_DT_I8>(p, i);
    case MF_DT_I4: return load_as_f32<MF_DT_I4>(p, i);
    case MF_DT_U64: return load_as_f32<MF_DT_U64>(p, i);
    case MF_DT_U32: return load_as_f32<MF_DT_U32>(p, i);
    case MF_DT_U16: return load_as_f32<MF_DT_U16>(p, i);
    default: return load_as_f32<MF_DT_U8>(p, i);
    }
}

template <int DST>
__global__ void __launch_bounds__(kThreads) convert_scalar_kernel(int src_dt, const void* __restrict__ src,
                                                                 void* __restrict__ dst, int64_t n,
                                                                 int compat) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        store_code<DST>(dst, i, encode_f32<DST>(decode_any(src_dt, src, i), compat));
    }
}

bool is_vector_format(int dt) {
    return dt == MF_DT_F32 || dt == MF_DT_F16 || dt == MF_DT_BF16 || dt == MF_DT_F8E4M3 || dt == MF_DT_F8E5M2;
}

template <int SRC, int DST>
cudaError_t launch_vec(const void* src, void* dst, int64_t n, int compat, cudaStream_t s) {
    StreamArgs<1> a{};
    single_chunk(a, src, dst, n, true, stream_tile_elems<dtype_bytes(SRC)>());
    if (compat) return launch_stream<ConvertOp<SRC, DST, 1>, 1>(a, state().sm_count, s);
    return launch_stream<ConvertOp<SRC, DST, 0>, 1>(a, state().sm_count, s);
}

template <int SRC>
cudaError_t dispatch_dst(int dst_dt, const void* src, void* dst, int64_t n, int compat, cudaStream_t s) {
    switch (dst_dt) {
    case MF_DT_F32: return launch_vec<SRC, MF_DT_F32>(src, dst, n, compat, s);
    case MF_DT_F16: return launch_vec<SRC, MF_DT_F16>(src, dst, n, compat, s);
    case MF_DT_BF16: return launch_vec<SRC, MF_DT_BF16>(src, dst, n, compat, s);
    case MF_DT_F8E4M3: return launch_vec<SRC, MF_DT_F8E4M3>(src, dst, n, compat, s);
    default: return launch_vec<SRC, MF_DT_F8E5M2>(src, dst, n, compat, s);
    }
}

template <int DST>
void launch_scalar(int src_dt, const void* src, void* dst, int64_t n, int compat, cudaStream_t s) {
    const int64_t blocks = stream_grid(n, kThreads, 8);
    convert_scalar_kernel<DST><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(src_dt, src, dst, n, compat);
}

}  // namespace
}  // namespace mf

using namespace mf;

extern "C" int mf_convert(int src_dtype, int dst_dtype, const void* src, void* dst, int64_t n, int compat,
                          mf_stream stream) {
    MF_ENTER();
    if (n < 0) return fail(MF_ERR_SHAPE_INVALID, "mf_convert: negative element count %lld", (long long)n);
    if (!is_decodable(src_dtype))
        return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_convert: unsupported source dtype %d", src_dtype);
    if (!is_float_store_dtype(dst_dtype) && !is_fp8(dst_dtype))
        return fail(MF_ERR_DTYPE_UNSUPPORTED, "mf_convert: unsupported destination dtype %d", dst_dtype);
    if (compat != MF_COMPAT_REFERENCE && compat != MF_COMPAT_OCP)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_convert: unknown compat mode %d", compat);
    if (n == 0) return MF_OK;
    if (!src || !dst) return fail(MF_ERR_INVALID_ARGUMENT, "mf_convert: NULL buffer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (is_vector_format(src_dtype) && aligned16(src) && aligned16(dst)) {
        cudaError_t err;
        switch (src_dtype) {
        case MF_DT_F32: err = dispatch_dst<MF_DT_F32>(dst_dtype, src, dst, n, compat, s); break;
        case MF_DT_F16: err = dispatch_dst<MF_DT_F16>(dst_dtype, src, dst, n, compat, s); break;
        case MF_DT_BF16: err = dispatch_dst<MF_DT_BF16>(dst_dtype, src, dst, n, compat, s); break;
        case MF_DT_F8E4M3: err = dispatch_dst<MF_DT_F8E4M3>(dst_dtype, src, dst, n, compat, s); break;
        default: err = dispatch_dst<MF_DT_F8E5M2>(dst_dtype, src, dst, n, compat, s); break;
        }
        if (err != cudaSuccess) return cuda_fail(err, "mf_convert launch");
    } else {
        switch (dst_dtype) {
        case MF_DT_F32: launch_scalar<MF_DT_F32>(src_dtype, src, dst, n, compat, s); break;
        case MF_DT_F16: launch_scalar<MF_DT_F16>(src_dtype, src, dst, n, compat, s); break;
        case MF_DT_BF16: launch_scalar<MF_DT_BF16>(src_dtype, src, dst, n, compat, s); break;
        case MF_DT_F8E4M3: launch_scalar<MF_DT_F8E4M3>(src_dtype, src, dst, n, compat, s); break;
        default: launch_scalar<MF_DT_F8E5M2>(src_dtype, src, dst, n, compat, s); break;
        }
    }
    MF_LAUNCH_CHECK("mf_convert launch");
    return MF_OK;
}
