// probe.cu -- HBM ceilings per access mix (mf_bw_probe).
//
// The kernels of this library read and write DRAM in fixed ratios: a FP8
// decode reads 1 byte for every 4 it writes, a BF16 -> FP8 cast reads 2 for
// every 1, the checkpoint's amax pass only reads.  A plain 1:1 copy is a poor
// denominator for them, because the DRAM's read and write bandwidths differ
// and the bus turnaround cost depends on the mix.  This probe moves bytes in
// a chosen mix with the same access forms those kernels use (16-byte
// non-coherent evict-first loads, 16-byte streaming stores, lane-contiguous
// warps, a grid of 8 blocks of 256 per SM) and does no other work, so its
// rate is the ceiling a kernel of that mix can reach.
//
// One step reads A vectors of 16 bytes and writes B: read k of step s is
// vector k * n_steps + s of src, write k is vector k * n_steps + s of dst,
// so every region is swept contiguously by consecutive lanes.  Stored values
// depend on the loaded ones (as in a conversion); a read-only probe folds
// what it reads into one word and writes it to d_sink only if it equals a
// value no input produces, which keeps the loads alive without traffic.
// Supported mixes (A, B): (1, 0) read-only, (0, 1) write-only, (1, 1) copy,
// (1, 4) decode-shaped, (2, 1) cast-shaped.
#include "mf_runtime.h"
#include "mf_vec.cuh"

namespace mf {
namespace {

constexpr int kThreads = 256;
constexpr int kSteps = 4;  // steps in flight per thread

template <int A, int B>
__global__ void __launch_bounds__(kThreads) bw_probe_kernel(const uint4* __restrict__ in, uint4* __restrict__ out,
                                                            int64_t n_steps, uint32_t* __restrict__ sink) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    uint32_t acc = 0x9e3779b9u ^ threadIdx.x;
    for (int64_t s = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; s < n_steps;
         s += kSteps * stride) {
        uint4 v[kSteps][A > 0 ? A : 1];
#pragma unroll
        for (int u = 0; u < kSteps; ++u) {
            const int64_t st = s + u * stride;
#pragma unroll
            for (int k = 0; k < A; ++k)
                if (st < n_steps) v[u][k] = ld_stream(in + k * n_steps + st);
        }
#pragma unroll
        for (int u = 0; u < kSteps; ++u) {
            const int64_t st = s + u * stride;
            if (st >= n_steps) break;
            uint32_t w = static_cast<uint32_t>(st);
#pragma unroll
            for (int k = 0; k < A; ++k) w ^= v[u][k].x ^ v[u][k].y ^ v[u][k].z ^ v[u][k].w;
            acc ^= w;
#pragma unroll
            for (int k = 0; k < B; ++k) st_stream(out + k * n_steps + st, make_uint4(w, w + 1u, w + 2u, w + 3u));
        }
    }
    if (B == 0 && acc == 0x5a5aa5a5u) *sink = acc;
}

template <int A, int B>
void launch(const void* src, void* dst, int64_t n_steps, uint32_t* sink, cudaStream_t s) {
    const int64_t blocks = stream_grid((n_steps + kSteps - 1) / kSteps, kThreads, 8);
    bw_probe_kernel<A, B><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), n_steps, sink);
}

}  // namespace
}  // namespace mf

using namespace mf;

extern "C" int mf_bw_probe(const void* src, int in_per_step, void* dst, int out_per_step, int64_t n_steps,
                           uint32_t* d_sink, mf_stream stream) {
    MF_ENTER();
    if (n_steps < 0) return fail(MF_ERR_SHAPE_INVALID, "mf_bw_probe: negative step count %lld", (long long)n_steps);
    if (n_steps == 0) return MF_OK;
    if ((in_per_step > 0 && (!src || !aligned16(src))) || (out_per_step > 0 && (!dst || !aligned16(dst))))
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_bw_probe: buffers must be non-NULL and 16-byte aligned");
    if (out_per_step == 0 && !d_sink) return fail(MF_ERR_INVALID_ARGUMENT, "mf_bw_probe: read-only probe needs d_sink");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int mix = in_per_step * 16 + out_per_step;
    switch (mix) {
    case 0x10: launch<1, 0>(src, dst, n_steps, d_sink, s); break;
    case 0x01: launch<0, 1>(src, dst, n_steps, d_sink, s); break;
    case 0x11: launch<1, 1>(src, dst, n_steps, d_sink, s); break;
    case 0x14: launch<1, 4>(src, dst, n_steps, d_sink, s); break;
    case 0x21: launch<2, 1>(src, dst, n_steps, d_sink, s); break;
    default:
        return fail(MF_ERR_INVALID_ARGUMENT,
                    "mf_bw_probe: mix (%d reads, %d writes) unsupported: (1,0) (0,1) (1,1) (1,4) (2,1)", in_per_step,
                    out_per_step);
    }
    MF_LAUNCH_CHECK("mf_bw_probe launch");
    return MF_OK;
}
