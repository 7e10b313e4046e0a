// probe.cu -- HBM ceilings per access mix (mf_bw_probe).
//
// The kernels of this library read and write DRAM in fixed ratios: a FP8
// decode reads 1 byte for every 4 it writes, a BF16 -> FP8 cast reads 2 for
// every 1, the checkpoint's amax pass only reads.  A plain 1:1 copy is a poor
// denominator for them, because the DRAM's read and write bandwidths differ
// and the bus turnaround cost depends on the mix.  This probe moves bytes in
// a chosen mix with the bulk-copy (TMA) engine alone -- 32 KB loads
// (cp.async.bulk global -> shared, completion on an mbarrier) and 32 KB stores
// (cp.async.bulk shared -> global, bulk groups), no thread touches the data --
// so its rate is the ceiling a kernel of that mix can reach on this GPU.
//
// One step reads A vectors of 16 bytes and writes B: read k of step s is
// vector k * n_steps + s of src, write k is vector k * n_steps + s of dst.
// Steps are moved 2048 at a time (a 32 KB piece of every region); each CTA
// owns a contiguous range of pieces.  One lane streams the loads into a ring
// of stages, one lane of another warp issues the stores of each landed stage
// (a store of piece k reads load k mod A of the stage; a write-only probe
// stores a zeroed tile) and releases the stage once its stores have read it.
// Supported mixes (A, B): (1, 0) read-only, (0, 1) write-only, (1, 1) copy,
// (1, 4) decode-shaped, (2, 1) cast-shaped.  Every mbarrier wait is bounded.
#include <algorithm>

#include "mf_runtime.h"
#include "mf_stream.cuh"

namespace mf {
namespace {

constexpr int kPieceVecs = 2048;                 // 16-byte vectors per piece (32 KB)
constexpr int kPieceBytes = kPieceVecs * 16;
constexpr int kProbeSmem = 192 * 1024;           // ring bytes per CTA (one CTA per SM)

__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int A, int B>
struct ProbeGeometry {
    static constexpr int kStageBytes = (A > 0 ? A : 1) * kPieceBytes;
    static constexpr int kStages = (kProbeSmem / kStageBytes) < 8 ? (kProbeSmem / kStageBytes) : 8;
    static constexpr int kSmemBytes = kStages * kStageBytes + 2 * kStages * 8;
};

template <int A, int B>
__global__ void __launch_bounds__(64, 1) bw_probe_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out,
                                                         int64_t n_steps, int* status) {
    using G = ProbeGeometry<A, B>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kStages * G::kStageBytes);
    uint64_t* empty = full + G::kStages;
    const int64_t pieces = (n_steps + kPieceVecs - 1) / kPieceVecs;
    const int64_t per = pieces / gridDim.x, extra = pieces % gridDim.x, b = blockIdx.x;
    const int64_t p0 = b * per + (b < extra ? b : extra);
    const int64_t np = per + (b < extra ? 1 : 0);
    const int64_t region = n_steps * 16;  // bytes of one region
    if (threadIdx.x == 0) {
        for (int s = 0; s < G::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_barrier_init();
    }
    if (A == 0) {
        for (int j = threadIdx.x; j < kPieceBytes / 16; j += blockDim.x)
            reinterpret_cast<uint4*>(smem)[j] = make_uint4(0, 0, 0, 0);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    if (np <= 0) return;
    auto piece_bytes = [&](int64_t p) -> uint32_t {
        const int64_t v = min(static_cast<int64_t>(kPieceVecs), n_steps - p * kPieceVecs);
        return static_cast<uint32_t>(v * 16);
    };
    if (threadIdx.x == 0) {
        // ---------------- loads
        if (A == 0) return;
        bool ok = true;
        int64_t i = 0;
        for (; i < np; ++i) {
            const int s = static_cast<int>(i % G::kStages);
            if (i >= G::kStages && !mbar_wait(&empty[s], static_cast<uint32_t>((i / G::kStages - 1) & 1))) {
                ok = false;
                break;
            }
            const int64_t p = p0 + i;
            const uint32_t bytes = piece_bytes(p);
            mbar_arrive_expect_tx(&full[s], A * bytes);
#pragma unroll
            for (int k = 0; k < A; ++k)
                bulk_g2s(smem + s * G::kStageBytes + k * kPieceBytes, in + k * region + p * kPieceBytes, bytes,
                         &full[s]);
        }
        if (!ok) atomicExch(status, kDeviceTimeout);
        for (int64_t j = (i > G::kStages ? i - G::kStages : 0); j < i; ++j)
            mbar_wait(&full[j % G::kStages], static_cast<uint32_t>((j / G::kStages) & 1));
    } else if (threadIdx.x == 32) {
        // ---------------- stores (and the release of each stage)
        for (int64_t i = 0; i < np; ++i) {
            const int s = static_cast<int>(i % G::kStages);
            const int64_t p = p0 + i;
            if (A > 0 && !mbar_wait(&full[s], static_cast<uint32_t>((i / G::kStages) & 1))) {
                atomicExch(status, kDeviceTimeout);
                break;
            }
            const uint32_t bytes = piece_bytes(p);
#pragma unroll
            for (int k = 0; k < B; ++k)
                bulk_s2g(out + k * region + p * kPieceBytes, smem + (A > 0 ? s * G::kStageBytes + (k % A) * kPieceBytes : 0),
                         bytes);
            bulk_commit();
            if (A > 0) {
                // the stores of the previous stage have read it: hand it back
                bulk_wait_read<1>();
                if (i >= 1) mbar_arrive(&empty[(i - 1) % G::kStages]);
            } else {
                bulk_wait_read<4>();
            }
        }
        bulk_wait_all();
    }
}

template <int A, int B>
cudaError_t launch(const void* src, void* dst, int64_t n_steps, int* status, cudaStream_t s) {
    using G = ProbeGeometry<A, B>;
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(bw_probe_kernel<A, B>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmemBytes);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    const int64_t pieces = (n_steps + kPieceVecs - 1) / kPieceVecs;
    const int64_t blocks = std::min<int64_t>(pieces, state().sm_count);
    bw_probe_kernel<A, B><<<static_cast<unsigned>(blocks), 64, G::kSmemBytes, s>>>(
        static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), n_steps, status);
    return cudaGetLastError();
}

}  // namespace
}  // namespace mf

using namespace mf;

extern "C" int mf_bw_probe(const void* src, int in_per_step, void* dst, int out_per_step, int64_t n_steps,
                           mf_stream stream) {
    MF_ENTER();
    if (n_steps < 0) return fail(MF_ERR_SHAPE_INVALID, "mf_bw_probe: negative step count %lld", (long long)n_steps);
    if (n_steps == 0) return MF_OK;
    if ((in_per_step > 0 && (!src || !aligned16(src))) || (out_per_step > 0 && (!dst || !aligned16(dst))))
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_bw_probe: buffers must be non-NULL and 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int* status = sticky_status_ptr();
    cudaError_t e;
    switch (in_per_step * 16 + out_per_step) {
    case 0x10: e = launch<1, 0>(src, dst, n_steps, status, s); break;
    case 0x01: e = launch<0, 1>(src, dst, n_steps, status, s); break;
    case 0x11: e = launch<1, 1>(src, dst, n_steps, status, s); break;
    case 0x14: e = launch<1, 4>(src, dst, n_steps, status, s); break;
    case 0x21: e = launch<2, 1>(src, dst, n_steps, status, s); break;
    default:
        return fail(MF_ERR_INVALID_ARGUMENT,
                    "mf_bw_probe: mix (%d reads, %d writes) unsupported: (1,0) (0,1) (1,1) (1,4) (2,1)", in_per_step,
                    out_per_step);
    }
    if (e != cudaSuccess) return cuda_fail(e, "mf_bw_probe launch");
    return MF_OK;
}
