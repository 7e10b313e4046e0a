// quant.cu -- K8 per-tensor amax-scaled FP8 cast and K9 grouped
// whole-checkpoint quantisation.
//
// The reference has no amax, scale or quantize operation (its only cast
// is shape.cast); the semantics here are composed from its primitives:
//   amax      = max |v| (NaN ignored, as Go's '>' never selects NaN)
//   scale     = fp8_max / amax in float32, 1 if amax is 0 or not finite
//   q         = NewF8E4M3FromFloat32(v * scale)   (dtype/fp8.go:77-136)
//               or NewF8E5M2FromFloat32           (dtype/fp8.go:190-249)
//   scale_inv = amax / fp8_max in float32, 1 if amax is 0 or not finite
//
// amax keeps a running magnitude key per lane: a BF16/F16 pair is folded
// with one max.xorsign.abs.{bf16,f16}x2 (max of the magnitudes per half, a
// NaN half never wins), float32 and FP8 on the integer bit patterns (|v|
// orders like bits & ~sign once NaN codes are excluded); the key is decoded
// once at the end.  Roofline: HBM; amax reads src once, the cast reads src
// and writes 1 B per element.
//
// Checkpoint quantisation: each rank owns one contiguous chunk of every
// tensor.  One descriptor table (passed by value as the kernel parameter,
// so nothing is allocated) lists the chunks; the chunks are cut into tiles
// (16384 elements of a 16-bit source, 8192 of a float32 one) and each CTA
// walks a contiguous range of tiles, so a
// CTA crosses few tensor boundaries and reduces its per-tensor maximum
// once per crossing.  Pass 1 (stream_amax_kernel, two CTAs per SM) has one
// producer lane per CTA pull 32 KB tiles through a 3-stage shared-memory ring with
// 1-D bulk copies; eight consumer warps copy a landed stage to registers,
// release it at once and fold.  Pass 1 (amax) and pass 2 (cast) are one launch each
// per 512 chunks; between them an NCCL max all-reduce of the amax vector
// makes the scales global.
#include <algorithm>
#include <mutex>
#include <vector>

#include "mf_internal.h"
#include "mf_runtime.h"
#include "mf_stream.cuh"

namespace mf {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------- amax

// Magnitude key of one element: monotone in |v|, 0 for NaN.
template <int DT>
struct MagKey;
template <>
struct MagKey<MF_DT_F32> {
    // running max of (bits & 0x7fffffff) over non-NaN values
    static __device__ __forceinline__ uint32_t fold(const RawChunk<4>& r, uint32_t m) {
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const uint32_t a = r.w[k] & 0x7fffffffu;
            m = (a <= 0x7f800000u && a > m) ? a : m;
        }
        return m;
    }
    static __device__ __forceinline__ float to_f32(uint32_t m) { return __uint_as_float(m); }
};
// Two halves per word: max(|a|, |b|) per half with one max.xorsign.abs (the
// maxNum rule: a NaN half never wins; the result's sign bits are the XOR of the
// inputs' and are cleared when the key is read).
template <int DT>
struct MagKey16 {
    static __device__ __forceinline__ uint32_t fold(const RawChunk<2>& r, uint32_t m) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            if constexpr (DT == MF_DT_BF16) asm("max.xorsign.abs.bf16x2 %0, %0, %1;" : "+r"(m) : "r"(r.w[k]));
            else asm("max.xorsign.abs.f16x2 %0, %0, %1;" : "+r"(m) : "r"(r.w[k]));
        }
        return m;
    }
};
template <>
struct MagKey<MF_DT_BF16> {
    static __device__ __forceinline__ uint32_t fold(const RawChunk<2>& r, uint32_t m) {
        return MagKey16<MF_DT_BF16>::fold(r, m);
    }
    static __device__ __forceinline__ float to_f32(uint32_t m) {
        const uint32_t h = max(m & 0x7fffu, (m >> 16) & 0x7fffu);
        return __uint_as_float(h << 16);
    }
};
template <>
struct MagKey<MF_DT_F16> {
    static __device__ __forceinline__ uint32_t fold(const RawChunk<2>& r, uint32_t m) {
        return MagKey16<MF_DT_F16>::fold(r, m);
    }
    static __device__ __forceinline__ float to_f32(uint32_t m) {
        const uint32_t h = max(m & 0x7fffu, (m >> 16) & 0x7fffu);
        return __uint_as_float(f16_to_f32bits(h));
    }
};
template <int DT>
struct MagKey8 {
    static __device__ __forceinline__ uint32_t fold(const RawChunk<1>& r, uint32_t m, uint32_t nan_floor4) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t a = r.w[k] & 0x7f7f7f7fu;
            const uint32_t nan_mask = __vcmpgtu4(a, nan_floor4);
            m = __vmaxu4(m, a & ~nan_mask);
        }
        return m;
    }
    static __device__ __forceinline__ uint32_t top(uint32_t m) {
        return max(max(m & 0xffu, (m >> 8) & 0xffu), max((m >> 16) & 0xffu, m >> 24));
    }
};
template <>
struct MagKey<MF_DT_F8E4M3> {
    static __device__ __forceinline__ uint32_t fold(const RawChunk<1>& r, uint32_t m) {
        return MagKey8<MF_DT_F8E4M3>::fold(r, m, 0x7e7e7e7eu);
    }
    static __device__ __forceinline__ float to_f32(uint32_t m) {
        return __uint_as_float(e4m3_to_f32bits(MagKey8<MF_DT_F8E4M3>::top(m)));
    }
};
template <>
struct MagKey<MF_DT_F8E5M2> {
    static __device__ __forceinline__ uint32_t fold(const RawChunk<1>& r, uint32_t m) {
        return MagKey8<MF_DT_F8E5M2>::fold(r, m, 0x7c7c7c7cu);
    }
    static __device__ __forceinline__ float to_f32(uint32_t m) {
        return __uint_as_float(e5m2_to_f32bits(MagKey8<MF_DT_F8E5M2>::top(m)));
    }
};

__device__ __forceinline__ float warp_max(float m) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    return m;
}

// Block-wide maximum of a non-negative float; result valid in thread 0.
__device__ __forceinline__ float block_max(float m) {
    __shared__ float partial[kThreads / 32];
    m = warp_max(m);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();  // partial[] may still be read by a previous call
    if (lane == 0) partial[warp] = m;
    __syncthreads();
    if (warp == 0) {
        m = lane < kThreads / 32 ? partial[lane] : 0.0f;
        m = warp_max(m);
    }
    return m;
}

__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
    if (v > 0.0f) atomicMax(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

// |v| of one element, NaN -> 0 (for scalar tails)
template <int DT>
__device__ __forceinline__ float abs_or_zero(const void* p, int64_t i) {
    const float a = fabsf(load_as_f32<DT>(p, i));
    return (a == a) ? a : 0.0f;
}

template <int SRC>
__global__ void __launch_bounds__(kThreads) amax_vec_kernel(const void* __restrict__ src, int64_t n,
                                                           float* __restrict__ amax) {
    const int64_t nchunks = n / kChunk;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    uint32_t key = 0;
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < nchunks; c += stride) {
        RawChunk<dtype_bytes(SRC)> r;
        load_raw<dtype_bytes(SRC)>(src, c, r);
        key = MagKey<SRC>::fold(r, key);
    }
    float m = MagKey<SRC>::to_f32(key);
    if (blockIdx.x == 0) {
        const int64_t i = nchunks * kChunk + threadIdx.x;
        if (i < n) m = fmaxf(m, abs_or_zero<SRC>(src, i));
    }
    m = block_max(m);
    if (threadIdx.x == 0) atomic_max_nonneg(amax, m);
}

template <int SRC>
__global__ void __launch_bounds__(kThreads) amax_scalar_kernel(const void* __restrict__ src, int64_t n,
                                                              float* __restrict__ amax) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    float m = 0.0f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        m = fmaxf(m, abs_or_zero<SRC>(src, i));
    m = block_max(m);
    if (threadIdx.x == 0) atomic_max_nonneg(amax, m);
}

// --------------------------------------------------------- scaled cast

template <int FP8>
__device__ __forceinline__ uint32_t encode_fp8(float v, int compat) {
    return encode_f32<FP8>(v, compat);
}

// scale_inv[t] = amax[t] / fp8_max (1 when amax is 0 or not finite) for every
// tensor of the call, including a tensor this rank holds no element of.
__global__ void scale_inv_kernel(const float* __restrict__ amax, float* __restrict__ scale_inv, int n, int fp8) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) scale_inv[t] = scale_inv_from_amax(amax[t], fp8);
}

int launch_scale_inv(const float* d_amax, float* d_scale_inv, int n, int fp8_dtype, cudaStream_t s) {
    if (!d_scale_inv || n <= 0) return MF_OK;
    scale_inv_kernel<<<(n + 255) / 256, 256, 0, s>>>(d_amax, d_scale_inv, n, fp8_dtype);
    MF_LAUNCH_CHECK("scale_inv launch");
    return MF_OK;
}

template <int SRC>
void amax_dispatch(const void* src, int64_t n, float* d_amax, cudaStream_t s) {
    if (aligned16(src)) {
        const int64_t blocks = stream_grid(n / kChunk + 1, kThreads, 8);
        amax_vec_kernel<SRC><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(src, n, d_amax);
    } else {
        const int64_t blocks = stream_grid(n, kThreads, 8);
        amax_scalar_kernel<SRC><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(src, n, d_amax);
    }
}

template <int SRC, int FP8>
cudaError_t cast_dispatch(const void* src, void* dst, int64_t n, const float* d_amax, int compat, cudaStream_t s) {
    StreamArgs<1> a{};
    single_chunk(a, src, dst, n, aligned16(src) && aligned16(dst), stream_tile_elems<dtype_bytes(SRC)>());
    a.amax = d_amax;
    if (compat) return launch_stream<CastOp<SRC, FP8, 1>, 1>(a, state().sm_count, s);
    return launch_stream<CastOp<SRC, FP8, 0>, 1>(a, state().sm_count, s);
}

template <int SRC>
cudaError_t cast_dispatch_fp8(int fp8_dtype, const void* src, void* dst, int64_t n, const float* d_amax, int compat,
                              cudaStream_t s) {
    if (fp8_dtype == MF_DT_F8E4M3) return cast_dispatch<SRC, MF_DT_F8E4M3>(src, dst, n, d_amax, compat, s);
    return cast_dispatch<SRC, MF_DT_F8E5M2>(src, dst, n, d_amax, compat, s);
}

// ----------------------------------------------------- grouped (ckpt)

constexpr int kGroupMaxChunks = 512;

// Per tile every thread owns 128 bytes of source: 4 chunks of 16 BF16/F16
// elements or 2 chunks of 16 float32.  One launch covers chunks of one
// source dtype, so each kernel body holds a single decode path.
template <int SRC>
struct Tile {
    static constexpr int kChunks = 128 / (kChunk * dtype_bytes(SRC));
    static constexpr int64_t kElems = int64_t(kThreads) * kChunks * kChunk;
};

struct AmaxChunk {
    const void* src;
    int64_t n;
    int64_t tile_begin;  // first tile of this chunk within the launch
    int32_t tensor;
    int32_t aligned;     // src 16-byte aligned
};

struct AmaxArgs {
    float* amax;
    int64_t total_tiles;
    int32_t n_chunks;
    int32_t publish;        // the launch's last CTA publishes `amax` through xchg (a plan's two-launch form)
    const AmaxXchg* xchg;
    int32_t epoch;
    int32_t pad;
    AmaxChunk chunk[kGroupMaxChunks];
};

__device__ __forceinline__ int find_chunk(const AmaxArgs& a, int64_t t) {
    int lo = 0, hi = a.n_chunks - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.chunk[mid].tile_begin <= t) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// This CTA's contiguous tile range [t0, t1).
__device__ __forceinline__ void tile_range(int64_t total, int64_t& t0, int64_t& t1) {
    const int64_t per = total / gridDim.x, extra = total % gridDim.x;
    const int64_t b = blockIdx.x;
    t0 = b * per + (b < extra ? b : extra);
    t1 = t0 + per + (b < extra ? 1 : 0);
}

// Pass 1 on the bulk-copy engine.  The amax fold is a few instructions per
// 16 bytes, so the pass is bound by how many bytes are in flight: one producer
// lane streams the CTA's tiles (32 KB each, contiguous tile ranges as above)
// through kAmaxStages shared-memory stages -- two CTAs per SM with three
// stages each, 192 KB in flight per SM (measured 2.25 ms on the 16 GB
// checkpoint, 0.97 of the bulk-copy read ceiling, against 2.41 ms for one CTA
// with six stages and 2.42 ms with seven: two producer lanes per SM keep more
// copies issued) -- and 256 consumer threads fold each landed tile from shared
// memory (lane-contiguous 16-byte reads) into a per-lane magnitude key.  A
// tensor's maximum is reduced per warp and folded into amax[tensor] with one
// atomicMax per warp when the CTA leaves the tensor.  Every mbarrier wait is
// bounded; a wait that runs out records MF_DEVICE_TIMEOUT.
// Compile-time tunables (the defaults are the measured choices): stages per CTA
// and CTAs per SM; their product times 32 KB must fit the SM's shared memory.
#ifndef MF_AMAX_STAGES
#define MF_AMAX_STAGES 3
#endif
#ifndef MF_AMAX_CTAS
#define MF_AMAX_CTAS 2
#endif
constexpr int kAmaxStages = MF_AMAX_STAGES;
constexpr int kAmaxCtas = MF_AMAX_CTAS;  // CTAs per SM
constexpr int kAmaxTileBytes = 32768;
constexpr int kAmaxSmem = kAmaxStages * kAmaxTileBytes + 2 * kAmaxStages * 8;

// Running per-lane magnitude key over one 16-byte word group (NaN never wins).
template <int SRC>
__device__ __forceinline__ uint32_t fold16(uint32_t key, const uint4& w) {
    if constexpr (SRC == MF_DT_F32) {
        const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t a = v[k] & 0x7fffffffu;
            key = (a <= 0x7f800000u && a > key) ? a : key;
        }
        return key;
    } else {
        const uint32_t v[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if constexpr (SRC == MF_DT_BF16) asm("max.xorsign.abs.bf16x2 %0, %0, %1;" : "+r"(key) : "r"(v[k]));
            else asm("max.xorsign.abs.f16x2 %0, %0, %1;" : "+r"(key) : "r"(v[k]));
        }
        return key;
    }
}

template <int SRC>
__device__ __forceinline__ void flush_amax(float* amax, int tensor, uint32_t key, float mel) {
    float m = warp_max(fmaxf(MagKey<SRC>::to_f32(key), mel));
    if ((threadIdx.x & 31) == 0 && m > 0.0f) atomicMax(reinterpret_cast<unsigned*>(amax + tensor), __float_as_uint(m));
}

// Warp 0 of every CTA of a publishing pass-1 launch, once the CTA's maxima are
// folded into a.amax: the last CTA to arrive stores this rank's maxima into
// its slot of every rank's exchange buffer (plain stores into peer memory
// opened with CUDA IPC; no multicast) and then releases its flag there with
// the run's epoch.
__device__ void amax_publish(const AmaxArgs& a) {
    const AmaxXchg& x = *a.xchg;
    const int lane = threadIdx.x & 31;
    const int par = a.epoch & 1;
    int last = 0;
    if (lane == 0) {
        __threadfence();
        last = atomicAdd(x.counter + par, 1) == static_cast<int>(gridDim.x) - 1;
    }
    if (!__shfl_sync(0xffffffffu, last, 0)) return;
    __threadfence();
    if (lane == 0) x.counter[par] = 0;
    for (int r = 0; r < x.world; ++r) {
        float* dst = x.slots[r] + (static_cast<int64_t>(par) * x.world + x.rank) * x.n_tensors;
        for (int t = lane; t < x.n_tensors; t += 32) dst[t] = ld_relaxed_gpu(a.amax + t);
    }
    __threadfence_system();
    __syncwarp();
    if (lane < x.world) st_release_sys(x.flags[lane] + x.rank, a.epoch);
}

template <int SRC>
__global__ void __launch_bounds__(kStreamBlock, 1) stream_amax_kernel(const __grid_constant__ AmaxArgs a, int* status) {
    using T = Tile<SRC>;
    constexpr int kIn = dtype_bytes(SRC);
    static_assert(T::kElems * kIn == kAmaxTileBytes, "tile geometry");
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kAmaxStages * kAmaxTileBytes);
    uint64_t* empty = full + kAmaxStages;
    int64_t t0, t1;
    tile_range(a.total_tiles, t0, t1);
    if (t0 >= t1) {
        if (a.publish && threadIdx.x < 32) amax_publish(a);
        return;
    }
    const int64_t nt = t1 - t0;
    if (threadIdx.x == 0) {
        for (int st = 0; st < kAmaxStages; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x >= kStreamThreads) {
        if (threadIdx.x != kStreamThreads) return;
        int k = find_chunk(a, t0);
        int64_t i = 0;
        bool ok = true;
        for (; i < nt; ++i) {
            const int st = static_cast<int>(i % kAmaxStages);
            if (i >= kAmaxStages && !mbar_wait(&empty[st], static_cast<uint32_t>((i / kAmaxStages - 1) & 1))) {
                ok = false;
                break;
            }
            const int64_t t = t0 + i;
            while (k + 1 < a.n_chunks && a.chunk[k + 1].tile_begin <= t) ++k;
            const AmaxChunk& ch = a.chunk[k];
            const int64_t e0 = (t - ch.tile_begin) * T::kElems;
            const int64_t cnt = min(T::kElems, ch.n - e0);
            const uint32_t bytes = static_cast<uint32_t>((cnt * kIn) & ~int64_t(15));
            if (ch.aligned && bytes > 0) {
                mbar_arrive_expect_tx(&full[st], bytes);
                bulk_g2s(smem + st * kAmaxTileBytes, static_cast<const uint8_t*>(ch.src) + e0 * kIn, bytes, &full[st]);
            } else {
                mbar_arrive(&full[st]);
            }
        }
        if (!ok) atomicExch(status, kDeviceTimeout);
        for (int64_t j = (i > kAmaxStages ? i - kAmaxStages : 0); j < i; ++j)
            mbar_wait(&full[j % kAmaxStages], static_cast<uint32_t>((j / kAmaxStages) & 1));
        return;
    }
    const int lane = threadIdx.x & 31;
    int k = find_chunk(a, t0);
    int cur = a.chunk[k].tensor;
    uint32_t key = 0;
    float mel = 0.0f;
    for (int64_t i = 0; i < nt; ++i) {
        const int st = static_cast<int>(i % kAmaxStages);
        if (!__all_sync(0xffffffffu, mbar_wait(&full[st], static_cast<uint32_t>((i / kAmaxStages) & 1)))) {
            if (lane == 0) atomicExch(status, kDeviceTimeout);
            break;  // the producer's own bounded waits end its loop; the warp still meets the CTA below
        }
        const int64_t t = t0 + i;
        while (k + 1 < a.n_chunks && a.chunk[k + 1].tile_begin <= t) ++k;
        const AmaxChunk& ch = a.chunk[k];
        if (ch.tensor != cur) {
            flush_amax<SRC>(a.amax, cur, key, mel);
            cur = ch.tensor;
            key = 0;
            mel = 0.0f;
        }
        const int64_t e0 = (t - ch.tile_begin) * T::kElems;
        const int64_t cnt = min(T::kElems, ch.n - e0);
        if (ch.aligned && cnt == T::kElems) {
            // pull the tile into registers and hand the stage back before folding it
            constexpr int kV = kAmaxTileBytes / 16 / kStreamThreads;
            const uint4* tp = reinterpret_cast<const uint4*>(smem + st * kAmaxTileBytes);
            uint4 w[kV];
#pragma unroll
            for (int v = 0; v < kV; ++v) w[v] = tp[threadIdx.x + v * kStreamThreads];
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
#pragma unroll
            for (int v = 0; v < kV; ++v) key = fold16<SRC>(key, w[v]);
            continue;
        }
        if (ch.aligned) {
            const int64_t copied = (cnt * kIn) & ~int64_t(15);
            const uint4* tp = reinterpret_cast<const uint4*>(smem + st * kAmaxTileBytes);
            {
                for (int v = threadIdx.x; v < copied / 16; v += kStreamThreads) key = fold16<SRC>(key, tp[v]);
                for (int64_t e = e0 + copied / kIn + threadIdx.x; e < e0 + cnt; e += kStreamThreads)
                    mel = fmaxf(mel, abs_or_zero<SRC>(ch.src, e));
            }
        } else {
            for (int64_t e = e0 + threadIdx.x; e < e0 + cnt; e += kStreamThreads)
                mel = fmaxf(mel, abs_or_zero<SRC>(ch.src, e));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    flush_amax<SRC>(a.amax, cur, key, mel);
    if (a.publish) {
        __threadfence();   // this warp's atomicMax results before the CTA's ticket
        consumers_sync();
        if (threadIdx.x < 32) amax_publish(a);
    }
}

// Launch pass 1 over one argument block (the grid is at most kAmaxCtas CTAs per SM).
template <int SRC>
cudaError_t launch_stream_amax(const AmaxArgs& args, int64_t tiles, cudaStream_t s) {
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(stream_amax_kernel<SRC>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAmaxSmem);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    // a publishing launch runs even without tiles (its one CTA publishes zeros)
    const unsigned blocks =
        static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(tiles, int64_t(state().sm_count) * kAmaxCtas)));
    stream_amax_kernel<SRC><<<blocks, kStreamBlock, kAmaxSmem, s>>>(args, sticky_status_ptr());
    return cudaGetLastError();
}

// Fill the amax / cast argument blocks with the chunks idx[first, first+count);
// return the number of tiles.
int64_t fill_amax(AmaxArgs& a, const mf_chunk_desc* chunks, const int32_t* idx, int first, int count,
                  int64_t tile_elems) {
    int64_t tiles = 0;
    for (int i = 0; i < count; ++i) {
        const mf_chunk_desc& d = chunks[idx[first + i]];
        AmaxChunk& r = a.chunk[i];
        r.src = d.src;
        r.n = d.n;
        r.tile_begin = tiles;
        r.tensor = d.tensor;
        r.aligned = aligned16(d.src) ? 1 : 0;
        tiles += (d.n + tile_elems - 1) / tile_elems;
    }
    a.n_chunks = count;
    a.total_tiles = tiles;
    return tiles;
}

int64_t fill_cast(StreamArgs<kGroupMaxChunks>& a, const mf_chunk_desc* chunks, const int32_t* idx, int first,
                  int count, int64_t tile_elems) {
    int64_t tiles = 0;
    for (int i = 0; i < count; ++i) {
        const mf_chunk_desc& d = chunks[idx[first + i]];
        ChunkRec& r = a.chunk[i];
        r.src = d.src;
        r.dst = d.dst;
        r.n = d.n;
        r.tile_begin = tiles;
        r.tensor = d.tensor;
        r.aligned = (aligned16(d.src) && aligned16(d.dst)) ? 1 : 0;
        tiles += (d.n + tile_elems - 1) / tile_elems;
    }
    a.n_chunks = count;
    a.total_tiles = tiles;
    return tiles;
}

}  // namespace

int launch_amax(const void* src, int src_dtype, int64_t n, float* d_amax, cudaStream_t s) {
    if (n == 0) return MF_OK;
    switch (src_dtype) {
    case MF_DT_F32: amax_dispatch<MF_DT_F32>(src, n, d_amax, s); break;
    case MF_DT_F16: amax_dispatch<MF_DT_F16>(src, n, d_amax, s); break;
    case MF_DT_BF16: amax_dispatch<MF_DT_BF16>(src, n, d_amax, s); break;
    case MF_DT_F8E4M3: amax_dispatch<MF_DT_F8E4M3>(src, n, d_amax, s); break;
    case MF_DT_F8E5M2: amax_dispatch<MF_DT_F8E5M2>(src, n, d_amax, s); break;
    default: return fail(MF_ERR_DTYPE_UNSUPPORTED, "amax: source dtype %d unsupported", src_dtype);
    }
    MF_LAUNCH_CHECK("amax launch");
    return MF_OK;
}

int launch_scaled_cast(const void* src, int src_dtype, void* dst, int fp8_dtype, const float* d_amax,
                       float* d_scale_inv, int64_t n, int compat, cudaStream_t s) {
    int rc = launch_scale_inv(d_amax, d_scale_inv, 1, fp8_dtype, s);
    if (rc || n == 0) return rc;
    cudaError_t err;
    switch (src_dtype) {
    case MF_DT_F32: err = cast_dispatch_fp8<MF_DT_F32>(fp8_dtype, src, dst, n, d_amax, compat, s); break;
    case MF_DT_F16: err = cast_dispatch_fp8<MF_DT_F16>(fp8_dtype, src, dst, n, d_amax, compat, s); break;
    case MF_DT_BF16: err = cast_dispatch_fp8<MF_DT_BF16>(fp8_dtype, src, dst, n, d_amax, compat, s); break;
    default: return fail(MF_ERR_DTYPE_UNSUPPORTED, "scaled cast: source dtype %d unsupported", src_dtype);
    }
    if (err != cudaSuccess) return cuda_fail(err, "scaled cast launch");
    return MF_OK;
}

}  // namespace mf

using namespace mf;

static int check_quant_args(const char* name, int src_dtype, int fp8_dtype, int compat, int64_t n) {
    if (n < 0) return fail(MF_ERR_SHAPE_INVALID, "%s: negative element count %lld", name, (long long)n);
    if (!is_fp8(fp8_dtype)) return fail(MF_ERR_DTYPE_UNSUPPORTED, "%s: destination dtype %d is not FP8", name, fp8_dtype);
    if (!is_float_store_dtype(src_dtype))
        return fail(MF_ERR_DTYPE_UNSUPPORTED, "%s: source dtype %d unsupported (F32, F16, BF16)", name, src_dtype);
    if (compat != MF_COMPAT_REFERENCE && compat != MF_COMPAT_OCP)
        return fail(MF_ERR_INVALID_ARGUMENT, "%s: unknown compat mode %d", name, compat);
    return MF_OK;
}

extern "C" int mf_amax(const void* src, int src_dtype, int64_t n, float* d_amax, mf_stream stream) {
    MF_ENTER();
    if (n < 0) return fail(MF_ERR_SHAPE_INVALID, "mf_amax: negative element count %lld", (long long)n);
    if (!d_amax) return fail(MF_ERR_INVALID_ARGUMENT, "mf_amax: d_amax is NULL");
    if (n > 0 && !src) return fail(MF_ERR_INVALID_ARGUMENT, "mf_amax: NULL source");
    return launch_amax(src, src_dtype, n, d_amax, static_cast<cudaStream_t>(stream));
}

extern "C" int mf_fp8_scaled_cast(const void* src, int src_dtype, void* dst, int fp8_dtype, const float* d_amax,
                                  float* d_scale_inv, int64_t n, int compat, mf_stream stream) {
    MF_ENTER();
    int rc = check_quant_args("mf_fp8_scaled_cast", src_dtype, fp8_dtype, compat, n);
    if (rc) return rc;
    if (!d_amax) return fail(MF_ERR_INVALID_ARGUMENT, "mf_fp8_scaled_cast: d_amax is NULL");
    if (n > 0 && (!src || !dst)) return fail(MF_ERR_INVALID_ARGUMENT, "mf_fp8_scaled_cast: NULL buffer");
    return launch_scaled_cast(src, src_dtype, dst, fp8_dtype, d_amax, d_scale_inv, n, compat,
                              static_cast<cudaStream_t>(stream));
}

extern "C" int mf_fp8_quantize(const void* src, int src_dtype, void* dst, int fp8_dtype, float* d_amax,
                               float* d_scale_inv, int64_t n, int compat, mf_stream stream) {
    MF_ENTER();
    int rc = check_quant_args("mf_fp8_quantize", src_dtype, fp8_dtype, compat, n);
    if (rc) return rc;
    if (!d_amax) return fail(MF_ERR_INVALID_ARGUMENT, "mf_fp8_quantize: d_amax is NULL");
    if (n > 0 && (!src || !dst)) return fail(MF_ERR_INVALID_ARGUMENT, "mf_fp8_quantize: NULL buffer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    MF_CUDA_CHECK(cudaMemsetAsync(d_amax, 0, sizeof(float), s));
    if (n == 0) return launch_scale_inv(d_amax, d_scale_inv, 1, fp8_dtype, s);
    rc = launch_amax(src, src_dtype, n, d_amax, s);
    if (rc) return rc;
    return launch_scaled_cast(src, src_dtype, dst, fp8_dtype, d_amax, d_scale_inv, n, compat, s);
}

extern "C" int mf_ckpt_partition(const int64_t* rows, int32_t n_tensors, int32_t world, int32_t rank,
                                 int64_t* first_row, int64_t* n_rows) {
    if (n_tensors < 0 || (n_tensors > 0 && (!rows || !first_row || !n_rows)))
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_partition: bad tensor table");
    if (world < 1 || rank < 0 || rank >= world)
        return fail(MF_ERR_INVALID_ARGUMENT, "mf_ckpt_partition: rank %d outside world %d", rank, world);
    for (int32_t t = 0; t < n_tensors; ++t) {
        if (rows[t] < 0) return fail(MF_ERR_SHAPE_INVALID, "mf_ckpt_partition: tensor %d has %lld rows", t, (long long)rows[t]);
        const int64_t base = rows[t] / world, extra = rows[t] % world;
        first_row[t] = rank * base + (rank < extra ? rank : extra);
        n_rows[t] = base + (rank < extra ? 1 : 0);
    }
    return MF_OK;
}

static int check_chunks(const char* name, const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors,
                        const float* d_amax) {
    if (n_chunks < 0 || n_tensors <= 0 || (n_chunks > 0 && !chunks))
        return fail(MF_ERR_INVALID_ARGUMENT, "%s: bad chunk table (%d chunks, %d tensors)", name, n_chunks, n_tensors);
    if (!d_amax) return fail(MF_ERR_INVALID_ARGUMENT, "%s: d_amax is NULL", name);
    for (int32_t i = 0; i < n_chunks; ++i) {
        const mf_chunk_desc& d = chunks[i];
        if (d.tensor < 0 || d.tensor >= n_tensors)
            return fail(MF_ERR_INVALID_ARGUMENT, "%s: chunk %d names tensor %d of %d", name, i, d.tensor, n_tensors);
        if (d.n < 0) return fail(MF_ERR_SHAPE_INVALID, "%s: chunk %d has %lld elements", name, i, (long long)d.n);
        if (!is_float_store_dtype(d.src_dtype))
            return fail(MF_ERR_DTYPE_UNSUPPORTED, "%s: chunk %d source dtype %d unsupported", name, i, d.src_dtype);
        if (d.n > 0 && (!d.src || !d.dst)) return fail(MF_ERR_INVALID_ARGUMENT, "%s: chunk %d has a NULL buffer", name, i);
    }
    return MF_OK;
}

static int check_fp8_mode(const char* name, int fp8_dtype, int compat) {
    if (!is_fp8(fp8_dtype)) return fail(MF_ERR_DTYPE_UNSUPPORTED, "%s: dtype %d is not FP8", name, fp8_dtype);
    if (compat != MF_COMPAT_REFERENCE && compat != MF_COMPAT_OCP)
        return fail(MF_ERR_INVALID_ARGUMENT, "%s: unknown compat mode %d", name, compat);
    return MF_OK;
}

namespace {
std::mutex g_group_mutex;
AmaxArgs g_amax_args;                           // ~16 KB, filled under the mutex
StreamArgs<kGroupMaxChunks> g_cast_args;        // ~20 KB, filled under the mutex

// Chunk indices with n > 0, grouped by source dtype (BF16, F16, F32), each
// group in table order.
void group_by_dtype(const mf_chunk_desc* chunks, int32_t n_chunks, std::vector<int32_t> (&by)[3]) {
    for (int32_t i = 0; i < n_chunks; ++i) {
        if (chunks[i].n <= 0) continue;
        const int d = chunks[i].src_dtype;
        by[d == MF_DT_BF16 ? 0 : d == MF_DT_F16 ? 1 : 2].push_back(i);
    }
}

template <int SRC>
int amax_launches(const mf_chunk_desc* chunks, const std::vector<int32_t>& idx, float* d_amax, cudaStream_t s) {
    AmaxArgs& args = g_amax_args;
    for (int first = 0; first < static_cast<int>(idx.size()); first += kGroupMaxChunks) {
        const int count = std::min<int>(kGroupMaxChunks, static_cast<int>(idx.size()) - first);
        args.amax = d_amax;
        args.publish = 0;
        const int64_t tiles = fill_amax(args, chunks, idx.data(), first, count, Tile<SRC>::kElems);
        if (tiles == 0) continue;
        const cudaError_t err = launch_stream_amax<SRC>(args, tiles, s);
        if (err != cudaSuccess) return cuda_fail(err, "checkpoint amax pass launch");
    }
    return MF_OK;
}

template <int SRC, int FP8>
cudaError_t cast_launch(const StreamArgs<kGroupMaxChunks>& args, int compat, cudaStream_t s) {
    if (compat) return launch_stream<CastOp<SRC, FP8, 1>, kGroupMaxChunks>(args, state().sm_count, s);
    return launch_stream<CastOp<SRC, FP8, 0>, kGroupMaxChunks>(args, state().sm_count, s);
}

template <int SRC>
int cast_launches(const mf_chunk_desc* chunks, const std::vector<int32_t>& idx, const float* d_amax, int fp8_dtype,
                  int compat, cudaStream_t s) {
    StreamArgs<kGroupMaxChunks>& args = g_cast_args;
    for (int first = 0; first < static_cast<int>(idx.size()); first += kGroupMaxChunks) {
        const int count = std::min<int>(kGroupMaxChunks, static_cast<int>(idx.size()) - first);
        args.amax = d_amax;
        args.status = sticky_status_ptr();
        const int64_t tiles = fill_cast(args, chunks, idx.data(), first, count, stream_tile_elems<dtype_bytes(SRC)>());
        if (tiles == 0) continue;
        const cudaError_t err = (fp8_dtype == MF_DT_F8E4M3) ? cast_launch<SRC, MF_DT_F8E4M3>(args, compat, s)
                                                            : cast_launch<SRC, MF_DT_F8E5M2>(args, compat, s);
        if (err != cudaSuccess) return cuda_fail(err, "checkpoint cast pass launch");
    }
    return MF_OK;
}

int launch_amax_pass(const mf_chunk_desc* chunks, int32_t n_chunks, float* d_amax, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(g_group_mutex);
    std::vector<int32_t> by[3];
    group_by_dtype(chunks, n_chunks, by);
    int rc = amax_launches<MF_DT_BF16>(chunks, by[0], d_amax, s);
    if (!rc) rc = amax_launches<MF_DT_F16>(chunks, by[1], d_amax, s);
    if (!rc) rc = amax_launches<MF_DT_F32>(chunks, by[2], d_amax, s);
    return rc;
}

int launch_cast_pass(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors, const float* d_amax,
                     float* d_scale_inv, int fp8_dtype, int compat, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(g_group_mutex);
    int rc = launch_scale_inv(d_amax, d_scale_inv, n_tensors, fp8_dtype, s);
    if (rc) return rc;
    std::vector<int32_t> by[3];
    group_by_dtype(chunks, n_chunks, by);
    rc = cast_launches<MF_DT_BF16>(chunks, by[0], d_amax, fp8_dtype, compat, s);
    if (!rc) rc = cast_launches<MF_DT_F16>(chunks, by[1], d_amax, fp8_dtype, compat, s);
    if (!rc) rc = cast_launches<MF_DT_F32>(chunks, by[2], d_amax, fp8_dtype, compat, s);
    return rc;
}

// ---- a checkpoint plan's two-launch form (one source dtype per plan)

// Pass 1 into this run's copy of the per-rank maxima; with several ranks the
// last launch publishes them (it runs, as one CTA, even when this rank holds
// no elements, so that the other ranks are never left waiting).
template <int SRC>
int plan_amax_launches(const mf_chunk_desc* chunks, const std::vector<int32_t>& idx, const AmaxXchg* xchg,
                       float* lam, int world, int32_t epoch, cudaStream_t s) {
    AmaxArgs& args = g_amax_args;
    const int n = static_cast<int>(idx.size());
    int first = 0;
    do {
        const int count = std::min<int>(kGroupMaxChunks, n - first);
        args.amax = lam;
        args.xchg = xchg;
        args.epoch = epoch;
        const int64_t tiles = fill_amax(args, chunks, idx.data(), first, count, Tile<SRC>::kElems);
        args.publish = (world > 1 && first + count >= n) ? 1 : 0;
        if (tiles > 0 || args.publish) {
            const cudaError_t err = launch_stream_amax<SRC>(args, tiles, s);
            if (err != cudaSuccess) return cuda_fail(err, "checkpoint plan amax pass launch");
        }
        first += count;
    } while (first < n);
    return MF_OK;
}

// Pass 2: the cast with the exchange in its prologue; the first launch is the
// writer of the amax / scale_inv outputs (it runs even without tiles).
template <int SRC, int FP8, int COMPAT>
int plan_cast_launches(const mf_chunk_desc* chunks, const std::vector<int32_t>& idx, const AmaxXchg* xchg,
                       int32_t epoch, float* d_amax, float* d_scale_inv, cudaStream_t s) {
    StreamArgs<kGroupMaxChunks>& args = g_cast_args;
    const int n = static_cast<int>(idx.size());
    int first = 0;
    do {
        const int count = std::min<int>(kGroupMaxChunks, n - first);
        args.amax = nullptr;
        args.status = sticky_status_ptr();
        args.xchg = xchg;
        args.epoch = epoch;
        args.out_amax = d_amax;
        args.out_scale_inv = d_scale_inv;
        args.writer = first == 0 ? 1 : 0;
        const int64_t tiles = fill_cast(args, chunks, idx.data(), first, count, stream_tile_elems<dtype_bytes(SRC)>());
        if (tiles > 0 || args.writer) {
            const cudaError_t err =
                launch_stream<CastXOp<SRC, FP8, COMPAT, kGroupMaxChunks>, kGroupMaxChunks>(args, state().sm_count, s);
            if (err != cudaSuccess) return cuda_fail(err, "checkpoint plan cast pass launch");
        }
        first += count;
    } while (first < n);
    return MF_OK;
}

template <int SRC>
int plan_cast_dispatch(const mf_chunk_desc* chunks, const std::vector<int32_t>& idx, const AmaxXchg* xchg,
                       int32_t epoch, float* d_amax, float* d_scale_inv, int fp8_dtype, int compat, cudaStream_t s) {
    if (fp8_dtype == MF_DT_F8E4M3)
        return compat ? plan_cast_launches<SRC, MF_DT_F8E4M3, 1>(chunks, idx, xchg, epoch, d_amax, d_scale_inv, s)
                      : plan_cast_launches<SRC, MF_DT_F8E4M3, 0>(chunks, idx, xchg, epoch, d_amax, d_scale_inv, s);
    return compat ? plan_cast_launches<SRC, MF_DT_F8E5M2, 1>(chunks, idx, xchg, epoch, d_amax, d_scale_inv, s)
                  : plan_cast_launches<SRC, MF_DT_F8E5M2, 0>(chunks, idx, xchg, epoch, d_amax, d_scale_inv, s);
}
}  // namespace

namespace mf {
int launch_plan_passes(const mf_chunk_desc* chunks, int32_t n_chunks, int src_dtype, const AmaxXchg* d_xchg,
                       float* d_local_amax, int world, int32_t epoch, int passes, float* d_amax, float* d_scale_inv,
                       int fp8_dtype, int compat, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(g_group_mutex);
    std::vector<int32_t> idx;
    for (int32_t i = 0; i < n_chunks; ++i)
        if (chunks[i].n > 0) idx.push_back(i);
    int rc = MF_OK;
    if (passes & 1) {
        switch (src_dtype) {
        case MF_DT_BF16: rc = plan_amax_launches<MF_DT_BF16>(chunks, idx, d_xchg, d_local_amax, world, epoch, s); break;
        case MF_DT_F16: rc = plan_amax_launches<MF_DT_F16>(chunks, idx, d_xchg, d_local_amax, world, epoch, s); break;
        case MF_DT_F32: rc = plan_amax_launches<MF_DT_F32>(chunks, idx, d_xchg, d_local_amax, world, epoch, s); break;
        default: return fail(MF_ERR_DTYPE_UNSUPPORTED, "checkpoint plan: source dtype %d unsupported", src_dtype);
        }
        if (rc) return rc;
    }
    if (passes & 2) {
        switch (src_dtype) {
        case MF_DT_BF16:
            rc = plan_cast_dispatch<MF_DT_BF16>(chunks, idx, d_xchg, epoch, d_amax, d_scale_inv, fp8_dtype, compat, s);
            break;
        case MF_DT_F16:
            rc = plan_cast_dispatch<MF_DT_F16>(chunks, idx, d_xchg, epoch, d_amax, d_scale_inv, fp8_dtype, compat, s);
            break;
        case MF_DT_F32:
            rc = plan_cast_dispatch<MF_DT_F32>(chunks, idx, d_xchg, epoch, d_amax, d_scale_inv, fp8_dtype, compat, s);
            break;
        default: return fail(MF_ERR_DTYPE_UNSUPPORTED, "checkpoint plan: source dtype %d unsupported", src_dtype);
        }
    }
    return rc;
}
}  // namespace mf

extern "C" int mf_ckpt_amax_pass(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors, float* d_amax,
                                 mf_stream stream) {
    MF_ENTER();
    int rc = check_chunks("mf_ckpt_amax_pass", chunks, n_chunks, n_tensors, d_amax);
    if (rc) return rc;
    return launch_amax_pass(chunks, n_chunks, d_amax, static_cast<cudaStream_t>(stream));
}

extern "C" int mf_ckpt_cast_pass(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors, const float* d_amax,
                                 float* d_scale_inv, int fp8_dtype, int compat, mf_stream stream) {
    MF_ENTER();
    int rc = check_chunks("mf_ckpt_cast_pass", chunks, n_chunks, n_tensors, d_amax);
    if (rc) return rc;
    rc = check_fp8_mode("mf_ckpt_cast_pass", fp8_dtype, compat);
    if (rc) return rc;
    return launch_cast_pass(chunks, n_chunks, n_tensors, d_amax, d_scale_inv, fp8_dtype, compat,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int mf_ckpt_quant_fp8(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors, float* d_amax,
                                 float* d_scale_inv, int fp8_dtype, int compat, mf_comm comm, mf_stream stream) {
    MF_ENTER();
    int rc = check_chunks("mf_ckpt_quant_fp8", chunks, n_chunks, n_tensors, d_amax);
    if (rc) return rc;
    rc = check_fp8_mode("mf_ckpt_quant_fp8", fp8_dtype, compat);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    MF_CUDA_CHECK(cudaMemsetAsync(d_amax, 0, sizeof(float) * n_tensors, s));
    rc = launch_amax_pass(chunks, n_chunks, d_amax, s);
    if (rc) return rc;
    if (comm) {
        rc = comm_allreduce_max(comm, d_amax, n_tensors, s);
        if (rc) return rc;
    }
    return launch_cast_pass(chunks, n_chunks, n_tensors, d_amax, d_scale_inv, fp8_dtype, compat, s);
}

// ---------------------------------------------------------------------------
// Allocation-free checkpoint quantisation (mf_ckpt_quant_fp8_noalloc).
//
// Some callers cannot give this library a device buffer for the per-tensor
// amax vector that mf_ckpt_quant_fp8 needs as scratch: a host whose device
// memory is entirely owned by another allocator -- for instance a Go program
// that runs manifesto graphs on the single workspace arena its planner sized
// in advance (ir.PlanWorkspace), where no port exists for scratch -- or a
// deployment that forbids cudaMalloc once set-up is over.  For them the amax
// vector lives in a file-scope device array instead.
//   * At most kNoAllocMaxTensors (4096) tensors per call (16 KB of scratch);
//     larger calls are rejected with MF_ERR_ALLOCATOR_EXHAUSTED.
//   * Every GPU that loads the library holds the array until the process
//     exits, and every call on a device shares it: calls that overlap on the
//     GPU (on streams with no ordering between them) race on it.
//   * Each call zeroes the entries it uses before pass 1.
//   * Every call looks up the array's device address with
//     cudaGetSymbolAddress, with the library's device current (no address is
//     kept between calls, so a context torn down and made again by the host
//     never leaves a stale one).  The first call on a device also loads the
//     module's device globals there; make that first call before any stream
//     capture begins.
//   * Nothing is allocated: no cudaMalloc/cudaFree and no host heap use (the
//     chunk table is scanned in place instead of being grouped into lists).
namespace mf {
namespace {

constexpr int kNoAllocMaxTensors = 4096;
__device__ __align__(256) float g_noalloc_amax[kNoAllocMaxTensors];

int noalloc_scratch(float** out) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_amax);
    if (err != cudaSuccess) return cuda_fail(err, "mf_ckpt_quant_fp8_noalloc: cudaGetSymbolAddress");
    *out = static_cast<float*>(p);
    return MF_OK;
}

// Pass 1 over the chunks of one source dtype, filling the argument block
// straight from the table.  Caller holds g_group_mutex.
template <int SRC>
int noalloc_amax_launches(const mf_chunk_desc* chunks, int32_t n_chunks, float* d_amax, cudaStream_t s) {
    AmaxArgs& args = g_amax_args;
    int32_t i = 0;
    while (i < n_chunks) {
        int count = 0;
        int64_t tiles = 0;
        for (; i < n_chunks && count < kGroupMaxChunks; ++i) {
            const mf_chunk_desc& d = chunks[i];
            if (d.n <= 0 || d.src_dtype != SRC) continue;
            AmaxChunk& r = args.chunk[count++];
            r.src = d.src;
            r.n = d.n;
            r.tile_begin = tiles;
            r.tensor = d.tensor;
            r.aligned = aligned16(d.src) ? 1 : 0;
            tiles += (d.n + Tile<SRC>::kElems - 1) / Tile<SRC>::kElems;
        }
        if (count == 0) continue;
        args.amax = d_amax;
        args.publish = 0;
        args.n_chunks = count;
        args.total_tiles = tiles;
        const cudaError_t err = launch_stream_amax<SRC>(args, tiles, s);
        if (err != cudaSuccess) return cuda_fail(err, "mf_ckpt_quant_fp8_noalloc amax pass launch");
    }
    return MF_OK;
}

// Pass 2 over the chunks of one source dtype.  Caller holds g_group_mutex.
template <int SRC>
int noalloc_cast_launches(const mf_chunk_desc* chunks, int32_t n_chunks, const float* d_amax, int fp8_dtype,
                          int compat, cudaStream_t s) {
    StreamArgs<kGroupMaxChunks>& args = g_cast_args;
    int32_t i = 0;
    while (i < n_chunks) {
        int count = 0;
        int64_t tiles = 0;
        for (; i < n_chunks && count < kGroupMaxChunks; ++i) {
            const mf_chunk_desc& d = chunks[i];
            if (d.n <= 0 || d.src_dtype != SRC) continue;
            ChunkRec& r = args.chunk[count++];
            r.src = d.src;
            r.dst = d.dst;
            r.n = d.n;
            r.tile_begin = tiles;
            r.tensor = d.tensor;
            r.aligned = (aligned16(d.src) && aligned16(d.dst)) ? 1 : 0;
            tiles += (d.n + stream_tile_elems<dtype_bytes(SRC)>() - 1) / stream_tile_elems<dtype_bytes(SRC)>();
        }
        if (count == 0) continue;
        args.amax = d_amax;
        args.status = sticky_status_ptr();
        args.n_chunks = count;
        args.total_tiles = tiles;
        const cudaError_t err = (fp8_dtype == MF_DT_F8E4M3) ? cast_launch<SRC, MF_DT_F8E4M3>(args, compat, s)
                                                            : cast_launch<SRC, MF_DT_F8E5M2>(args, compat, s);
        if (err != cudaSuccess) return cuda_fail(err, "mf_ckpt_quant_fp8_noalloc cast pass launch");
    }
    return MF_OK;
}

}  // namespace
}  // namespace mf

extern "C" int mf_ckpt_quant_fp8_noalloc(const mf_chunk_desc* chunks, int32_t n_chunks, int32_t n_tensors,
                                         float* d_scale_inv, int fp8_dtype, int compat, mf_comm comm,
                                         mf_stream stream) {
    MF_ENTER();
    if (n_tensors > kNoAllocMaxTensors)
        return fail(MF_ERR_ALLOCATOR_EXHAUSTED,
                    "mf_ckpt_quant_fp8_noalloc: %d tensors exceed the static amax scratch of %d tensors; "
                    "split the checkpoint or use mf_ckpt_quant_fp8 with a caller buffer",
                    n_tensors, kNoAllocMaxTensors);
    float* amax = nullptr;
    int rc = noalloc_scratch(&amax);
    if (rc) return rc;
    rc = check_chunks("mf_ckpt_quant_fp8_noalloc", chunks, n_chunks, n_tensors, amax);
    if (rc) return rc;
    rc = check_fp8_mode("mf_ckpt_quant_fp8_noalloc", fp8_dtype, compat);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    MF_CUDA_CHECK(cudaMemsetAsync(amax, 0, sizeof(float) * n_tensors, s));
    {
        std::lock_guard<std::mutex> lock(g_group_mutex);
        rc = noalloc_amax_launches<MF_DT_BF16>(chunks, n_chunks, amax, s);
        if (!rc) rc = noalloc_amax_launches<MF_DT_F16>(chunks, n_chunks, amax, s);
        if (!rc) rc = noalloc_amax_launches<MF_DT_F32>(chunks, n_chunks, amax, s);
    }
    if (rc) return rc;
    if (comm) {
        rc = comm_allreduce_max(comm, amax, n_tensors, s);
        if (rc) return rc;
    }
    rc = launch_scale_inv(amax, d_scale_inv, n_tensors, fp8_dtype, s);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_group_mutex);
    rc = noalloc_cast_launches<MF_DT_BF16>(chunks, n_chunks, amax, fp8_dtype, compat, s);
    if (!rc) rc = noalloc_cast_launches<MF_DT_F16>(chunks, n_chunks, amax, fp8_dtype, compat, s);
    if (!rc) rc = noalloc_cast_launches<MF_DT_F32>(chunks, n_chunks, amax, fp8_dtype, compat, s);
    return rc;
}
