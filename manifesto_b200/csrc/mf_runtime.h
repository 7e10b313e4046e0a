// mf_runtime.h -- internal helpers shared by the C-ABI translation units:
// thread-local error reporting, device/launch configuration and the
// argument checks every entry point performs before it launches.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "../../include/mfcuda.h"

namespace mf {

// Record a failure message for mf_last_error() on this thread and return code.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Map a CUDA error to MF_ERR_CUDA with the call site in the message.
int cuda_fail(cudaError_t err, const char* what);

struct DeviceState {
    int device = -1;
    int sm_count = 0;
    int max_threads_per_sm = 0;
    bool open = false;
};
DeviceState& state();

// Make the library's device current on the calling thread; returns MF_OK or
// MF_ERR_BACKEND_CLOSED when mf_init has not run (or mf_shutdown has).
int enter();

// Grid size for a grid-stride streaming kernel of `threads` per block over
// `work_items` items per thread-iteration: capped at `waves` full
// occupancy waves over all SMs.
int64_t stream_grid(int64_t work_items, int threads, int blocks_per_sm);

// Device address of the sticky status word (0 = OK).  Kernels that detect a
// condition the host could not rule out write a nonzero code there; the
// host reads and clears it in mf_device_status.
int* sticky_status_ptr();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline bool is_float_store_dtype(int dt) {
    return dt == MF_DT_F32 || dt == MF_DT_BF16 || dt == MF_DT_F16;
}
inline bool is_fp8(int dt) { return dt == MF_DT_F8E4M3 || dt == MF_DT_F8E5M2; }
inline bool is_decodable(int dt) {
    return dt >= MF_DT_F64 && dt <= MF_DT_U8;
}

}  // namespace mf

#define MF_CUDA_CHECK(expr)                                  \
    do {                                                     \
        cudaError_t mf_err_ = (expr);                        \
        if (mf_err_ != cudaSuccess) return ::mf::cuda_fail(mf_err_, #expr); \
    } while (0)

#define MF_LAUNCH_CHECK(name)                                \
    do {                                                     \
        cudaError_t mf_err_ = cudaGetLastError();            \
        if (mf_err_ != cudaSuccess) return ::mf::cuda_fail(mf_err_, name); \
    } while (0)

#define MF_ENTER()                                           \
    do {                                                     \
        int mf_rc_ = ::mf::enter();                          \
        if (mf_rc_ != MF_OK) return mf_rc_;                  \
    } while (0)
