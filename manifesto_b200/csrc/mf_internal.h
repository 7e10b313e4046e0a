// mf_internal.h -- host-side functions shared between translation units of
// libmfcuda.so (not exported; the C ABI is include/mfcuda.h).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/mfcuda.h"

namespace mf {

// Launch the amax-scaled FP8 cast of n elements of src_dtype (quant.cu).
int launch_scaled_cast(const void* src, int src_dtype, void* dst, int fp8_dtype, const float* d_amax,
                       float* d_scale_inv, int64_t n, int compat, cudaStream_t s);
// Fold max|src| into *d_amax (quant.cu).
int launch_amax(const void* src, int src_dtype, int64_t n, float* d_amax, cudaStream_t s);
// In-place float32 max all-reduce over the communicator (comm.cu).
int comm_allreduce_max(mf_comm comm, float* d_vec, int64_t count, cudaStream_t s);

}  // namespace mf
