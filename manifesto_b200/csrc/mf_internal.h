// mf_internal.h -- host-side functions shared between translation units of
// libmfcuda.so (not exported; the C ABI is include/mfcuda.h).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/mfcuda.h"

namespace mf {

// Launch the amax-scaled FP8 cast of n elements of src_dtype (quant.cu).
int launch_scaled_cast(const void* src, int src_dtype, void* dst, int fp8_dtype, const float* d_amax,
                       float* d_scale_inv, int64_t n, int compat, cudaStream_t s);
// Fold max|src| into *d_amax (quant.cu).
int launch_amax(const void* src, int src_dtype, int64_t n, float* d_amax, cudaStream_t s);
// The two launches of a checkpoint plan's split form (quant.cu): passes bit 0
// folds this rank's maxima into d_local_amax (the run's copy) and, world > 1,
// publishes them through the exchange; bit 1 waits for every rank's maxima
// and casts, the first launch writing d_amax / d_scale_inv.
struct AmaxXchg;
int launch_plan_passes(const mf_chunk_desc* chunks, int32_t n_chunks, int src_dtype, const AmaxXchg* d_xchg,
                       float* d_local_amax, int world, int32_t epoch, int passes, float* d_amax, float* d_scale_inv,
                       int fp8_dtype, int compat, cudaStream_t s);
// In-place float32 max all-reduce over the communicator (comm.cu).
int comm_allreduce_max(mf_comm comm, float* d_vec, int64_t count, cudaStream_t s);

// A validated fused program (postfix) as the CUDA codegen target sees it (fused_jit.cu).
struct JitSpec {
    int n_nodes;
    const int8_t* op;
    const int8_t* arg;
    int n_consts;
    const uint32_t* const_bits;  // float32(node value) bit patterns
    int n_inputs;
    const int32_t* in_dtype;
    const int64_t* in_bcast;     // 0: full size; L: read at index i mod L
    int out_dtype;
};
struct JitKernel;
// Emit CUDA source for the program and compile it with NVRTC; NULL (and the
// reason in *why) when NVRTC is unavailable or the compile fails.
JitKernel* jit_compile(const JitSpec& spec, std::string* why);
void jit_release(JitKernel* k);
// Launch the generated kernel (8 elements per lane when every buffer allows it).
int jit_launch(JitKernel* k, const void* const* inputs, void* out, int64_t n, float* d_amax, cudaStream_t s);
// Whether jit_launch runs the bulk-copy pipeline for these buffers and this size.
bool jit_pipeline_applies(const JitKernel* k, const void* const* inputs, const void* out, int64_t n);

}  // namespace mf
