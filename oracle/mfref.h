/*
 * mfref.h -- CPU oracle for the manifesto hot path.  TEST INFRASTRUCTURE:
 * only the tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * load this library, and only as the checker / the timed CPU baseline.
 * The product (libmfcuda.so) never links or calls it.
 *
 * Each function restates the manifesto Go scalar code it names
 * (paths are inside the manifesto Go module).  Build flags:
 * -O2 -ffp-contract=off -fno-fast-math, so float arithmetic is the plain
 * IEEE single/double rounding Go uses on amd64.
 *
 * Parity is pinned by the known-answer vectors of the reference's own Go
 * tests (dtype/fp8_test.go, dtype/bfloat16_test.go, dtype/float16_test.go,
 * dtype/int4_test.go, dtype/convert/convert_test.go, codegen/codegen_test.go,
 * runtime/axpy_test.go) transcribed into tests/golden/, plus cross-checks
 * against numpy / ml_dtypes outside the documented quirk bands.  The Go
 * code itself cannot run here (no Go toolchain).
 */
#ifndef MFREF_H
#define MFREF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* scalar codecs: f32 values are passed as their bit patterns */
uint32_t ref_e4m3_decode(uint8_t code);
uint8_t ref_e4m3_encode(uint32_t f32bits);
uint8_t ref_e4m3_encode_ocp(uint32_t f32bits);
uint32_t ref_e5m2_decode(uint8_t code);
uint8_t ref_e5m2_encode(uint32_t f32bits);
uint8_t ref_e5m2_encode_ocp(uint32_t f32bits);
uint16_t ref_bf16_encode(uint32_t f32bits);
uint32_t ref_bf16_decode(uint16_t h);
uint16_t ref_f16_encode(uint32_t f32bits);
uint32_t ref_f16_decode(uint16_t h);
int8_t ref_int4_lo(uint8_t pair);
int8_t ref_int4_hi(uint8_t pair);
uint8_t ref_int4_pair(int8_t lo, int8_t hi);

/* slice drivers (return 0 or a negative status) */
int ref_decode_f32(int src_dtype, const void* src, float* dst, int64_t begin, int64_t n);
int ref_encode_f32(int dst_dtype, const float* src, void* dst, int64_t begin, int64_t n, int compat);
int ref_convert(int src_dtype, int dst_dtype, const void* src, void* dst,
                int64_t begin, int64_t n, int compat);

int ref_int4_dequant_grouped(const uint8_t* q, const void* scales, int scale_dtype,
                             void* out, int out_dtype, int64_t rows, int64_t cols,
                             int64_t group, int64_t row_begin, int64_t row_end);

int ref_axpy(void* y, const void* x, int64_t begin, int64_t n, float alpha, int dtype, int fused_fma);

int ref_linspace(float start, float stop, int64_t count, int endpoint, void* dst, int dst_dtype,
                 int64_t begin, int64_t n);
int ref_scalar_broadcast(const void* src, int src_dtype, void* dst, int dst_dtype,
                         int64_t begin, int64_t n, float scalar, int op);

/* Fused evaluator over a FusionAST given as a node table:
 * type[k] (optimizer.NodeType), value[k] (Constant), input[k] (Input),
 * child0[k], child1[k] (-1 if absent); root is the root node index.
 * inputs are raw buffers of in_dtype[j]; in_bcast[j] = 0 full, L > 0 index
 * i mod L.  Writes out (out_dtype) for elements [begin, begin+n). */
int ref_fused_eval(int n_nodes, const int32_t* type, const double* value, const int32_t* input,
                   const int32_t* child0, const int32_t* child1, int root,
                   int n_inputs, const void* const* inputs, const int32_t* in_dtype,
                   const int64_t* in_bcast, void* out, int out_dtype, int64_t begin, int64_t n);

/* amax over [begin, begin+n) (NaN ignored) as float32 bits */
uint32_t ref_amax(const void* src, int src_dtype, int64_t begin, int64_t n);
/* scale rule of the amax-scaled FP8 cast */
float ref_fp8_scale(float amax, int fp8_dtype);
int ref_scaled_cast(const void* src, int src_dtype, void* dst, int fp8_dtype, float amax,
                    int64_t begin, int64_t n, int compat);

#ifdef __cplusplus
}
#endif

#endif
