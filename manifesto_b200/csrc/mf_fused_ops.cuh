// mf_fused_ops.cuh -- element semantics of a fused elementwise chain.
//
// One place for the per-node rules of manifesto's evalCPU
// (codegen/cpu.go:126-212), shared by the runtime interpreter (fused.cu) and
// by the CUDA source the CUDA codegen target emits for each FusionAST and
// compiles at run time (fused_jit.cu), so the two cannot drift apart:
//   Add/Sub/Mul/Div/Max/Min/Neg/Abs/ReLU/LeakyReLU in float32, nothing
//   contracted (Max: l > r ? l : r, :144-151; Min :153-160; Abs :165-170;
//   ReLU v < 0 ? 0 : v, :178-184; LeakyReLU slope 0.01, :201-206);
//   Sqrt/Exp/Log/Sigmoid/Tanh/SiLU/GELU in float64, then float32(...) with
//   the amd64 NaN rule (:172-200); GELU's sqrt(2/pi) folded in float64 (:198).
// Unknown nodes evaluate to 0 (:208-210).
#pragma once

#include "mf_numerics.cuh"

// optimizer.NodeType values, optimizer/fusion_ast.go:32-65
enum NodeType : int32_t {
    NODE_INVALID = 0, NODE_INPUT, NODE_CONSTANT, NODE_ADD, NODE_SUB, NODE_MUL, NODE_DIV, NODE_MAX, NODE_MIN,
    NODE_NEG, NODE_ABS, NODE_SQRT, NODE_EXP, NODE_LOG, NODE_RELU, NODE_SIGMOID, NODE_TANH, NODE_SILU,
    NODE_GELU, NODE_LEAKY_RELU
};

namespace mf {

// sqrt(2/pi) in float64: Go folds the constant 2/math.Pi exactly and math.Sqrt
// rounds once (codegen/cpu.go:198).
__device__ __forceinline__ double gelu_k() { return sqrt(0.63661977236758134307553505349005744813783858296182579499); }

template <int OP>
__device__ __forceinline__ float fused_unary(float v) {
    if constexpr (OP == NODE_NEG) return -v;
    else if constexpr (OP == NODE_ABS) return v < 0.0f ? -v : v;
    else if constexpr (OP == NODE_SQRT) return f64_to_f32(sqrt(static_cast<double>(v)));
    else if constexpr (OP == NODE_EXP) return f64_to_f32(exp(static_cast<double>(v)));
    else if constexpr (OP == NODE_LOG) return f64_to_f32(log(static_cast<double>(v)));
    else if constexpr (OP == NODE_RELU) return v < 0.0f ? 0.0f : v;
    else if constexpr (OP == NODE_SIGMOID) return f64_to_f32(__drcp_rn(__dadd_rn(1.0, exp(-static_cast<double>(v)))));
    else if constexpr (OP == NODE_TANH) return f64_to_f32(tanh(static_cast<double>(v)));
    else if constexpr (OP == NODE_SILU) {
        const double d = static_cast<double>(v);
        return f64_to_f32(__ddiv_rn(d, __dadd_rn(1.0, exp(-d))));
    } else if constexpr (OP == NODE_GELU) {
        const double d = static_cast<double>(v);
        const double cube = __dmul_rn(__dmul_rn(__dmul_rn(0.044715, d), d), d);
        const double inner = __dmul_rn(gelu_k(), __dadd_rn(d, cube));
        return f64_to_f32(__dmul_rn(__dmul_rn(0.5, d), __dadd_rn(1.0, tanh(inner))));
    } else if constexpr (OP == NODE_LEAKY_RELU) return v >= 0.0f ? v : __fmul_rn(0.01f, v);
    else return 0.0f;
}

template <int OP>
__device__ __forceinline__ float fused_binary(float a, float b) {
    if constexpr (OP == NODE_ADD) return __fadd_rn(a, b);
    else if constexpr (OP == NODE_SUB) return __fsub_rn(a, b);
    else if constexpr (OP == NODE_MUL) return __fmul_rn(a, b);
    else if constexpr (OP == NODE_DIV) return __fdiv_rn(a, b);
    else if constexpr (OP == NODE_MAX) return a > b ? a : b;
    else if constexpr (OP == NODE_MIN) return a < b ? a : b;
    else return 0.0f;
}

// ------------------------------------------- float32 forms for 16-bit outputs
//
// A chain whose output is BF16 or F16 is held to 1 ulp of that format after the
// final cast (2^-8 or 2^-11 relative), far coarser than float32.  For a node whose
// value reaches such an output only through operations that keep relative error
// (Mul, Div, Neg, Abs, ReLU, LeakyReLU, Max, Min -- the code generator checks the
// path), the generated code evaluates the float64 rule in float32 on the SFU,
// inside ranges where both this form and the reference's float64 value are
// accurate to better than 2^-16 relative.  Outside them (NaN, overflow edges,
// GELU far below zero, where the reference's 1 + tanh(u) in float64 keeps only a
// few significant bits) the float64 rule runs.  ex2/rcp flush subnormals; inside
// the ranges their arguments and results are normal.
__device__ __forceinline__ float sfu_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float sfu_rcp(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int OP>
__device__ __forceinline__ float fused_unary_fast(float v) {
    constexpr float kLog2e = 1.4426950408889634f;
    if constexpr (OP == NODE_EXP) {
        if (v >= -80.0f && v <= 88.0f) return sfu_ex2(__fmul_rn(v, kLog2e));
    } else if constexpr (OP == NODE_SIGMOID) {
        if (v >= -80.0f) return sfu_rcp(__fadd_rn(1.0f, sfu_ex2(__fmul_rn(v, -kLog2e))));
    } else if constexpr (OP == NODE_SILU) {
        if (v >= -80.0f) return __fmul_rn(v, sfu_rcp(__fadd_rn(1.0f, sfu_ex2(__fmul_rn(v, -kLog2e)))));
    } else if constexpr (OP == NODE_TANH) {
        if (v == v) return tanhf(v);
    } else if constexpr (OP == NODE_LOG) {
        if (v >= 1.0e-30f && v <= 1.0e30f) return logf(v);
    } else if constexpr (OP == NODE_SQRT) {
        if (v >= 0.0f) return __fsqrt_rn(v);
    } else if constexpr (OP == NODE_GELU) {
        // 0.5 x (1 + tanh(u)) = x / (1 + e^(-2u)), u = sqrt(2/pi) (x + 0.044715 x^3)
        const float u =
            __fmul_rn(0.7978845608028654f, __fadd_rn(v, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v)));
        if (u >= -9.0f && v <= 3.0e38f)
            return __fmul_rn(v, sfu_rcp(__fadd_rn(1.0f, sfu_ex2(__fmul_rn(u, -2.0f * kLog2e)))));
    }
    return fused_unary<OP>(v);
}

// fused_unary_fast without the branch: always the float32 form, and `bad` set
// when the input lies outside its range.  The caller re-evaluates an element
// that set it with fused_unary_fast (one branch per group of elements instead
// of one per element).
template <int OP>
__device__ __forceinline__ float fused_unary_try(float v, bool& bad) {
    constexpr float kLog2e = 1.4426950408889634f;
    if constexpr (OP == NODE_EXP) {
        bad |= !(v >= -80.0f && v <= 88.0f);
        return sfu_ex2(__fmul_rn(v, kLog2e));
    } else if constexpr (OP == NODE_SIGMOID) {
        bad |= !(v >= -80.0f);
        return sfu_rcp(__fadd_rn(1.0f, sfu_ex2(__fmul_rn(v, -kLog2e))));
    } else if constexpr (OP == NODE_SILU) {
        bad |= !(v >= -80.0f);
        return __fmul_rn(v, sfu_rcp(__fadd_rn(1.0f, sfu_ex2(__fmul_rn(v, -kLog2e)))));
    } else if constexpr (OP == NODE_TANH) {
        bad |= (v != v);
        return tanhf(v);
    } else if constexpr (OP == NODE_LOG) {
        bad |= !(v >= 1.0e-30f && v <= 1.0e30f);
        return logf(v);
    } else if constexpr (OP == NODE_SQRT) {
        bad |= !(v >= 0.0f);
        return __fsqrt_rn(v);
    } else if constexpr (OP == NODE_GELU) {
        const float u =
            __fmul_rn(0.7978845608028654f, __fadd_rn(v, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v)));
        bad |= !(u >= -9.0f && v <= 3.0e38f);
        return __fmul_rn(v, sfu_rcp(__fadd_rn(1.0f, sfu_ex2(__fmul_rn(u, -2.0f * kLog2e)))));
    } else {
        return fused_unary<OP>(v);
    }
}

// Pairs of elements.  Multiplies use Blackwell's packed float32 multiply (each
// lane rounds like __fmul_rn); adds stay scalar __fadd_rn, which is never merged
// into a fused multiply-add.  A packed multiply feeding a packed add was measured
// on B200 to be contracted into one (a single rounding) in some compiled
// contexts, even written as PTX with .rn, where the reference rounds the product
// and the sum separately.  The generated code uses these for chains with a
// 16-bit output, where NaN is compared as a class.
template <int OP>
__device__ __forceinline__ float2 fused_binary2(float2 a, float2 b) {
    if constexpr (OP == NODE_ADD) return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
    else if constexpr (OP == NODE_SUB) return make_float2(__fsub_rn(a.x, b.x), __fsub_rn(a.y, b.y));
    else if constexpr (OP == NODE_MUL) return __fmul2_rn(a, b);
    else return make_float2(fused_binary<OP>(a.x, b.x), fused_binary<OP>(a.y, b.y));
}
template <int OP>
__device__ __forceinline__ float2 fused_unary2(float2 v) {
    return make_float2(fused_unary<OP>(v.x), fused_unary<OP>(v.y));
}
// fused_unary_try on both lanes (GELU's polynomial packed).
template <int OP>
__device__ __forceinline__ float2 fused_unary2_try(float2 v, bool& bad) {
    if constexpr (OP == NODE_GELU) {
        constexpr float kM2Log2e = -2.0f * 1.4426950408889634f;
        const float2 c3 = make_float2(0.044715f, 0.044715f), k = make_float2(0.7978845608028654f, 0.7978845608028654f);
        // the float32 approximation's own arithmetic (held to the 1-ulp bar of the 16-bit
        // output, not to a reference rounding): packed throughout
        const float2 u = __fmul2_rn(k, __fadd2_rn(v, __fmul2_rn(__fmul2_rn(__fmul2_rn(c3, v), v), v)));
        const float2 a = __fmul2_rn(u, make_float2(kM2Log2e, kM2Log2e));
        bad |= !(u.x >= -9.0f && v.x <= 3.0e38f && u.y >= -9.0f && v.y <= 3.0e38f);
        return __fmul2_rn(v, make_float2(sfu_rcp(__fadd_rn(1.0f, sfu_ex2(a.x))), sfu_rcp(__fadd_rn(1.0f, sfu_ex2(a.y)))));
    } else {
        const float x = fused_unary_try<OP>(v.x, bad);
        return make_float2(x, fused_unary_try<OP>(v.y, bad));
    }
}

// The same with the node type known only at run time (the interpreter).
__device__ __forceinline__ float fused_unary_rt(int op, float v) {
    switch (op) {
    case NODE_NEG: return fused_unary<NODE_NEG>(v);
    case NODE_ABS: return fused_unary<NODE_ABS>(v);
    case NODE_SQRT: return fused_unary<NODE_SQRT>(v);
    case NODE_EXP: return fused_unary<NODE_EXP>(v);
    case NODE_LOG: return fused_unary<NODE_LOG>(v);
    case NODE_RELU: return fused_unary<NODE_RELU>(v);
    case NODE_SIGMOID: return fused_unary<NODE_SIGMOID>(v);
    case NODE_TANH: return fused_unary<NODE_TANH>(v);
    case NODE_SILU: return fused_unary<NODE_SILU>(v);
    case NODE_GELU: return fused_unary<NODE_GELU>(v);
    case NODE_LEAKY_RELU: return fused_unary<NODE_LEAKY_RELU>(v);
    default: return 0.0f;
    }
}
__device__ __forceinline__ float fused_binary_rt(int op, float a, float b) {
    switch (op) {
    case NODE_ADD: return fused_binary<NODE_ADD>(a, b);
    case NODE_SUB: return fused_binary<NODE_SUB>(a, b);
    case NODE_MUL: return fused_binary<NODE_MUL>(a, b);
    case NODE_DIV: return fused_binary<NODE_DIV>(a, b);
    case NODE_MAX: return fused_binary<NODE_MAX>(a, b);
    case NODE_MIN: return fused_binary<NODE_MIN>(a, b);
    default: return 0.0f;
    }
}

// |stored value| of an output code, NaN ignored (0): the amax fold of a chain
// whose output is then cast to FP8.
template <int ODT>
__device__ __forceinline__ float stored_abs(uint32_t code) {
    float a;
    if constexpr (ODT == MF_DT_F32) a = fabsf(__uint_as_float(code));
    else if constexpr (ODT == MF_DT_BF16) a = fabsf(__uint_as_float(code << 16));
    else a = fabsf(__uint_as_float(f16_to_f32bits(code)));
    return (a == a) ? a : 0.0f;
}

}  // namespace mf
