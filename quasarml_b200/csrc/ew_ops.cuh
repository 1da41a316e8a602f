// Elementwise operators with their exact rounding: the one definition used
// by the precompiled kernels (through ew_common.cuh) and, as source text, by
// the runtime-compiled fused kernels (ew_jit.cu).  Device code only, no
// includes when compiled by NVRTC (the JIT prologue defines the QSML_OP_* /
// QSML_UN_* codes and the integer types).
#pragma once

#ifndef __CUDACC_RTC__
#include <cstdint>

#include "qsml_cuda.h"
#endif

namespace qsml {
namespace ew {

// ---------------------------------------------------------------------------
// Operators
// ---------------------------------------------------------------------------
// binary64 pow rounded once; kept out of line so kernels that expand many
// operator instances do not inline one copy per instance.
static __device__ __noinline__ float pow_general(float x, float y) {
    return __double2float_rn(pow(static_cast<double>(x), static_cast<double>(y)));
}

__device__ __forceinline__ float pow_f32(float x, float y) {
    // Exponent 2 is the single correctly rounded product; any other exponent
    // goes through binary64 pow (error far below 1 binary32 ulp) rounded once.
    if (y == 2.0f) return __fmul_rn(x, x);
    return pow_general(x, y);
}

template <int OP> struct BinOp {
    __device__ __forceinline__ float operator()(float a, float b) const {
        if (OP == QSML_OP_ADD) return __fadd_rn(a, b);
        if (OP == QSML_OP_SUB) return __fsub_rn(a, b);
        if (OP == QSML_OP_MUL) return __fmul_rn(a, b);
        if (OP == QSML_OP_DIV) return __fdiv_rn(a, b);
        return pow_f32(a, b);
    }
    __device__ __forceinline__ int32_t operator()(int32_t a, int32_t b) const {
        uint32_t ua = static_cast<uint32_t>(a), ub = static_cast<uint32_t>(b);
        if (OP == QSML_OP_ADD) return static_cast<int32_t>(ua + ub);
        if (OP == QSML_OP_SUB) return static_cast<int32_t>(ua - ub);
        if (OP == QSML_OP_MUL) return static_cast<int32_t>(ua * ub);
        if (OP == QSML_OP_DIV) {
            if (b == 0) return 0;
            if (a == INT32_MIN && b == -1) return INT32_MIN;
            return a / b;
        }
        return 0;
    }
};

template <int OP> struct UnOp {
    __device__ __forceinline__ float operator()(float x) const {
        switch (OP) {
            case QSML_UN_RELU: return (x != x) ? x : (x > 0.0f ? x : 0.0f);
            case QSML_UN_NEG: return -x;
            case QSML_UN_ABS: return fabsf(x);
            case QSML_UN_SQRT: return __fsqrt_rn(x);
            case QSML_UN_EXP: return expf(x);
            case QSML_UN_LOG: return logf(x);
            case QSML_UN_SIN: return sinf(x);
            case QSML_UN_COS: return cosf(x);
            case QSML_UN_TANH: return tanhf(x);
            case QSML_UN_SIGMOID:
                // Ops/Elementwise.cpp:77: 1 / (1 + exp(-x))
                return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
            case QSML_UN_GELU: {
                // Ops/Elementwise.cpp:93, evaluated left to right:
                // 0.5*x*(1 + tanh(0.7978845608*(x + 0.044715*x*x*x)))
                float c = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
                float t = tanhf(__fmul_rn(0.7978845608f, __fadd_rn(x, c)));
                return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
            }
        }
        return x;
    }
    __device__ __forceinline__ int32_t operator()(int32_t x) const {
        switch (OP) {
            case QSML_UN_RELU: return x > 0 ? x : 0;
            case QSML_UN_NEG: return static_cast<int32_t>(0u - static_cast<uint32_t>(x));
            case QSML_UN_ABS: return x < 0 ? static_cast<int32_t>(0u - static_cast<uint32_t>(x)) : x;
        }
        return x;
    }
};

}  // namespace ew
}  // namespace qsml
