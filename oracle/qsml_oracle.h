/*
 * qsml_oracle.h -- CPU restatement of QuasarML's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * backend: only the test suite, the smoke check and the CPU-baseline leg of
 * the benchmark may load it.  The product path (libqsml_cuda.so and the C++
 * QuasarML layer) never links, loads or calls anything in this directory.
 *
 * Every routine is scalar IEEE-754 binary32/binary64 C, compiled with
 * -ffp-contract=off (no FMA contraction) and never with -ffast-math, so the
 * rounding of each operation is the one the C source spells out.
 *
 * Citations are file:line inside the QuasarML reference project.
 *
 * Parity status: the reference snapshot cannot be built here (Vulkan SDK,
 * shaderc and spdlog are absent and no graphics stack exists), so the oracle
 * is pinned only by the known-answer vectors of the reference's own unit
 * tests (unit-tests/src/_test_comprehensive.cpp, _test_qsml_functionality.cpp,
 * _test_minimal.cpp).  Broadcasting, pow, axis min/max, argmax/argmin,
 * softmax values, strided slicing, layer norm, fp16 and batched matmul have
 * no reference implementation or test of their values: for those ops the
 * oracle restates NumPy semantics (or the reference shader's formula) and is
 * "parity unpinned".
 */
#ifndef QSML_ORACLE_H
#define QSML_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Operation codes shared with include/qsml_cuda.h. */
enum { ORC_ADD = 0, ORC_SUB = 1, ORC_MUL = 2, ORC_DIV = 3, ORC_POW = 4 };
enum { ORC_SUM = 0, ORC_MEAN = 1, ORC_MAX = 2, ORC_MIN = 3, ORC_PROD = 4 };

/* Element conversions (IEEE binary16 <-> binary32, round-to-nearest-even). */
float    orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f);
void     orc_half_to_float_n(const uint16_t* in, float* out, int64_t n);
void     orc_float_to_half_n(const float* in, uint16_t* out, int64_t n);

/* NumPy broadcasting of two shapes (right-aligned).  Returns 0 and fills
 * out_shape/out_ndim on success, -1 if the shapes are incompatible. */
int orc_broadcast_shape(const int64_t* a_shape, int a_ndim,
                        const int64_t* b_shape, int b_ndim,
                        int64_t* out_shape, int* out_ndim);

/* out = a (op) b with broadcasting; a, b and out contiguous row-major.
 * op in {ADD, SUB, MUL, DIV, POW}.  Returns 0, or -1 on a shape error. */
int orc_binary_f32(int op, const float* a, const int64_t* a_shape, int a_ndim,
                   const float* b, const int64_t* b_shape, int b_ndim, float* out);
/* binary16 variant: each result is the binary32 result rounded to binary16
 * (correctly rounded for add/sub/mul/div because 24 >= 2*11+2). */
int orc_binary_f16(int op, const uint16_t* a, const int64_t* a_shape, int a_ndim,
                   const uint16_t* b, const int64_t* b_shape, int b_ndim, uint16_t* out);
/* int32 variant (add/sub/mul with two's-complement wraparound). */
int orc_binary_i32(int op, const int32_t* a, const int64_t* a_shape, int a_ndim,
                   const int32_t* b, const int64_t* b_shape, int b_ndim, int32_t* out);

/* Scalar-operand ops: out[i] = x[i] (op) s.  op in {ADD, SUB, MUL, DIV, POW}. */
void orc_binary_scalar_f32(int op, const float* x, int64_t n, float s, float* out);

/* Single-element semantics, exported for the tests. */
float orc_pow_f32(float x, float y);
float orc_relu_f32(float x);
float orc_max_f32(float a, float b);
float orc_min_f32(float a, float b);

void orc_relu_f32_n(const float* x, int64_t n, float* out);

/* Unary ops in the order of include/qsml_cuda.h's QSML_UN_* codes:
 * relu, neg, abs, sqrt, exp, log, sin, cos, tanh, sigmoid, gelu
 * (Ops/Elementwise.cpp:243-417); libm for the transcendental ones. */
enum { ORC_UN_RELU = 0, ORC_UN_NEG, ORC_UN_ABS, ORC_UN_SQRT, ORC_UN_EXP, ORC_UN_LOG,
       ORC_UN_SIN, ORC_UN_COS, ORC_UN_TANH, ORC_UN_SIGMOID, ORC_UN_GELU };
int orc_unary_f32(int op, const float* x, int64_t n, float* out);
void orc_relu_f16_n(const uint16_t* x, int64_t n, uint16_t* out);

/* Reduction of x viewed as [outer, k, inner] over the middle axis.
 * out32: the reference's own order (k ascending, binary32 accumulator);
 * out64: the same in binary64 (the truth the tolerances are measured from).
 * Either output pointer may be NULL.  mean multiplies by 1.0f/(float)k.
 * min/max: IEEE 754-2019 maximum/minimum (-0 < +0, any NaN -> NaN).
 * absum (optional): sum of |x| per output, the natural scale of the
 * summation error. */
void orc_reduce_f32(int op, const float* x, int64_t outer, int64_t k, int64_t inner,
                    float* out32, double* out64, double* absum);
void orc_reduce_f16(int op, const uint16_t* x, int64_t outer, int64_t k, int64_t inner,
                    float* out32, double* out64, double* absum);

/* argmax (op 0) / argmin (op 1) of x viewed as [outer, k, inner] over the
 * middle axis, k >= 1; dtype is a QSML_* code (F32 .. U8).  out[o*inner+i]
 * is the first index of the largest (smallest) value; values compare
 * numerically (-0 == +0) and a NaN counts as larger (smaller) than every
 * number, so the first NaN wins. */
void orc_argreduce(int op, int dtype, const void* x, int64_t outer, int64_t k, int64_t inner, int64_t* out);

/* Softmax of x viewed as [outer, k, inner] over the middle axis, in binary64:
 * m = max (any NaN -> NaN), e = exp(x - m), out = e / sum(e)
 * (Ops/Elementwise.cpp:98-135 restated for any axis).  x is binary32 or
 * binary16 (f16 != 0). */
void orc_softmax(const void* x, int f16, int64_t outer, int64_t k, int64_t inner, double* out);

/* Strided gather: copies the view (base, ndim, shape, strides in elements,
 * possibly negative) of esize-byte elements into contiguous out. */
void orc_gather(const void* base, int esize, int ndim, const int64_t* shape,
                const int64_t* strides, void* out);

/* Layer norm over the last dim of x[rows, cols] with biased variance,
 * computed in binary64 (two-pass) and rounded once to the output type. */
void orc_layer_norm_f32(const float* x, const float* gamma, const float* beta,
                        int64_t rows, int64_t cols, float eps, float* y);
void orc_layer_norm_f16(const uint16_t* x, const float* gamma, const float* beta,
                        int64_t rows, int64_t cols, float eps, uint16_t* y);

/* C[b] = A[b] * B[b], row-major, batch strides in elements (0 = shared).
 * _fma: the reference's binary32 fma chain, k ascending.
 * _f64: binary64 accumulation of the binary32 inputs (the truth).
 * _f16in_f64: inputs given as binary16, binary64 accumulation. */
void orc_matmul_f32_fma(const float* A, const float* B, float* C,
                        int64_t batch, int64_t M, int64_t K, int64_t N,
                        int64_t sA, int64_t sB, int64_t sC);
void orc_matmul_f64(const float* A, const float* B, double* C,
                    int64_t batch, int64_t M, int64_t K, int64_t N,
                    int64_t sA, int64_t sB, int64_t sC);
void orc_matmul_f16in_f64(const uint16_t* A, const uint16_t* B, double* C,
                          int64_t batch, int64_t M, int64_t K, int64_t N,
                          int64_t sA, int64_t sB, int64_t sC);

/* CPU-baseline helpers: same arithmetic spread over OpenMP threads.
 * Full reductions split into fixed chunks (partials combined in chunk
 * order), so their binary32 order differs from the serial one. */
int  orc_num_threads(void);
void orc_set_num_threads(int n);
void orc_reduce_f32_par(int op, const float* x, int64_t outer, int64_t k, int64_t inner, float* out32);
void orc_reduce_f16_par(int op, const uint16_t* x, int64_t outer, int64_t k, int64_t inner, float* out32);

#ifdef __cplusplus
}
#endif
#endif
