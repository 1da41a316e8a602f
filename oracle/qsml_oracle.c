/*
 * qsml_oracle.c -- CPU restatement of QuasarML's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA backend, loaded by the
 * test suite, the smoke check and the benchmark's CPU-baseline leg, never by
 * the product path.  Build with -ffp-contract=off and without -ffast-math
 * (see oracle/Makefile): every binary32 operation below is rounded exactly
 * once, as written.
 *
 * Reference citations are file:line inside the QuasarML project.
 */
#include "qsml_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* binary16 <-> binary32                                                      */
/* ------------------------------------------------------------------------ */

/* binary16 -> binary32 is exact. */
float orc_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        /* zero or subnormal: m * 2^-24 is exact in binary32 */
        float v = (float)m * 5.9604644775390625e-08f;
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e - 15u + 127u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* binary32 -> binary16, round to nearest, ties to even; overflow -> inf. */
uint16_t orc_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {
        if (man) return (uint16_t)(sign | 0x7e00u | (man >> 13));
        return (uint16_t)(sign | 0x7c00u);
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e >= 1) {
        uint32_t h = ((uint32_t)e << 10) | (man >> 13);
        uint32_t rem = man & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    /* half subnormal (or zero): value = m_full * 2^(e-14) units of 2^-24 */
    if (exp == 0) return (uint16_t)sign; /* binary32 zero/subnormal < 2^-126 */
    uint32_t m_full = man | 0x800000u;
    int s = 14 - e;
    if (s >= 25) return (uint16_t)sign;
    uint32_t h = m_full >> s;
    uint32_t rem = m_full & ((1u << s) - 1u);
    uint32_t half = 1u << (s - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

static float g_h2f[65536];
static int g_h2f_ready = 0;

static void h2f_table_init(void) {
    if (g_h2f_ready) return;
    for (uint32_t i = 0; i < 65536u; ++i) g_h2f[i] = orc_half_to_float((uint16_t)i);
    g_h2f_ready = 1;
}

static inline float h2f(uint16_t h) { return g_h2f[h]; }

void orc_half_to_float_n(const uint16_t* in, float* out, int64_t n) {
    h2f_table_init();
    for (int64_t i = 0; i < n; ++i) out[i] = h2f(in[i]);
}

void orc_float_to_half_n(const float* in, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = orc_float_to_half(in[i]);
}

/* ------------------------------------------------------------------------ */
/* Element semantics                                                          */
/* ------------------------------------------------------------------------ */

static inline float canonical_nan(void) {
    uint32_t b = 0x7fffffffu;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* pow has no counterpart in the reference snapshot (no symbol in
 * Ops/Elementwise.h:10-30).  Semantics: C99 powf, with exponent 2 computed
 * as the single correctly rounded product x*x. */
float orc_pow_f32(float x, float y) {
    if (y == 2.0f) return x * x;
    return powf(x, y);
}

/* relu follows Ops/Elementwise.cpp:53-66 (`max(x, 0)`), with the cases GLSL
 * max leaves open pinned: NaN propagates unchanged, -0 and +0 give +0. */
float orc_relu_f32(float x) {
    if (x != x) return x;
    return x > 0.0f ? x : 0.0f;
}

/* IEEE 754-2019 maximum/minimum: NaN if either operand is NaN (returned as
 * the canonical quiet NaN 0x7fffffff), and -0 < +0.  Order-independent, so
 * any combine tree gives the same bits. */
float orc_max_f32(float a, float b) {
    if (a != a || b != b) return canonical_nan();
    if (a > b) return a;
    if (b > a) return b;
    return signbit(a) ? b : a;
}

float orc_min_f32(float a, float b) {
    if (a != a || b != b) return canonical_nan();
    if (a < b) return a;
    if (b < a) return b;
    return signbit(a) ? a : b;
}

/* One binary op in binary32: Ops/ShaderGen.cpp:40-53 (`a[idx] op b[idx]`),
 * scalar form Ops/Elementwise.cpp:39-51. */
static inline float apply_f32(int op, float a, float b) {
    switch (op) {
        case ORC_ADD: return a + b;
        case ORC_SUB: return a - b;
        case ORC_MUL: return a * b;
        case ORC_DIV: return a / b;
        case ORC_POW: return orc_pow_f32(a, b);
    }
    return canonical_nan();
}

static inline int32_t apply_i32(int op, int32_t a, int32_t b) {
    uint32_t ua = (uint32_t)a, ub = (uint32_t)b;
    switch (op) {
        case ORC_ADD: return (int32_t)(ua + ub);
        case ORC_SUB: return (int32_t)(ua - ub);
        case ORC_MUL: return (int32_t)(ua * ub);
        case ORC_DIV: return b == 0 ? 0 : (a == INT32_MIN && b == -1 ? INT32_MIN : a / b);
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Broadcasting                                                               */
/* ------------------------------------------------------------------------ */

/* Two-sided NumPy broadcasting.  The reference only has the one-sided test
 * Tensor::is_broadcastable (Core/Tensor.cpp:142-151: right-aligned, each
 * pair equal or one of them 1), which nothing calls; binary ops there
 * assert equal shapes (Ops/Elementwise.cpp:140). */
int orc_broadcast_shape(const int64_t* a_shape, int a_ndim,
                        const int64_t* b_shape, int b_ndim,
                        int64_t* out_shape, int* out_ndim) {
    int n = a_ndim > b_ndim ? a_ndim : b_ndim;
    for (int i = 0; i < n; ++i) {
        int ia = a_ndim - n + i, ib = b_ndim - n + i;
        int64_t da = ia >= 0 ? a_shape[ia] : 1;
        int64_t db = ib >= 0 ? b_shape[ib] : 1;
        if (da != db && da != 1 && db != 1) return -1;
        out_shape[i] = da == 1 ? db : da;
    }
    *out_ndim = n;
    return 0;
}

/* Contiguous strides of `shape` right-aligned into an n-dim frame, with 0
 * for broadcast dims. */
static void bcast_strides(const int64_t* shape, int ndim,
                          int n, int64_t* st) {
    int64_t s = 1;
    for (int i = n - 1; i >= 0; --i) {
        int j = ndim - n + i;
        if (j < 0) { st[i] = 0; continue; }
        st[i] = shape[j] == 1 ? 0 : s;
        s *= shape[j];
    }
}

typedef struct {
    int n;
    int64_t shape[16];
    int64_t sa[16], sb[16];
    int64_t total;
} bplan;

static int make_plan(const int64_t* a_shape, int a_ndim, const int64_t* b_shape,
                     int b_ndim, bplan* p) {
    if (a_ndim > 16 || b_ndim > 16) return -1;
    if (orc_broadcast_shape(a_shape, a_ndim, b_shape, b_ndim, p->shape, &p->n)) return -1;
    bcast_strides(a_shape, a_ndim, p->n, p->sa);
    bcast_strides(b_shape, b_ndim, p->n, p->sb);
    p->total = 1;
    for (int i = 0; i < p->n; ++i) p->total *= p->shape[i];
    return 0;
}

/* Offsets of output element `idx` in a and b. */
static inline void plan_offsets(const bplan* p, int64_t idx, int64_t* oa, int64_t* ob) {
    int64_t a = 0, b = 0;
    for (int i = p->n - 1; i >= 0; --i) {
        int64_t c = idx % p->shape[i];
        idx /= p->shape[i];
        a += c * p->sa[i];
        b += c * p->sb[i];
    }
    *oa = a;
    *ob = b;
}

int orc_binary_f32(int op, const float* a, const int64_t* a_shape, int a_ndim,
                   const float* b, const int64_t* b_shape, int b_ndim, float* out) {
    bplan p;
    if (make_plan(a_shape, a_ndim, b_shape, b_ndim, &p)) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < p.total; ++i) {
        int64_t oa, ob;
        plan_offsets(&p, i, &oa, &ob);
        out[i] = apply_f32(op, a[oa], b[ob]);
    }
    return 0;
}

int orc_binary_f16(int op, const uint16_t* a, const int64_t* a_shape, int a_ndim,
                   const uint16_t* b, const int64_t* b_shape, int b_ndim, uint16_t* out) {
    bplan p;
    if (make_plan(a_shape, a_ndim, b_shape, b_ndim, &p)) return -1;
    h2f_table_init();
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < p.total; ++i) {
        int64_t oa, ob;
        plan_offsets(&p, i, &oa, &ob);
        out[i] = orc_float_to_half(apply_f32(op, h2f(a[oa]), h2f(b[ob])));
    }
    return 0;
}

int orc_binary_i32(int op, const int32_t* a, const int64_t* a_shape, int a_ndim,
                   const int32_t* b, const int64_t* b_shape, int b_ndim, int32_t* out) {
    bplan p;
    if (make_plan(a_shape, a_ndim, b_shape, b_ndim, &p)) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < p.total; ++i) {
        int64_t oa, ob;
        plan_offsets(&p, i, &oa, &ob);
        out[i] = apply_i32(op, a[oa], b[ob]);
    }
    return 0;
}

/* add_scalar / multiply_scalar: Ops/Elementwise.cpp:207-241 with the shader
 * of Ops/Elementwise.cpp:39-51 (`in_data[idx] op scalar`). */
void orc_binary_scalar_f32(int op, const float* x, int64_t n, float s, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = apply_f32(op, x[i], s);
}

void orc_relu_f32_n(const float* x, int64_t n, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = orc_relu_f32(x[i]);
}

/* Ops/Elementwise.cpp:243-417: neg/abs/sqrt/exp/log/sin/cos/tanh map to the
 * GLSL built-ins; sigmoid is `1 / (1 + exp(-x))` (:77) and gelu is
 * `0.5 * x * (1 + tanh(0.7978845608 * (x + 0.044715 * x * x * x)))` (:93),
 * both evaluated left to right in binary32. */
static float unary1(int op, float x) {
    switch (op) {
        case ORC_UN_RELU: return orc_relu_f32(x);
        case ORC_UN_NEG: return -x;
        case ORC_UN_ABS: return fabsf(x);
        case ORC_UN_SQRT: return sqrtf(x);
        case ORC_UN_EXP: return expf(x);
        case ORC_UN_LOG: return logf(x);
        case ORC_UN_SIN: return sinf(x);
        case ORC_UN_COS: return cosf(x);
        case ORC_UN_TANH: return tanhf(x);
        case ORC_UN_SIGMOID: return 1.0f / (1.0f + expf(-x));
        case ORC_UN_GELU: {
            float c = 0.044715f * x * x * x;
            return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + c)));
        }
    }
    return canonical_nan();
}

int orc_unary_f32(int op, const float* x, int64_t n, float* out) {
    if (op < ORC_UN_RELU || op > ORC_UN_GELU) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = unary1(op, x[i]);
    return 0;
}

void orc_relu_f16_n(const uint16_t* x, int64_t n, uint16_t* out) {
    h2f_table_init();
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        uint16_t h = x[i];
        float f = h2f(h);
        /* NaN keeps its payload; everything not > 0 becomes +0 */
        out[i] = (f != f) ? h : (f > 0.0f ? h : (uint16_t)0);
    }
}

/* ------------------------------------------------------------------------ */
/* Reductions                                                                 */
/* ------------------------------------------------------------------------ */

/* Axis reduction: Ops/Reduction.cpp:293-345.  The reference decomposes the
 * tensor into [outer, axis_size, inner] (Reduction.cpp:310-312) and runs,
 * per output, `for k in 0..axis_size-1: acc += in[(o*axis_size+k)*inner+i]`
 * in the tensor's own type (Reduction.cpp:328); mean multiplies that sum by
 * 1.0f/(f32)n (Reduction.cpp:347-356).  Full sum/max/min
 * (Reduction.cpp:21-211) is the same with outer = inner = 1; its combine
 * order is implementation-defined there, so binary64 is the truth.  Axis
 * max/min are stubs in the reference (Reduction.cpp:366-382) and are defined
 * here with IEEE 754-2019 maximum/minimum. */
#define REDUCE_BODY(LOAD)                                                       \
    for (int64_t o = 0; o < outer; ++o) {                                       \
        for (int64_t i = 0; i < inner; ++i) {                                   \
            float a32;                                                          \
            double a64 = 0.0, aabs = 0.0;                                       \
            if (op == ORC_MAX) a32 = -INFINITY;                                 \
            else if (op == ORC_MIN) a32 = INFINITY;                             \
            else if (op == ORC_PROD) { a32 = 1.0f; a64 = 1.0; }                 \
            else a32 = 0.0f;                                                    \
            const int64_t base = o * k * inner + i;                             \
            for (int64_t kk = 0; kk < k; ++kk) {                                \
                float v = LOAD(base + kk * inner);                              \
                if (op == ORC_MAX) a32 = orc_max_f32(a32, v);                   \
                else if (op == ORC_MIN) a32 = orc_min_f32(a32, v);              \
                else if (op == ORC_PROD) { a32 = a32 * v; a64 *= (double)v; }   \
                else { a32 = a32 + v; a64 += (double)v; aabs += fabs((double)v); } \
            }                                                                   \
            int64_t j = o * inner + i;                                          \
            if (op == ORC_MEAN) {                                               \
                a32 = a32 * (1.0f / (float)k);                                  \
                a64 = a64 / (double)k;                                          \
                aabs = aabs / (double)k;                                        \
            }                                                                   \
            if (op == ORC_MAX || op == ORC_MIN) { a64 = (double)a32; aabs = fabs(a64); } \
            if (op == ORC_PROD) aabs = fabs(a64);                               \
            if (out32) out32[j] = a32;                                          \
            if (out64) out64[j] = a64;                                          \
            if (absum) absum[j] = aabs;                                         \
        }                                                                       \
    }

#define LOAD_F32(idx) (x[(idx)])
#define LOAD_F16(idx) (h2f(x[(idx)]))

void orc_reduce_f32(int op, const float* x, int64_t outer, int64_t k, int64_t inner,
                    float* out32, double* out64, double* absum) {
    REDUCE_BODY(LOAD_F32)
}

void orc_reduce_f16(int op, const uint16_t* x, int64_t outer, int64_t k, int64_t inner,
                    float* out32, double* out64, double* absum) {
    h2f_table_init();
    REDUCE_BODY(LOAD_F16)
}

/* ------------------------------------------------------------------------ */
/* argmax / argmin                                                            */
/* ------------------------------------------------------------------------ */

/* The reference's argmax/argmin (Ops/Reduction.cpp:388-396) ignore the axis
 * and return max/min values, not indices.  This restates what the names
 * promise, with NumPy's argmax/argmin conventions: scan k in ascending
 * order, keep the first strictly better value; a NaN beats every number and
 * the first NaN is kept.  Values are read as double (exact for every
 * QSML dtype). */
static inline double arg_load(int dtype, const void* x, int64_t i) {
    switch (dtype) {
        case 0: return ((const float*)x)[i];
        case 1: return h2f(((const uint16_t*)x)[i]);
        case 2: return ((const int32_t*)x)[i];
        case 3: return ((const int16_t*)x)[i];
        case 4: return ((const int8_t*)x)[i];
        case 5: return ((const uint32_t*)x)[i];
        case 6: return ((const uint16_t*)x)[i];
        default: return ((const uint8_t*)x)[i];
    }
}

void orc_argreduce(int op, int dtype, const void* x, int64_t outer, int64_t k, int64_t inner, int64_t* out) {
    if (dtype == 1) h2f_table_init();
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < outer; ++o) {
        for (int64_t i = 0; i < inner; ++i) {
            const int64_t base = o * k * inner + i;
            double best = arg_load(dtype, x, base);
            int64_t bi = 0;
            for (int64_t j = 1; j < k && best == best; ++j) {
                const double v = arg_load(dtype, x, base + j * inner);
                const int better = v != v || (op == 0 ? v > best : v < best);
                if (better) {
                    best = v;
                    bi = j;
                }
            }
            out[o * inner + i] = bi;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Softmax                                                                    */
/* ------------------------------------------------------------------------ */

/* The reference's shader (Ops/Elementwise.cpp:98-135): row max, sum of
 * exp(x - max), then exp(x - max) / sum; here in binary64 over any axis. */
void orc_softmax(const void* x, int f16, int64_t outer, int64_t k, int64_t inner, double* out) {
    if (f16) h2f_table_init();
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < outer; ++o) {
        for (int64_t i = 0; i < inner; ++i) {
            const int64_t base = o * k * inner + i;
            double m = -INFINITY;
            int nan = 0;
            for (int64_t j = 0; j < k; ++j) {
                const int64_t q = base + j * inner;
                const double v = f16 ? (double)h2f(((const uint16_t*)x)[q]) : (double)((const float*)x)[q];
                if (v != v) nan = 1;
                if (v > m) m = v;
            }
            double s = 0.0;
            for (int64_t j = 0; j < k; ++j) {
                const int64_t q = base + j * inner;
                const double v = f16 ? (double)h2f(((const uint16_t*)x)[q]) : (double)((const float*)x)[q];
                s += exp(v - m);
            }
            for (int64_t j = 0; j < k; ++j) {
                const int64_t q = base + j * inner;
                const double v = f16 ? (double)h2f(((const uint16_t*)x)[q]) : (double)((const float*)x)[q];
                out[q] = nan ? NAN : exp(v - m) / s;
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Strided gather                                                             */
/* ------------------------------------------------------------------------ */

/* Materialises a strided view.  The reference's slice (Ops/Manipulation.cpp:
 * 146-161) copies one contiguous byte range through the host (correct for
 * axis 0 only, no step) and its copy kernel (Manipulation.cpp:18-30,
 * 171-184) is a flat element copy; this restates NumPy view semantics:
 * out[i0,...,in] = base[sum_d i_d * strides[d]]. */
void orc_gather(const void* base, int esize, int ndim, const int64_t* shape,
                const int64_t* strides, void* out) {
    int64_t total = 1;
    for (int d = 0; d < ndim; ++d) total *= shape[d];
    const char* src = (const char*)base;
    char* dst = (char*)out;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < total; ++idx) {
        int64_t rem = idx, off = 0;
        for (int d = ndim - 1; d >= 0; --d) {
            int64_t c = rem % shape[d];
            rem /= shape[d];
            off += c * strides[d];
        }
        memcpy(dst + idx * esize, src + off * esize, (size_t)esize);
    }
}

/* ------------------------------------------------------------------------ */
/* Layer norm                                                                 */
/* ------------------------------------------------------------------------ */

/* Layer norm has no counterpart in the reference snapshot.  Definition:
 * y = (x - mean) / sqrt(var + eps) * gamma + beta over the last dim, with
 * the biased (population) variance, evaluated in binary64 by two passes. */
static void ln_row_f64(const double* xr, const float* gamma, const float* beta,
                       int64_t cols, float eps, double* yr) {
    double mean = 0.0;
    for (int64_t c = 0; c < cols; ++c) mean += xr[c];
    mean /= (double)cols;
    double var = 0.0;
    for (int64_t c = 0; c < cols; ++c) {
        double d = xr[c] - mean;
        var += d * d;
    }
    var /= (double)cols;
    double rstd = 1.0 / sqrt(var + (double)eps);
    for (int64_t c = 0; c < cols; ++c)
        yr[c] = (xr[c] - mean) * rstd * (double)gamma[c] + (double)beta[c];
}

void orc_layer_norm_f32(const float* x, const float* gamma, const float* beta,
                        int64_t rows, int64_t cols, float eps, float* y) {
#pragma omp parallel
    {
        double* xr = (double*)malloc(sizeof(double) * (size_t)cols);
        double* yr = (double*)malloc(sizeof(double) * (size_t)cols);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            for (int64_t c = 0; c < cols; ++c) xr[c] = (double)x[r * cols + c];
            ln_row_f64(xr, gamma, beta, cols, eps, yr);
            for (int64_t c = 0; c < cols; ++c) y[r * cols + c] = (float)yr[c];
        }
        free(xr);
        free(yr);
    }
}

void orc_layer_norm_f16(const uint16_t* x, const float* gamma, const float* beta,
                        int64_t rows, int64_t cols, float eps, uint16_t* y) {
    h2f_table_init();
#pragma omp parallel
    {
        double* xr = (double*)malloc(sizeof(double) * (size_t)cols);
        double* yr = (double*)malloc(sizeof(double) * (size_t)cols);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            for (int64_t c = 0; c < cols; ++c) xr[c] = (double)h2f(x[r * cols + c]);
            ln_row_f64(xr, gamma, beta, cols, eps, yr);
            for (int64_t c = 0; c < cols; ++c) y[r * cols + c] = orc_float_to_half((float)yr[c]);
        }
        free(xr);
        free(yr);
    }
}

/* ------------------------------------------------------------------------ */
/* Matmul                                                                     */
/* ------------------------------------------------------------------------ */

/* Ops/LinAlg.cpp:84-158 (matmul_shader_blocked): C[r][c] accumulates
 * fma(A[r][k], B[k][c], acc) for k ascending (K-tiles of 16, 4 k per
 * unrolled step, all in order), row-major A[M,K], B[K,N], C[M,N].
 * batch_matmul (LinAlg.cpp:273-290) is broken in the reference; here each
 * batch entry is its own matmul. */
void orc_matmul_f32_fma(const float* A, const float* B, float* C,
                        int64_t batch, int64_t M, int64_t K, int64_t N,
                        int64_t sA, int64_t sB, int64_t sC) {
    for (int64_t bi = 0; bi < batch; ++bi) {
        const float* a = A + bi * sA;
        const float* b = B + bi * sB;
        float* c = C + bi * sC;
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < M; ++r) {
            for (int64_t col = 0; col < N; ++col) {
                float acc = 0.0f;
                for (int64_t kk = 0; kk < K; ++kk) acc = fmaf(a[r * K + kk], b[kk * N + col], acc);
                c[r * N + col] = acc;
            }
        }
    }
}

void orc_matmul_f64(const float* A, const float* B, double* C,
                    int64_t batch, int64_t M, int64_t K, int64_t N,
                    int64_t sA, int64_t sB, int64_t sC) {
    for (int64_t bi = 0; bi < batch; ++bi) {
        const float* a = A + bi * sA;
        const float* b = B + bi * sB;
        double* c = C + bi * sC;
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < M; ++r) {
            for (int64_t col = 0; col < N; ++col) c[r * N + col] = 0.0;
            for (int64_t kk = 0; kk < K; ++kk) {
                double av = (double)a[r * K + kk];
                const float* brow = b + kk * N;
                double* crow = c + r * N;
                for (int64_t col = 0; col < N; ++col) crow[col] += av * (double)brow[col];
            }
        }
    }
}

void orc_matmul_f16in_f64(const uint16_t* A, const uint16_t* B, double* C,
                          int64_t batch, int64_t M, int64_t K, int64_t N,
                          int64_t sA, int64_t sB, int64_t sC) {
    h2f_table_init();
    for (int64_t bi = 0; bi < batch; ++bi) {
        const uint16_t* a = A + bi * sA;
        const uint16_t* b = B + bi * sB;
        double* c = C + bi * sC;
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < M; ++r) {
            for (int64_t col = 0; col < N; ++col) c[r * N + col] = 0.0;
            for (int64_t kk = 0; kk < K; ++kk) {
                double av = (double)h2f(a[r * K + kk]);
                const uint16_t* brow = b + kk * N;
                double* crow = c + r * N;
                for (int64_t col = 0; col < N; ++col) crow[col] += av * (double)h2f(brow[col]);
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* CPU-baseline variants (OpenMP over outputs / fixed chunks)                 */
/* ------------------------------------------------------------------------ */

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

#define PAR_CHUNK 65536

static inline float comb(int op, float a, float v) {
    if (op == ORC_MAX) return orc_max_f32(a, v);
    if (op == ORC_MIN) return orc_min_f32(a, v);
    if (op == ORC_PROD) return a * v;
    return a + v;
}

static inline float ident(int op) {
    if (op == ORC_MAX) return -INFINITY;
    if (op == ORC_MIN) return INFINITY;
    if (op == ORC_PROD) return 1.0f;
    return 0.0f;
}

#define PAR_REDUCE_BODY(LOAD)                                                   \
    if (outer * inner == 1) {                                                   \
        int64_t nchunks = (k + PAR_CHUNK - 1) / PAR_CHUNK;                      \
        float* part = (float*)malloc(sizeof(float) * (size_t)nchunks);          \
        _Pragma("omp parallel for schedule(static)")                           \
        for (int64_t c = 0; c < nchunks; ++c) {                                 \
            int64_t lo = c * PAR_CHUNK, hi = lo + PAR_CHUNK < k ? lo + PAR_CHUNK : k; \
            float a = ident(op);                                                \
            for (int64_t j = lo; j < hi; ++j) a = comb(op, a, LOAD(j));         \
            part[c] = a;                                                        \
        }                                                                       \
        float a = ident(op);                                                    \
        for (int64_t c = 0; c < nchunks; ++c) a = comb(op, a, part[c]);         \
        if (op == ORC_MEAN) a = a * (1.0f / (float)k);                          \
        out32[0] = a;                                                           \
        free(part);                                                             \
        return;                                                                 \
    }                                                                           \
    if (inner == 1) {                                                           \
        _Pragma("omp parallel for schedule(static)")                           \
        for (int64_t o = 0; o < outer; ++o) {                                   \
            float a = ident(op);                                                \
            for (int64_t kk = 0; kk < k; ++kk) a = comb(op, a, LOAD(o * k + kk)); \
            if (op == ORC_MEAN) a = a * (1.0f / (float)k);                      \
            out32[o] = a;                                                       \
        }                                                                       \
        return;                                                                 \
    }                                                                           \
    /* column reduction: rows of `inner` accumulate in k order, vectorisable */ \
    {                                                                           \
        int64_t tiles = (inner + 255) / 256;                                    \
        _Pragma("omp parallel for schedule(static)")                           \
        for (int64_t t = 0; t < outer * tiles; ++t) {                           \
            int64_t o = t / tiles, i0 = (t % tiles) * 256;                      \
            int64_t i1 = i0 + 256 < inner ? i0 + 256 : inner;                   \
            float acc[256];                                                     \
            for (int64_t i = i0; i < i1; ++i) acc[i - i0] = ident(op);          \
            for (int64_t kk = 0; kk < k; ++kk) {                                \
                int64_t base = (o * k + kk) * inner;                            \
                for (int64_t i = i0; i < i1; ++i)                               \
                    acc[i - i0] = comb(op, acc[i - i0], LOAD(base + i));        \
            }                                                                   \
            for (int64_t i = i0; i < i1; ++i) {                                 \
                float a = acc[i - i0];                                          \
                if (op == ORC_MEAN) a = a * (1.0f / (float)k);                  \
                out32[o * inner + i] = a;                                       \
            }                                                                   \
        }                                                                       \
    }

void orc_reduce_f32_par(int op, const float* x, int64_t outer, int64_t k, int64_t inner,
                        float* out32) {
    PAR_REDUCE_BODY(LOAD_F32)
}

void orc_reduce_f16_par(int op, const uint16_t* x, int64_t outer, int64_t k, int64_t inner,
                        float* out32) {
    h2f_table_init();
    PAR_REDUCE_BODY(LOAD_F16)
}
