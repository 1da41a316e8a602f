// Element type conversion: out = (out dtype) src, elementwise, for binary32
// <-> binary16 (round to nearest even; binary16 -> binary32 is exact) and the
// identity copies.  The reference has no conversion op: its tensors keep the
// dtype they were created with, and an fp16 copy of data has to be built on
// the host and uploaded.  A contiguous conversion is one HBM pass with 16-byte
// loads and stores (8 elements per thread step).
#include "qsml_internal.cuh"

namespace qsml {
namespace {

struct alignas(16) F32x8 {
    float4 a, b;
};

__global__ void __launch_bounds__(256) k_cast_f32_f16(const float* __restrict__ x, __half* __restrict__ y, int64_t n,
                                                      int vec) {
    pdl_begin();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vec) {
        const int64_t n8 = n / 8;
        for (int64_t i = t; i < n8; i += stride) {
            const F32x8 v = reinterpret_cast<const F32x8*>(x)[i];
            __half2 h[4] = {__floats2half2_rn(v.a.x, v.a.y), __floats2half2_rn(v.a.z, v.a.w),
                            __floats2half2_rn(v.b.x, v.b.y), __floats2half2_rn(v.b.z, v.b.w)};
            reinterpret_cast<uint4*>(y)[i] = *reinterpret_cast<const uint4*>(h);
        }
        for (int64_t i = n8 * 8 + t; i < n; i += stride) y[i] = __float2half_rn(x[i]);
    } else {
        for (int64_t i = t; i < n; i += stride) y[i] = __float2half_rn(x[i]);
    }
}

__global__ void __launch_bounds__(256) k_cast_f16_f32(const __half* __restrict__ x, float* __restrict__ y, int64_t n,
                                                      int vec) {
    pdl_begin();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vec) {
        const int64_t n8 = n / 8;
        for (int64_t i = t; i < n8; i += stride) {
            const uint4 raw = reinterpret_cast<const uint4*>(x)[i];
            const __half2* h = reinterpret_cast<const __half2*>(&raw);
            F32x8 v;
            const float2 f0 = __half22float2(h[0]), f1 = __half22float2(h[1]), f2 = __half22float2(h[2]),
                         f3 = __half22float2(h[3]);
            v.a = make_float4(f0.x, f0.y, f1.x, f1.y);
            v.b = make_float4(f2.x, f2.y, f3.x, f3.y);
            reinterpret_cast<F32x8*>(y)[i] = v;
        }
        for (int64_t i = n8 * 8 + t; i < n; i += stride) y[i] = __half2float(x[i]);
    } else {
        for (int64_t i = t; i < n; i += stride) y[i] = __half2float(x[i]);
    }
}

unsigned cast_grid(const Context* ctx, int64_t n) {
    int64_t g = (n / 8 + 255) / 256;
    const int64_t cap = static_cast<int64_t>(ctx->num_sms) * 16;
    if (g > cap) g = cap;
    return static_cast<unsigned>(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace qsml

using namespace qsml;

extern "C" qsml_status_t qsml_cast(qsml_ctx* handle, const qsml_tdesc* src, const qsml_tdesc* out) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, src, "src"));
    QSML_TRY_STATUS(check_desc(C_, out, "out"));
    if (src->ndim != out->ndim) return set_error(C_, QSML_E_SHAPE, "qsml_cast: src and out shapes differ");
    for (int i = 0; i < src->ndim; ++i)
        if (src->shape[i] != out->shape[i]) return set_error(C_, QSML_E_SHAPE, "qsml_cast: src and out shapes differ");
    if (!is_contiguous(src) || !is_contiguous(out))
        return set_error(C_, QSML_E_UNSUPPORTED, "qsml_cast: src and out must be contiguous (gather a view first)");
    const int64_t n = numel(out);
    if (n == 0) return QSML_OK;
    if (src->dtype == out->dtype) {
        if (src->data == out->data) return QSML_OK;
        return check_cuda(C_, cudaMemcpyAsync(out->data, src->data, static_cast<size_t>(n) * dtype_size(src->dtype),
                                              cudaMemcpyDeviceToDevice, C_->stream),
                          "qsml_cast copy");
    }
    const int vec = aligned16(src->data) && aligned16(out->data) ? 1 : 0;
    cudaError_t e;
    if (src->dtype == QSML_F32 && out->dtype == QSML_F16) {
        e = launch_pdl(k_cast_f32_f16, dim3(cast_grid(C_, n)), dim3(256), 0, C_->stream,
                       static_cast<const float*>(src->data), static_cast<__half*>(out->data), n, vec);
        if (e != cudaSuccess) return check_cuda(C_, e, "k_cast_f32_f16");
        return after_launch(C_, "k_cast_f32_f16");
    }
    if (src->dtype == QSML_F16 && out->dtype == QSML_F32) {
        e = launch_pdl(k_cast_f16_f32, dim3(cast_grid(C_, n)), dim3(256), 0, C_->stream,
                       static_cast<const __half*>(src->data), static_cast<float*>(out->data), n, vec);
        if (e != cudaSuccess) return check_cuda(C_, e, "k_cast_f16_f32");
        return after_launch(C_, "k_cast_f16_f32");
    }
    return set_error(C_, QSML_E_DTYPE, "qsml_cast: F32 <-> F16 (or the same dtype) only");
}
