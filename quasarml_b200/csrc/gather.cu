// Strided gather: materialise any strided view into a contiguous tensor.
//
// Reference: Ops::slice copies one contiguous byte range through the host
// (Ops/Manipulation.cpp:146-161: axis 0 only, no step), Ops::copy runs a flat
// element copy shader (Manipulation.cpp:18-30, 171-184) and Ops::transpose a
// 2-D shader with uncoalesced writes (Ops/LinAlg.cpp:160-175, 329-351).
// Here views (slices with steps, transposes) are zero-copy descriptors and
// this entry point turns one into contiguous memory.  After dropping unit
// dims and merging dims that are contiguous in the source, one of:
//   * one contiguous run            -> cudaMemcpyAsync (device to device);
//   * inner source stride 1         -> k_gather_rows, 16-byte vectors when
//                                      every row start is 16-byte aligned;
//   * small inner stride (|s| <= 32) -> k_gather_small: each thread writes one
//                                      16-byte output vector from |s|-spaced
//                                      loads; a warp's loads cover whole
//                                      32-byte sectors, so DRAM reads are the
//                                      sector footprint and no more;
//   * large inner stride, another dim with a smaller one (a transpose)
//                                   -> k_gather_tiled: a 128 (small-stride
//                                      dim) x 32 (output dim) tile staged in
//                                      shared memory, read along the
//                                      small-stride dim and written along the
//                                      contiguous output dim;
//   * anything else                 -> k_gather_generic.
// Every path is a bit copy of the element, so results are bit-exact.
#include "qsml_internal.cuh"

namespace qsml {
namespace {

template <int ES> struct EType;
template <> struct EType<1> { using T = uint8_t; };
template <> struct EType<2> { using T = uint16_t; };
template <> struct EType<4> { using T = uint32_t; };
template <> struct EType<8> { using T = uint64_t; };

struct GPlan {
    int nd;
    int64_t shape[kMaxDims];
    int64_t st[kMaxDims];
};

// Source offset of the first element of collapsed row `row` (all dims but
// the innermost).
__device__ __forceinline__ int64_t g_row_offset(const GPlan& p, int64_t row) {
    int64_t off = 0;
    for (int d = p.nd - 2; d >= 1; --d) {
        int64_t c = row % p.shape[d];
        row /= p.shape[d];
        off += c * p.st[d];
    }
    if (p.nd >= 2) off += row * p.st[0];
    return off;
}

constexpr int kGT = 256;
constexpr int kGU = 4;

// Inner stride 1: copy rows, VEC = whole 16-byte packs.
template <typename T, bool VEC>
__global__ void __launch_bounds__(kGT) k_gather_rows(const T* __restrict__ src, T* __restrict__ dst, GPlan p,
                                                     int64_t items, int64_t per_row, int defer) {
    pdl_start(defer);
    const int64_t base = static_cast<int64_t>(blockIdx.x) * (kGT * kGU) + threadIdx.x;
    if (VEC) {
        constexpr int PV = 16 / sizeof(T);
        uint4 v[kGU];
        int64_t it[kGU];
#pragma unroll
        for (int u = 0; u < kGU; ++u) {
            it[u] = base + static_cast<int64_t>(u) * kGT;
            if (it[u] >= items) continue;
            int64_t row = it[u] / per_row, cv = it[u] - row * per_row;
            v[u] = *reinterpret_cast<const uint4*>(src + g_row_offset(p, row) + cv * PV);
        }
#pragma unroll
        for (int u = 0; u < kGU; ++u)
            if (it[u] < items) reinterpret_cast<uint4*>(dst)[it[u]] = v[u];
    } else {
        T v[kGU];
        int64_t it[kGU];
#pragma unroll
        for (int u = 0; u < kGU; ++u) {
            it[u] = base + static_cast<int64_t>(u) * kGT;
            if (it[u] >= items) continue;
            int64_t row = it[u] / per_row, c = it[u] - row * per_row;
            v[u] = src[g_row_offset(p, row) + c];
        }
#pragma unroll
        for (int u = 0; u < kGU; ++u)
            if (it[u] < items) dst[it[u]] = v[u];
    }
    pdl_end(defer);
}

// Small inner stride: G consecutive outputs per item from G loads spaced by
// the inner stride; one G-element store (16 bytes when G*sizeof(T) == 16).
template <typename T, int G>
__global__ void __launch_bounds__(kGT) k_gather_small(const T* __restrict__ src, T* __restrict__ dst, GPlan p,
                                                      int64_t items, int64_t per_row, int defer) {
    pdl_start(defer);
    struct alignas(G * sizeof(T)) Out { T v[G]; };
    const int64_t s = p.st[p.nd - 1];
    const int64_t base = static_cast<int64_t>(blockIdx.x) * (kGT * 2) + threadIdx.x;
    Out o[2];
    int64_t it[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        it[u] = base + static_cast<int64_t>(u) * kGT;
        if (it[u] >= items) continue;
        int64_t row = it[u] / per_row, cg = it[u] - row * per_row;
        const T* r = src + g_row_offset(p, row) + cg * G * s;
#pragma unroll
        for (int g = 0; g < G; ++g) o[u].v[g] = r[g * s];
    }
#pragma unroll
    for (int u = 0; u < 2; ++u)
        if (it[u] < items) reinterpret_cast<Out*>(dst)[it[u]] = o[u];
    pdl_end(defer);
}

// Transpose-like: tile over (P = small-stride dim, Q = innermost dim).  128
// along P: each of a tile's 32 source lines is read over 128 elements (2 KiB
// of X.T[::4, :]'s int32 rows), which measured 5 % faster on that gather than
// 64 x 64 tiles (32 x 32: 8 % slower).
constexpr int kTileP = 128, kTileQ = 32;
template <typename T>
__global__ void __launch_bounds__(256) k_gather_tiled(const T* __restrict__ src, T* __restrict__ dst, GPlan p,
                                                      int dP, int64_t ptiles, int64_t qtiles, int defer) {
    pdl_start(defer);
    __shared__ T tile[kTileQ][kTileP + 1];
    const int tx = threadIdx.x, ty = threadIdx.y;  // (32, 8)
    const int dQ = p.nd - 1;
    int64_t bid = blockIdx.x;
    const int64_t qt = bid % qtiles;
    bid /= qtiles;
    const int64_t pt = bid % ptiles;
    int64_t batch = bid / ptiles;
    // Batch dims: every dim except dP and dQ.  Output is contiguous, so the
    // output stride of each dim is the product of the extents after it.
    int64_t soff = 0, ooff = 0, ostride = 1;
    int64_t ostr[kMaxDims];
    for (int d = p.nd - 1; d >= 0; --d) {
        ostr[d] = ostride;
        ostride *= p.shape[d];
    }
    for (int d = p.nd - 1; d >= 0; --d) {
        if (d == dP || d == dQ) continue;
        int64_t c = batch % p.shape[d];
        batch /= p.shape[d];
        soff += c * p.st[d];
        ooff += c * ostr[d];
    }
    const int64_t P = p.shape[dP], Q = p.shape[dQ];
    const int64_t p0 = pt * kTileP, q0 = qt * kTileQ;
    const int64_t sP = p.st[dP], sQ = p.st[dQ];
    // Load: lanes walk P (the small source stride).
#pragma unroll
    for (int qi = ty; qi < kTileQ; qi += 8) {
#pragma unroll
        for (int ph = 0; ph < kTileP; ph += 32) {
            int pi = tx + ph;
            int64_t pp = p0 + pi, qq = q0 + qi;
            if (pp < P && qq < Q) tile[qi][pi] = src[soff + pp * sP + qq * sQ];
        }
    }
    __syncthreads();
    // Store: lanes walk Q (contiguous in the output).
    const int64_t oP = ostr[dP];
#pragma unroll
    for (int pi = ty; pi < kTileP; pi += 8) {
#pragma unroll
        for (int qh = 0; qh < kTileQ; qh += 32) {
            int qi = tx + qh;
            int64_t pp = p0 + pi, qq = q0 + qi;
            if (pp < P && qq < Q) dst[ooff + pp * oP + qq] = tile[qi][pi];
        }
    }
    pdl_end(defer);
}

template <typename T>
__global__ void __launch_bounds__(kGT) k_gather_generic(const T* __restrict__ src, T* __restrict__ dst, GPlan p,
                                                        int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kGT + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * kGT) {
        int64_t rem = i, off = 0;
        for (int d = p.nd - 1; d >= 0; --d) {
            int64_t c = rem % p.shape[d];
            rem /= p.shape[d];
            off += c * p.st[d];
        }
        dst[i] = src[off];
    }
}

// Strided destination (a slice of a larger tensor, e.g. concat/stack): both
// sides decomposed per element.
struct CopyPlan {
    int nd;
    int64_t shape[kMaxDims];
    int64_t ss[kMaxDims];  // source strides
    int64_t ds[kMaxDims];  // destination strides
};

template <typename T>
__global__ void __launch_bounds__(kGT) k_copy_strided(const T* __restrict__ src, T* __restrict__ dst, CopyPlan p,
                                                      int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kGT + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * kGT) {
        int64_t rem = i, so = 0, dof = 0;
        for (int d = p.nd - 1; d >= 0; --d) {
            int64_t c = rem % p.shape[d];
            rem /= p.shape[d];
            so += c * p.ss[d];
            dof += c * p.ds[d];
        }
        dst[dof] = src[so];
    }
}

template <int ES>
qsml_status_t copy_strided_typed(Context* ctx, const CopyPlan& p, const void* src, void* dst, int64_t n) {
    using T = typename EType<ES>::T;
    int64_t blocks = (n + kGT - 1) / kGT;
    int64_t cap = static_cast<int64_t>(ctx->num_sms) * 16;
    if (blocks > cap) blocks = cap;
    k_copy_strided<T><<<static_cast<unsigned>(blocks), kGT, 0, ctx->stream>>>(static_cast<const T*>(src),
                                                                                static_cast<T*>(dst), p, n);
    return after_launch(ctx, "k_copy_strided");
}

template <int ES>
qsml_status_t gather_typed(Context* ctx, const GPlan& p, const void* srcv, void* dstv, int64_t n,
                           const Footprint& fp) {
    using T = typename EType<ES>::T;
    const T* src = static_cast<const T*>(srcv);
    T* dst = static_cast<T*>(dstv);
    const int last = p.nd - 1;
    const int64_t C = p.shape[last];
    const int64_t s = p.st[last];
    constexpr int PV = 16 / ES;

    if (s == 1) {
        bool vec = aligned16(src) && aligned16(dst) && C % PV == 0;
        for (int d = 0; d < last && vec; ++d)
            if ((p.st[d] * ES) % 16 != 0) vec = false;
        if (vec) {
            int64_t per_row = C / PV, items = n / PV;
            int64_t blocks = (items + kGT * kGU - 1) / (kGT * kGU);
            {
                const int defer = plan_launch(ctx, fp);
                const cudaError_t e = launch_pdl(k_gather_rows<T, true>, dim3(static_cast<unsigned>(blocks)),
                                                 dim3(kGT), 0, ctx->stream, src, dst, p, items, per_row, defer);
                if (e != cudaSuccess) return check_cuda(ctx, e, "k_gather_rows");
            }
        } else {
            int64_t blocks = (n + kGT * kGU - 1) / (kGT * kGU);
            {
                const int defer = plan_launch(ctx, fp);
                const cudaError_t e = launch_pdl(k_gather_rows<T, false>, dim3(static_cast<unsigned>(blocks)),
                                                 dim3(kGT), 0, ctx->stream, src, dst, p, n, C, defer);
                if (e != cudaSuccess) return check_cuda(ctx, e, "k_gather_rows");
            }
        }
        return after_launch(ctx, "k_gather_rows");
    }

    // A transpose: the innermost output dim walks memory with a large stride
    // while some other dim walks it with a small one.
    int dP = -1;
    const int64_t as = s < 0 ? -s : s;
    for (int d = 0; d < last; ++d) {
        int64_t ad = p.st[d] < 0 ? -p.st[d] : p.st[d];
        if (p.shape[d] >= 8 && ad < as && (dP < 0 || ad < (p.st[dP] < 0 ? -p.st[dP] : p.st[dP]))) dP = d;
    }
    if (as > 32 && dP >= 0) {
        int64_t ptiles = (p.shape[dP] + kTileP - 1) / kTileP, qtiles = (C + kTileQ - 1) / kTileQ;
        int64_t batch = n / (p.shape[dP] * C);
        int64_t blocks = ptiles * qtiles * batch;
        if (blocks > INT32_MAX) return set_error(ctx, QSML_E_UNSUPPORTED, "gather too large");
        {
            const int defer = plan_launch(ctx, fp);
            const cudaError_t e = launch_pdl(k_gather_tiled<T>, dim3(static_cast<unsigned>(blocks)), dim3(32, 8), 0,
                                             ctx->stream, src, dst, p, dP, ptiles, qtiles, defer);
            if (e != cudaSuccess) return check_cuda(ctx, e, "k_gather_tiled");
        }
        return after_launch(ctx, "k_gather_tiled");
    }

    if (as <= 32 && C % PV == 0 && aligned16(dst)) {
        int64_t per_row = C / PV, items = n / PV;
        int64_t blocks = (items + kGT * 2 - 1) / (kGT * 2);
        {
            const int defer = plan_launch(ctx, fp);
            const cudaError_t e = launch_pdl(k_gather_small<T, PV>, dim3(static_cast<unsigned>(blocks)), dim3(kGT), 0,
                                             ctx->stream, src, dst, p, items, per_row, defer);
            if (e != cudaSuccess) return check_cuda(ctx, e, "k_gather_small");
        }
        return after_launch(ctx, "k_gather_small");
    }

    int64_t blocks = (n + kGT - 1) / kGT;
    int64_t cap = static_cast<int64_t>(ctx->num_sms) * 16;
    if (blocks > cap) blocks = cap;
    k_gather_generic<T><<<static_cast<unsigned>(blocks), kGT, 0, ctx->stream>>>(src, dst, p, n);
    return after_launch(ctx, "k_gather_generic");
}

}  // namespace
}  // namespace qsml

using namespace qsml;

extern "C" qsml_status_t qsml_gather(qsml_ctx* handle, const qsml_tdesc* src, const qsml_tdesc* out) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, src, "src"));
    QSML_TRY_STATUS(check_desc(C_, out, "out"));
    if (src->dtype != out->dtype) return set_error(C_, QSML_E_DTYPE, "qsml_gather: dtype mismatch");
    if (src->ndim != out->ndim) return set_error(C_, QSML_E_SHAPE, "qsml_gather: rank mismatch");
    for (int d = 0; d < src->ndim; ++d)
        if (src->shape[d] != out->shape[d]) return set_error(C_, QSML_E_SHAPE, "qsml_gather: shape mismatch");
    const int64_t n = numel(src);
    if (n == 0) return QSML_OK;
    const int es = dtype_size(src->dtype);
    if (!is_contiguous(out)) {
        // Strided destination: an element-wise copy between two views.
        CopyPlan cp;
        cp.nd = src->ndim;
        for (int d = 0; d < src->ndim; ++d) {
            cp.shape[d] = src->shape[d];
            cp.ss[d] = src->stride[d];
            cp.ds[d] = out->stride[d];
        }
        switch (es) {
            case 1: return copy_strided_typed<1>(C_, cp, src->data, out->data, n);
            case 2: return copy_strided_typed<2>(C_, cp, src->data, out->data, n);
            case 4: return copy_strided_typed<4>(C_, cp, src->data, out->data, n);
            case 8: return copy_strided_typed<8>(C_, cp, src->data, out->data, n);
        }
        return set_error(C_, QSML_E_DTYPE, "qsml_gather: unsupported element size");
    }

    GPlan p;
    int nd = 0;
    for (int d = 0; d < src->ndim; ++d) {
        if (src->shape[d] == 1) continue;
        if (nd > 0 && p.st[nd - 1] == src->stride[d] * src->shape[d]) {
            p.shape[nd - 1] *= src->shape[d];
            p.st[nd - 1] = src->stride[d];
            continue;
        }
        p.shape[nd] = src->shape[d];
        p.st[nd] = src->stride[d];
        ++nd;
    }
    if (nd == 0) {
        p.shape[0] = 1;
        p.st[0] = 1;
        nd = 1;
    }
    p.nd = nd;
    Footprint fp;  // what the launch reads and writes, for overlap
    fp.read(view_span(src)).write(span_of(out->data, static_cast<size_t>(n) * es));
    if (nd == 1 && p.st[0] == 1)
        return check_cuda(C_, cudaMemcpyAsync(out->data, src->data, static_cast<size_t>(n) * es,
                                              cudaMemcpyDeviceToDevice, C_->stream),
                          "qsml_gather copy");
    switch (es) {
        case 1: return gather_typed<1>(C_, p, src->data, out->data, n, fp);
        case 2: return gather_typed<2>(C_, p, src->data, out->data, n, fp);
        case 4: return gather_typed<4>(C_, p, src->data, out->data, n, fp);
        case 8: return gather_typed<8>(C_, p, src->data, out->data, n, fp);
    }
    return set_error(C_, QSML_E_DTYPE, "qsml_gather: unsupported element size");
}
