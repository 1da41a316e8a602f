/*
 * qsml_cuda.h -- extern "C" ABI of the B200 (sm_100a) backend for QuasarML.
 *
 * libqsml_cuda.so replaces QuasarML's Vulkan backend (the abstract Backend of
 * QuasarML/src/Backend/BackendInterface.h:43-85 with its VulkanBackend
 * implementation) together with the per-op GLSL generation of
 * the op files under QuasarML/src/Ops.  The C++ QuasarML layer (Tensor, Device, Ops::*,
 * qsml::) calls these entry points; any other host language can bind them
 * directly (plain pointers, sizes and POD descriptors, no C++ types).
 *
 * Conventions
 *  - Every entry point returns a qsml_status_t and never throws or aborts.
 *    On failure qsml_last_error(ctx) gives a message; the C++ layer turns it
 *    into std::runtime_error, the reference's error convention
 *    (QuasarML/src/Common/Assert.h:8-13).
 *  - Work is enqueued on the context's CUDA stream and is asynchronous with
 *    respect to the host until qsml_synchronize() or a device->host copy,
 *    as in the reference (QuasarML/src/Core/Device.cpp:96-102).
 *  - Tensors are described by qsml_tdesc: `data` points at the view's first
 *    element (storage offset already applied), shape/stride are in elements,
 *    strides may be 0 (broadcast) or negative on inputs.  Outputs must be
 *    contiguous row-major and must not partially overlap an input.
 *  - Outputs are caller-allocated (the reference's Ops allocate the result
 *    tensor first, e.g. QuasarML/src/Ops/Elementwise.cpp:143).
 *  - There is no CPU fallback: an unsupported case returns an error status.
 */
#ifndef QSML_CUDA_H
#define QSML_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define QSML_API __declspec(dllexport)
#else
#define QSML_API __attribute__((visibility("default")))
#endif

typedef int32_t qsml_status_t;

#define QSML_OK 0
#define QSML_E_INVALID 1     /* bad argument (null pointer, bad enum)         */
#define QSML_E_SHAPE 2       /* incompatible shapes / axis out of range       */
#define QSML_E_DTYPE 3       /* dtype not supported by this op                */
#define QSML_E_OOM 4         /* device allocation failed                      */
#define QSML_E_CUDA 5        /* CUDA runtime error                            */
#define QSML_E_NCCL 6        /* collective error                              */
#define QSML_E_TIMEOUT 7     /* bounded device-side wait expired              */
#define QSML_E_UNSUPPORTED 8 /* valid request the library does not implement */

/* Element types, same order and sizes as QuasarML::DataType
 * (QuasarML/src/Common/Types.h:80-103). */
#define QSML_F32 0
#define QSML_F16 1
#define QSML_I32 2
#define QSML_I16 3
#define QSML_I8 4
#define QSML_U32 5
#define QSML_U16 6
#define QSML_U8 7

#define QSML_MAX_DIMS 8

typedef struct qsml_tdesc {
    void* data;                      /* device pointer to element [0,...,0]   */
    int32_t dtype;                   /* QSML_F32 ...                          */
    int32_t ndim;                    /* 0..QSML_MAX_DIMS (0 = scalar)         */
    int64_t shape[QSML_MAX_DIMS];
    int64_t stride[QSML_MAX_DIMS];   /* in elements                           */
} qsml_tdesc;

typedef struct qsml_ctx qsml_ctx;

/* Binary element ops (qsml_binary, qsml_binary_scalar). */
#define QSML_OP_ADD 0
#define QSML_OP_SUB 1
#define QSML_OP_MUL 2
#define QSML_OP_DIV 3
#define QSML_OP_POW 4

/* Unary element ops (qsml_unary). */
#define QSML_UN_RELU 0
#define QSML_UN_NEG 1
#define QSML_UN_ABS 2
#define QSML_UN_SQRT 3
#define QSML_UN_EXP 4
#define QSML_UN_LOG 5
#define QSML_UN_SIN 6
#define QSML_UN_COS 7
#define QSML_UN_TANH 8
#define QSML_UN_SIGMOID 9
#define QSML_UN_GELU 10

/* Reductions (qsml_reduce). */
#define QSML_RED_SUM 0
#define QSML_RED_MEAN 1
#define QSML_RED_MAX 2
#define QSML_RED_MIN 3
#define QSML_RED_PROD 4
#define QSML_AXIS_ALL (-1000)

/* arg-reduction ops (qsml_arg_reduce) */
#define QSML_ARG_MAX 0
#define QSML_ARG_MIN 1

/* Matmul precisions (qsml_matmul). */
#define QSML_MM_AUTO 0          /* F32 inputs -> FP32_FFMA, F16 -> FP16_F32ACC */
#define QSML_MM_FP32_FFMA 1     /* fp32 CUDA-core fma, k ascending             */
#define QSML_MM_FP32_3XTF32 2   /* fp32 via three tf32 tensor-core products    */
#define QSML_MM_FP16_F32ACC 3   /* fp16 inputs, fp32 accumulate (tcgen05)      */

/* ---- device / context ------------------------------------------------- */

/* Number of CUDA devices.  Replaces DeviceManager::enumerate
 * (QuasarML/src/Core/DeviceManager.cpp:20-50). */
QSML_API qsml_status_t qsml_device_count(int32_t* count);

/* Device name into buf (NUL-terminated).  Replaces
 * DeviceManager::device_names (QuasarML/src/Core/DeviceManager.cpp:68-106). */
QSML_API qsml_status_t qsml_device_name(int32_t device, char* buf, size_t len);

/* Creates a context on `device`: a CUDA stream, a caching allocator and the
 * op scratch space.  Replaces Device::Device -> create_vulkan_backend ->
 * VulkanBackend::init (QuasarML/src/Core/Device.cpp:9-17,
 * QuasarML/src/Backend/Vulkan/VulkanBackend.cpp:82-180). */
QSML_API qsml_status_t qsml_init(int32_t device, qsml_ctx** ctx);

/* Releases the context, its cached blocks and its stream.  Replaces
 * Device::~Device (QuasarML/src/Core/Device.cpp:19-23). */
QSML_API qsml_status_t qsml_destroy(qsml_ctx* ctx);

/* Makes the context enqueue on `stream`, a cudaStream_t used as given: NULL
 * is the CUDA legacy default stream (stream 0).  The context's own stream
 * is what qsml_get_stream returns on a fresh context.  Pending work on the
 * previous stream is waited for first, so cached blocks stay
 * stream-ordered.  No reference counterpart (the reference owns one Vulkan
 * queue per device). */
QSML_API qsml_status_t qsml_set_stream(qsml_ctx* ctx, void* stream);
QSML_API qsml_status_t qsml_get_stream(qsml_ctx* ctx, void** stream);

/* Blocks until all work enqueued on the context has finished, then reports
 * QSML_E_TIMEOUT (and clears it) if a kernel gave up a bounded device-side
 * wait since the previous call.  Replaces Device::synchronize /
 * flush_pending (QuasarML/src/Core/Device.cpp:96-102,
 * QuasarML/src/Backend/Vulkan/VulkanBackend.cpp:613-658). */
QSML_API qsml_status_t qsml_synchronize(qsml_ctx* ctx);

/* Limit, in SM clock cycles, after which a kernel that waits for data on an
 * mbarrier (the one-SM tensor-core GEMM, the layer-norm and softmax row
 * pipelines) gives up: it stops, lets every copy and MMA it already issued
 * finish, records QSML_E_TIMEOUT for the next qsml_synchronize and returns,
 * so the context stays usable.  0 restores the default (2e9 cycles, about
 * 1 s).  Stream-ordered: applies to kernels enqueued after the call.  Meant
 * for failure-detection tests and watchdogs; a limit below a kernel's
 * normal wait times makes it give up on healthy work.  No reference
 * counterpart (its fence waits are unbounded,
 * QuasarML/src/Backend/Vulkan/VulkanBackend.cpp:613-658). */
QSML_API qsml_status_t qsml_set_wait_limit(qsml_ctx* ctx, int64_t cycles);

/* Overlap of independent calls on the context's stream (off by default).
 * With enable = 1, a memory-bound call (qsml_reduce, qsml_arg_reduce,
 * qsml_layer_norm, qsml_softmax, qsml_gather, qsml_binary, qsml_unary,
 * qsml_binary_scalar on vectorisable layouts, and qsml_elementwise_fused
 * when it runs a runtime-compiled kernel) whose inputs, outputs and
 * scratch share no byte with the library kernels that may still be running
 * on the stream starts reading at once instead of waiting for them to
 * finish; it waits for them only at its end, so kernels still complete in
 * stream order and every other call sees the same results as without
 * overlap.  A call that reads what such a kernel writes (or writes what it
 * reads or writes) waits at its start as usual.  The library tracks its own kernels
 * only: enable this when nothing else on the stream launches kernels that
 * trigger programmatic dependent launch early (plain kernel launches,
 * copies, memsets and events are fine).  Measured on B200: binary16 column
 * reductions of 64 MiB 13.2 -> 10.5 us per launch.  No reference counterpart
 * (its dispatches each end with a fence wait, VulkanBackend.cpp:613-658). */
QSML_API qsml_status_t qsml_set_overlap(qsml_ctx* ctx, int32_t enable);
/* Launches planned for overlap on this context so far, and how many of them
 * overlapped the kernels before them (either pointer may be NULL). */
QSML_API qsml_status_t qsml_overlap_stats(qsml_ctx* ctx, uint64_t* planned, uint64_t* deferred);

/* Message of the last failed call on ctx (or of the last failed
 * context-free call when ctx is NULL).  Never NULL. */
QSML_API const char* qsml_last_error(qsml_ctx* ctx);

/* ---- memory ------------------------------------------------------------ */

/* Device allocation from the context's caching allocator (256-byte aligned,
 * size-binned, reused in stream order).  Replaces
 * Backend::create_storage_buffer / destroy_buffer
 * (QuasarML/src/Backend/Vulkan/VulkanBackend.cpp:254-325). */
QSML_API qsml_status_t qsml_alloc(qsml_ctx* ctx, size_t bytes, void** ptr);
QSML_API qsml_status_t qsml_free(qsml_ctx* ctx, void* ptr);
/* Returns every cached, unused block to the driver. */
QSML_API qsml_status_t qsml_empty_cache(qsml_ctx* ctx);

/* Host<->device copies on the context stream.  qsml_h2d is asynchronous for
 * pinned host memory; from pageable memory it returns once the source may be
 * reused (copies of 8 MiB and more are staged through the context's pinned
 * buffers by several host threads, the DMAs stay ordered on the stream).
 * qsml_d2h waits for the data before returning (pageable destinations of
 * 8 MiB and more are staged the same way).  Replace Backend::upload_buffer /
 * download_buffer / copy_buffer
 * (QuasarML/src/Backend/Vulkan/VulkanBackend.cpp:327-373). */
QSML_API qsml_status_t qsml_h2d(qsml_ctx* ctx, void* dst, const void* src, size_t bytes);
QSML_API qsml_status_t qsml_d2h(qsml_ctx* ctx, void* dst, const void* src, size_t bytes);
QSML_API qsml_status_t qsml_d2h_async(qsml_ctx* ctx, void* dst, const void* src, size_t bytes);
QSML_API qsml_status_t qsml_d2d(qsml_ctx* ctx, void* dst, const void* src, size_t bytes);

/* Page-locked host memory for fast, asynchronous transfers. */
QSML_API qsml_status_t qsml_host_alloc(size_t bytes, void** ptr);
QSML_API qsml_status_t qsml_host_free(void* ptr);

/* Fills `count` elements of `elem_size` bytes (1, 2, 4 or 8) with the
 * pattern at `value`.  Replaces Tensor::fill / Tensor::zero, which upload a
 * host-built buffer (QuasarML/src/Core/Tensor.cpp:100-112). */
QSML_API qsml_status_t qsml_fill(qsml_ctx* ctx, void* dst, const void* value,
                                 int32_t elem_size, int64_t count);

/* ---- ops --------------------------------------------------------------- */

/* out = a (op) b with NumPy broadcasting; out.shape must equal the
 * broadcast shape.  F32, F16 (computed in fp32, rounded once) and I32
 * (add/sub/mul/div).  Add/sub/mul/div are IEEE-correctly rounded with no FMA
 * contraction; POW uses x*x for exponent 2 and a binary64 pow rounded once
 * otherwise.  Replaces Ops::add/subtract/multiply/divide
 * (QuasarML/src/Ops/Elementwise.cpp:139-205, shader
 * QuasarML/src/Ops/ShaderGen.cpp:40-53), which require equal shapes. */
QSML_API qsml_status_t qsml_binary(qsml_ctx* ctx, int32_t op, const qsml_tdesc* a,
                                   const qsml_tdesc* b, const qsml_tdesc* out);

/* out = a (op) s.  Replaces Ops::add_scalar / multiply_scalar
 * (QuasarML/src/Ops/Elementwise.cpp:207-241, shader :39-51); SUB, DIV and
 * POW (scalar exponent, the new qsml::pow(x, f32)) use the same kernel. */
QSML_API qsml_status_t qsml_binary_scalar(qsml_ctx* ctx, int32_t op, const qsml_tdesc* a,
                                          float s, const qsml_tdesc* out);

/* out = f(a).  Replaces Ops::relu (QuasarML/src/Ops/Elementwise.cpp:347-361,
 * shader :53-66) and neg/abs/sqrt/exp/log/sin/cos/tanh/sigmoid/gelu
 * (QuasarML/src/Ops/Elementwise.cpp:243-345,363-395).  relu(NaN) = NaN,
 * relu(-0) = +0. */
QSML_API qsml_status_t qsml_unary(qsml_ctx* ctx, int32_t op, const qsml_tdesc* a,
                                  const qsml_tdesc* out);

/* Sum / mean / max / min / prod over one axis (negative counts from the end) or
 * over all elements (axis = QSML_AXIS_ALL).  out has the reduced shape
 * (keepdims keeps the axis as 1; the full reduction gives shape [1]) and the
 * input's dtype; F16 input accumulates in fp32.  mean = sum * (1.0f/(float)n).
 * max/min follow IEEE 754-2019 maximum/minimum (NaN propagates as 0x7fffffff,
 * -0 < +0).  The combine order is fixed by the shape alone, so results are
 * run-to-run deterministic.  `a` may be a strided view (slices with a step,
 * transposes, negative or zero strides): it is read in place, with the
 * dims other than the reduced one merged where their strides chain; a view
 * that leaves more than four such dims returns QSML_E_UNSUPPORTED (gather it
 * with qsml_gather first).  Replaces Ops::sum/mean/max/min
 * (QuasarML/src/Ops/Reduction.cpp:285-382), whose axis max/min are stubs. */
QSML_API qsml_status_t qsml_reduce(qsml_ctx* ctx, int32_t op, const qsml_tdesc* a,
                                   int32_t axis, int32_t keepdims, const qsml_tdesc* out);

/* Index of the largest (QSML_ARG_MAX) or smallest (QSML_ARG_MIN) element
 * over one axis (negative counts from the end) or over all elements (axis =
 * QSML_AXIS_ALL, an index into the flattened tensor).  Any input dtype,
 * contiguous; out is I32 or U32 with the reduced shape (keepdims as in
 * qsml_reduce).  Ties give the first index; values compare numerically
 * (-0 == +0) and a NaN counts as beyond every number, so the first NaN wins
 * (NumPy's argmax/argmin).  The reduced axis must be non-empty and shorter
 * than 2^31 (I32 out) or 2^32 - 1 (U32 out).  Replaces Ops::argmax/argmin
 * (QuasarML/src/Ops/Reduction.cpp:388-396), stubs there that ignore the axis
 * and return the max/min value. */
QSML_API qsml_status_t qsml_arg_reduce(qsml_ctx* ctx, int32_t op, const qsml_tdesc* a,
                                       int32_t axis, int32_t keepdims, const qsml_tdesc* out);

/* Fused elementwise expression: out = the value of the last node, computed
 * per element in one kernel that reads every input once and writes only out.
 * Nodes form a DAG in topological order (operands are earlier nodes):
 *   QSML_FUSE_INPUT   inputs[code]
 *   QSML_FUSE_CONST   the binary32 `value`
 *   QSML_FUSE_BINARY  QSML_OP_<code>(node a, node b)
 *   QSML_FUSE_UNARY   QSML_UN_<code>(node a)
 * Inputs broadcast to out's shape (NumPy rules; out must be exactly their
 * broadcast shape) and share out's dtype, F32 or F16.  Every node computes
 * what qsml_binary / qsml_unary computes for that element and rounds to the
 * dtype, and a CONST operand acts like qsml_binary_scalar's `s` (used as
 * binary32), so the result is bit-identical to the unfused sequence of calls.
 * At most QSML_FUSE_MAX_NODES nodes and QSML_FUSE_MAX_INPUTS inputs; very
 * deep or heavily shared expressions may exceed the kernel's program limits
 * (48 instructions after expanding shared nodes, 16 distinct constants, 3
 * temporaries) and return QSML_E_UNSUPPORTED.  The reference has no fusion
 * (README.md:78 lists it as not done): each of its ops is a dispatch that
 * writes a full intermediate (QuasarML/src/Ops/Elementwise.cpp:139-417). */
#define QSML_FUSE_INPUT 0
#define QSML_FUSE_CONST 1
#define QSML_FUSE_BINARY 2
#define QSML_FUSE_UNARY 3
#define QSML_FUSE_MAX_NODES 64
#define QSML_FUSE_MAX_INPUTS 6

typedef struct {
    int32_t kind;   /* QSML_FUSE_*                                   */
    int32_t code;   /* input index, QSML_OP_* or QSML_UN_*            */
    int32_t a, b;   /* operand node indices (b: binary nodes only)    */
    float value;    /* QSML_FUSE_CONST                                */
} qsml_fuse_node;

QSML_API qsml_status_t qsml_elementwise_fused(qsml_ctx* ctx, const qsml_fuse_node* nodes, int32_t n_nodes,
                                              const qsml_tdesc* inputs, int32_t n_inputs,
                                              const qsml_tdesc* out);

/* Which kernel runs a fused expression.  AUTO (the default): a kernel
 * generated for the expression and compiled at run time with NVRTC (first
 * use of each expression / dtype / layout class; cached per device) when the
 * collapsed layout is at most 2-D with every input contiguous or broadcast
 * along the inner dim, else the precompiled interpreter kernel.  INTERP:
 * always the interpreter.  JIT: the compiled kernel or QSML_E_UNSUPPORTED.
 * All paths give bit-identical results.  The reference compiles a generated
 * shader per op at run time (QuasarML/src/Ops/ShaderGen.cpp,
 * Backend/Vulkan/VulkanBackend.cpp:44-80). */
#define QSML_FUSE_MODE_AUTO 0
#define QSML_FUSE_MODE_INTERP 1
#define QSML_FUSE_MODE_JIT 2
QSML_API qsml_status_t qsml_set_fuse_mode(qsml_ctx* ctx, int32_t mode);

/* Fused launches on this context by kernel kind, and the number of
 * expression kernels compiled so far in the process. */
QSML_API qsml_status_t qsml_fuse_stats(qsml_ctx* ctx, uint64_t* jit_launches, uint64_t* interp_launches,
                                       uint64_t* jit_kernels);

/* Materialises a strided view (any strides, including 0 and negative) into
 * `out` of the same shape and dtype, bit-exactly.  `out` is normally
 * contiguous (the fast paths); a strided `out` (a slice of a larger tensor,
 * as concat/stack/broadcast_to need) is also accepted and must not overlap
 * itself or `src`.  Replaces
 * Ops::copy (QuasarML/src/Ops/Manipulation.cpp:171-184), Ops::slice's host
 * round trip (QuasarML/src/Ops/Manipulation.cpp:146-161) and the
 * materialising transpose (QuasarML/src/Ops/LinAlg.cpp:329-351). */
QSML_API qsml_status_t qsml_gather(qsml_ctx* ctx, const qsml_tdesc* src, const qsml_tdesc* out);

/* out = src converted to out's dtype, elementwise: F32 -> F16 rounds to
 * nearest even (values beyond the binary16 range become +-inf), F16 -> F32
 * is exact, equal dtypes copy.  src and out contiguous, same shape.  No
 * reference counterpart (the reference's tensors keep their creation dtype;
 * an fp16 copy of data is built and uploaded from the host). */
QSML_API qsml_status_t qsml_cast(qsml_ctx* ctx, const qsml_tdesc* src, const qsml_tdesc* out);

/* y = exp(x - max) / sum(exp(x - max)) over one axis (negative counts from
 * the end); x and y F32 or F16 with the same contiguous shape, binary32
 * arithmetic (max, subtract, expf, sum, then multiply by the correctly
 * rounded reciprocal of the sum).  A NaN in a
 * slice makes that slice NaN.  Replaces Ops::softmax
 * (QuasarML/src/Ops/Elementwise.cpp:395-417, shader :98-135), whose indexing
 * is right for the last axis only. */
QSML_API qsml_status_t qsml_softmax(qsml_ctx* ctx, const qsml_tdesc* x, int32_t axis, const qsml_tdesc* y);

/* y = (x - mean) / sqrt(var + eps) * gamma + beta over the last dim (biased
 * variance).  x/y F32 or F16; gamma/beta F32 or the dtype of x, shape
 * [last dim].  No reference counterpart (layer norm is absent from the
 * reference snapshot). */
QSML_API qsml_status_t qsml_layer_norm(qsml_ctx* ctx, const qsml_tdesc* x, const qsml_tdesc* gamma,
                                       const qsml_tdesc* beta, float eps, const qsml_tdesc* y);

/* C = A * B for rank-2 A[M,K], B[K,N] -> C[M,N], or batched rank-3
 * A[b,M,K], B[b,K,N] -> C[b,M,N] (batch strides may be 0).  A and B must have
 * unit stride in their last dim.  F32 inputs give F32 C; F16 inputs give
 * F32 (or F16) C with fp32 accumulation.  Replaces Ops::matmul and
 * Ops::batch_matmul (QuasarML/src/Ops/LinAlg.cpp:221-290; the reference's
 * batched version is broken). */
QSML_API qsml_status_t qsml_matmul(qsml_ctx* ctx, const qsml_tdesc* a, const qsml_tdesc* b,
                                   const qsml_tdesc* c, int32_t precision);

/* ---- Multi-GPU groups (NCCL) ------------------------------------------------
 * The reference is single-GPU; sharded execution combines per-GPU partial
 * results with an in-place all-reduce.  Two ways to form a group:
 *   one process per GPU   -- one rank calls qsml_group_unique_id, the host
 *                            shares the bytes, every rank calls
 *                            qsml_group_init_rank with its context;
 *   one process, n GPUs   -- qsml_group_init_all over n contexts (rank i =
 *                            ctxs[i]); collectives for several of them from
 *                            one thread go between qsml_group_start and
 *                            qsml_group_end.
 * Collectives run on the rank's context stream, in order with its kernels.
 * Every wait on NCCL is bounded by QSML_NCCL_TIMEOUT_MS (default 60000): a
 * rank that never joins, or a collective that makes no progress, returns
 * QSML_E_TIMEOUT; qsml_group_destroy then aborts the communicators. */
#define QSML_UNIQUE_ID_BYTES 128
typedef struct qsml_group qsml_group;

QSML_API qsml_status_t qsml_group_unique_id(uint8_t* id /* QSML_UNIQUE_ID_BYTES */);
QSML_API qsml_status_t qsml_group_init_rank(qsml_ctx* ctx, const uint8_t* id, int32_t nranks, int32_t rank,
                                            qsml_group** group);
QSML_API qsml_status_t qsml_group_init_all(qsml_ctx* const* ctxs, int32_t n, qsml_group** group);
QSML_API qsml_status_t qsml_group_size(qsml_group* group, int32_t* nranks, int32_t* local_ranks);
QSML_API qsml_status_t qsml_group_start(void);
QSML_API qsml_status_t qsml_group_end(void);
/* In-place all-reduce of `count` elements at buf (device memory of local rank
 * `local`'s context; 0 for init_rank groups): op QSML_RED_SUM, MEAN (the sum
 * divided by the number of ranks), MAX, MIN or PROD; dtype F32, F16, I32,
 * U32, I8 or U8. */
QSML_API qsml_status_t qsml_allreduce(qsml_group* group, int32_t local, void* buf, int64_t count, int32_t dtype,
                                      int32_t op);
QSML_API qsml_status_t qsml_group_destroy(qsml_group* group);

/* ---- Sharded reductions -----------------------------------------------------
 * A tensor split by rows (axis 0) over the ranks of a group, each rank holding
 * its own row block (blocks may differ in length; the other dims agree).  A
 * reduction over any other axis needs no exchange: qsml_reduce of the block is
 * the rank's row block of the global result.  A reduction over axis 0 or over
 * all elements combines one partial per rank:
 *   1. qsml_reduce with a binary32 `out` (F16 input is fine) gives the rank's
 *      partial: SUM for sum and mean, MAX / MIN for max / min;
 *   2. qsml_allreduce_partials combines the partials of all ranks in place,
 *      several reductions' partials at once if the caller packs them into one
 *      buffer;
 *   3. qsml_finish_partial writes the result in out's dtype; a mean is the
 *      combined sum * (1.0f / (float)n), n = the elements reduced into each
 *      output over all ranks, the reference's definition of mean
 *      (QuasarML/src/Ops/Reduction.cpp:347-356).
 * qsml_reduce_sharded does all three for one reduction.  Sums combine in
 * binary32 (binary16 inputs are never summed in binary16); max / min cross
 * the group as order-preserving 32-bit keys, so NaN propagation (as
 * 0x7fffffff) and -0 < +0 are exactly those of qsml_reduce on one GPU.  The
 * reference has no multi-GPU path (README.md:84, Core/DeviceManager.cpp:52-66
 * open independent devices); these replace nothing there. */

/* In place over `count` binary32 partials at buf (device memory of local
 * rank `local`'s context), on that context's stream: op SUM or MEAN adds,
 * MAX / MIN take the IEEE 754-2019 maximum / minimum.  One process driving
 * several GPUs from one thread brackets its ranks' calls with
 * qsml_group_start / qsml_group_end (the combine, and for max / min the
 * decoding of the keys after it, then complete in stream order once
 * qsml_group_end returns). */
QSML_API qsml_status_t qsml_allreduce_partials(qsml_group* group, int32_t local, int32_t op, void* buf,
                                               int64_t count);

/* out (F32 or F16, as many elements as `partial`, F32) from combined
 * partials: SUM / MAX / MIN as they are, MEAN times 1.0f / (float)n; rounded
 * once to out's dtype.  out may be `partial` itself. */
QSML_API qsml_status_t qsml_finish_partial(qsml_ctx* ctx, int32_t op, const qsml_tdesc* partial, int64_t n,
                                           const qsml_tdesc* out);

/* One sharded reduction (sum, mean, max or min) of this rank's row block `a`
 * with qsml_reduce's axis / keepdims / out rules; out is identical on every
 * rank for axis 0 and QSML_AXIS_ALL.  global_rows = the rows of all ranks
 * together (0: this rank's rows times the number of ranks).  A rank without
 * rows contributes 0 to sums and the identity (-inf / +inf) to max / min.
 * Not inside qsml_group_start / qsml_group_end (it finishes right after its
 * combine): one process driving several GPUs from one thread uses the three
 * steps above, with the combines bracketed. */
QSML_API qsml_status_t qsml_reduce_sharded(qsml_group* group, int32_t local, int32_t op, const qsml_tdesc* a,
                                           int32_t axis, int32_t keepdims, const qsml_tdesc* out,
                                           int64_t global_rows);

/* Rows [*begin, *begin + *count) of `rows` that rank `rank` of `nranks` holds
 * under the balanced contiguous split every sharded workload here uses (the
 * first rows % nranks ranks hold one row more). */
QSML_API qsml_status_t qsml_shard_rows(int64_t rows, int32_t nranks, int32_t rank, int64_t* begin, int64_t* count);

/* Allocation-free sum / mean / max / min over all elements (axis =
 * QSML_AXIS_ALL) or over an axis followed only by unit dims, for callers that
 * cannot allocate device memory at that point: latency-critical paths that
 * must not block in the driver's allocator (cudaMalloc and cudaFree can
 * synchronise the device), hosts whose own allocator already owns all of
 * HBM, and plugins handed only a stream.  It needs no qsml_ctx:
 * it enqueues on `stream` (a cudaStream_t of the current device; NULL = the
 * legacy default stream) and never calls cudaMalloc, cudaFree or any
 * allocating routine.  It runs qsml_reduce's segment kernel with the same
 * slicing, so its results are bit-identical to qsml_reduce's wherever
 * qsml_reduce picks that kernel too: the full reduction, a single row, or
 * fewer than 592 rows of at least 8192 elements each.  For other shapes
 * (many short rows, where qsml_reduce uses a warp per row) the two agree
 * within the reductions' rounding tolerance but not bit for bit.  An empty
 * reduced axis is rejected with QSML_E_SHAPE (qsml_reduce instead writes 0
 * for sum and NaN for mean).
 *
 * Its scratch is a fixed 64 KiB device array inside this library, which every
 * GPU that loads the library holds until the process exits; it limits a call
 * to at most 64 output rows (larger requests return QSML_E_UNSUPPORTED with a
 * message).  The first call in each CUDA context looks up that array's
 * device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture; after a device reset the next call looks it up again.
 * All calls share the array and clear its counters before each launch:
 * calls on the same GPU whose work overlaps race on it.  Errors are reported
 * through qsml_last_error(NULL).  No counterpart in the reference. */
QSML_API qsml_status_t qsml_reduce_noalloc(void* stream, int32_t op, const qsml_tdesc* a, int32_t axis,
                                           int32_t keepdims, const qsml_tdesc* out);

/* ---- counters ---------------------------------------------------------- */

/* Kernels this context has launched since qsml_init. */
QSML_API qsml_status_t qsml_launch_count(qsml_ctx* ctx, uint64_t* count);
/* Name of the last kernel this context launched ("" before the first), at
 * most len-1 characters and a terminating NUL into buf: which of an op's
 * kernels the shape selected (e.g. "k_reduce_cols_wide", "k_gemm_tc2<f16>"). */
QSML_API qsml_status_t qsml_last_kernel(qsml_ctx* ctx, char* buf, size_t len);
/* Ops that ran on the CPU instead of the GPU: always 0 (there is no CPU
 * path).  Backs qsml::cpu_fallback_count(). */
QSML_API qsml_status_t qsml_cpu_fallback_count(qsml_ctx* ctx, uint64_t* count);
/* Caching-allocator statistics: cudaMalloc calls (misses), cache hits,
 * bytes currently held from the driver, bytes currently handed out. */
QSML_API qsml_status_t qsml_allocator_stats(qsml_ctx* ctx, uint64_t* misses, uint64_t* hits,
                                            uint64_t* reserved_bytes, uint64_t* live_bytes);

#ifdef __cplusplus
}
#endif
#endif
