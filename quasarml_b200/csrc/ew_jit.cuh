// Runtime-compiled fused elementwise kernels (ew_jit.cu), used by
// qsml_elementwise_fused when the collapsed layout is at most 2-D and every
// input is either contiguous along the inner dim or broadcast along it.
#pragma once

#include "qsml_internal.cuh"

namespace qsml {

struct JitInput {
    const void* ptr;
    int64_t row_stride;  // elements between consecutive collapsed rows (0 = broadcast rows)
    bool vec;            // inner stride 1 (vector loads); false: inner stride 0 (one value per row)
};

// Runs the expression (already validated) with a kernel compiled for exactly
// this expression, dtype and input layout classes; the compiled kernel is
// cached per device.  items = output elements / V (V = 16 bytes / element
// size), cpr = vectors per collapsed row.  *ran = false (with QSML_OK) when no
// runtime compiler is available or compilation failed: the caller then uses
// the precompiled interpreter kernel.
qsml_status_t fused_jit(Context* ctx, const qsml_fuse_node* nodes, int n_nodes, const JitInput* ins, int nin,
                        bool half, void* out, int64_t items, int64_t cpr, bool* ran);

// Kernels compiled so far in this process (all devices).
uint64_t fused_jit_kernels();

}  // namespace qsml
