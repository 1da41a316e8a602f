// Tensor-core fp16 matmul (tcgen05 / TMEM / TMA) -- placeholder until the
// kernel lands: every shape is reported as outside the kernel's range.
#include "matmul.cuh"

namespace qsml {
qsml_status_t matmul_tc_f16(Context*, const MatmulArgs&, bool) { return QSML_E_UNSUPPORTED; }
}  // namespace qsml
