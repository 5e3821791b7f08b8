// linear.cu -- chooses the kernel for one packed linear.
#include "../../include/clq.h"
#include "clq_internal.h"

namespace clq {

cudaError_t launch_linear(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                          float* out, int64_t ldo, unsigned flags, cudaStream_t stream) {
    (void)flags;
    if (gemv_mma_supported(w, m)) return launch_gemv_mma(w, rows, x, xtype, m, out, ldo, stream);
    return launch_linear_generic(w, rows, x, xtype, m, out, ldo, stream);
}

}  // namespace clq
