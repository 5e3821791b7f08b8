// linear.cu -- chooses the kernel for one packed linear, and provides the
// scratch the prefill GEMM stages its activations in.
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/clq.h"
#include "clq_internal.h"

namespace clq {
namespace {

// Activation rows from which the tensor-core GEMM replaces the GEMV: past 16
// rows the GEMVs' cost grows with every row while the GEMM's (its weight
// conversion) does not (Llama-3.2-1B shapes, Q4_0 + Q4_K, fp32 activations:
// 4.46 ms on the GEMV against 2.78 on the exact GEMM at 32 rows; at 16 rows
// the GEMV is still ahead on Q4_0 / Q8_0, 2.44 against 2.73 ms).
int64_t gemm_min_m() {
    static int64_t v = -1;
    if (v < 0) {
        const char* e = getenv("CLQ_GEMM_MIN_M");  // tuning knob
        v = e ? atoll(e) : 17;
        if (v < 1) v = 1;
    }
    return v;
}

}  // namespace

// Scratch for one GEMM (or attention) call comes from the device's
// stream-ordered pool: it is allocated and released on the call's stream
// (graph memory nodes when the stream is being captured), so concurrent
// streams never share it.  The pool keeps released memory for reuse instead
// of returning it at each sync.
cudaError_t keep_pool_memory() {
    static std::mutex mu;
    static std::map<int, bool> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (done[dev]) return cudaSuccess;
    cudaMemPool_t pool;
    if ((e = cudaDeviceGetDefaultMemPool(&pool, dev)) != cudaSuccess) return e;
    uint64_t keep = UINT64_MAX;
    if ((e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep)) != cudaSuccess) return e;
    done[dev] = true;
    return cudaSuccess;
}

// Every request of at least CLQ_GEMM_MIN_M rows: fp32 activations without
// CLQ_MATH_FAST take the exact form (fp32-class products), 16-bit ones (or
// CLQ_MATH_FAST) the fp16-operand form unless CLQ_MATH_EXACT asks otherwise.
bool uses_gemm_tc(const WeightView& w, int xtype, int64_t m, unsigned flags) {
    (void)xtype;
    (void)flags;
    return m >= gemm_min_m() && gemm_tc_supported(w, m);
}
bool gemm_exact(int xtype, unsigned flags) {
    return (flags & CLQ_MATH_EXACT) || (xtype == CLQ_X_F32 && !(flags & CLQ_MATH_FAST));
}

cudaError_t launch_linear(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                          float* out, int64_t ldo, unsigned flags, cudaStream_t stream) {
    if (uses_gemm_tc(w, xtype, m, flags)) {
        const bool exact = gemm_exact(xtype, flags);
        const GemmPlan g = plan_gemm_tc(w.dtype, rows, w.k, m, exact, exact && xtype == CLQ_X_F32);
        cudaError_t e = keep_pool_memory();
        if (e != cudaSuccess) return e;
        void* scratch = nullptr;
        if ((e = cudaMallocAsync(&scratch, gemm_tc_scratch_bytes(g), stream)) != cudaSuccess) return e;
        e = launch_gemm_tc(w, rows, x, xtype, m, out, ldo, (uint8_t*)scratch, g, stream);
        cudaError_t f = cudaFreeAsync(scratch, stream);
        return e != cudaSuccess ? e : f;
    }
    if (gemv_mma_supported(w, m)) return launch_gemv_mma(w, rows, x, xtype, m, out, ldo, stream);
    return launch_linear_generic(w, rows, x, xtype, m, out, ldo, stream);
}

}  // namespace clq
