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

// Activation rows from which the tensor-core GEMM replaces the GEMV when the
// activations are 16-bit or the caller accepts fp16 rounding (CLQ_MATH_FAST).
int64_t gemm_min_m() {
    static int64_t v = -1;
    if (v < 0) {
        const char* e = getenv("CLQ_GEMM_MIN_M");  // tuning knob
        v = e ? atoll(e) : 64;
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

bool uses_gemm_tc(const WeightView& w, int xtype, int64_t m, unsigned flags) {
    const bool sixteen_bit = xtype != CLQ_X_F32 || (flags & CLQ_MATH_FAST);
    return sixteen_bit && m >= gemm_min_m() && gemm_tc_supported(w, m);
}

cudaError_t launch_linear(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                          float* out, int64_t ldo, unsigned flags, cudaStream_t stream) {
    if (uses_gemm_tc(w, xtype, m, flags)) {
        const GemmPlan g = plan_gemm_tc(w.dtype, rows, w.k, m);
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
