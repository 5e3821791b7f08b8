// linear.cu -- chooses the kernel for one packed linear, and provides the
// scratch the prefill GEMM stages its activations in.
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/clq.h"
#include "clq_internal.h"
#include "formats.cuh"

namespace clq {
namespace {

// Activation rows from which the tensor-core GEMM replaces the GEMV
// (CLQ_GEMM_MIN_M, a tuning knob, sets one threshold for every case).  The
// GEMVs' cost grows with every row, the GEMM's (its weight conversion) does
// not.  Measured with fp32 activations and the exact GEMM: Q4_0 / Q8_0 from
// 17 rows (Llama-3.2-1B shapes at 32 rows: 4.46 ms on the register-fed GEMV
// against 2.78); Q4_K / Q6_K from 25, since the per-warp GEMV in passes of
// eight rows holds out longer (Llama-3-8B step at 24 rows: 9.5 against 12.7
// ms; even at 32).  16-bit activations keep the fp32-class GEMVs below 64
// rows: the fp16-operand GEMM misses the 1e-3 norm-relative gate there on
// N(0, 0.02) weights quantized to Q4_K (1.2e-3 at 24 rows).
int64_t gemm_min_m(const WeightView& w, bool exact) {
    static int64_t v = -2;
    if (v == -2) {
        const char* e = getenv("CLQ_GEMM_MIN_M");
        v = e ? atoll(e) : -1;
        if (e && v < 1) v = 1;
    }
    if (v > 0) return v;
    if (!exact) return 64;
    return w.dtype == kQ4_K || w.dtype == kQ6_K ? 25 : 17;
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
bool gemm_exact(int xtype, unsigned flags) {
    return (flags & CLQ_MATH_EXACT) || (xtype == CLQ_X_F32 && !(flags & CLQ_MATH_FAST));
}
bool uses_gemm_tc(const WeightView& w, int xtype, int64_t m, unsigned flags) {
    return m >= gemm_min_m(w, gemm_exact(xtype, flags)) && gemm_tc_supported(w, m);
}

cudaError_t launch_linear_group_gemm(const WeightView* const* w, const int64_t* rows, int count, const void* x,
                                     int xtype, int64_t m, float* const* out, const int64_t* ldo, unsigned flags,
                                     cudaStream_t stream) {
    if (count < 1 || count > 4 || !uses_gemm_tc(*w[0], xtype, m, flags)) return cudaErrorNotSupported;
    const bool exact = gemm_exact(xtype, flags);
    GemmPlan g[4];
    size_t scratch_bytes = 0;
    for (int i = 0; i < count; i++) {
        if (w[i]->dtype != w[0]->dtype || w[i]->k != w[0]->k || !uses_gemm_tc(*w[i], xtype, m, flags))
            return cudaErrorNotSupported;
        g[i] = plan_gemm_tc(w[i]->dtype, rows[i], w[i]->k, m, exact, exact && xtype == CLQ_X_F32);
        // one activation image for all: the same tokens per tile and image layout
        if (g[i].tn != g[0].tn || g[i].xs_bytes != g[0].xs_bytes || g[i].us_bytes != g[0].us_bytes ||
            g[i].xlo != g[0].xlo)
            return cudaErrorNotSupported;
        const size_t b = gemm_tc_scratch_bytes(g[i]);
        if (b > scratch_bytes) scratch_bytes = b;
    }
    cudaError_t e = keep_pool_memory();
    if (e != cudaSuccess) return e;
    void* scratch = nullptr;
    if ((e = cudaMallocAsync(&scratch, scratch_bytes, stream)) != cudaSuccess) return e;
    for (int i = 0; i < count && e == cudaSuccess; i++)
        e = launch_gemm_tc(*w[i], rows[i], x, xtype, m, out[i], ldo[i], (uint8_t*)scratch, g[i], stream, i > 0);
    const cudaError_t f = cudaFreeAsync(scratch, stream);
    return e != cudaSuccess ? e : f;
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
