// linear.cu -- chooses the kernel for one packed linear, and owns the
// per-stream scratch the prefill GEMM stages its activations in.
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

// Grow-only device scratch per (device, stream).  Calls on one stream are
// ordered, so they can share it; growing frees the old buffer (cudaFree waits
// for the device), which cannot happen while a graph is being captured.
std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> g_scratch;

cudaError_t scratch_for(cudaStream_t stream, size_t bytes, uint8_t** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    auto& slot = g_scratch[{dev, stream}];
    if (slot.second < bytes) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(stream, &cap) == cudaSuccess && cap != cudaStreamCaptureStatusNone)
            return cudaErrorStreamCaptureUnsupported;
        if (slot.first) cudaFree(slot.first);
        slot = {nullptr, 0};
        const size_t want = bytes + bytes / 4;
        void* p = nullptr;
        if ((e = cudaMalloc(&p, want)) != cudaSuccess) return e;
        slot = {p, want};
    }
    *out = (uint8_t*)slot.first;
    return cudaSuccess;
}

}  // namespace

bool uses_gemm_tc(const WeightView& w, int xtype, int64_t m, unsigned flags) {
    const bool sixteen_bit = xtype != CLQ_X_F32 || (flags & CLQ_MATH_FAST);
    return sixteen_bit && m >= gemm_min_m() && gemm_tc_supported(w, m);
}

cudaError_t launch_linear(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                          float* out, int64_t ldo, unsigned flags, cudaStream_t stream) {
    if (uses_gemm_tc(w, xtype, m, flags)) {
        const GemmPlan g = plan_gemm_tc(rows, w.k, m);
        uint8_t* scratch = nullptr;
        cudaError_t e = scratch_for(stream, gemm_tc_scratch_bytes(g), &scratch);
        if (e != cudaSuccess) return e;
        return launch_gemm_tc(w, rows, x, xtype, m, out, ldo, scratch, g, stream);
    }
    if (gemv_mma_supported(w, m)) return launch_gemv_mma(w, rows, x, xtype, m, out, ldo, stream);
    return launch_linear_generic(w, rows, x, xtype, m, out, ldo, stream);
}

}  // namespace clq
