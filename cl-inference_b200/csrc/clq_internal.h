// clq_internal.h -- launchers shared between the C ABI layer and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace clq {

// A packed weight as the kernels see it: N rows of K/elems blocks in the
// re-tiled device planes of layout.cuh, offset to the view's first row.
struct WeightView {
    int dtype;
    int64_t rows;          // rows available from row 0 of the view
    int64_t k;             // elements per row
    int64_t nb;            // blocks per row
    const uint8_t* q;      // planes (see layout.cuh), already offset to row 0
    const uint8_t* s;
    const uint8_t* d;
};

bool geometry(int dtype, int* elems, int* block_bytes);

// Records the formatted message as this thread's clq_last_error and returns CODE.
int set_error(int code, const char* fmt, ...);
// Makes the current device's stream-ordered pool keep released memory (once per device).
cudaError_t keep_pool_memory();

// Re-tile NBLOCKS native GGUF blocks (N rows of NB blocks) into the planes at
// DST (layout.cuh); the planes' tail must be zeroed by the caller.
cudaError_t launch_retile(const uint8_t* native, int dtype, int64_t n, int64_t nb, uint8_t* dst,
                          cudaStream_t stream);

// Writes into *first_bad the smallest block index whose fp16 scale has
// exponent 31, or leaves it untouched (caller initialises it to ~0ull).
cudaError_t launch_validate_scales(const uint8_t* dev, int dtype, int64_t nblocks,
                                   unsigned long long* first_bad, cudaStream_t stream);

cudaError_t launch_dequantize(const WeightView& w, int64_t rows, float* out, bool transposed,
                              cudaStream_t stream);

// Rows ids[i] of w; an id outside [0, w.rows) yields a row of quiet NaNs.
cudaError_t launch_gather(const WeightView& w, const int32_t* ids, int64_t count, float* out,
                          cudaStream_t stream);

// BYTES (a multiple of 16) from page-locked host memory mapped into the
// device's address space (SRC_MAPPED, its device pointer) to device DST, both
// 16-byte aligned, by a kernel that lets the next one start early.
cudaError_t launch_copy_in(void* dst, const void* src_mapped, size_t bytes, cudaStream_t stream);

// out[i*ldo + j] = sum_c x[i, c] * W[j, c], i < m, j < rows.
// Returns cudaErrorNotSupported when no kernel covers the request.
cudaError_t launch_linear(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                          float* out, int64_t ldo, unsigned flags, cudaStream_t stream);

// Tensor-core fused dequant + GEMV (K a multiple of 256).
bool gemv_mma_supported(const WeightView& w, int64_t m);
bool gemv_pdl_enabled();
// The streaming decode GEMVs: Q4_K / Q6_K on the per-warp streams (m <= 8 in
// one pass, or two passes for 9 <= m <= 16 and for 5 <= m <= 8 when one pass
// does not fit), else the bulk-copy kernel (m <= 8).  cudaErrorNotSupported
// for shapes none of them takes, before anything is launched.
cudaError_t launch_gemv_bulk_group(const WeightView* const* w, const int64_t* rows, int count, const void* x,
                                   int xtype, int64_t m, float* const* out, const int64_t* ldo,
                                   cudaStream_t stream);
// Peer-memory links of one rank of a tensor-parallel group (max 8 ranks), for
// the GEMV whose epilogue all-reduces over NVLink.  recv buffers hold 8-byte
// (epoch, value) words, [2 parities][world writer ranks][kMaxTpCtas][cap]: a
// fixed region per CTA index, written and read only by that CTA index on every
// rank.  epochs holds one call counter per CTA index (local only).
constexpr int kMaxRanks = 8;
constexpr int kMaxTpCtas = 160;
struct TpLink {
    uint2* peer_recv[kMaxRanks];    // each rank's recv buffer, mapped here
    uint2* my_recv;
    uint32_t* epochs;               // [kMaxTpCtas]
    int rank, world;
    int64_t cap;                    // words per (parity, writer, CTA) region
    uint32_t wait_polls;            // polls of one peer word before the wait gives up
};
// out = sum over ranks of x_r W_r^T (the row-parallel shard product of each
// rank), computed by the bulk GEMV with the reduction over peer memory fused
// into its epilogue.  cudaErrorNotSupported for shapes it does not take.
cudaError_t launch_gemv_bulk_allreduce(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                                       float* out, int64_t ldo, const TpLink& tp, cudaStream_t stream);

// Work fused around a linear (local/blocks.lisp:115-116, 151-154, 387-392):
// the product's input is h = (gate ? silu(gate) * x : x), then, with norm_w,
// h * norm_w / sqrt(mean(h^2) + norm_eps) per activation row; with res,
// out = res + h W^T (res row stride ldr; single-weight calls only).
struct Fusion {
    const float* norm_w = nullptr;
    float norm_eps = 0.f;
    const void* gate = nullptr;
    const float* res = nullptr;
    int64_t ldr = 0;
    bool any() const { return norm_w || gate || res; }
};

// The decode GEMV with one weight stream per warp (Q4_K / Q6_K, m <= 8), with
// the all-reduce over TP's ranks fused in when TP is non-null and the
// prologue / epilogue of FUSE (m <= 2) when that is non-null;
// cudaErrorNotSupported for shapes it does not take, before anything is launched.
cudaError_t launch_gemv_warp(const WeightView* const* w, const int64_t* rows, int count, const void* x, int xtype,
                             int64_t m, float* const* out, const int64_t* ldo, const TpLink* tp,
                             cudaStream_t stream, const Fusion* fuse = nullptr);
// The unfused forms, for every other kernel: H (fp32 [m, k]) = the fused input
// of X; OUT[t, j] = RES[t, j] + PART[t, j] for j < rows (OUT may be RES).
cudaError_t launch_fuse_input(const void* x, int xtype, int64_t m, int64_t k, const Fusion& f, float* h,
                              cudaStream_t stream);
cudaError_t launch_add_residual(float* out, int64_t ldo, const float* part, int64_t ldp, const float* res,
                                int64_t ldr, int64_t m, int64_t rows, cudaStream_t stream);
// Streaming multiprocessors of the current device (cached).
int sm_count();

// Device address of the current device's sticky status word (0 = no kernel
// reported a problem; else a CLQ_ERR_* code), or nullptr if it cannot be found.
int* device_status_word();
cudaError_t launch_gemv_mma(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                            float* out, int64_t ldo, cudaStream_t stream);
// Up to 4 weights of one dtype and K sharing x, in one launch.
cudaError_t launch_gemv_mma_group(const WeightView* const* w, const int64_t* rows, int count, const void* x,
                                  int xtype, int64_t m, float* const* out, const int64_t* ldo,
                                  cudaStream_t stream);

// Tensor-core (tcgen05) prefill GEMM: tiling and scratch layout for one call.
struct GemmPlan {
    int tn;                // tokens per tile
    int row_tile;          // weight rows per CTA: 128, or 256 (the Q4_K kernel)
    int64_t token_tiles, row_tiles;
    int splits;            // K splits (partials reduced in a second kernel)
    int kb_per_split;      // 64-wide K blocks per split
    bool exact, xlo;       // fp32-class products: weights (and activations, xlo) as hi + lo
    int stages;            // pipeline depth
    size_t xs_bytes, us_bytes, part_bytes;
    size_t smem;           // dynamic shared memory per CTA
};
// DTYPE picks the kernel: Q4_K weights of at least 256 rows may take the one
// with 256-row tiles (a tuning knob).  EXACT: fp32-class products, the weights
// split into fp16 hi + lo parts and, with XLO, the activations too.
GemmPlan plan_gemm_tc(int dtype, int64_t rows, int64_t k, int64_t m, bool exact, bool xlo);
size_t gemm_tc_scratch_bytes(const GemmPlan& g);
// plan_gemm_tc with fewer K splits until the scratch fits in CAP bytes;
// splits = 0 when it cannot fit.
GemmPlan plan_gemm_tc_capped(int dtype, int64_t rows, int64_t k, int64_t m, size_t cap);
bool gemm_tc_supported(const WeightView& w, int64_t m);
// SCRATCH: gemm_tc_scratch_bytes(g) device bytes, 256-byte aligned, private to
// this call until it completes on STREAM.  PREPPED: SCRATCH already holds
// the activation image of X for a plan with the same tn, image sizes and
// exactness (an earlier call of a group), so it is not formed again.
cudaError_t launch_gemm_tc(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m, float* out,
                           int64_t ldo, uint8_t* scratch, const GemmPlan& g, cudaStream_t stream,
                           bool prepped = false);
// Weights sharing one activation X (q/k/v, gate/up) through the tensor-core
// GEMM with the activation image formed once; cudaErrorNotSupported (nothing
// launched) when the members' plans do not share one image.
cudaError_t launch_linear_group_gemm(const WeightView* const* w, const int64_t* rows, int count, const void* x,
                                     int xtype, int64_t m, float* const* out, const int64_t* ldo, unsigned flags,
                                     cudaStream_t stream);

// Whether launch_linear takes the tensor-core GEMM for this request.
bool uses_gemm_tc(const WeightView& w, int xtype, int64_t m, unsigned flags);

// The generic (any alignment, any M) kernel, also used as a fallback by launch_linear.
cudaError_t launch_linear_generic(const WeightView& w, int64_t rows, const void* x, int xtype,
                                  int64_t m, float* out, int64_t ldo, cudaStream_t stream);

}  // namespace clq
