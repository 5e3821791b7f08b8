// kernels_basic.cu -- scale validation, bit-exact dequantize/gather, the
// generic linear kernel (any row alignment, any number of activation rows) and
// the host-call path's copy of its inputs from mapped page-locked memory.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/clq.h"
#include "clq_internal.h"
#include "formats.cuh"
#include "fusion.cuh"
#include "layout.cuh"

namespace clq {

bool geometry(int dtype, int* elems, int* block_bytes) {
    switch (dtype) {
    case kQ4_0: *elems = 32; *block_bytes = 18; return true;
    case kQ8_0: *elems = 32; *block_bytes = 34; return true;
    case kQ4_K: *elems = 256; *block_bytes = 144; return true;
    case kQ6_K: *elems = 256; *block_bytes = 210; return true;
    default: return false;
    }
}

namespace {

constexpr int kThreads = 256;

Planes planes_of(const WeightView& w) { return Planes{w.q, w.s, w.d, w.nb}; }

int grid_for(int64_t work, int threads) {
    int64_t blocks = (work + threads - 1) / threads;
    // 148 SMs x 8 resident blocks of 256 threads covers the machine; grid-stride beyond.
    return (int)(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

// mlx/gguf/weights.lisp:19-23 checks (byte & 0x7C) == 0x7C on each scale's high byte.
__global__ void validate_scales_kernel(const uint8_t* __restrict__ w, int64_t nblocks,
                                       int block_bytes, int off0, int off1, int noff,
                                       unsigned long long* first_bad) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nblocks;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint8_t* b = w + i * block_bytes;
        bool bad = (b[off0 + 1] & 0x7C) == 0x7C;
        if (noff > 1) bad = bad || (b[off1 + 1] & 0x7C) == 0x7C;
        if (bad) atomicMin(first_bad, (unsigned long long)i);
    }
}

template <int D>
__global__ void dequantize_kernel(Planes p, int64_t k, int64_t rows, float* __restrict__ out,
                                  int transposed) {
    int64_t total = rows * k;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i / k, c = i - r * k;
        float v = element_planar<D>(p, r, c);
        if (transposed) out[c * rows + r] = v;
        else out[i] = v;
    }
}

template <int D>
__global__ void gather_kernel(Planes p, int64_t k, int64_t nrows, const int32_t* __restrict__ ids,
                              int64_t count, float* __restrict__ out) {
    int64_t total = count * k;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = i / k, c = i - t * k;
        int64_t r = ids[t];
        out[i] = (r >= 0 && r < nrows) ? element_planar<D>(p, r, c) : __int_as_float(0x7fc00000);
    }
}

// One thread per native block: scatter its bytes into the planes.
template <int D>
__global__ void retile_kernel(const uint8_t* __restrict__ native, int64_t n, int64_t nb,
                              uint8_t* __restrict__ q, uint8_t* __restrict__ s, uint8_t* __restrict__ d) {
    constexpr int B = Geometry<D>::kBytes;
    const int64_t total = n * nb;
    for (int64_t blk = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; blk < total;
         blk += (int64_t)gridDim.x * blockDim.x) {
        const uint8_t* src = native + blk * B;
        const int64_t row = blk / nb, j = blk % nb;
        if (D == kQ4_K) {
            for (int i = 0; i < 144; i++) q[blk * 144 + i] = src[i];
        } else if (D == kQ4_0) {
            d[2 * blk] = src[0]; d[2 * blk + 1] = src[1];
            for (int i = 0; i < 16; i++) q[row * nb * 16 + chunk_code_offset<16>(nb, j, i)] = src[2 + i];
        } else if (D == kQ8_0) {
            d[2 * blk] = src[0]; d[2 * blk + 1] = src[1];
            for (int i = 0; i < 32; i++) q[row * nb * 32 + chunk_code_offset<32>(nb, j, i)] = src[2 + i];
        } else {  // Q6_K
            for (int i = 0; i < 128; i++) {  // ql: element (h, grp, l) low bits
                const int h = i / 64, p = (i % 64) / 32, l = i % 32;
                const int half = l / 16, t = (l % 16) / 4, bw = l % 4;
                q[blk * 192 + t * 48 + (2 * h + half) * 12 + 4 * p + bw] = src[i];
            }
            for (int i = 0; i < 64; i++) {  // qh
                const int h = i / 32, l = i % 32;
                const int half = l / 16, t = (l % 16) / 4, bw = l % 4;
                q[blk * 192 + t * 48 + (2 * h + half) * 12 + 8 + bw] = src[128 + i];
            }
            for (int i = 0; i < 16; i++) s[blk * 16 + i] = src[192 + i];
            d[2 * blk] = src[208]; d[2 * blk + 1] = src[209];
        }
    }
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// One warp per weight row; lanes stride over 32-element units of the row and
// decode each element with the reference formula.  Up to MT activation rows
// per grid.y slice.  Slow but valid for every alignment and shape.
template <int D, typename XT, int MT>
__global__ void linear_generic_kernel(Planes p, int64_t k, int64_t rows, const XT* __restrict__ x,
                                      int64_t m, float* __restrict__ out, int64_t ldo) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int64_t m0 = (int64_t)blockIdx.y * MT;
    float acc[MT];
#pragma unroll
    for (int t = 0; t < MT; t++) acc[t] = 0.f;
    const int64_t units = k / 32;
    for (int64_t u = lane; u < units; u += 32) {
        const int64_t e0 = u * 32;
        for (int i = 0; i < 32; i++) {
            float wv = element_planar<D>(p, row, e0 + i);
#pragma unroll
            for (int t = 0; t < MT; t++)
                if (m0 + t < m) acc[t] = fmaf(to_f32(x[(m0 + t) * k + e0 + i]), wv, acc[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < MT; t++) {
        float v = acc[t];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && m0 + t < m) out[(m0 + t) * ldo + row] = v;
    }
}

template <int D, typename XT>
cudaError_t generic_launch(const WeightView& w, int64_t rows, const XT* x, int64_t m, float* out,
                           int64_t ldo, cudaStream_t s) {
    constexpr int MT = 4, WARPS = 4;
    dim3 grid((unsigned)((rows + WARPS - 1) / WARPS), (unsigned)((m + MT - 1) / MT));
    if (grid.y > 65535) return cudaErrorInvalidConfiguration;
    linear_generic_kernel<D, XT, MT><<<grid, WARPS * 32, 0, s>>>(planes_of(w), w.k, rows, x, m, out, ldo);
    return cudaGetLastError();
}

template <typename XT>
cudaError_t generic_by_dtype(const WeightView& w, int64_t rows, const XT* x, int64_t m, float* out,
                             int64_t ldo, cudaStream_t s) {
    switch (w.dtype) {
    case kQ4_0: return generic_launch<kQ4_0, XT>(w, rows, x, m, out, ldo, s);
    case kQ8_0: return generic_launch<kQ8_0, XT>(w, rows, x, m, out, ldo, s);
    case kQ4_K: return generic_launch<kQ4_K, XT>(w, rows, x, m, out, ldo, s);
    case kQ6_K: return generic_launch<kQ6_K, XT>(w, rows, x, m, out, ldo, s);
    default: return cudaErrorInvalidValue;
    }
}

// N16 16-byte words from SRC (page-locked host memory mapped into the device's
// address space) to DST, every load in flight before any store.  The next
// kernel in the stream may start at once under programmatic dependent launch:
// it prefetches its weights and waits (griddepcontrol.wait) for this copy
// before it reads DST.
__global__ void __launch_bounds__(kThreads) copy_in_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                                           int64_t n16) {
    asm volatile("griddepcontrol.launch_dependents;");
    constexpr int B = 4;
    for (int64_t i0 = blockIdx.x * (int64_t)kThreads * B + threadIdx.x; i0 < n16;
         i0 += (int64_t)gridDim.x * kThreads * B) {
        uint4 v[B];
#pragma unroll
        for (int b = 0; b < B; b++)
            if (i0 + b * kThreads < n16) v[b] = src[i0 + b * kThreads];
#pragma unroll
        for (int b = 0; b < B; b++)
            if (i0 + b * kThreads < n16) dst[i0 + b * kThreads] = v[b];
    }
}

}  // namespace

cudaError_t launch_copy_in(void* dst, const void* src_mapped, size_t bytes, cudaStream_t s) {
    if (bytes == 0) return cudaSuccess;
    if (bytes % 16 || (uintptr_t)dst % 16 || (uintptr_t)src_mapped % 16) return cudaErrorInvalidValue;
    const int64_t n16 = (int64_t)(bytes / 16);
    int64_t blocks = (n16 + kThreads * 4 - 1) / (kThreads * 4);
    if (blocks > 64) blocks = 64;
    copy_in_kernel<<<(unsigned)blocks, kThreads, 0, s>>>(static_cast<uint4*>(dst), static_cast<const uint4*>(src_mapped),
                                                        n16);
    return cudaGetLastError();
}

cudaError_t launch_validate_scales(const uint8_t* dev, int dtype, int64_t nblocks,
                                   unsigned long long* first_bad, cudaStream_t stream) {
    int elems, bb, off[2] = {0, 0};
    if (!geometry(dtype, &elems, &bb)) return cudaErrorInvalidValue;
    int noff = scale_offsets(dtype, off);
    if (nblocks <= 0) return cudaSuccess;
    validate_scales_kernel<<<grid_for(nblocks, kThreads), kThreads, 0, stream>>>(
        dev, nblocks, bb, off[0], off[1], noff, first_bad);
    return cudaGetLastError();
}

cudaError_t launch_retile(const uint8_t* native, int dtype, int64_t n, int64_t nb, uint8_t* dst,
                          cudaStream_t s) {
    if (n * nb == 0) return cudaSuccess;
    size_t s_off, d_off, total;
    plane_offsets(dtype, n * nb, &s_off, &d_off, &total);
    uint8_t *q = dst, *sp = dst + s_off, *dp = dst + d_off;
    int g = grid_for(n * nb, kThreads);
    switch (dtype) {
    case kQ4_0: retile_kernel<kQ4_0><<<g, kThreads, 0, s>>>(native, n, nb, q, sp, dp); break;
    case kQ8_0: retile_kernel<kQ8_0><<<g, kThreads, 0, s>>>(native, n, nb, q, sp, dp); break;
    case kQ4_K: retile_kernel<kQ4_K><<<g, kThreads, 0, s>>>(native, n, nb, q, sp, dp); break;
    case kQ6_K: retile_kernel<kQ6_K><<<g, kThreads, 0, s>>>(native, n, nb, q, sp, dp); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequantize(const WeightView& w, int64_t rows, float* out, bool transposed,
                              cudaStream_t s) {
    if (rows <= 0 || w.k <= 0) return cudaSuccess;
    int g = grid_for(rows * w.k, kThreads);
    int t = transposed ? 1 : 0;
    switch (w.dtype) {
    case kQ4_0: dequantize_kernel<kQ4_0><<<g, kThreads, 0, s>>>(planes_of(w), w.k, rows, out, t); break;
    case kQ8_0: dequantize_kernel<kQ8_0><<<g, kThreads, 0, s>>>(planes_of(w), w.k, rows, out, t); break;
    case kQ4_K: dequantize_kernel<kQ4_K><<<g, kThreads, 0, s>>>(planes_of(w), w.k, rows, out, t); break;
    case kQ6_K: dequantize_kernel<kQ6_K><<<g, kThreads, 0, s>>>(planes_of(w), w.k, rows, out, t); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_gather(const WeightView& w, const int32_t* ids, int64_t count, float* out,
                          cudaStream_t s) {
    if (count <= 0 || w.k <= 0) return cudaSuccess;
    int g = grid_for(count * w.k, kThreads);
    switch (w.dtype) {
    case kQ4_0: gather_kernel<kQ4_0><<<g, kThreads, 0, s>>>(planes_of(w), w.k, w.rows, ids, count, out); break;
    case kQ8_0: gather_kernel<kQ8_0><<<g, kThreads, 0, s>>>(planes_of(w), w.k, w.rows, ids, count, out); break;
    case kQ4_K: gather_kernel<kQ4_K><<<g, kThreads, 0, s>>>(planes_of(w), w.k, w.rows, ids, count, out); break;
    case kQ6_K: gather_kernel<kQ6_K><<<g, kThreads, 0, s>>>(planes_of(w), w.k, w.rows, ids, count, out); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

namespace {

__device__ __forceinline__ float act(const float* p) { return *p; }
__device__ __forceinline__ float act(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float act(const __half* p) { return __half2float(*p); }

// One CTA per activation row: h = silu(gate) * x (with a gate), then times
// norm_w / sqrt(mean(h^2) + eps) (with norm_w): the per-element arithmetic of
// the decode GEMV's fused prologue (its sum of squares runs in another order).
template <typename XT>
__global__ void fuse_input_kernel(const XT* x, const XT* gate, const float* norm_w, float eps, int64_t k,
                                  float* h) {
    constexpr int T = 256;
    __shared__ float red[T / 32];
    const int64_t row = blockIdx.x;
    const XT* xr = x + row * k;
    const XT* gr = gate ? gate + row * k : nullptr;
    float* hr = h + row * k;
    auto in = [&](int64_t e) {
        float v = act(xr + e);
        if (gr) {
            const float g = act(gr + e);
            v = swiglu(g, v);
        }
        return v;
    };
    if (!norm_w) {
        for (int64_t e = threadIdx.x; e < k; e += T) hr[e] = in(e);
        return;
    }
    float ss = 0.f;
    for (int64_t e = threadIdx.x; e < k; e += T) {
        const float v = in(e);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < T / 32; w++) tot += red[w];
    const float r = 1.f / sqrtf(tot / (float)k + eps);
    for (int64_t e = threadIdx.x; e < k; e += T) hr[e] = in(e) * r * norm_w[e];
}

// out = res + part, element by element (OUT may be RES: each element is read
// before it is written, by the same thread).
__global__ void add_residual_kernel(float* out, int64_t ldo, const float* part, int64_t ldp, const float* res,
                                    int64_t ldr, int64_t m, int64_t rows) {
    const int64_t n = m * rows;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / rows, j = i - t * rows;
        out[t * ldo + j] = res[t * ldr + j] + part[t * ldp + j];
    }
}

}  // namespace

cudaError_t launch_fuse_input(const void* x, int xtype, int64_t m, int64_t k, const Fusion& f, float* h,
                              cudaStream_t s) {
    if (m <= 0 || k <= 0) return cudaSuccess;
    switch (xtype) {
    case CLQ_X_F32:
        fuse_input_kernel<float><<<(unsigned)m, 256, 0, s>>>((const float*)x, (const float*)f.gate, f.norm_w,
                                                             f.norm_eps, k, h);
        break;
    case CLQ_X_BF16:
        fuse_input_kernel<__nv_bfloat16><<<(unsigned)m, 256, 0, s>>>((const __nv_bfloat16*)x,
                                                                     (const __nv_bfloat16*)f.gate, f.norm_w,
                                                                     f.norm_eps, k, h);
        break;
    case CLQ_X_F16:
        fuse_input_kernel<__half><<<(unsigned)m, 256, 0, s>>>((const __half*)x, (const __half*)f.gate, f.norm_w,
                                                              f.norm_eps, k, h);
        break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_add_residual(float* out, int64_t ldo, const float* part, int64_t ldp, const float* res,
                                int64_t ldr, int64_t m, int64_t rows, cudaStream_t s) {
    if (m <= 0 || rows <= 0) return cudaSuccess;
    add_residual_kernel<<<grid_for(m * rows, kThreads), kThreads, 0, s>>>(out, ldo, part, ldp, res, ldr, m, rows);
    return cudaGetLastError();
}

cudaError_t launch_linear_generic(const WeightView& w, int64_t rows, const void* x, int xtype,
                                  int64_t m, float* out, int64_t ldo, cudaStream_t s) {
    if (rows <= 0 || m <= 0) return cudaSuccess;
    switch (xtype) {
    case CLQ_X_F32: return generic_by_dtype(w, rows, (const float*)x, m, out, ldo, s);
    case CLQ_X_BF16: return generic_by_dtype(w, rows, (const __nv_bfloat16*)x, m, out, ldo, s);
    case CLQ_X_F16: return generic_by_dtype(w, rows, (const __half*)x, m, out, ldo, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace clq
