// attention.cu -- the decode layer's work between the linears on the device:
// the KV cache (f32 or the Q8 codec of local/kv-cache.lisp), RoPE
// (local/blocks.lisp:172-214) and grouped-query attention over the cache
// prefix with the causal mask (local/blocks.lisp:282-325).
//
// Cache layout in HBM, per layer, keys and values alike: [n_ctx][kv_heads]
// [head_dim] -- f32 elements, or int8 codes plus one f32 scale per 32-element
// group ([n_ctx][kv_heads][ceil(head_dim / 32)]), the reference buffers'
// order, so a position's row of every head is one contiguous span.
//
// Attention is split over positions (flash-decoding): a CTA takes one query
// row, one KV head and a range of positions, reads each key and value row
// once for all the query heads of that KV head (coalesced: lanes over the
// head dimension), and leaves the range's softmax maximum, sum and weighted
// value sum; a second kernel merges the ranges of each (row, head).  The
// cache is read once per query row -- the step is bound by HBM.
#include <cfloat>
#include <cmath>
#include <cstdint>

#include <cuda_runtime.h>

#include "../../include/clq.h"
#include "clq_internal.h"

namespace clq {
namespace {

constexpr int kQ8Group = 32;          // local/kv-cache.lisp:20
constexpr int kAttnThreads = 128;     // 4 warps per CTA
constexpr int kMaxGroup = 16;         // query heads per KV head
constexpr int kSplitRows = 64;        // positions per CTA, staged in shared memory
constexpr int kMaxSplits = 1024;      // position ranges merged per (row, head)
constexpr int kMaxHeadDim = 256;

// ---- the Q8 codec --------------------------------------------------------

// A code back to f32: code * scale in single precision when that cannot
// overflow, else the double product clamped to the finite range
// (local/kv-cache.lisp:62-78).
__device__ __forceinline__ float q8_decode(int8_t code, float scale) {
    const double limit = (double)FLT_MAX / 127.0;
    if ((double)scale <= limit) return __fmul_rn((float)code, scale);
    double v = (double)code * (double)scale;
    v = fmin(fmax(v, -(double)FLT_MAX), (double)FLT_MAX);
    return (float)v;
}

// One warp per (position, head, group of 32): the group's peak magnitude
// sets scale = max(FLT_MIN, peak / 127) (1 for an all-zero group), and each
// value becomes clamp(round-half-even(value / scale), -127, 127)
// (local/kv-cache.lisp:37-60).  A non-finite value sets *ERR.
// Keys (blockIdx.y = 0) and values (1) in one launch.
struct KvStore {
    const float* src[2];
    uint8_t* buf[2];
    size_t code_bytes;
};

__global__ void kv_store_q8_kernel(const KvStore S, int64_t count, int kvh, int hd, int64_t ps, int64_t hs,
                                   int64_t start, int* err) {
    const int groups = (hd + kQ8Group - 1) / kQ8Group;
    const float* __restrict__ src = S.src[blockIdx.y];
    int8_t* __restrict__ codes = reinterpret_cast<int8_t*>(S.buf[blockIdx.y]);
    float* __restrict__ scales = reinterpret_cast<float*>(S.buf[blockIdx.y] + S.code_bytes);
    const int64_t items = count * kvh * groups;
    const int lane = threadIdx.x & 31;
    for (int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; w < items;
         w += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        const int grp = (int)(w % groups);
        const int head = (int)((w / groups) % kvh);
        const int64_t row = w / ((int64_t)groups * kvh);
        const int i = grp * kQ8Group + lane;
        const bool in = i < hd;
        const float v = in ? src[row * ps + head * hs + i] : 0.f;
        if (in && !isfinite(v)) atomicExch(err, CLQ_ERR_NONFINITE_VALUE);
        const uint32_t peak_bits = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v)));
        const float peak = __uint_as_float(peak_bits);
        float scale = 1.f;
        if (peak != 0.f) scale = (float)fmax((double)FLT_MIN, (double)peak / 127.0);
        const int64_t slot = (start + row) * kvh + head;
        if (lane == 0) scales[slot * groups + grp] = scale;
        if (in) {
            float c = rintf(__fdiv_rn(v, scale));
            c = fminf(fmaxf(c, -127.f), 127.f);
            codes[slot * hd + i] = (int8_t)c;
        }
    }
}

__global__ void kv_store_f32_kernel(const KvStore S, int64_t count, int kvh, int hd, int64_t ps, int64_t hs,
                                    int64_t start) {
    const float* __restrict__ src = S.src[blockIdx.y];
    float* __restrict__ dst = reinterpret_cast<float*>(S.buf[blockIdx.y]);
    const int64_t total = count * kvh * hd;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(e % hd);
        const int head = (int)((e / hd) % kvh);
        const int64_t row = e / ((int64_t)hd * kvh);
        dst[((start + row) * kvh + head) * hd + i] = src[row * ps + head * hs + i];
    }
}

__global__ void kv_read_q8_kernel(float* __restrict__ out, const int8_t* __restrict__ codes,
                                  const float* __restrict__ scales, int64_t end, int kvh, int hd) {
    const int groups = (hd + kQ8Group - 1) / kQ8Group;
    const int64_t total = end * kvh * hd;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(e % hd);
        const int64_t slot = e / hd;
        out[e] = q8_decode(codes[e], scales[slot * groups + i / kQ8Group]);
    }
}

// ---- RoPE ------------------------------------------------------------------

// One thread per (position, head, pair i < rope_dims / 2): frequency
// theta^(-2i / rope_dims) / factor_i and angle (start + position) * frequency
// in double, cos and sin rounded to f32 (the reference's tables), then the
// rotation in f32 with each product and sum rounded on its own.  Pairs are
// (2i, 2i + 1) (adjacent) or (i, i + rope_dims / 2) (neox).
__global__ void rope_kernel(float* __restrict__ x, int64_t count, int heads, int64_t ps, int64_t hs, int rope_dims,
                            int64_t start, double theta, const float* __restrict__ factors, int neox) {
    const int half = rope_dims / 2;
    const int64_t total = count * heads * half;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(e % half);
        const int head = (int)((e / half) % heads);
        const int64_t pos = e / ((int64_t)half * heads);
        double freq = pow(theta, (-2.0 * (double)i) / (double)rope_dims);
        if (factors) freq /= (double)factors[i];
        const double angle = (double)(start + pos) * freq;
        const float c = (float)cos(angle), s = (float)sin(angle);
        float* row = x + pos * ps + head * hs;
        const int j0 = neox ? i : 2 * i, j1 = neox ? i + half : 2 * i + 1;
        const float x0 = row[j0], x1 = row[j1];
        row[j0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        row[j1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
}

// ---- attention -------------------------------------------------------------

struct AttnParams {
    const float* q;        // [count][n_heads][hd], position stride q_ps
    int64_t q_ps;
    const void* keys;      // layer's key buffer (f32 or int8 codes)
    const void* values;
    const float* kscale;   // Q8: [n_ctx][kvh][groups]
    const float* vscale;
    int64_t end;           // keys in the prefix
    int64_t query_start;   // position of query row 0
    int n_heads, kvh, hd, groups;
    int splits;
    int64_t per_split;
    float scale;           // 1 / sqrt(hd), rounded to f32
    float* part;           // [count][n_heads][splits][hd + 2]: weighted sum, then max, sum
};

// The split's rows of one KV head, keys and values, into shared memory as
// f32: every thread issues its 16-byte loads (4 f32 or 16 codes) before any
// is used, so the split costs about one memory round trip.
template <bool Q8>
__device__ __forceinline__ void stage_rows(const AttnParams& P, const void* buf, const float* scl, int64_t p0, int np,
                                           int kv, float* dst) {
    const int hd = P.hd;
    if (hd % (Q8 ? 16 : 4)) {  // rows off the 16-byte grid: element by element
        for (int e = threadIdx.x; e < np * hd; e += kAttnThreads) {
            const int j = e / hd, d = e - j * hd;
            const int64_t slot = (p0 + j) * P.kvh + kv;
            if constexpr (Q8) {
                dst[e] = q8_decode(reinterpret_cast<const int8_t*>(buf)[slot * hd + d], scl[slot * P.groups + d / kQ8Group]);
            } else {
                dst[e] = reinterpret_cast<const float*>(buf)[slot * hd + d];
            }
        }
        return;
    }
    // vector rows: eight 16-byte loads per thread in flight before any store
    constexpr int B = 8;
    if constexpr (Q8) {
        const int per_row = hd / 16, n = np * per_row;
        for (int e0 = threadIdx.x; e0 < n; e0 += B * kAttnThreads) {
            uint4 w[B];
            float sc[B];
#pragma unroll
            for (int b = 0; b < B; b++) {
                const int e = e0 + b * kAttnThreads;
                if (e < n) {
                    const int j = e / per_row, c = e - j * per_row;
                    const int64_t slot = (p0 + j) * P.kvh + kv;
                    w[b] = *reinterpret_cast<const uint4*>(reinterpret_cast<const int8_t*>(buf) + slot * hd + c * 16);
                    sc[b] = scl[slot * P.groups + (c * 16) / kQ8Group];
                }
            }
#pragma unroll
            for (int b = 0; b < B; b++) {
                const int e = e0 + b * kAttnThreads;
                if (e < n) {
                    const int j = e / per_row, c = e - j * per_row;
                    const uint32_t ws[4] = {w[b].x, w[b].y, w[b].z, w[b].w};
                    float* o = dst + j * hd + c * 16;
#pragma unroll
                    for (int i = 0; i < 16; i++) o[i] = q8_decode((int8_t)(ws[i >> 2] >> (8 * (i & 3))), sc[b]);
                }
            }
        }
    } else {
        const int per_row = hd / 4, n = np * per_row;
        for (int e0 = threadIdx.x; e0 < n; e0 += B * kAttnThreads) {
            float4 v[B];
#pragma unroll
            for (int b = 0; b < B; b++) {
                const int e = e0 + b * kAttnThreads;
                if (e < n) {
                    const int j = e / per_row, c = e - j * per_row;
                    const int64_t slot = (p0 + j) * P.kvh + kv;
                    v[b] = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(buf) + slot * hd + c * 4);
                }
            }
#pragma unroll
            for (int b = 0; b < B; b++) {
                const int e = e0 + b * kAttnThreads;
                if (e < n) {
                    const int j = e / per_row, c = e - j * per_row;
                    *reinterpret_cast<float4*>(dst + j * hd + c * 4) = v[b];
                }
            }
        }
    }
}

// CTA (split, kv head, query row).  The split's unmasked positions (key
// position <= query_start + row) are staged; scores s = (q . k) * scale for
// the group's query heads; then the split's maximum m, the sum l of
// exp(s - m) and the sum of exp(s - m) * v.
template <bool Q8, int G>
__global__ void __launch_bounds__(kAttnThreads) attend_split_kernel(const AttnParams P) {
    extern __shared__ __align__(16) float sh[];
    const int split = blockIdx.x, kv = blockIdx.y;
    const int64_t row = blockIdx.z;
    const int hd = P.hd;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int NW = kAttnThreads / 32;
    float* qs = sh;                                 // [G][hd]
    float* sc = qs + G * hd;                        // [G][kSplitRows]
    float* ks = sc + G * kSplitRows;                // [kSplitRows][hd]
    float* vs = ks + kSplitRows * hd;               // [kSplitRows][hd]
    const int64_t last = P.query_start + row + 1 < P.end ? P.query_start + row + 1 : P.end;  // causal
    const int64_t p0 = (int64_t)split * P.per_split;
    int64_t p1 = p0 + P.per_split;
    if (p1 > last) p1 = last;
    const int np = p1 > p0 ? (int)(p1 - p0) : 0;

    for (int e = threadIdx.x; e < G * hd; e += kAttnThreads) {
        const int g = e / hd, d = e - g * hd;
        qs[e] = P.q[row * P.q_ps + (int64_t)(kv * G + g) * hd + d];
    }
    stage_rows<Q8>(P, P.keys, P.kscale, p0, np, kv, ks);
    stage_rows<Q8>(P, P.values, P.vscale, p0, np, kv, vs);
    __syncthreads();

    // scores: a warp per position, lanes over the head dimension
    for (int j = warp; j < np; j += NW) {
        float dot[G];
#pragma unroll
        for (int g = 0; g < G; g++) dot[g] = 0.f;
        for (int d = lane; d < hd; d += 32) {
            const float k = ks[j * hd + d];
#pragma unroll
            for (int g = 0; g < G; g++) dot[g] = fmaf(qs[g * hd + d], k, dot[g]);
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            float v = dot[g];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) sc[g * kSplitRows + j] = __fmul_rn(v, P.scale);
        }
    }
    __syncthreads();

    // the split's maximum and sum per query head: warp g handles heads g, g + NW, ...
    for (int g = warp; g < G; g += NW) {
        float m = -INFINITY;
        for (int j = lane; j < np; j += 32) m = fmaxf(m, sc[g * kSplitRows + j]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        float l = 0.f;
        for (int j = lane; j < np; j += 32) {
            const float p = expf(sc[g * kSplitRows + j] - m);
            sc[g * kSplitRows + j] = p;
            l += p;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (lane == 0) {
            float* out = P.part + (((row * P.n_heads) + kv * G + g) * P.splits + split) * (int64_t)(hd + 2);
            out[hd] = m;
            out[hd + 1] = l;
        }
    }
    __syncthreads();

    // weighted value sums: each thread owns dimensions d = threadIdx.x, + 128, ...
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
        float acc[G];
#pragma unroll
        for (int g = 0; g < G; g++) acc[g] = 0.f;
        for (int j = 0; j < np; j++) {
            const float v = vs[j * hd + d];
#pragma unroll
            for (int g = 0; g < G; g++) acc[g] = fmaf(sc[g * kSplitRows + j], v, acc[g]);
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            P.part[(((row * P.n_heads) + kv * G + g) * P.splits + split) * (int64_t)(hd + 2) + d] = acc[g];
        }
    }
}

size_t attend_smem(int G, int hd) {
    return ((size_t)G * hd + (size_t)G * kSplitRows + 2 * (size_t)kSplitRows * hd) * sizeof(float);
}

// Merges the splits of (query row, head) for a slice of 32 dimensions (one
// warp per CTA): M = max m_s, output sum_s exp(m_s - M) acc_s / sum_s
// exp(m_s - M) l_s into out[row][head * hd + d].  Every load is issued before
// any is used (the kernel is one round trip to L2, not one per split).
__global__ void __launch_bounds__(32) attend_merge_kernel(const float* __restrict__ part, int n_heads, int hd,
                                                          int splits, float* __restrict__ out, int64_t ldo) {
    __shared__ float wgt[kMaxSplits];
    __shared__ float lsum[kMaxSplits];
    const int head = blockIdx.x, lane = threadIdx.x;
    const int64_t row = blockIdx.y;
    const int d = blockIdx.z * 32 + lane;
    const int64_t stride = hd + 2;
    const float* base = part + ((row * n_heads) + head) * (int64_t)splits * stride;
    constexpr int B = 16;
    float m = -INFINITY;
    for (int s0 = 0; s0 < splits; s0 += 32 * B) {
        float lv[B], mv[B];
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int s = s0 + b * 32 + lane;
            lv[b] = s < splits ? base[s * stride + hd + 1] : 0.f;
            mv[b] = s < splits ? base[s * stride + hd] : -INFINITY;
        }
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int s = s0 + b * 32 + lane;
            if (s < splits) {
                lsum[s] = lv[b];
                wgt[s] = lv[b] > 0.f ? mv[b] : -INFINITY;
                m = fmaxf(m, wgt[s]);
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    __syncwarp();
    float L = 0.f;
    for (int s = lane; s < splits; s += 32) {
        const float w = lsum[s] > 0.f ? expf(wgt[s] - m) : 0.f;
        wgt[s] = w;
        L = fmaf(w, lsum[s], L);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    __syncwarp();
    if (d >= hd) return;
    float a = 0.f;
    for (int s0 = 0; s0 < splits; s0 += B) {
        float v[B];
#pragma unroll
        for (int b = 0; b < B; b++) v[b] = s0 + b < splits ? base[(s0 + b) * stride + d] : 0.f;
#pragma unroll
        for (int b = 0; b < B; b++)
            if (s0 + b < splits) a = fmaf(wgt[s0 + b], v[b], a);
    }
    out[row * ldo + (int64_t)head * hd + d] = a / L;
}

__global__ void fill_kernel(float* __restrict__ p, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
}

template <typename Kern>
cudaError_t attend_smem_limit(Kern kern, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

// The split kernel for G query heads per KV head (1, 2, 4, 8 or 16).
template <bool Q8>
cudaError_t launch_split(int G, dim3 grid, size_t smem, cudaStream_t s, const AttnParams& P) {
    cudaError_t e = cudaErrorNotSupported;
    switch (G) {
#define CLQ_SPLIT_CASE(n)                                                        \
    case n:                                                                     \
        e = attend_smem_limit(attend_split_kernel<Q8, n>, smem);                \
        if (e == cudaSuccess) attend_split_kernel<Q8, n><<<grid, kAttnThreads, smem, s>>>(P); \
        break;
        CLQ_SPLIT_CASE(1)
        CLQ_SPLIT_CASE(2)
        CLQ_SPLIT_CASE(4)
        CLQ_SPLIT_CASE(8)
        CLQ_SPLIT_CASE(16)
#undef CLQ_SPLIT_CASE
    }
    return e;
}

unsigned grid_for(int64_t work, int threads) {
    int64_t b = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)sm_count() * 8;
    if (b > cap) b = cap;
    return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace
}  // namespace clq

// ---------------------------------------------------------------------------

struct clq_kv_cache {
    int device;
    int64_t n_ctx;
    int layers, kvh, hd, type, groups;
    uint8_t* mem;      // every layer's keys then values
    size_t layer_bytes;  // one buffer (keys or values) of one layer
    size_t code_bytes;   // Q8: the codes of one buffer; scales follow
    int* err;          // sticky status of the Q8 stores
};

namespace {

int kv_fail(int code, const char* what) { return clq::set_error(code, "%s", what); }

// True when rows of WIDTH unit-stride elements at (position, head) offsets
// p * PS + h * HS never overlap: the inner of the two strides spans a row,
// the outer spans all of the inner ones (either order).
bool rows_disjoint(int64_t count, int64_t ps, int heads, int64_t hs, int width) {
    int64_t s_in = ps, n_in = count, s_out = hs, n_out = heads;
    if (hs < ps || (hs == ps && heads <= count)) {
        s_in = hs, n_in = heads, s_out = ps, n_out = count;
    }
    if (n_in > 1 && s_in < width) return false;
    if (n_out > 1 && s_out < (n_in > 1 ? s_in * n_in : width)) return false;
    return s_in >= 0 && s_out >= 0;
}

uint8_t* kv_buffer(const clq_kv_cache* c, int layer, int which) {
    return c->mem + ((size_t)layer * 2 + which) * c->layer_bytes;
}

int kv_check_device(const clq_kv_cache* c) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return kv_fail(CLQ_ERR_NO_DEVICE, "no CUDA device");
    if (dev != c->device) return clq::set_error(CLQ_ERR_ARGUMENT, "cache lives on device %d, current device is %d", c->device, dev);
    return CLQ_OK;
}

}  // namespace

extern "C" {

int clq_kv_cache_create(int64_t n_ctx, int layers, int kv_heads, int head_dim, int cache_type, clq_kv_cache** out) {
    if (!out) return kv_fail(CLQ_ERR_ARGUMENT, "null result pointer");
    *out = nullptr;
    if (n_ctx < 1 || layers < 1 || kv_heads < 1 || head_dim < 1)
        return clq::set_error(CLQ_ERR_SHAPE, "cache of %lld positions, %d layers, %d heads of %d", (long long)n_ctx, layers,
                              kv_heads, head_dim);
    if (cache_type != CLQ_KV_F32 && cache_type != CLQ_KV_Q8)
        return clq::set_error(CLQ_ERR_ARGUMENT, "unknown cache type %d (f32 %d, q8 %d)", cache_type, CLQ_KV_F32, CLQ_KV_Q8);
    clq_kv_cache* c = new clq_kv_cache{};
    if (cudaGetDevice(&c->device) != cudaSuccess) {
        delete c;
        return kv_fail(CLQ_ERR_NO_DEVICE, "no CUDA device");
    }
    c->n_ctx = n_ctx;
    c->layers = layers;
    c->kvh = kv_heads;
    c->hd = head_dim;
    c->type = cache_type;
    c->groups = (head_dim + clq::kQ8Group - 1) / clq::kQ8Group;
    const size_t slots = (size_t)n_ctx * kv_heads;
    if (cache_type == CLQ_KV_F32) {
        c->layer_bytes = slots * head_dim * sizeof(float);
    } else {
        c->code_bytes = (slots * head_dim + 255) & ~(size_t)255;
        c->layer_bytes = (c->code_bytes + slots * c->groups * sizeof(float) + 255) & ~(size_t)255;
    }
    cudaError_t e = cudaMalloc((void**)&c->mem, c->layer_bytes * 2 * layers);
    if (e == cudaSuccess) e = cudaMalloc((void**)&c->err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(c->mem, 0, c->layer_bytes * 2 * layers);
    if (e == cudaSuccess) e = cudaMemset(c->err, 0, sizeof(int));
    if (e == cudaSuccess && cache_type == CLQ_KV_Q8) {
        // unused scales read as 1, as the reference's buffers start (kv-cache.lisp:28-33)
        for (int b = 0; b < 2 * layers && e == cudaSuccess; b++) {
            float* sc = reinterpret_cast<float*>(c->mem + (size_t)b * c->layer_bytes + c->code_bytes);
            const int64_t n = (int64_t)slots * c->groups;
            clq::fill_kernel<<<clq::grid_for(n, 256), 256>>>(sc, n, 1.f);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    if (e != cudaSuccess) {
        if (c->mem) cudaFree(c->mem);
        if (c->err) cudaFree(c->err);
        delete c;
        return clq::set_error(e == cudaErrorMemoryAllocation ? CLQ_ERR_OUT_OF_MEMORY : CLQ_ERR_CUDA, "KV cache allocation: %s",
                              cudaGetErrorString(e));
    }
    *out = c;
    return CLQ_OK;
}

int clq_kv_cache_destroy(clq_kv_cache* c) {
    if (!c) return CLQ_OK;
    cudaFree(c->mem);
    cudaFree(c->err);
    delete c;
    return CLQ_OK;
}

int clq_kv_cache_info(const clq_kv_cache* c, int64_t* n_ctx, int* layers, int* kv_heads, int* head_dim, int* cache_type) {
    if (!c) return kv_fail(CLQ_ERR_ARGUMENT, "null cache");
    if (n_ctx) *n_ctx = c->n_ctx;
    if (layers) *layers = c->layers;
    if (kv_heads) *kv_heads = c->kvh;
    if (head_dim) *head_dim = c->hd;
    if (cache_type) *cache_type = c->type;
    return CLQ_OK;
}

int clq_kv_cache_update(clq_kv_cache* c, int layer, const float* k, const float* v, int64_t count, int64_t pos_stride,
                        int64_t head_stride, int64_t start, void* stream) {
    if (!c) return kv_fail(CLQ_ERR_ARGUMENT, "null cache");
    if (layer < 0 || layer >= c->layers) return clq::set_error(CLQ_ERR_ARGUMENT, "layer %d outside 0..%d", layer, c->layers - 1);
    if (count < 0 || start < 0) return clq::set_error(CLQ_ERR_SHAPE, "%lld rows at %lld", (long long)count, (long long)start);
    if (start + count > c->n_ctx)
        return clq::set_error(CLQ_ERR_CONTEXT, "Positions up to %lld do not fit in a context of %lld",
                              (long long)(start + count), (long long)c->n_ctx);
    if (count == 0) return CLQ_OK;
    if (!k || !v) return kv_fail(CLQ_ERR_ARGUMENT, "null key or value rows");
    if (head_stride < 0 || pos_stride < 0)
        return clq::set_error(CLQ_ERR_SHAPE, "negative row strides (%lld, %lld)", (long long)pos_stride, (long long)head_stride);
    int rc;
    if ((rc = kv_check_device(c))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    clq::KvStore S;
    S.src[0] = k;
    S.src[1] = v;
    S.buf[0] = kv_buffer(c, layer, 0);
    S.buf[1] = kv_buffer(c, layer, 1);
    S.code_bytes = c->code_bytes;
    if (c->type == CLQ_KV_F32) {
        const int64_t n = count * c->kvh * c->hd;
        clq::kv_store_f32_kernel<<<dim3(clq::grid_for(n, 256), 2), 256, 0, s>>>(S, count, c->kvh, c->hd, pos_stride,
                                                                                 head_stride, start);
    } else {
        const int64_t warps = count * c->kvh * c->groups;
        clq::kv_store_q8_kernel<<<dim3(clq::grid_for(warps * 32, 256), 2), 256, 0, s>>>(S, count, c->kvh, c->hd, pos_stride,
                                                                                         head_stride, start, c->err);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "KV cache store: %s", cudaGetErrorString(e));
    return CLQ_OK;
}

int clq_kv_cache_status(clq_kv_cache* c, int* status) {
    if (!c || !status) return kv_fail(CLQ_ERR_ARGUMENT, "null cache or status pointer");
    int rc;
    if ((rc = kv_check_device(c))) return rc;
    cudaError_t e = cudaDeviceSynchronize();
    int v = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&v, c->err, sizeof v, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && v) e = cudaMemset(c->err, 0, sizeof v);
    if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "KV cache status: %s", cudaGetErrorString(e));
    *status = v;
    return CLQ_OK;
}

int clq_kv_cache_read(const clq_kv_cache* c, int layer, int64_t end, float* keys, float* values, void* stream) {
    if (!c) return kv_fail(CLQ_ERR_ARGUMENT, "null cache");
    if (layer < 0 || layer >= c->layers) return clq::set_error(CLQ_ERR_ARGUMENT, "layer %d outside 0..%d", layer, c->layers - 1);
    if (end < 0 || end > c->n_ctx) return clq::set_error(CLQ_ERR_SHAPE, "prefix %lld of a %lld context", (long long)end, (long long)c->n_ctx);
    if (end == 0) return CLQ_OK;
    int rc;
    if ((rc = kv_check_device(c))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    for (int which = 0; which < 2; which++) {
        float* dst = which ? values : keys;
        if (!dst) continue;
        const uint8_t* buf = kv_buffer(c, layer, which);
        const int64_t n = end * c->kvh * c->hd;
        cudaError_t e;
        if (c->type == CLQ_KV_F32) {
            e = cudaMemcpyAsync(dst, buf, (size_t)n * sizeof(float), cudaMemcpyDeviceToDevice, s);
        } else {
            clq::kv_read_q8_kernel<<<clq::grid_for(n, 256), 256, 0, s>>>(
                dst, reinterpret_cast<const int8_t*>(buf), reinterpret_cast<const float*>(buf + c->code_bytes), end, c->kvh, c->hd);
            e = cudaGetLastError();
        }
        if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "KV cache read: %s", cudaGetErrorString(e));
    }
    return CLQ_OK;
}

int clq_rope_device(float* x, int64_t count, int heads, int head_dim, int64_t pos_stride, int64_t head_stride, int rope_dims,
                    int64_t start, double theta, const float* factors, int pairing, void* stream) {
    if (count < 0 || heads < 1 || head_dim < 1 || start < 0)
        return clq::set_error(CLQ_ERR_SHAPE, "%lld rows of %d heads of %d at %lld", (long long)count, heads, head_dim,
                              (long long)start);
    if (rope_dims < 2 || rope_dims > head_dim || rope_dims % 2)
        return clq::set_error(CLQ_ERR_SHAPE, "rotated dimensions %d of a %d-wide head", rope_dims, head_dim);
    if (pairing != CLQ_ROPE_ADJACENT && pairing != CLQ_ROPE_NEOX)
        return clq::set_error(CLQ_ERR_ARGUMENT, "unknown pairing %d", pairing);
    if (!(theta > 0.0)) return kv_fail(CLQ_ERR_ARGUMENT, "RoPE theta must be positive");
    if (count == 0) return CLQ_OK;
    if (!x) return kv_fail(CLQ_ERR_ARGUMENT, "null rows");
    if (!rows_disjoint(count, pos_stride, heads, head_stride, head_dim))
        return clq::set_error(CLQ_ERR_SHAPE, "rows of strides (%lld, %lld) overlap (%lld positions, %d heads of %d)",
                              (long long)pos_stride, (long long)head_stride, (long long)count, heads, head_dim);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return kv_fail(CLQ_ERR_NO_DEVICE, "no CUDA device");
    const int64_t n = count * heads * (rope_dims / 2);
    clq::rope_kernel<<<clq::grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(
        x, count, heads, pos_stride, head_stride, rope_dims, start, theta, factors, pairing == CLQ_ROPE_NEOX);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "RoPE launch: %s", cudaGetErrorString(e));
    return CLQ_OK;
}

int clq_attend_device(const float* q, int64_t count, int n_heads, int64_t q_pos_stride, const clq_kv_cache* c, int layer,
                      int64_t end, int64_t query_start, float* out, int64_t ldo, void* stream) {
    if (!c) return kv_fail(CLQ_ERR_ARGUMENT, "null cache");
    if (layer < 0 || layer >= c->layers) return clq::set_error(CLQ_ERR_ARGUMENT, "layer %d outside 0..%d", layer, c->layers - 1);
    if (count < 0 || query_start < 0) return kv_fail(CLQ_ERR_SHAPE, "negative query rows or start");
    if (n_heads < c->kvh || n_heads % c->kvh || n_heads / c->kvh > clq::kMaxGroup ||
        ((n_heads / c->kvh) & (n_heads / c->kvh - 1)))
        return clq::set_error(CLQ_ERR_SHAPE, "%d query heads over %d KV heads (groups of 1, 2, 4, 8 or 16)", n_heads, c->kvh);
    if (c->hd > clq::kMaxHeadDim) return clq::set_error(CLQ_ERR_UNSUPPORTED, "head dimension %d above %d", c->hd, clq::kMaxHeadDim);
    if (end < 1 || end > c->n_ctx) return clq::set_error(CLQ_ERR_SHAPE, "prefix %lld of a %lld context", (long long)end, (long long)c->n_ctx);
    if (q_pos_stride < (int64_t)n_heads * c->hd || ldo < (int64_t)n_heads * c->hd)
        return clq::set_error(CLQ_ERR_SHAPE, "query or output row stride below %d heads of %d", n_heads, c->hd);
    if (count == 0) return CLQ_OK;
    if (!q || !out) return kv_fail(CLQ_ERR_ARGUMENT, "null query or output");
    int rc;
    if ((rc = kv_check_device(c))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    clq::AttnParams P = {};
    P.q = q;
    P.q_ps = q_pos_stride;
    const uint8_t* kb = kv_buffer(c, layer, 0);
    const uint8_t* vb = kv_buffer(c, layer, 1);
    P.keys = kb;
    P.values = vb;
    P.kscale = c->type == CLQ_KV_Q8 ? reinterpret_cast<const float*>(kb + c->code_bytes) : nullptr;
    P.vscale = c->type == CLQ_KV_Q8 ? reinterpret_cast<const float*>(vb + c->code_bytes) : nullptr;
    P.end = end;
    P.query_start = query_start;
    P.n_heads = n_heads;
    P.kvh = c->kvh;
    P.hd = c->hd;
    P.groups = c->groups;
    P.scale = 1.f / sqrtf((float)c->hd);  // local/blocks.lisp:311
    // positions split so that the grid covers the SMs about twice, at most 64 a CTA
    const int64_t ctas_per_split = (int64_t)c->kvh * count;
    int64_t splits = (2 * (int64_t)clq::sm_count() + ctas_per_split - 1) / ctas_per_split;
    const int64_t min_splits = (end + clq::kSplitRows - 1) / clq::kSplitRows;
    if (splits < min_splits) splits = min_splits;
    if (splits > (end + 15) / 16) splits = (end + 15) / 16 > min_splits ? (end + 15) / 16 : min_splits;
    if (splits > clq::kMaxSplits)
        return clq::set_error(CLQ_ERR_UNSUPPORTED, "prefix %lld above %d positions", (long long)end,
                              clq::kMaxSplits * clq::kSplitRows);
    if (splits > 65535 || count > 65535) return kv_fail(CLQ_ERR_UNSUPPORTED, "too many query rows or positions for one launch");
    P.splits = (int)splits;
    P.per_split = (end + splits - 1) / splits;
    float* part = nullptr;
    cudaError_t e = clq::keep_pool_memory();
    if (e == cudaSuccess) e = cudaMallocAsync((void**)&part, (size_t)count * n_heads * splits * (c->hd + 2) * sizeof(float), s);
    if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "attention scratch: %s", cudaGetErrorString(e));
    P.part = part;
    const dim3 grid((unsigned)splits, (unsigned)c->kvh, (unsigned)count);
    const int G = n_heads / c->kvh;
    const size_t smem = clq::attend_smem(G, c->hd);
    e = c->type == CLQ_KV_Q8 ? clq::launch_split<true>(G, grid, smem, s, P) : clq::launch_split<false>(G, grid, smem, s, P);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e == cudaSuccess) {
        clq::attend_merge_kernel<<<dim3((unsigned)n_heads, (unsigned)count, (unsigned)((c->hd + 31) / 32)), 32, 0, s>>>(
            part, n_heads, c->hd, (int)splits, out, ldo);
        e = cudaGetLastError();
    }
    const cudaError_t f = cudaFreeAsync(part, s);
    if (e == cudaSuccess) e = f;
    if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
    return CLQ_OK;
}

}  // extern "C"
