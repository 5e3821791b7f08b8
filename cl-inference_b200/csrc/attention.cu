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
#include <mutex>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/clq.h"
#include "clq_internal.h"

namespace clq {
namespace {

constexpr int kQ8Group = 32;          // local/kv-cache.lisp:20
constexpr int kAttnThreads = 128;     // 4 warps per CTA
constexpr int kMaxGroup = 16;         // query heads per KV head
constexpr int kMaxPerSplit = 256;     // positions per CTA
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
__global__ void kv_store_q8_kernel(int8_t* __restrict__ codes, float* __restrict__ scales,
                                   const float* __restrict__ src, int64_t count, int kvh, int hd,
                                   int64_t ps, int64_t hs, int64_t start, int* err) {
    const int groups = (hd + kQ8Group - 1) / kQ8Group;
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

__global__ void kv_store_f32_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t count, int kvh,
                                    int hd, int64_t ps, int64_t hs, int64_t start) {
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

template <bool Q8>
__device__ __forceinline__ float kv_at(const AttnParams& P, const void* buf, const float* scl, int64_t pos, int kv,
                                       int e) {
    const int64_t slot = pos * P.kvh + kv;
    if constexpr (Q8) {
        const int8_t c = reinterpret_cast<const int8_t*>(buf)[slot * P.hd + e];
        return q8_decode(c, scl[slot * P.groups + e / kQ8Group]);
    } else {
        return reinterpret_cast<const float*>(buf)[slot * P.hd + e];
    }
}

// CTA (split, kv head, query row).  Scores s = (q . k) * scale for the
// group's query heads over the split's unmasked positions (key position <=
// query_start + row), kept in shared memory; then the split's maximum m,
// the sum l of exp(s - m) and the sum of exp(s - m) * v.
template <bool Q8>
__global__ void __launch_bounds__(kAttnThreads) attend_split_kernel(const AttnParams P) {
    __shared__ float qs[kMaxGroup * kMaxHeadDim];
    __shared__ float sc[kMaxGroup * kMaxPerSplit];
    const int split = blockIdx.x, kv = blockIdx.y;
    const int64_t row = blockIdx.z;
    const int G = P.n_heads / P.kvh, hd = P.hd;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int NW = kAttnThreads / 32;
    const int64_t last = P.query_start + row + 1 < P.end ? P.query_start + row + 1 : P.end;  // causal
    const int64_t p0 = (int64_t)split * P.per_split;
    int64_t p1 = p0 + P.per_split;
    if (p1 > last) p1 = last;
    const int np = p1 > p0 ? (int)(p1 - p0) : 0;

    for (int e = threadIdx.x; e < G * hd; e += kAttnThreads) {
        const int g = e / hd, d = e - g * hd;
        qs[e] = P.q[row * P.q_ps + (int64_t)(kv * G + g) * hd + d];
    }
    __syncthreads();

    // scores: a warp per position, lanes over the head dimension
    for (int j = warp; j < np; j += NW) {
        float dot[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) dot[g] = 0.f;
        for (int d = lane; d < hd; d += 32) {
            const float k = kv_at<Q8>(P, P.keys, P.kscale, p0 + j, kv, d);
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++)
                if (g < G) dot[g] = fmaf(qs[g * hd + d], k, dot[g]);
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g >= G) break;
            float v = dot[g];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) sc[g * kMaxPerSplit + j] = __fmul_rn(v, P.scale);
        }
    }
    __syncthreads();

    // the split's maximum and sum per query head: warp g handles heads g, g + NW, ...
    for (int g = warp; g < G; g += NW) {
        float m = -INFINITY;
        for (int j = lane; j < np; j += 32) m = fmaxf(m, sc[g * kMaxPerSplit + j]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        float l = 0.f;
        for (int j = lane; j < np; j += 32) {
            const float p = expf(sc[g * kMaxPerSplit + j] - m);
            sc[g * kMaxPerSplit + j] = p;
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
        float acc[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) acc[g] = 0.f;
        for (int j = 0; j < np; j++) {
            const float v = kv_at<Q8>(P, P.values, P.vscale, p0 + j, kv, d);
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++)
                if (g < G) acc[g] = fmaf(sc[g * kMaxPerSplit + j], v, acc[g]);
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g >= G) break;
            P.part[(((row * P.n_heads) + kv * G + g) * P.splits + split) * (int64_t)(hd + 2) + d] = acc[g];
        }
    }
}

// One CTA per (query row, head): merges the splits -- M = max m_s, output
// sum_s exp(m_s - M) acc_s / sum_s exp(m_s - M) l_s -- into out[row][head * hd + d].
__global__ void attend_merge_kernel(const float* __restrict__ part, int n_heads, int hd, int splits,
                                    float* __restrict__ out, int64_t ldo) {
    const int head = blockIdx.x;
    const int64_t row = blockIdx.y;
    const float* base = part + ((row * n_heads) + head) * (int64_t)splits * (hd + 2);
    float M = -INFINITY;
    for (int s = 0; s < splits; s++) {
        const float l = base[s * (int64_t)(hd + 2) + hd + 1];
        if (l > 0.f) M = fmaxf(M, base[s * (int64_t)(hd + 2) + hd]);
    }
    float L = 0.f;
    for (int s = 0; s < splits; s++) {
        const float l = base[s * (int64_t)(hd + 2) + hd + 1];
        if (l > 0.f) L += expf(base[s * (int64_t)(hd + 2) + hd] - M) * l;
    }
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float a = 0.f;
        for (int s = 0; s < splits; s++) {
            const float l = base[s * (int64_t)(hd + 2) + hd + 1];
            if (l > 0.f) a += expf(base[s * (int64_t)(hd + 2) + hd] - M) * base[s * (int64_t)(hd + 2) + d];
        }
        out[row * ldo + (int64_t)head * hd + d] = a / L;
    }
}

__global__ void fill_kernel(float* __restrict__ p, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
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
    for (int which = 0; which < 2; which++) {
        const float* src = which ? v : k;
        uint8_t* buf = kv_buffer(c, layer, which);
        if (c->type == CLQ_KV_F32) {
            const int64_t n = count * c->kvh * c->hd;
            clq::kv_store_f32_kernel<<<clq::grid_for(n, 256), 256, 0, s>>>(reinterpret_cast<float*>(buf), src, count, c->kvh,
                                                                            c->hd, pos_stride, head_stride, start);
        } else {
            const int64_t warps = count * c->kvh * c->groups;
            clq::kv_store_q8_kernel<<<clq::grid_for(warps * 32, 256), 256, 0, s>>>(
                reinterpret_cast<int8_t*>(buf), reinterpret_cast<float*>(buf + c->code_bytes), src, count, c->kvh, c->hd,
                pos_stride, head_stride, start, c->err);
        }
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "KV cache store: %s", cudaGetErrorString(e));
    }
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
    if (n_heads < c->kvh || n_heads % c->kvh || n_heads / c->kvh > clq::kMaxGroup)
        return clq::set_error(CLQ_ERR_SHAPE, "%d query heads over %d KV heads (groups of at most %d)", n_heads, c->kvh,
                              clq::kMaxGroup);
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
    // positions split so that the grid covers the SMs about twice, at most 256 a CTA
    const int64_t ctas_per_split = (int64_t)c->kvh * count;
    int64_t splits = (2 * (int64_t)clq::sm_count() + ctas_per_split - 1) / ctas_per_split;
    const int64_t min_splits = (end + clq::kMaxPerSplit - 1) / clq::kMaxPerSplit;
    if (splits < min_splits) splits = min_splits;
    if (splits > (end + 15) / 16) splits = (end + 15) / 16 > min_splits ? (end + 15) / 16 : min_splits;
    if (splits > 65535 || count > 65535) return kv_fail(CLQ_ERR_UNSUPPORTED, "too many query rows or positions for one launch");
    P.splits = (int)splits;
    P.per_split = (end + splits - 1) / splits;
    float* part = nullptr;
    cudaError_t e = clq::keep_pool_memory();
    if (e == cudaSuccess) e = cudaMallocAsync((void**)&part, (size_t)count * n_heads * splits * (c->hd + 2) * sizeof(float), s);
    if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "attention scratch: %s", cudaGetErrorString(e));
    P.part = part;
    const dim3 grid((unsigned)splits, (unsigned)c->kvh, (unsigned)count);
    if (c->type == CLQ_KV_Q8) clq::attend_split_kernel<true><<<grid, clq::kAttnThreads, 0, s>>>(P);
    else clq::attend_split_kernel<false><<<grid, clq::kAttnThreads, 0, s>>>(P);
    e = cudaGetLastError();
    if (e == cudaSuccess) {
        clq::attend_merge_kernel<<<dim3((unsigned)n_heads, (unsigned)count), 128, 0, s>>>(part, n_heads, c->hd, (int)splits,
                                                                                          out, ldo);
        e = cudaGetLastError();
    }
    const cudaError_t f = cudaFreeAsync(part, s);
    if (e == cudaSuccess) e = f;
    if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
    return CLQ_OK;
}

}  // extern "C"
