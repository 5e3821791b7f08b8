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
// Attention is split over positions (flash-decoding): a CTA takes a block of
// query rows, one KV head and a range of 32 or 64 positions, stages each
// key and value row of the range once (bulk copies for f32 rows) for all the
// query heads of that KV head and all the rows of the block, and leaves the
// range's softmax maximum, sum and weighted value sum; a second launch merges
// the ranges of each (row, head).  A prefix that fits one range is written
// directly.  The cache is read once per block of query rows.
#include <cfloat>
#include <cmath>
#include <cstdint>

#include <cstdlib>
#include <cuda_runtime.h>

#include "../../include/clq.h"
#include "clq_internal.h"
#include "pipeline.cuh"

namespace clq {
namespace {

constexpr int kQ8Group = 32;          // local/kv-cache.lisp:20
constexpr int kMergeThreads = 256;
constexpr int kMaxGroup = 16;         // query heads per KV head
// A CTA stages SR = 32 or 64 positions and runs SR / 8 warps (8 positions each).
constexpr int kMaxSplits = 2048;      // position ranges merged per (row, head)
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
    pipe::allow_dependents();
    pipe::grid_dependency_wait();  // the rows may come from the previous kernel
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
    pipe::allow_dependents();
    pipe::grid_dependency_wait();  // the rows may come from the previous kernel
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
// (2i, 2i + 1) (adjacent) or (i, i + rope_dims / 2) (neox).  Under
// programmatic dependent launch the first angle's cos and sin are formed
// before the wait for the kernel that wrote the rows.
__global__ void rope_kernel(float* __restrict__ x, int64_t count, int heads, int64_t ps, int64_t hs, int rope_dims,
                            int64_t start, double theta, const float* __restrict__ factors, int neox) {
    pipe::allow_dependents();
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
        pipe::grid_dependency_wait();  // returns at once after the first time
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
    int64_t count;         // query rows
    int64_t end;           // keys in the prefix
    int64_t query_start;   // position of query row 0
    int n_heads, kvh, hd, groups;
    int gshift;            // log2 of the query heads per KV head
    int rows;              // query rows per CTA: rows << gshift query vectors
    int splits;
    int64_t per_split;
    float scale;           // 1 / sqrt(hd), rounded to f32
    float* acc;            // [count][n_heads][splits][hd]: the splits' weighted value sums
    float2* ml;            // [count][n_heads][splits]: their (max, sum)
    float* out;            // one split: the output rows, stride ldo
    int64_t ldo;
    int bulk;              // f32 rows staged by bulk copies
    int* err;              // device status word (a staging wait that gave up)
};

// Staged key rows are hd + 16 floats apart, so that the two positions of a
// quarter warp (4 lanes each, float4 columns 16 apart) fall in distinct banks.
__host__ __device__ constexpr int key_ld(int hd) { return hd + 16; }
// Query rows in shared memory: hd rounded up to 4 floats (16-byte rows).
__host__ __device__ constexpr int query_ld(int hd) { return (hd + 3) & ~3; }

// The split's key and value rows of one KV head into shared memory as f32
// (key rows LDK floats apart, value rows hd apart): every thread issues its
// 16-byte loads (4 f32 or 16 codes) of both before any is used, so the split
// costs about one memory round trip.
template <bool Q8, int T>
__device__ __forceinline__ void stage_kv(const AttnParams& P, int64_t p0, int np, int kv, float* ks, int ldk, float* vs) {
    const int hd = P.hd;
    if (hd % (Q8 ? 16 : 4)) {  // rows off the 16-byte grid: element by element
        const int n = np * hd;
        for (int e = threadIdx.x; e < 2 * n; e += T) {
            const bool val = e >= n;
            const int f = val ? e - n : e, j = f / hd, d = f - j * hd;
            const int64_t slot = (p0 + j) * P.kvh + kv;
            float* dst = val ? vs + j * hd + d : ks + j * ldk + d;
            if constexpr (Q8) {
                const int8_t* codes = reinterpret_cast<const int8_t*>(val ? P.values : P.keys);
                *dst = q8_decode(codes[slot * hd + d], (val ? P.vscale : P.kscale)[slot * P.groups + d / kQ8Group]);
            } else {
                *dst = reinterpret_cast<const float*>(val ? P.values : P.keys)[slot * hd + d];
            }
        }
        return;
    }
    // vector rows: eight 16-byte loads per thread in flight before any store
    constexpr int B = 8;
    const int per_row = hd / (Q8 ? 16 : 4), n = np * per_row;
    for (int e0 = threadIdx.x; e0 < 2 * n; e0 += B * T) {
        uint4 w[B];
        float sc[B];
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int e = e0 + b * T;
            if (e < 2 * n) {
                const bool val = e >= n;
                const int f = val ? e - n : e, j = f / per_row, c = f - j * per_row;
                const int64_t slot = (p0 + j) * P.kvh + kv;
                const int8_t* row = reinterpret_cast<const int8_t*>(val ? P.values : P.keys) + slot * hd * (Q8 ? 1 : 4);
                w[b] = *reinterpret_cast<const uint4*>(row + c * 16);
                if constexpr (Q8) sc[b] = (val ? P.vscale : P.kscale)[slot * P.groups + (c * 16) / kQ8Group];
            }
        }
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int e = e0 + b * T;
            if (e < 2 * n) {
                const bool val = e >= n;
                const int f = val ? e - n : e, j = f / per_row, c = f - j * per_row;
                if constexpr (Q8) {
                    const uint32_t ws[4] = {w[b].x, w[b].y, w[b].z, w[b].w};
                    float4* o = reinterpret_cast<float4*>((val ? vs + j * hd : ks + j * ldk) + c * 16);
                    // q8_decode's single-precision case for all 16 codes at once
                    const bool fast = (double)sc[b] <= (double)FLT_MAX / 127.0;
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        float f[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int8_t code = (int8_t)(ws[q] >> (8 * i));
                            f[i] = fast ? __fmul_rn((float)code, sc[b]) : q8_decode(code, sc[b]);
                        }
                        o[q] = make_float4(f[0], f[1], f[2], f[3]);
                    }
                } else {
                    *reinterpret_cast<uint4*>((val ? vs + j * hd : ks + j * ldk) + c * 4) = w[b];
                }
            }
        }
    }
}

__device__ __forceinline__ void fma4(float4& a, float p, const float4& x) {
    a.x = fmaf(p, x.x, a.x);
    a.y = fmaf(p, x.y, a.y);
    a.z = fmaf(p, x.z, a.z);
    a.w = fmaf(p, x.w, a.w);
}

// CTA (split, KV head, block of query rows): the QV = rows * G query vectors
// of `rows` consecutive query rows and the G query heads of one KV head.  The
// split's key and value rows are staged once -- f32 rows by bulk copies on one
// barrier, otherwise by 16-byte vector loads -- and serve every query vector:
//   scores   4 lanes per position, each a quarter of the head dimension
//            (float4 columns 16 apart), summed by two shuffles, times scale;
//   softmax  a warp per query vector over its unmasked positions (key
//            position <= query_start + row): m = max, p = exp(s - m), l = sum p;
//   values   a thread per (query vector, 4 dimensions) and share of the
//            positions; the shares summed in a fixed order.
// One split writes acc / l to the output rows; otherwise (acc, m, l) go to
// scratch for attend_merge_kernel.  HD: the head dimension when it is 64 or
// 128 (constant strides and trip counts), 0 for any other.  Under
// programmatic dependent launch nothing is read before the previous grid
// completes.
template <bool Q8, int QV, int HD, int SR>
__global__ void __launch_bounds__(SR * 4, SR == 32 ? 4 : 2) attend_split_kernel(const AttnParams P) {
    extern __shared__ __align__(16) float sh[];
    constexpr int T = SR * 4, NW = T / 32;  // one pass of 8 positions per warp covers a split
    const int split = blockIdx.x, kv = blockIdx.y;
    const int64_t r0 = (int64_t)blockIdx.z * P.rows;
    const int hd = HD ? HD : P.hd, ld = key_ld(hd), qld = query_ld(hd);
    const int gs = P.gshift, G = 1 << gs;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sh);  // the bulk copies' barrier (16 bytes)
    float* qs = sh + 4;                     // [QV][qld]
    float* sc = qs + QV * qld;              // [QV][SR]: scores, then weights
    float* mls = sc + QV * SR;      // [QV][4]: max, sum
    float* ks = mls + 4 * QV;               // [SR][ld]; after the scores, value partials
    float* vs = ks + SR * ld;       // [SR][hd]

    // positions [p0, p1) of this split that some row of the block may attend
    const int64_t last_row = (r0 + P.rows < P.count ? r0 + P.rows : P.count) - 1;
    const int64_t lim = P.query_start + last_row + 1 < P.end ? P.query_start + last_row + 1 : P.end;  // causal
    const int64_t p0 = (int64_t)split * P.per_split;
    const int64_t p1 = p0 + P.per_split < lim ? p0 + P.per_split : lim;
    const int np = p1 > p0 ? (int)(p1 - p0) : 0;

    const bool bulk = !Q8 && P.bulk;
    if (bulk && threadIdx.x == 0) {
        pipe::mbar_init(bar, 1);
        pipe::mbar_init_fence();
    }
    pipe::grid_dependency_wait();  // the queries and the cache rows may come from the previous kernels
    if (bulk) {
        __syncthreads();
        if (warp == 0 && np > 0) {  // every row of the split in flight on one barrier
            const uint32_t rb = (uint32_t)hd * 4u;
            if (lane == 0) pipe::mbar_arrive_tx(bar, 2u * (uint32_t)np * rb);
            __syncwarp();
            for (int j = lane; j < np; j += 32) {
                const int64_t slot = (p0 + j) * P.kvh + kv;
                pipe::bulk_copy(ks + j * ld, reinterpret_cast<const float*>(P.keys) + slot * hd, rb, bar);
                pipe::bulk_copy(vs + j * hd, reinterpret_cast<const float*>(P.values) + slot * hd, rb, bar);
            }
        }
    }
    for (int e = threadIdx.x; e < QV * hd; e += T) {
        const int v = e / hd, d = e - v * hd;
        const int64_t row = r0 + (v >> gs);
        qs[v * qld + d] = row < P.count ? P.q[row * P.q_ps + (int64_t)(kv * G + (v & (G - 1))) * hd + d] : 0.f;
    }
    if (bulk) {
        if (np > 0 && !pipe::mbar_wait(bar, 0, P.err)) pipe::mbar_drain(bar, 0);
    } else {
        stage_kv<Q8, T>(P, p0, np, kv, ks, ld, vs);
    }
    __syncthreads();
    pipe::allow_dependents();

    // scores: position j = 8 warp + lane / 4, lane c = lane % 4 takes the
    // float4 columns 16 i + 4 c (and the scalar tail d = c mod 4)
    {
        const int c = lane & 3, j = warp * 8 + (lane >> 2);
        const int nfull = (hd & 3) ? 0 : hd >> 4;
        const float* kr = ks + j * ld;
        float dot[QV];
#pragma unroll
        for (int v = 0; v < QV; v++) dot[v] = 0.f;
        for (int i = 0; i < nfull; i++) {
            const int d = 16 * i + 4 * c;
            const float4 k = *reinterpret_cast<const float4*>(kr + d);
#pragma unroll
            for (int v = 0; v < QV; v++) {
                const float4 q = *reinterpret_cast<const float4*>(qs + v * qld + d);
                dot[v] = fmaf(q.x, k.x, dot[v]);
                dot[v] = fmaf(q.y, k.y, dot[v]);
                dot[v] = fmaf(q.z, k.z, dot[v]);
                dot[v] = fmaf(q.w, k.w, dot[v]);
            }
        }
        for (int d = 16 * nfull + c; d < hd; d += 4) {
            const float k = kr[d];
#pragma unroll
            for (int v = 0; v < QV; v++) dot[v] = fmaf(qs[v * qld + d], k, dot[v]);
        }
#pragma unroll
        for (int v = 0; v < QV; v++) {
            dot[v] += __shfl_xor_sync(0xffffffffu, dot[v], 1);
            dot[v] += __shfl_xor_sync(0xffffffffu, dot[v], 2);
            if ((v & 3) == c && j < np) sc[v * SR + j] = __fmul_rn(dot[v], P.scale);
        }
    }
    __syncthreads();

    // softmax pieces per query vector: a warp each
    for (int v = warp; v < QV; v += NW) {
        const int64_t row = r0 + (v >> gs);
        int nv = 0;  // this vector's unmasked positions of the split
        if (row < P.count) {
            const int64_t lv = P.query_start + row + 1 < P.end ? P.query_start + row + 1 : P.end;
            nv = lv - p0 < 0 ? 0 : (lv - p0 > np ? np : (int)(lv - p0));
        }
        float* s = sc + v * SR;
        float m = -INFINITY;
        for (int j = lane; j < nv; j += 32) m = fmaxf(m, s[j]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        float l = 0.f;
        for (int j = lane; j < SR; j += 32) {
            const float p = j < nv ? expf(s[j] - m) : 0.f;
            s[j] = p;
            l += p;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (lane == 0) {
            mls[4 * v] = m;
            mls[4 * v + 1] = l;
            if (P.splits > 1 && row < P.count)
                P.ml[(row * P.n_heads + kv * G + (v & (G - 1))) * P.splits + split] = make_float2(m, l);
        }
    }
    __syncthreads();

    // weighted value sums: W = QV x (hd / cw) columns of cw dimensions, each
    // over the positions j = share (mod PS); the PS shares then summed in order
    const int cw = (hd & 3) ? 1 : 4, nc = hd / cw, W = QV * nc;
    const int PS = W >= T ? 1 : T / W;
    float4* red = reinterpret_cast<float4*>(ks);  // [PS][W], the keys being done with
    auto emit = [&](int w, float4 a) {
        const int v = w / nc, col = w - v * nc;
        const int64_t row = r0 + (v >> gs);
        if (row >= P.count) return;
        const int head = kv * G + (v & (G - 1));
        const float o[4] = {a.x, a.y, a.z, a.w};
        if (P.splits == 1) {
            const float l = mls[4 * v + 1];
            float* dst = P.out + row * P.ldo + (int64_t)head * hd + col * cw;
            for (int i = 0; i < cw; i++) dst[i] = o[i] / l;
        } else {
            float* dst = P.acc + ((row * P.n_heads + head) * P.splits + split) * (int64_t)hd + col * cw;
            if (cw == 4) *reinterpret_cast<float4*>(dst) = a;
            else dst[0] = o[0];
        }
    };
    for (int t = threadIdx.x; t < PS * W; t += T) {
        const int w = t % W, ps = t / W;
        const int v = w / nc, col = w - v * nc;
        const float* pv = sc + v * SR;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        if (cw == 4) {
            for (int j = ps; j < np; j += PS) fma4(a, pv[j], *reinterpret_cast<const float4*>(vs + j * hd + 4 * col));
        } else {
            for (int j = ps; j < np; j += PS) a.x = fmaf(pv[j], vs[j * hd + col], a.x);
        }
        if (PS > 1) red[t] = a;
        else emit(w, a);
    }
    if (PS > 1) {
        __syncthreads();
        for (int w = threadIdx.x; w < W; w += T) {
            float4 a = red[w];
            for (int ps = 1; ps < PS; ps++) {
                const float4 b = red[ps * W + w];
                a.x += b.x;
                a.y += b.y;
                a.z += b.z;
                a.w += b.w;
            }
            emit(w, a);
        }
    }
}

size_t attend_smem(int QV, int hd, int SR) {
    return 16 + ((size_t)QV * query_ld(hd) + (size_t)QV * SR + 4 * (size_t)QV + (size_t)SR * key_ld(hd) + (size_t)SR * hd) *
                    sizeof(float);
}

// CTA per (head, query row): thread (column, split group) first puts the
// weighted sums of its first eight splits in flight; meanwhile every split's
// (m, l) gives M = max m_s over the non-empty splits, the weights
// w_s = exp(m_s - M) (0 for an empty split) and L = sum w_s l_s.  Each thread
// sums w_s acc_s over its splits, the groups are summed in order, and the
// output is acc / L.
__global__ void __launch_bounds__(kMergeThreads) attend_merge_kernel(const float* __restrict__ acc,
                                                                     const float2* __restrict__ ml, int n_heads, int hd,
                                                                     int splits, float* __restrict__ out, int64_t ldo) {
    __shared__ float wgt[kMaxSplits];
    __shared__ float lsum[kMaxSplits];
    __shared__ float4 part[kMergeThreads];
    __shared__ float red[kMergeThreads / 32];
    constexpr int NW = kMergeThreads / 32, B = 8;
    static_assert(kMaxHeadDim <= kMergeThreads, "one (column, split group) per thread");
    const int head = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row = blockIdx.y;
    const int64_t base = (row * n_heads + head) * (int64_t)splits;
    const int cw = (hd & 3) ? 1 : 4, nc = hd / cw, SG = kMergeThreads / nc;
    const int col = threadIdx.x % nc, sg = threadIdx.x / nc;
    const bool active = sg < SG;
    const float* src = acc + base * hd + col * cw;
    auto load = [&](float4* x, int s0) {
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int s = s0 + b * SG;
            x[b] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (active && s < splits) {
                if (cw == 4) x[b] = *reinterpret_cast<const float4*>(src + (int64_t)s * hd);
                else x[b].x = src[(int64_t)s * hd];
            }
        }
    };

    pipe::grid_dependency_wait();  // the split kernel's partials
    pipe::allow_dependents();
    float4 x[B];
    load(x, sg);
    float m = -INFINITY;
    for (int s = threadIdx.x; s < splits; s += kMergeThreads) {
        const float2 v = ml[base + s];
        lsum[s] = v.y;
        wgt[s] = v.y > 0.f ? v.x : -INFINITY;
        m = fmaxf(m, wgt[s]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int w = 1; w < NW; w++) m = fmaxf(m, red[w]);
    __syncthreads();
    float L = 0.f;
    for (int s = threadIdx.x; s < splits; s += kMergeThreads) {
        const float w = lsum[s] > 0.f ? expf(wgt[s] - m) : 0.f;
        wgt[s] = w;
        L = fmaf(w, lsum[s], L);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    if (lane == 0) red[warp] = L;
    __syncthreads();
    L = red[0];
#pragma unroll
    for (int w = 1; w < NW; w++) L += red[w];

    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = sg;; s0 += B * SG) {  // splits s0, s0 + SG, ... in order
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int s = s0 + b * SG;
            if (active && s < splits) fma4(a, wgt[s], x[b]);
        }
        if (s0 + B * SG >= splits) break;
        load(x, s0 + B * SG);
    }
    if (active) part[threadIdx.x] = a;
    __syncthreads();
    if (threadIdx.x < nc) {
        a = part[threadIdx.x];
        for (int g = 1; g < SG; g++) {
            const float4 b = part[g * nc + threadIdx.x];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        const float o[4] = {a.x, a.y, a.z, a.w};
        float* dst = out + row * ldo + (int64_t)head * hd + threadIdx.x * cw;
        for (int i = 0; i < cw; i++) dst[i] = o[i] / L;
    }
}

__global__ void fill_kernel(float* __restrict__ p, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
}

template <typename Kern>
cudaError_t attend_smem_limit(Kern kern, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

// KERN<<<GRID, THREADS, SMEM, S>>>(ARGS...), a programmatic dependent launch
// unless CLQ_PDL=0.
template <typename... Args>
cudaError_t launch_pdl(void (*kern)(Args...), dim3 grid, int threads, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = gemv_pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <bool Q8, int QV, int HD, int SR>
cudaError_t launch_split_sr(dim3 grid, size_t smem, cudaStream_t s, const AttnParams& P) {
    const cudaError_t e = attend_smem_limit(attend_split_kernel<Q8, QV, HD, SR>, smem);
    return e != cudaSuccess ? e : launch_pdl(attend_split_kernel<Q8, QV, HD, SR>, grid, SR * 4, smem, s, P);
}
template <bool Q8, int QV, int HD>
cudaError_t launch_split_hd(int sr, dim3 grid, size_t smem, cudaStream_t s, const AttnParams& P) {
    return sr == 32 ? launch_split_sr<Q8, QV, HD, 32>(grid, smem, s, P) : launch_split_sr<Q8, QV, HD, 64>(grid, smem, s, P);
}
template <bool Q8, int QV>
cudaError_t launch_split_qv(int sr, dim3 grid, size_t smem, cudaStream_t s, const AttnParams& P) {
    switch (P.hd) {
    case 64: return launch_split_hd<Q8, QV, 64>(sr, grid, smem, s, P);
    case 128: return launch_split_hd<Q8, QV, 128>(sr, grid, smem, s, P);
    default: return launch_split_hd<Q8, QV, 0>(sr, grid, smem, s, P);
    }
}
// The split kernel for QV query vectors (1, 2, 4, 8 or 16) and SR positions per CTA.
template <bool Q8>
cudaError_t launch_split(int QV, int sr, dim3 grid, size_t smem, cudaStream_t s, const AttnParams& P) {
    switch (QV) {
    case 1: return launch_split_qv<Q8, 1>(sr, grid, smem, s, P);
    case 2: return launch_split_qv<Q8, 2>(sr, grid, smem, s, P);
    case 4: return launch_split_qv<Q8, 4>(sr, grid, smem, s, P);
    case 8: return launch_split_qv<Q8, 8>(sr, grid, smem, s, P);
    case 16: return launch_split_qv<Q8, 16>(sr, grid, smem, s, P);
    default: return cudaErrorNotSupported;
    }
}

// CLQ_ATTN_BULK=0 stages f32 key and value rows with vector loads instead of
// bulk copies.
bool attn_bulk_enabled() {
    static const bool on = [] {
        const char* v = getenv("CLQ_ATTN_BULK");
        return !(v && v[0] == '0');
    }();
    return on;
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
    cudaError_t e;
    if (c->type == CLQ_KV_F32) {
        const int64_t n = count * c->kvh * c->hd;
        e = clq::launch_pdl(clq::kv_store_f32_kernel, dim3(clq::grid_for(n, 256), 2), 256, 0, s, S, (int64_t)count,
                            (int)c->kvh, (int)c->hd, (int64_t)pos_stride, (int64_t)head_stride, (int64_t)start);
    } else {
        const int64_t warps = count * c->kvh * c->groups;
        e = clq::launch_pdl(clq::kv_store_q8_kernel, dim3(clq::grid_for(warps * 32, 256), 2), 256, 0, s, S,
                            (int64_t)count, (int)c->kvh, (int)c->hd, (int64_t)pos_stride, (int64_t)head_stride,
                            (int64_t)start, (int*)c->err);
    }
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
    const cudaError_t e = clq::launch_pdl(clq::rope_kernel, dim3(clq::grid_for(n, 256)), 256, 0, (cudaStream_t)stream, x,
                                          (int64_t)count, (int)heads, (int64_t)pos_stride, (int64_t)head_stride,
                                          (int)rope_dims, (int64_t)start, (double)theta, (const float*)factors,
                                          (int)(pairing == CLQ_ROPE_NEOX));
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
    const int G = n_heads / c->kvh;
    const bool q8 = c->type == CLQ_KV_Q8;
    P.count = count;
    P.bulk = !q8 && clq::attn_bulk_enabled() && c->hd % 4 == 0 && ((uintptr_t)kb | (uintptr_t)vb) % 16 == 0;
    P.err = clq::device_status_word();
    // query rows per CTA: up to 16 query vectors (rows x G) share one staging
    int rows = 1;
    while (rows * 2 * G <= 16 && rows < count) rows *= 2;
    P.rows = rows;
    while ((1 << P.gshift) < G) P.gshift++;
    const int QV = rows * G;
    const int64_t blocks = (count + rows - 1) / rows;
    // positions per CTA: 32 (twice the CTAs, each with less to do) unless
    // blocks of many query vectors over a long prefix, where the partials'
    // traffic grows with the split count
    int sr = QV <= 4 || end <= 1024 ? 32 : 64;
    if ((end + sr - 1) / sr > clq::kMaxSplits) sr = 64;
    // positions split so that the grid covers the SMs about twice, at most sr a CTA
    const int64_t ctas_per_split = (int64_t)c->kvh * blocks;
    int64_t splits = (2 * (int64_t)clq::sm_count() + ctas_per_split - 1) / ctas_per_split;
    const int64_t min_splits = (end + sr - 1) / sr;
    if (splits < min_splits) splits = min_splits;
    if (splits > (end + 15) / 16) splits = (end + 15) / 16 > min_splits ? (end + 15) / 16 : min_splits;
    if (splits > clq::kMaxSplits)
        return clq::set_error(CLQ_ERR_UNSUPPORTED, "prefix %lld above %d positions", (long long)end, clq::kMaxSplits * 64);
    if (blocks > 65535 || count > 65535) return kv_fail(CLQ_ERR_UNSUPPORTED, "too many query rows for one launch");
    P.splits = (int)splits;
    P.per_split = (end + splits - 1) / splits;
    P.out = out;
    P.ldo = ldo;
    const dim3 grid((unsigned)splits, (unsigned)c->kvh, (unsigned)blocks);
    const size_t smem = clq::attend_smem(QV, c->hd, sr);
    cudaError_t e = cudaSuccess;
    void* scratch = nullptr;
    if (splits > 1) {  // the splits' partials, merged by a second launch
        const size_t acc_bytes = ((size_t)count * n_heads * splits * c->hd * sizeof(float) + 15) & ~(size_t)15;
        e = clq::keep_pool_memory();
        if (e == cudaSuccess) e = cudaMallocAsync(&scratch, acc_bytes + (size_t)count * n_heads * splits * sizeof(float2), s);
        if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "attention scratch: %s", cudaGetErrorString(e));
        P.acc = static_cast<float*>(scratch);
        P.ml = reinterpret_cast<float2*>(static_cast<uint8_t*>(scratch) + acc_bytes);
    }
    e = q8 ? clq::launch_split<true>(QV, sr, grid, smem, s, P) : clq::launch_split<false>(QV, sr, grid, smem, s, P);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e == cudaSuccess && splits > 1) {
        e = clq::launch_pdl(clq::attend_merge_kernel, dim3((unsigned)n_heads, (unsigned)count), clq::kMergeThreads, 0, s,
                            (const float*)P.acc, (const float2*)P.ml, n_heads, c->hd, (int)splits, out, ldo);
    }
    if (scratch) {
        const cudaError_t f = cudaFreeAsync(scratch, s);
        if (e == cudaSuccess) e = f;
    }
    if (e != cudaSuccess) return clq::set_error(CLQ_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
    return CLQ_OK;
}

}  // extern "C"
