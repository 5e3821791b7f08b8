// gemv_mma.cu -- fused dequant + GEMV/skinny-GEMM for packed weights on the
// warp-level tensor-core MMA (mma.sync m16n8k16, fp16 operands, fp32 accumulate).
//
// Each warp owns 16 weight rows (the MMA's M) x 256 columns (one "chunk": a
// K-quant superblock or 8 Q4_0/Q8_0 blocks) per step of its loop; the
// activation rows (tokens) are the MMA's N, 8 per n-tile.  The fp16 operands
// are exact:
//   A  weight codes unpacked in registers with prmt/lop3 (OR the code bits into
//      the mantissa of 1024.0 or 64.0) and one f16x2 fma/sub to remove the bias
//      -- for Q4_K also times the 6-bit sub-block scale, sc*q < 2^10;
//   B  activations split as hi + lo fp16 (x = hi + lo to ~22 bits) after a
//      power-of-two scaling per (chunk, token) that puts max|x| in [2^14, 2^15).
// Block scales (fp16 d, dmin, Q6_K int8 sub-scales) multiply the fp32 MMA
// results, so the result carries fp32-class error, like an fp32 dot product.
// The CTA splits K across warps and reduces through shared memory; activations
// are staged once per CTA into shared memory in MMA-fragment order.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/clq.h"
#include "clq_internal.h"
#include "layout.cuh"

namespace clq {
namespace {

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// f16x2 constants
constexpr uint32_t kMagic = 0x64646464u;  // high byte of 1024.0 in every byte
constexpr uint32_t kH1024 = 0x64006400u;
constexpr uint32_t kH1032 = 0x64086408u;  // 1024 + 8
constexpr uint32_t kH1056 = 0x64206420u;  // 1024 + 32
constexpr uint32_t kH1152 = 0x64806480u;  // 1024 + 128
constexpr uint32_t kHSixteenth = 0x2C002C00u;
constexpr uint32_t kHNeg72 = 0xD480D480u;
constexpr uint32_t kHNeg96 = 0xD600D600u;
constexpr uint32_t kHNeg1024 = 0xE400E400u;
constexpr uint32_t kHNeg64 = 0xD400D400u;
constexpr uint32_t kLoNib = 0x640F640Fu;   // keep 0x64 exponent byte + low nibble
constexpr uint32_t kHiNib = 0x64F064F0u;   // keep 0x64 exponent byte + high nibble
constexpr uint32_t kSelLo = 0x4140u;       // bytes [a0, b0, a1, b0]
constexpr uint32_t kSelHi = 0x4342u;       // bytes [a2, b0, a3, b0]

// Element index (within the 256-element chunk) of the first of the 4
// consecutive elements lane-quad t feeds at MMA step s, and its inverse.
template <int D> struct Steps;
template <> struct Steps<kQ4_K> {  // s = 2j + h: sub-block 2t+h, l = 4j..4j+3
    __device__ static int pos(int s, int t) { return 32 * (2 * t + (s & 1)) + 4 * (s >> 1); }
    __device__ static void inv(int q, int& s, int& t) { int G = q >> 3, j = q & 7; t = G >> 1; s = 2 * j + (G & 1); }
};
template <> struct Steps<kQ6_K> {  // s = (2h + half)*4 + grp: l = 16 half + 4t
    __device__ static int pos(int s, int t) {
        int hh = s >> 2, grp = s & 3;
        return 128 * (hh >> 1) + 32 * grp + 16 * (hh & 1) + 4 * t;
    }
    __device__ static void inv(int q, int& s, int& t) {
        int h = q >> 5, grp = (q >> 3) & 3, half = (q >> 2) & 1;
        t = q & 3;
        s = (2 * h + half) * 4 + grp;
    }
};
template <> struct Steps<kQ4_0> {  // s = 2b + hn: block b, elements 16hn + 4t..
    __device__ static int pos(int s, int t) { return 32 * (s >> 1) + 16 * (s & 1) + 4 * t; }
    __device__ static void inv(int q, int& s, int& t) { t = q & 3; s = 2 * (q >> 3) + ((q >> 2) & 1); }
};
template <> struct Steps<kQ8_0> : Steps<kQ4_0> {};

// 32-bit words of weight data per thread per row per chunk.
template <int D> struct Words;
template <> struct Words<kQ4_K> { static constexpr int n = 12; };  // 16 B header + 32 B codes
template <> struct Words<kQ6_K> { static constexpr int n = 16; };  // 48 B codes + 16 B sub-scales
template <> struct Words<kQ4_0> { static constexpr int n = 12; };  // 32 B codes + 16 B d[8]
template <> struct Words<kQ8_0> { static constexpr int n = 20; };  // 64 B codes + 16 B d[8]

#define CLQ_PUT4(w, i, v) do { (w)[(i)] = (v).x; (w)[(i) + 1] = (v).y; (w)[(i) + 2] = (v).z; (w)[(i) + 3] = (v).w; } while (0)

template <int D>
__device__ __forceinline__ void load_chunk(const Planes& p, int64_t row, int64_t c, int t,
                                           uint32_t (&w)[Words<D>::n], uint32_t& dbits) {
    if (D == kQ4_K) {
        const uint8_t* b = p.q + (row * p.nb + c) * 144;
        uint4 v0 = ldg_stream(b), v1 = ldg_stream(b + 16 + 32 * t), v2 = ldg_stream(b + 32 + 32 * t);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2);
    } else if (D == kQ6_K) {
        const int64_t blk = row * p.nb + c;
        const uint8_t* b = p.q + blk * 192 + 48 * t;
        uint4 v0 = ldg_stream(b), v1 = ldg_stream(b + 16), v2 = ldg_stream(b + 32), v3 = ldg_stream(p.s + blk * 16);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2); CLQ_PUT4(w, 12, v3);
        dbits = *reinterpret_cast<const unsigned short*>(p.d + 2 * blk);
    } else if (D == kQ4_0) {
        const uint8_t* b = p.q + row * p.nb * 16 + c * 128 + 32 * t;
        uint4 v0 = ldg_stream(b), v1 = ldg_stream(b + 16), v2 = ldg_stream(p.d + 2 * (row * p.nb + 8 * c));
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2);
    } else {
        const uint8_t* b = p.q + row * p.nb * 32 + c * 256 + 64 * t;
        uint4 v0 = ldg_stream(b), v1 = ldg_stream(b + 16), v2 = ldg_stream(b + 32), v3 = ldg_stream(b + 48),
              v4 = ldg_stream(p.d + 2 * (row * p.nb + 8 * c));
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2); CLQ_PUT4(w, 12, v3); CLQ_PUT4(w, 16, v4);
    }
}

__device__ __forceinline__ float lo_half(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFF))); }
__device__ __forceinline__ float hi_half(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

template <typename XT> __device__ __forceinline__ float xload(const XT* p);
template <> __device__ __forceinline__ float xload<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float xload<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <> __device__ __forceinline__ float xload<__half>(const __half* p) { return __half2float(*p); }

// hi + lo split of two scaled fp32 values into f16x2 words.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
    hi = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
    lo = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
}

struct Params {
    Planes p;
    int64_t rows, k, m, ldo;
    const void* x;
    float* out;
    int xtype;
    int part_chunks;  // chunks of x staged per pass
};

// Stage chunks [c0, c0 + pc) of activation rows [tok0, tok0 + ntok) into
// shared memory: fragments xf, unscale factors us, and (Q4_K) scaled sub-block
// sums sxf for the min term.
template <int D, typename XT, int WARPS>
__device__ void stage_x(const Params& P, int64_t c0, int pc, int64_t tok0, int ntok, uint4* xf,
                        float* us, uint2* sxf) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const XT* x = reinterpret_cast<const XT*>(P.x);
    for (int u = warp; u < pc * ntok; u += WARPS) {
        const int cc = u / ntok, tok = u % ntok;
        const XT* src = x + (tok0 + tok) * P.k + (c0 + cc) * 256 + 8 * lane;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = xload(src + i);
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        int sexp = 0;
        if (amax > 0.f) {
            int e = (int)((__float_as_uint(amax) >> 23) & 255) - 127;
            sexp = 14 - e;
            sexp = sexp < -120 ? -120 : (sexp > 120 ? 120 : sexp);
        }
        const float scale = __uint_as_float((uint32_t)(127 + sexp) << 23);
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] *= scale;
#pragma unroll
        for (int qq = 0; qq < 2; qq++) {
            int s, t;
            Steps<D>::inv(2 * lane + qq, s, t);
            uint4 f;
            split2(v[4 * qq], v[4 * qq + 1], f.x, f.z);
            split2(v[4 * qq + 2], v[4 * qq + 3], f.y, f.w);
            xf[((cc * 16 + s) * 4 + t) * ntok + tok] = f;
        }
        if (D == kQ4_K) {
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) sum += v[i];
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);   // lanes 4G..4G+3: sub-block G sum
            sum *= 0.015625f;                              // 2^-6 keeps it inside fp16 range
            const float other = __shfl_down_sync(0xffffffffu, sum, 4);  // sub-block G+1
            if ((lane & 7) == 0) {
                uint2 f;
                split2(sum, other, f.x, f.y);
                sxf[(cc * 4 + (lane >> 3)) * ntok + tok] = f;
            }
        }
        if (lane == 0) us[cc * ntok + tok] = __uint_as_float((uint32_t)(127 - sexp) << 23);
    }
}

template <int D, typename XT, int MT, int R, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) gemv_mma_kernel(Params P) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int NW = Words<D>::n;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int64_t tile0 = (int64_t)blockIdx.x * R;
    const int64_t tok0 = (int64_t)blockIdx.y * 8 * MT;
    const int ntok = (int)((P.m - tok0) < 8 * MT ? (P.m - tok0) : 8 * MT);
    const int64_t nchunks = P.k / 256;
    const int pc_max = P.part_chunks;

    uint4* xf = reinterpret_cast<uint4*>(smem);
    uint2* sxf = reinterpret_cast<uint2*>(xf + (size_t)pc_max * 64 * ntok);
    float* us = reinterpret_cast<float*>(sxf + (D == kQ4_K ? (size_t)pc_max * 4 * ntok : 0));

    float acc[R][MT][4];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int n = 0; n < MT; n++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[r][n][i] = 0.f;

    int64_t rowA[R], rowB[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        int64_t base = (tile0 + r) * 16 + g;
        rowA[r] = base < P.rows ? base : P.rows - 1;
        rowB[r] = base + 8 < P.rows ? base + 8 : P.rows - 1;
    }

    for (int64_t c0 = 0; c0 < nchunks; c0 += pc_max) {
        const int pc = (int)((nchunks - c0) < pc_max ? (nchunks - c0) : pc_max);
        __syncthreads();  // previous pass finished reading the staged activations
        stage_x<D, XT, WARPS>(P, c0, pc, tok0, ntok, xf, us, sxf);
        __syncthreads();

        for (int cc = warp; cc < pc; cc += WARPS) {
            const int64_t c = c0 + cc;
            uint32_t w[R][2][NW];
            uint32_t db[R][2];
#pragma unroll
            for (int r = 0; r < R; r++) {
                load_chunk<D>(P.p, rowA[r], c, t, w[r][0], db[r][0]);
                load_chunk<D>(P.p, rowB[r], c, t, w[r][1], db[r][1]);
            }
            float ut[MT][2];  // unscale of tokens 2t, 2t+1 of each n-tile
#pragma unroll
            for (int n = 0; n < MT; n++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    int tok = 8 * n + 2 * t + j;
                    ut[n][j] = tok < ntok ? us[cc * ntok + tok] : 0.f;
                }

            if constexpr (D == kQ4_K) {
#pragma unroll
                for (int r = 0; r < R; r++) {
                    uint32_t SCL[2], NL[2], SCH[2], NH[2], MN[2];
                    float dd[2], dm[2];
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const uint32_t* W = w[r][h];
                        const int sh = 16 * (t & 1);
                        const uint32_t A = (W[1] >> sh) & 0xFFFF, Bw = (W[2] >> sh) & 0xFFFF,
                                       Cw = (W[3] >> sh) & 0xFFFF;
                        const uint32_t sc = t < 2 ? (A & 0x3F3F) : ((Cw & 0x0F0F) | ((A >> 2) & 0x3030));
                        const uint32_t mn = t < 2 ? (Bw & 0x3F3F) : (((Cw >> 4) & 0x0F0F) | ((Bw >> 2) & 0x3030));
                        SCL[h] = hsub2(prmt(sc, kMagic, 0x4040), kH1024);
                        SCH[h] = hsub2(prmt(sc, kMagic, 0x4141), kH1024);
                        NL[h] = hmul2(SCL[h], kHNeg1024);
                        NH[h] = hmul2(SCH[h], kHNeg64);
                        SCH[h] = hmul2(SCH[h], kHSixteenth);
                        MN[h] = hsub2(prmt(mn, kMagic, kSelLo), kH1024);
                        dd[h] = lo_half(W[0]);
                        dm[h] = hi_half(W[0]);
                    }
                    float csb[MT][4], cmn[MT][4];
#pragma unroll
                    for (int n = 0; n < MT; n++)
#pragma unroll
                        for (int i = 0; i < 4; i++) csb[n][i] = cmn[n][i] = 0.f;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        uint32_t lo01[2], lo23[2], hi01[2], hi23[2];
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const uint32_t Wd = w[r][h][4 + j];
                            const uint32_t p01 = prmt(Wd, kMagic, kSelLo), p23 = prmt(Wd, kMagic, kSelHi);
                            lo01[h] = hfma2(p01 & kLoNib, SCL[h], NL[h]);
                            lo23[h] = hfma2(p23 & kLoNib, SCL[h], NL[h]);
                            hi01[h] = hfma2(p01 & kHiNib, SCH[h], NH[h]);
                            hi23[h] = hfma2(p23 & kHiNib, SCH[h], NH[h]);
                        }
#pragma unroll
                        for (int n = 0; n < MT; n++) {
                            const int tok = 8 * n + g;
                            const uint4 z = make_uint4(0, 0, 0, 0);
                            const uint4 b0 = tok < ntok ? xf[((cc * 16 + 2 * j) * 4 + t) * ntok + tok] : z;
                            const uint4 b1 = tok < ntok ? xf[((cc * 16 + 2 * j + 1) * 4 + t) * ntok + tok] : z;
                            mma16816(csb[n], lo01[0], lo01[1], lo23[0], lo23[1], b0.x, b0.y);
                            mma16816(csb[n], lo01[0], lo01[1], lo23[0], lo23[1], b0.z, b0.w);
                            mma16816(csb[n], hi01[0], hi01[1], hi23[0], hi23[1], b1.x, b1.y);
                            mma16816(csb[n], hi01[0], hi01[1], hi23[0], hi23[1], b1.z, b1.w);
                        }
                    }
#pragma unroll
                    for (int n = 0; n < MT; n++) {
                        const int tok = 8 * n + g;
                        const uint2 sx = tok < ntok ? sxf[(cc * 4 + t) * ntok + tok] : make_uint2(0, 0);
                        mma16816(cmn[n], MN[0], MN[1], 0u, 0u, sx.x, 0u);
                        mma16816(cmn[n], MN[0], MN[1], 0u, 0u, sx.y, 0u);
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int h = i >> 1;
                            const float v = fmaf(-64.f * dm[h], cmn[n][i], dd[h] * csb[n][i]);
                            acc[r][n][i] = fmaf(ut[n][i & 1], v, acc[r][n][i]);
                        }
                    }
                }
            } else {
                // Q6_K: scale per 16-element step; Q4_0 / Q8_0: scale per 32-element block (2 steps).
#pragma unroll
                for (int r = 0; r < R; r++) {
                    float cacc[MT][4];
#pragma unroll
                    for (int n = 0; n < MT; n++)
#pragma unroll
                        for (int i = 0; i < 4; i++) cacc[n][i] = 0.f;
#pragma unroll
                    for (int grpi = 0; grpi < (D == kQ6_K ? 4 : 8); grpi++) {
                        // grpi: Q6_K (h,half) word triple -> 4 steps; Q4_0/Q8_0 block -> 2 steps
                        constexpr int SPG = D == kQ6_K ? 4 : 2;
                        uint32_t a01[SPG][2], a23[SPG][2];
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const uint32_t* W = w[r][h];
                            if constexpr (D == kQ6_K) {
                                const uint32_t W0 = W[3 * grpi], W1 = W[3 * grpi + 1], QH = W[3 * grpi + 2];
                                const uint32_t p0a = prmt(W0, kMagic, kSelLo), p0b = prmt(W0, kMagic, kSelHi);
                                const uint32_t p1a = prmt(W1, kMagic, kSelLo), p1b = prmt(W1, kMagic, kSelHi);
                                const uint32_t qa = prmt(QH, 0u, kSelLo), qb = prmt(QH, 0u, kSelHi);
                                const uint32_t qa4 = qa << 4, qa2 = qa << 2, qb4 = qb << 4, qb2 = qb << 2;
                                a01[0][h] = hsub2((p0a & kLoNib) | (qa4 & 0x00300030u), kH1056);
                                a23[0][h] = hsub2((p0b & kLoNib) | (qb4 & 0x00300030u), kH1056);
                                a01[1][h] = hsub2((p1a & kLoNib) | (qa2 & 0x00300030u), kH1056);
                                a23[1][h] = hsub2((p1b & kLoNib) | (qb2 & 0x00300030u), kH1056);
                                a01[2][h] = hfma2((p0a & kHiNib) | (qa4 & 0x03000300u), kHSixteenth, kHNeg96);
                                a23[2][h] = hfma2((p0b & kHiNib) | (qb4 & 0x03000300u), kHSixteenth, kHNeg96);
                                a01[3][h] = hfma2((p1a & kHiNib) | (qa2 & 0x03000300u), kHSixteenth, kHNeg96);
                                a23[3][h] = hfma2((p1b & kHiNib) | (qb2 & 0x03000300u), kHSixteenth, kHNeg96);
                            } else if constexpr (D == kQ4_0) {
                                const uint32_t Wd = W[grpi];
                                const uint32_t pa = prmt(Wd, kMagic, kSelLo), pb = prmt(Wd, kMagic, kSelHi);
                                a01[0][h] = hsub2(pa & kLoNib, kH1032);
                                a23[0][h] = hsub2(pb & kLoNib, kH1032);
                                a01[1][h] = hfma2(pa & kHiNib, kHSixteenth, kHNeg72);
                                a23[1][h] = hfma2(pb & kHiNib, kHSixteenth, kHNeg72);
                            } else {  // Q8_0
#pragma unroll
                                for (int hf = 0; hf < 2; hf++) {
                                    const uint32_t Wd = W[2 * grpi + hf] ^ 0x80808080u;
                                    a01[hf][h] = hsub2(prmt(Wd, kMagic, kSelLo), kH1152);
                                    a23[hf][h] = hsub2(prmt(Wd, kMagic, kSelHi), kH1152);
                                }
                            }
                        }
                        float f[SPG][2];  // per-step (Q6_K) or per-block scale of rows g, g+8
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            if constexpr (D == kQ6_K) {
                                const uint32_t* S = &w[r][h][12];
#pragma unroll
                                for (int grp = 0; grp < 4; grp++) {
                                    // sub-scale index 8h + 2grp + half with (h, half) = grpi
                                    const int idx = 8 * (grpi >> 1) + 2 * grp + (grpi & 1);
                                    f[grp][h] = (float)(int)(int8_t)(S[idx >> 2] >> (8 * (idx & 3)));
                                }
                            } else {
                                const uint32_t dw = w[r][h][(D == kQ4_0 ? 8 : 16) + (grpi >> 1)];
                                f[0][h] = (grpi & 1) ? hi_half(dw) : lo_half(dw);
                            }
                        }
#pragma unroll
                        for (int n = 0; n < MT; n++) {
                            const int tok = 8 * n + g;
                            float cs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                            for (int st = 0; st < SPG; st++) {
                                const int s = SPG * grpi + st;
                                const uint4 b = tok < ntok ? xf[((cc * 16 + s) * 4 + t) * ntok + tok]
                                                           : make_uint4(0, 0, 0, 0);
                                if constexpr (D == kQ6_K) {
#pragma unroll
                                    for (int i = 0; i < 4; i++) cs[i] = 0.f;
                                }
                                mma16816(cs, a01[st][0], a01[st][1], a23[st][0], a23[st][1], b.x, b.y);
                                mma16816(cs, a01[st][0], a01[st][1], a23[st][0], a23[st][1], b.z, b.w);
                                if constexpr (D == kQ6_K) {
#pragma unroll
                                    for (int i = 0; i < 4; i++) cacc[n][i] = fmaf(f[st][i >> 1], cs[i], cacc[n][i]);
                                }
                            }
                            if constexpr (D != kQ6_K) {
#pragma unroll
                                for (int i = 0; i < 4; i++) cacc[n][i] = fmaf(f[0][i >> 1], cs[i], cacc[n][i]);
                            }
                        }
                    }
                    float dsb[2] = {1.f, 1.f};
                    if constexpr (D == kQ6_K) {
                        dsb[0] = __half2float(__ushort_as_half((unsigned short)db[r][0]));
                        dsb[1] = __half2float(__ushort_as_half((unsigned short)db[r][1]));
                    }
#pragma unroll
                    for (int n = 0; n < MT; n++)
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            acc[r][n][i] = fmaf(ut[n][i & 1] * dsb[i >> 1], cacc[n][i], acc[r][n][i]);
                }
            }
        }
    }

    // K-split reduction across warps through shared memory.
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int n = 0; n < MT; n++)
#pragma unroll
            for (int i = 0; i < 4; i++) red[(((warp * R + r) * MT + n) * 4 + i) * 32 + lane] = acc[r][n][i];
    __syncthreads();
    for (int idx = threadIdx.x; idx < R * MT * 128; idx += WARPS * 32) {
        float sum = 0.f;
#pragma unroll 4
        for (int wv = 0; wv < WARPS; wv++) sum += red[wv * R * MT * 128 + idx];
        const int ln = idx & 31, i = (idx >> 5) & 3, n = (idx >> 7) % MT, r = idx / (MT * 128);
        const int64_t row = (tile0 + r) * 16 + (ln >> 2) + 8 * (i >> 1);
        const int64_t tok = tok0 + 8 * n + 2 * (ln & 3) + (i & 1);
        if (row < P.rows && tok < P.m) P.out[tok * P.ldo + row] = sum;
    }
}

template <int D, typename XT, int MT, int R, int WARPS>
cudaError_t launch_one(const Params& P, cudaStream_t stream) {
    const int64_t tiles = (P.rows + 15) / 16;
    const int ntok_max = (int)(P.m < 8 * MT ? P.m : 8 * MT);
    const size_t per_chunk = (size_t)ntok_max * (1024 + (D == kQ4_K ? 32 : 0) + 4);
    const size_t red = (size_t)WARPS * R * MT * 128 * sizeof(float);
    const int64_t nchunks = P.k / 256;
    Params q = P;
    const size_t budget = 96 * 1024;
    int64_t pc = (int64_t)(budget / per_chunk);
    if (pc < 1) pc = 1;
    if (pc > nchunks) pc = nchunks;
    q.part_chunks = (int)pc;
    size_t smem = pc * per_chunk;
    if (smem < red) smem = red;
    auto kern = gemv_mma_kernel<D, XT, MT, R, WARPS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)((tiles + R - 1) / R), (unsigned)((P.m + 8 * MT - 1) / (8 * MT)));
    if (grid.y > 65535) return cudaErrorInvalidConfiguration;
    kern<<<grid, WARPS * 32, smem, stream>>>(q);
    return cudaGetLastError();
}

template <int D, typename XT>
cudaError_t launch_shape(const Params& P, cudaStream_t s) {
    const int64_t tiles = (P.rows + 15) / 16;
    const int64_t nchunks = P.k / 256;
    const bool two_tiles = tiles >= 4 * 148;
    const bool many_warps = nchunks >= 16 && tiles < 8 * 148;
    if (P.m <= 8) {
        if (two_tiles) return many_warps ? launch_one<D, XT, 1, 2, 16>(P, s) : launch_one<D, XT, 1, 2, 8>(P, s);
        return many_warps ? launch_one<D, XT, 1, 1, 16>(P, s) : launch_one<D, XT, 1, 1, 8>(P, s);
    }
    return many_warps ? launch_one<D, XT, 2, 1, 16>(P, s) : launch_one<D, XT, 2, 1, 8>(P, s);
}

template <typename XT>
cudaError_t launch_dtype(const Params& P, int dtype, cudaStream_t s) {
    switch (dtype) {
    case kQ4_K: return launch_shape<kQ4_K, XT>(P, s);
    case kQ6_K: return launch_shape<kQ6_K, XT>(P, s);
    case kQ4_0: return launch_shape<kQ4_0, XT>(P, s);
    case kQ8_0: return launch_shape<kQ8_0, XT>(P, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool gemv_mma_supported(const WeightView& w, int64_t m) {
    return w.k > 0 && w.k % 256 == 0 && m > 0;
}

cudaError_t launch_gemv_mma(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                            float* out, int64_t ldo, cudaStream_t stream) {
    Params P;
    P.p = Planes{w.q, w.s, w.d, w.nb};
    P.rows = rows;
    P.k = w.k;
    P.m = m;
    P.ldo = ldo;
    P.x = x;
    P.out = out;
    P.xtype = xtype;
    P.part_chunks = 1;
    switch (xtype) {
    case CLQ_X_F32: return launch_dtype<float>(P, w.dtype, stream);
    case CLQ_X_BF16: return launch_dtype<__nv_bfloat16>(P, w.dtype, stream);
    case CLQ_X_F16: return launch_dtype<__half>(P, w.dtype, stream);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace clq
