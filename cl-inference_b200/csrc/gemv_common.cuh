// gemv_common.cuh -- device code shared by the GEMV kernels: exact fp16
// unpacking of the packed codes, the activation staging (power-of-two scaled
// hi + lo fp16 fragments) and the per-chunk tensor-core product.
//
// A warp owns 16 weight rows (the MMA's M) x 256 columns (one "chunk": a
// K-quant superblock or 8 Q4_0/Q8_0 blocks) per unit; the activation rows
// (tokens) are the MMA's N, each as a hi and a lo column.  The fp16 operands
// are exact:
//   A  weight codes unpacked in registers with prmt/lop3 (OR the code bits into
//      the mantissa of 1024.0 or 64.0) and one f16x2 fma/sub to remove the bias
//      -- for Q4_K also times the 6-bit sub-block scale, sc*q < 2^10;
//   B  activations split as hi + lo fp16 (x = hi + lo to ~22 bits) after a
//      power-of-two scaling per (chunk, token) that puts max|x| in [2^14, 2^15).
// Block scales (fp16 d, dmin, Q6_K int8 sub-scales) multiply the fp32 MMA
// results, so the result carries fp32-class error, like an fp32 dot product.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/clq.h"
#include "clq_internal.h"
#include "layout.cuh"
#include "pipeline.cuh"

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

// Bytes per 256-column chunk in each plane, and this lane's offset in the q plane.
template <int D> struct ChunkBytes;
template <> struct ChunkBytes<kQ4_K> { static constexpr int q = 144, s = 0, d = 0; };
template <> struct ChunkBytes<kQ6_K> { static constexpr int q = 192, s = 16, d = 2; };
template <> struct ChunkBytes<kQ4_0> { static constexpr int q = 128, s = 0, d = 16; };
template <> struct ChunkBytes<kQ8_0> { static constexpr int q = 256, s = 0, d = 16; };

// Start of one weight row in each plane (row-major planes, nb blocks per row).
struct RowPtr {
    const uint8_t* q;
    const uint8_t* s;
    const uint8_t* d;
};

template <int D>
__device__ __forceinline__ RowPtr row_ptr(const Planes& p, int64_t row) {
    const int64_t chunks = p.nb / (D == kQ4_K || D == kQ6_K ? 1 : 8);
    RowPtr r;
    r.q = p.q + row * chunks * ChunkBytes<D>::q;
    r.s = p.s + row * chunks * ChunkBytes<D>::s;
    r.d = p.d + row * chunks * ChunkBytes<D>::d;
    return r;
}

template <int D>
__device__ __forceinline__ void load_chunk(const RowPtr& rp, int c, int t, uint32_t (&w)[Words<D>::n],
                                           uint32_t& dbits) {
    const uint8_t* b = rp.q + c * ChunkBytes<D>::q;
    if (D == kQ4_K) {
        uint4 v0 = ldg_stream(b), v1 = ldg_stream(b + 16 + 32 * t), v2 = ldg_stream(b + 32 + 32 * t);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2);
    } else if (D == kQ6_K) {
        b += 48 * t;
        uint4 v0 = ldg_stream(b), v1 = ldg_stream(b + 16), v2 = ldg_stream(b + 32), v3 = ldg_stream(rp.s + c * 16);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2); CLQ_PUT4(w, 12, v3);
        dbits = *reinterpret_cast<const unsigned short*>(rp.d + 2 * c);
    } else if (D == kQ4_0) {
        b += 32 * t;
        uint4 v0 = ldg_stream(b), v1 = ldg_stream(b + 16), v2 = ldg_stream(rp.d + 16 * c);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2);
    } else {
        b += 64 * t;
        uint4 v0 = ldg_stream(b), v1 = ldg_stream(b + 16), v2 = ldg_stream(b + 32), v3 = ldg_stream(b + 48),
              v4 = ldg_stream(rp.d + 16 * c);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2); CLQ_PUT4(w, 12, v3); CLQ_PUT4(w, 16, v4);
    }
}

__device__ __forceinline__ float lo_half(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFF))); }
__device__ __forceinline__ float hi_half(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

template <typename XT> __device__ __forceinline__ float xload(const XT* p);
template <> __device__ __forceinline__ float xload<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float xload<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <> __device__ __forceinline__ float xload<__half>(const __half* p) { return __half2float(*p); }

// Eight consecutive activations from a 16-byte aligned address.
__device__ __forceinline__ void xload8(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ float2 to_float2(__half2 h) { return __half22float2(h); }
__device__ __forceinline__ float2 to_float2(__nv_bfloat162 h) { return __bfloat1622float2(h); }
template <typename H2>
__device__ __forceinline__ void xload8_h(const void* p, float (&v)[8]) {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        H2 h = *reinterpret_cast<const H2*>(&w[i]);
        float2 f = to_float2(h);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void xload8(const __half* p, float (&v)[8]) { xload8_h<__half2>(p, v); }
__device__ __forceinline__ void xload8(const __nv_bfloat16* p, float (&v)[8]) { xload8_h<__nv_bfloat162>(p, v); }

// hi + lo split of two scaled fp32 values into f16x2 words.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
    hi = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
    lo = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
}

// Up to kGroup weights of one dtype and K that share the activations run as
// one launch; their 16-row tiles are numbered consecutively.
constexpr int kGroup = 4;

struct Member {
    Planes p;
    int64_t rows;
    float* out;
    int64_t ldo;
    int64_t tile_begin;  // first global tile of this member
};


template <typename PT>
__device__ __forceinline__ int member_of(const PT& P, int64_t tile) {
    int i = 0;
#pragma unroll
    for (int j = 1; j < kGroup; j++)
        if (j < P.nmem && tile >= P.mem[j].tile_begin) i = j;
    return i;
}

// Stage chunks [c0, c0 + pc) of activation rows [tok0, tok0 + ntok) into
// shared memory: fragments xf, unscale factors us, and (Q4_K) scaled sub-block
// sums sxf for the min term.
// Layout (token-major, PC = part_chunks): xf[(tok*PC + cc)*64 + s*4 + t],
// sxf[(tok*PC + cc)*4 + t], us[tok*PC + cc].
template <int D, typename XT, int WARPS>
__device__ void stage_x(const void* xv, int64_t k, int x_aligned, int PC, int64_t c0, int pc, int64_t tok0,
                        int ntok, uint4* xf, float* us, uint2* sxf) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const XT* x = reinterpret_cast<const XT*>(xv);
    for (int u = warp; u < pc * ntok; u += WARPS) {
        const int cc = u / ntok, tok = u % ntok;
        const XT* src = x + (tok0 + tok) * k + (c0 + cc) * 256 + 8 * lane;
        float v[8];
        if (x_aligned) {
            xload8(src, v);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = xload(src + i);
        }
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
            xf[(tok * PC + cc) * 64 + s * 4 + t] = f;
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
                sxf[(tok * PC + cc) * 4 + (lane >> 3)] = f;
            }
        }
        if (lane == 0) us[tok * PC + cc] = __uint_as_float((uint32_t)(127 - sexp) << 23);
    }
}

// One 16-row tile x one 256-column chunk: acc[n][i] += this chunk's products.
// w[h]: the rows g (h = 0) and g + 8 (h = 1) words of load_chunk; cc: the
// chunk's index among the staged ones.
// MMA columns carry (token, part): column 2u + p of n-tile n is token 4n + u,
// activation part p (0 = hi, 1 = lo), so one MMA yields both partial sums and
// lane t's accumulators c[2h], c[2h+1] are token 4n + t's hi and lo sums for
// row g + 8h.
// xq[n]: the (hi or lo) fragment pair of this lane's column for the chunk,
// indexed by step * 8 uint2 (token clamped to a staged one; padding columns are
// computed and discarded); sq[n]: its Q4_K sub-block sums; ut[n]: unscale of
// token 4n + t.  acc[n][h]: row g + 8h, token 4n + t.
template <int D, int MT>
__device__ __forceinline__ void compute_chunk(const uint32_t (&w)[2][Words<D>::n], const uint32_t (&db)[2],
                                              int t, const uint2* const (&xq)[MT],
                                              const uint32_t* const (&sq)[MT], const float (&ut)[MT],
                                              float (&acc)[MT][2]) {
    if constexpr (D == kQ4_K) {
        uint32_t SCL[2], NL[2], SCH[2], NH[2], MN[2];
        float dd[2], dm[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t* W = w[h];
            const int sh = 16 * (t & 1);
            const uint32_t A = (W[1] >> sh) & 0xFFFF, Bw = (W[2] >> sh) & 0xFFFF, Cw = (W[3] >> sh) & 0xFFFF;
            const uint32_t sc = t < 2 ? (A & 0x3F3F) : ((Cw & 0x0F0F) | ((A >> 2) & 0x3030));
            const uint32_t mn = t < 2 ? (Bw & 0x3F3F) : (((Cw >> 4) & 0x0F0F) | ((Bw >> 2) & 0x3030));
            const uint32_t scp = hsub2(prmt(sc, kMagic, kSelLo), kH1024);  // (sc_lo, sc_hi)
            SCL[h] = prmt(scp, scp, 0x1010);
            SCH[h] = prmt(scp, scp, 0x3232);
            NL[h] = hmul2(SCL[h], kHNeg1024);
            NH[h] = hmul2(SCH[h], kHNeg64);
            SCH[h] = hmul2(SCH[h], kHSixteenth);
            MN[h] = hsub2(prmt(mn, kMagic, kSelLo), kH1024);
            dd[h] = lo_half(W[0]);
            dm[h] = hi_half(W[0]);
        }
        // two independent accumulator chains (low / high code nibbles)
        float c2[2][MT][4], cm[MT][4];
#pragma unroll
        for (int n = 0; n < MT; n++)
#pragma unroll
            for (int i = 0; i < 4; i++) c2[0][n][i] = c2[1][n][i] = cm[n][i] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t lo01[2], lo23[2], hi01[2], hi23[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t Wd = w[h][4 + j];
                const uint32_t p01 = prmt(Wd, kMagic, kSelLo), p23 = prmt(Wd, kMagic, kSelHi);
                lo01[h] = hfma2(p01 & kLoNib, SCL[h], NL[h]);
                lo23[h] = hfma2(p23 & kLoNib, SCL[h], NL[h]);
                hi01[h] = hfma2(p01 & kHiNib, SCH[h], NH[h]);
                hi23[h] = hfma2(p23 & kHiNib, SCH[h], NH[h]);
            }
#pragma unroll
            for (int n = 0; n < MT; n++) {
                const uint2 b0 = xq[n][(2 * j) * 8], b1 = xq[n][(2 * j + 1) * 8];
                mma16816(c2[0][n], lo01[0], lo01[1], lo23[0], lo23[1], b0.x, b0.y);
                mma16816(c2[1][n], hi01[0], hi01[1], hi23[0], hi23[1], b1.x, b1.y);
            }
        }
#pragma unroll
        for (int n = 0; n < MT; n++) {
            mma16816(cm[n], MN[0], MN[1], 0u, 0u, *sq[n], 0u);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const float csb = (c2[0][n][2 * h] + c2[1][n][2 * h]) + (c2[0][n][2 * h + 1] + c2[1][n][2 * h + 1]);
                const float cmn = cm[n][2 * h] + cm[n][2 * h + 1];
                const float v = fmaf(-64.f * dm[h], cmn, dd[h] * csb);
                acc[n][h] = fmaf(ut[n], v, acc[n][h]);
            }
        }
    } else {
        // Q6_K: scale per 16-element step; Q4_0 / Q8_0: scale per 32-element block (2 steps).
        constexpr int SPG = D == kQ6_K ? 4 : 2;
        float cacc[MT][2];
#pragma unroll
        for (int n = 0; n < MT; n++) cacc[n][0] = cacc[n][1] = 0.f;
#pragma unroll
        for (int grpi = 0; grpi < (D == kQ6_K ? 4 : 8); grpi++) {
            // grpi: Q6_K (h,half) word triple -> 4 steps; Q4_0/Q8_0 block -> 2 steps
            uint32_t a01[SPG][2], a23[SPG][2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t* W = w[h];
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
                    const uint32_t* S = &w[h][12];
#pragma unroll
                    for (int grp = 0; grp < 4; grp++) {
                        // sub-scale index 8h + 2grp + half with (h, half) = grpi
                        const int idx = 8 * (grpi >> 1) + 2 * grp + (grpi & 1);
                        f[grp][h] = (float)(int)(int8_t)(S[idx >> 2] >> (8 * (idx & 3)));
                    }
                } else {
                    const uint32_t dw = w[h][(D == kQ4_0 ? 8 : 16) + (grpi >> 1)];
                    f[0][h] = (grpi & 1) ? hi_half(dw) : lo_half(dw);
                }
            }
#pragma unroll
            for (int n = 0; n < MT; n++) {
                float cs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int st = 0; st < SPG; st++) {
                    const uint2 b = xq[n][(SPG * grpi + st) * 8];
                    if constexpr (D == kQ6_K) {
                        float c1[4] = {0.f, 0.f, 0.f, 0.f};
                        mma16816(c1, a01[st][0], a01[st][1], a23[st][0], a23[st][1], b.x, b.y);
#pragma unroll
                        for (int h = 0; h < 2; h++) cacc[n][h] = fmaf(f[st][h], c1[2 * h] + c1[2 * h + 1], cacc[n][h]);
                    } else {
                        mma16816(cs, a01[st][0], a01[st][1], a23[st][0], a23[st][1], b.x, b.y);
                    }
                }
                if constexpr (D != kQ6_K) {
#pragma unroll
                    for (int h = 0; h < 2; h++) cacc[n][h] = fmaf(f[0][h], cs[2 * h] + cs[2 * h + 1], cacc[n][h]);
                }
            }
        }
        float dsb[2] = {1.f, 1.f};
        if constexpr (D == kQ6_K) {
            dsb[0] = __half2float(__ushort_as_half((unsigned short)db[0]));
            dsb[1] = __half2float(__ushort_as_half((unsigned short)db[1]));
        }
#pragma unroll
        for (int n = 0; n < MT; n++)
#pragma unroll
            for (int h = 0; h < 2; h++) acc[n][h] = fmaf(ut[n] * dsb[h], cacc[n][h], acc[n][h]);
    }
}

// One 8-byte (epoch, value) word to / from another GPU's memory, as ONE 64-bit
// scalar access (epoch in the low half, the value's bits in the high half).
// The PTX memory model makes an aligned scalar access single-copy atomic
// (a vector access is a set of element accesses in no set order), so a word
// read with the expected epoch also carries that call's value: no fences or
// flags are needed.
__device__ __forceinline__ void st_word(uint2* p, uint32_t ep, float v) {
    const unsigned long long w = (unsigned long long)ep | ((unsigned long long)__float_as_uint(v) << 32);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint2 ld_word(const uint2* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return make_uint2((uint32_t)w, (uint32_t)(w >> 32));
}

// The all-reduce tail of the tensor-parallel GEMVs: this CTA's outputs are the
// tiles [t_begin, t_end) of member 0, NTOK tokens each, and every rank's CTA
// with this index has written its partials of them into this rank's receive
// buffer as (EP, value) words.  Waits (bounded) for each word and sums the
// ranks in rank order.
template <typename TP>
__device__ void tp_gather_sum(const TP& tp, const Member& M, int t_begin, int t_end, int ntok, uint32_t ep,
                              int* err) {
    const uint2* slots = tp.my_recv + ((int64_t)(ep & 1u) * tp.world * kMaxTpCtas + blockIdx.x) * tp.cap;
    const int64_t rank_stride = (int64_t)kMaxTpCtas * tp.cap;
    const int64_t per_tile = (int64_t)ntok * 16;
    const int64_t n_el = (int64_t)(t_end - t_begin) * per_tile;
    for (int64_t i = threadIdx.x; i < n_el; i += blockDim.x) {
        const int tile = t_begin + (int)(i / per_tile);
        const int idx = (int)(i - (int64_t)(tile - t_begin) * per_tile);
        const int64_t row = (int64_t)(tile - (int)M.tile_begin) * 16 + (idx & 15);
        if (row >= M.rows) continue;
        float sum = 0.f;
        for (int q = 0; q < tp.world; q++) {  // fixed rank order
            const uint2* src = slots + q * rank_stride + i;
            uint2 w = ld_word(src);
            for (uint32_t it = 0; w.x != ep && it < tp.wait_polls; it++) {
                if (*(volatile int*)err) break;
                if (it > 32) __nanosleep(32);
                w = ld_word(src);
            }
            if (w.x != ep) atomicExch(err, CLQ_ERR_TIMEOUT);
            sum += __uint_as_float(w.y);
        }
        M.out[(int64_t)(idx >> 4) * M.ldo + row] = sum;
    }
}

// This rank's partial SUM of output IDX of tile TL of CTA index CTA's region
// (its tiles counted from its first), into that region of every rank's receive
// buffer, tagged EP (the region owner's epoch).
template <typename TP>
__device__ __forceinline__ void tp_put(const TP& tp, uint32_t ep, int cta, int64_t tl, int ntok, int idx, float sum) {
    const int64_t off =
        (((int64_t)(ep & 1u) * tp.world + tp.rank) * kMaxTpCtas + cta) * tp.cap + tl * ntok * 16 + idx;
    for (int q = 0; q < tp.world; q++) st_word(tp.peer_recv[q] + off, ep, sum);
}

using pipe::allow_dependents;
using pipe::grid_dependency_wait;

}  // namespace
}  // namespace clq
