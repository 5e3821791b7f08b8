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
#include <cstdlib>

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

struct Params {
    Member mem[kGroup];
    int nmem;
    int64_t tiles;      // total tiles over the members
    int64_t k, m;
    const void* x;
    int x_aligned;      // x and its rows start on 16-byte boundaries
    int part_chunks;    // chunks of x staged per pass (all of K when it fits)
    int tiles_per_cta;  // 16-row tiles each CTA owns
};

__device__ __forceinline__ int member_of(const Params& P, int64_t tile) {
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
__device__ void stage_x(const Params& P, int64_t c0, int pc, int64_t tok0, int ntok, uint4* xf,
                        float* us, uint2* sxf) {
    const int PC = P.part_chunks;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const XT* x = reinterpret_cast<const XT*>(P.x);
    for (int u = warp; u < pc * ntok; u += WARPS) {
        const int cc = u / ntok, tok = u % ntok;
        const XT* src = x + (tok0 + tok) * P.k + (c0 + cc) * 256 + 8 * lane;
        float v[8];
        if (P.x_aligned) {
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

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Each CTA owns tiles_per_cta consecutive 16-row tiles for one slice of up to
// 8*MT activation rows.  The activations are staged once per pass over K; each
// warp then streams a flat list of (tile, chunk) units -- its chunks are
// warp, warp + WARPS, ... -- with the next unit's weights loaded while the
// current one is computed.  Per-(warp, tile) partial sums stay in shared
// memory and one barrier at the end precedes the cross-warp sum.
// Launched with programmatic dependent launch: weight loads do not depend on
// the previous kernel, so only the activation staging waits for it.
template <int D, typename XT, int MT, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 16 / WARPS) gemv_mma_kernel(Params P) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int NW = Words<D>::n;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int TL = P.tiles_per_cta;
    const int64_t tiles = P.tiles;
    const int64_t tile0 = (int64_t)blockIdx.x * TL;
    const int tlc = (int)((tiles - tile0) < TL ? (tiles - tile0) : TL);
    const int64_t tok0 = (int64_t)blockIdx.y * 4 * MT;
    const int ntok = (int)((P.m - tok0) < 4 * MT ? (P.m - tok0) : 4 * MT);
    const int64_t nchunks = P.k / 256;
    const int PC = P.part_chunks;

    uint4* xf = reinterpret_cast<uint4*>(smem);
    uint2* sxf = reinterpret_cast<uint2*>(xf + (size_t)PC * 64 * ntok);
    float* us = reinterpret_cast<float*>(sxf + (D == kQ4_K ? (size_t)PC * 4 * ntok : 0));
    float* part = us + (size_t)PC * ntok;  // [WARPS][TL][ntok][16]

    // Per n-tile: the staged token of this lane's B column (4n + g/2, clamped)
    // and the token of its accumulators (4n + t, clamped); padding is dropped.
    int xtok[MT], utok[MT];
#pragma unroll
    for (int n = 0; n < MT; n++) {
        xtok[n] = min(4 * n + (g >> 1), ntok - 1);
        utok[n] = min(4 * n + t, ntok - 1);
    }
    const int part_sel = g & 1;  // 0: hi fragment pair, 1: lo

    allow_dependents();

    for (int64_t c0 = 0; c0 < nchunks; c0 += PC) {
        const int pc = (int)((nchunks - c0) < PC ? (nchunks - c0) : PC);
        const int my_chunks = warp < pc ? (pc - warp + WARPS - 1) / WARPS : 0;
        const int nunits = tlc * my_chunks;

        // unit (tl, ci): tile tile0 + tl, chunk c0 + warp + ci * WARPS
        int ltl = -1;
        RowPtr rpa, rpb;
        auto load_unit = [&](int tl, int ci, uint32_t (&w)[2][NW], uint32_t (&db)[2]) {
            if (tl != ltl) {  // warp-uniform: rows of a new tile
                ltl = tl;
                const int64_t base = (tile0 + tl) * 16 + g;
                const int mi = member_of(P, tile0 + tl);
                const Member& M = P.mem[mi];
                const int64_t lr = base - M.tile_begin * 16;
                rpa = row_ptr<D>(M.p, lr < M.rows ? lr : M.rows - 1);
                rpb = row_ptr<D>(M.p, lr + 8 < M.rows ? lr + 8 : M.rows - 1);
            }
            const int c = (int)c0 + warp + ci * WARPS;
            load_chunk<D>(rpa, c, t, w[0], db[0]);
            load_chunk<D>(rpb, c, t, w[1], db[1]);
        };
        uint32_t bufA[2][NW], bufB[2][NW], dbA[2] = {0, 0}, dbB[2] = {0, 0};
        if (nunits > 0) load_unit(0, 0, bufA, dbA);  // independent of the previous kernel
        if (c0 > 0) __syncthreads();                 // everyone finished with the previous pass
        else grid_dependency_wait();                 // activations may come from the previous kernel
        stage_x<D, XT, WARPS>(P, c0, pc, tok0, ntok, xf, us, sxf);
        __syncthreads();

        float acc[MT][2];
#pragma unroll
        for (int n = 0; n < MT; n++) acc[n][0] = acc[n][1] = 0.f;

        int tl = 0, ci = 0;  // current unit
        auto run_unit = [&](const uint32_t (&w)[2][NW], const uint32_t (&db)[2]) {
            const int cc = warp + ci * WARPS;
            const uint2* xq[MT];
            const uint32_t* sq[MT];
            float ut[MT];
#pragma unroll
            for (int n = 0; n < MT; n++) {
                xq[n] = reinterpret_cast<const uint2*>(xf + (xtok[n] * PC + cc) * 64 + t) + part_sel;
                sq[n] = reinterpret_cast<const uint32_t*>(sxf + (xtok[n] * PC + cc) * 4 + t) + part_sel;
                ut[n] = us[utok[n] * PC + cc];
            }
            compute_chunk<D, MT>(w, db, t, xq, sq, ut, acc);
            if (++ci == my_chunks) {
#pragma unroll
                for (int n = 0; n < MT; n++)
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int tok = 4 * n + t;
                        if (tok < ntok) {
                            float* dst = &part[((warp * TL + tl) * ntok + tok) * 16 + g + 8 * h];
                            *dst = c0 == 0 ? acc[n][h] : *dst + acc[n][h];
                        }
                        acc[n][h] = 0.f;
                    }
                ci = 0;
                ++tl;
            }
        };
        // the unit after (tl, ci)
        auto next_of = [&](int a_tl, int a_ci, int& n_tl, int& n_ci) {
            n_ci = a_ci + 1;
            n_tl = a_tl;
            if (n_ci == my_chunks) { n_ci = 0; ++n_tl; }
        };
        for (int u = 0; u < nunits; u += 2) {
            int t1, c1, t2, c2;
            next_of(tl, ci, t1, c1);
            if (u + 1 < nunits) load_unit(t1, c1, bufB, dbB);
            run_unit(bufA, dbA);
            if (u + 1 >= nunits) break;
            next_of(t1, c1, t2, c2);
            if (u + 2 < nunits) load_unit(t2, c2, bufA, dbA);
            run_unit(bufB, dbB);
        }
        if (c0 == 0 && my_chunks == 0) {  // a warp without chunks contributes zeros
            for (int i = lane; i < tlc * ntok * 16; i += 32) part[(warp * TL) * ntok * 16 + i] = 0.f;
        }
    }

    __syncthreads();
    for (int idx = threadIdx.x; idx < tlc * ntok * 16; idx += WARPS * 32) {
        float sum = 0.f;
#pragma unroll 4
        for (int wv = 0; wv < WARPS; wv++) sum += part[wv * TL * ntok * 16 + idx];
        const int r16 = idx & 15, tok = (idx >> 4) % ntok, tl = idx / (16 * ntok);
        const int mi = member_of(P, tile0 + tl);
        const Member& M = P.mem[mi];
        const int64_t row = (tile0 + tl - M.tile_begin) * 16 + r16;
        if (row < M.rows) M.out[(tok0 + tok) * M.ldo + row] = sum;
    }
}

// Programmatic dependent launch (on unless CLQ_PDL=0): the next kernel in the
// stream may start its weight prefetch while this one drains.
bool pdl_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("CLQ_PDL");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

int sm_count() {
    static int count = 0;
    if (!count) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || count <= 0)
            count = 148;
    }
    return count;
}

template <int D, typename XT, int MT, int WARPS>
cudaError_t launch_one(const Params& P, cudaStream_t stream) {
    const int64_t tiles = P.tiles;
    const int ntok_max = (int)(P.m < 4 * MT ? P.m : 4 * MT);
    const size_t per_chunk = (size_t)ntok_max * (1024 + (D == kQ4_K ? 32 : 0) + 4);
    const int64_t nchunks = P.k / 256;
    Params q = P;
    int64_t pc = (int64_t)((64 * 1024) / per_chunk);
    if (pc < 1) pc = 1;
    if (pc > nchunks) pc = nchunks;
    // 16 resident warps per SM; partial sums at most 32 KB
    const int64_t slots = (16 / WARPS) * (int64_t)sm_count();
    int64_t tl = (tiles + slots - 1) / slots;
    const int64_t tl_cap = (32 * 1024) / ((int64_t)WARPS * ntok_max * 16 * 4);
    if (tl > tl_cap) tl = tl_cap;
    if (tl < 1) tl = 1;
    q.part_chunks = (int)pc;
    q.tiles_per_cta = (int)tl;
    const size_t smem = pc * per_chunk + (size_t)WARPS * tl * ntok_max * 16 * 4;
    auto kern = gemv_mma_kernel<D, XT, MT, WARPS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)((tiles + tl - 1) / tl), (unsigned)((P.m + 4 * MT - 1) / (4 * MT)));
    if (grid.y > 65535) return cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, q);
}

int gemv_warps() {
    static int w = -1;
    if (w < 0) {
        const char* e = getenv("CLQ_GEMV_WARPS");  // tuning knob: 4 or 8 warps per CTA
        w = (e && atoi(e) == 4) ? 4 : 8;
    }
    return w;
}

template <int D, typename XT>
cudaError_t launch_shape(const Params& P, cudaStream_t s) {
    // MT n-tiles of 4 activation rows (each row uses a hi and a lo column)
    if (gemv_warps() == 4) {
        if (P.m <= 4) return launch_one<D, XT, 1, 4>(P, s);
        if (P.m <= 8) return launch_one<D, XT, 2, 4>(P, s);
        return launch_one<D, XT, 4, 4>(P, s);
    }
    if (P.m <= 4) return launch_one<D, XT, 1, 8>(P, s);
    if (P.m <= 8) return launch_one<D, XT, 2, 8>(P, s);
    return launch_one<D, XT, 4, 8>(P, s);
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

cudaError_t launch_gemv_mma_group(const WeightView* const* w, const int64_t* rows, int count, const void* x,
                                  int xtype, int64_t m, float* const* out, const int64_t* ldo,
                                  cudaStream_t stream) {
    if (count < 1 || count > kGroup) return cudaErrorInvalidValue;
    Params P = {};
    P.nmem = count;
    int64_t tiles = 0;
    for (int i = 0; i < count; i++) {
        if (w[i]->dtype != w[0]->dtype || w[i]->k != w[0]->k) return cudaErrorInvalidValue;
        P.mem[i].p = Planes{w[i]->q, w[i]->s, w[i]->d, w[i]->nb};
        P.mem[i].rows = rows[i];
        P.mem[i].out = out[i];
        P.mem[i].ldo = ldo[i];
        P.mem[i].tile_begin = tiles;
        tiles += (rows[i] + 15) / 16;
    }
    P.tiles = tiles;
    P.k = w[0]->k;
    P.m = m;
    P.x = x;
    P.part_chunks = 1;
    P.tiles_per_cta = 1;
    const int esize = xtype == CLQ_X_F32 ? 4 : 2;
    P.x_aligned = ((uintptr_t)x % 16 == 0) && ((P.k * esize) % 16 == 0);
    switch (xtype) {
    case CLQ_X_F32: return launch_dtype<float>(P, w[0]->dtype, stream);
    case CLQ_X_BF16: return launch_dtype<__nv_bfloat16>(P, w[0]->dtype, stream);
    case CLQ_X_F16: return launch_dtype<__half>(P, w[0]->dtype, stream);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv_mma(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                            float* out, int64_t ldo, cudaStream_t stream) {
    const WeightView* wp = &w;
    return launch_gemv_mma_group(&wp, &rows, 1, x, xtype, m, &out, &ldo, stream);
}

}  // namespace clq
