// gemv_i8.cuh -- decode GEMV compute on the integer tensor-core MMA for Q4_K,
// Q6_K, Q4_0 and Q8_0 at one or two activation rows, and at up to four pairs
// of rows.
//
// Codes become unsigned bytes with one AND per four weights (Q4_K high nibbles
// stay in place as 16 q; Q6_K adds a shift and an OR for its high bits) -- no
// conversion to fp16 -- and run
// through mma.sync m16n8k32 (Q4_K, one 32-element sub-block per MMA) or
// m16n8k16 (Q6_K, one 16-element sub-scale group per MMA), u8 x s8 -> s32.
// The activations of a 256-column chunk are scaled by a power of two per
// (chunk, token) to a 30-bit integer image X = rint(x * 2^e) and split into
// four balanced base-256 digits, X = D3 2^24 + D2 2^16 + D1 2^8 + D0 (one add,
// one XOR and a byte transpose per four elements); MMA column
// n carries token n / 4, digit 3 - n % 4, so lane t's two accumulator columns
// are (D3, D2) for even t and (D1, D0) for odd t of token t / 2.  Every integer
// product and sum is exact; the sub-block scales are applied as one integer
// multiply-add per accumulator (|sum| < 2^31), and the chunk's fp16 scales in
// fp32.  Q4_K's min term (dmin * sum_s m_s X_s) and Q6_K's offset term
// (-32 d sum_j sc_j X_j) are one fp16 MMA per chunk on hi + lo halves of the
// sub-block sums, as in gemv_common.cuh.  The result carries fp32-class error:
// the fixed-point image keeps 30 bits relative to the chunk's largest
// activation, and the digit and term sums are formed in fp32.  Q4_0 and Q8_0
// take one m16n8k32 MMA per 32-element block (Q8_0 codes as signed bytes, s8 x
// s8) and apply each block's fp16 scale in fp32; Q4_0's offset term
// (-8 sum_b d_b X_b) is one fp16 MMA per chunk like Q4_K's min term.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemv_common.cuh"

namespace clq {
namespace {

__device__ __forceinline__ void imma_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
// The same with signed A bytes (Q8_0 codes).
__device__ __forceinline__ void imma_k32_ss(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void imma_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// Staged activations of one (chunk, token): digit fragments (1024 bytes), the
// sub-block / group sum fragments of the fp16 correction MMA, and the unscale
// factor (padded to 16 bytes).
template <int D> struct I8Block;
template <> struct I8Block<kQ4_K> { static constexpr int sf = 32, bytes = 1024 + 32 + 16; };
template <> struct I8Block<kQ6_K> { static constexpr int sf = 64, bytes = 1024 + 64 + 16; };
// Q4_0 / Q8_0: 32-element blocks like Q4_K's sub-blocks, digits in the
// blocks' own element order (below)
template <> struct I8Block<kQ4_0> { static constexpr int sf = 32, bytes = 1024 + 32 + 16; };
template <> struct I8Block<kQ8_0> { static constexpr int sf = 32, bytes = 1024 + 32 + 16; };

// The four balanced base-256 digits of X (|X| < 2^30) as the bytes of one word,
// least significant first: adding 128 to each of the three low digit positions
// turns the carries of the balanced form into plain byte arithmetic, and the
// XOR maps each low byte y to the signed byte y - 128.  The top byte is the
// signed top digit (|D3| <= 64).
__device__ __forceinline__ uint32_t digits_of(int X) { return ((uint32_t)X + 0x00808080u) ^ 0x00808080u; }

// 4 x 4 byte transpose: out[d] holds byte d of v0..v3 (in that order), i.e.
// digit d of four consecutive elements.
__device__ __forceinline__ void transpose4(uint32_t v0, uint32_t v1, uint32_t v2, uint32_t v3, uint32_t (&out)[4]) {
    const uint32_t t0 = prmt(v0, v1, 0x5140u), t1 = prmt(v0, v1, 0x7362u);
    const uint32_t t2 = prmt(v2, v3, 0x5140u), t3 = prmt(v2, v3, 0x7362u);
    out[0] = prmt(t0, t2, 0x5410u);
    out[1] = prmt(t0, t2, 0x7632u);
    out[2] = prmt(t1, t3, 0x5410u);
    out[3] = prmt(t1, t3, 0x7632u);
}

// Stage chunks [c0, c0 + pc) of activation rows 0..ntok-1; block
// (cc, u) at STAGE + (cc * ntok + u) * I8Block<D>::bytes holds
//   [0, 1024)   the digit fragments, 16 bytes per (lane, MMA pair / quad):
//               digit dg (0 = most significant) of 8 elements per 8 bytes;
//               Q4_K uint4 at ((j*4 + dg)*4 + tt) = sub-blocks 2j and 2j+1,
//               elements 8tt..8tt+7 of each (k-slots 4tt.. and 16+4tt..);
//               Q6_K uint4 at ((hh*4 + dg)*4 + tt) = word grp (0..3) for group
//               hh*4 + grp, elements 16 half + 4tt.. of (h, half) = hh
//               (k-slots 4tt..4tt+3);
//               Q4_0 / Q8_0 uint4 at ((j*4 + dg)*4 + tt) = blocks 2j and 2j+1,
//               elements 4tt..4tt+3 and 16+4tt..16+4tt+3 of each (k-slot =
//               element, the order of the lane-major code planes);
//   [1024, +sf) hi / lo fp16 halves of the sums S of X over the sub-blocks
//               (Q4_K: uint32 pair (S_2t, S_2t+1) at (t*2 + part)) or groups
//               (Q6_K: uint2 at (t*2 + part), pairs (2t, 2t+1) and (8+2t, 9+2t)),
//               times 2^-21;
//   [.., +4)    the unscale 2^-e.
// The lane-to-fragment order makes every 8-lane phase of the consumers'
// 16-byte reads touch 128 consecutive bytes (no bank conflicts).
// One (chunk, token) block from this lane's eight activations V (elements
// 8 lane .. 8 lane + 7 of the chunk) into BASE.
template <int D>
__device__ __forceinline__ void stage_block_i8(const float (&v)[8], unsigned char* base) {
    const int lane = threadIdx.x & 31;
    float lmax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) lmax = fmaxf(lmax, fabsf(v[i]));
    // the bit patterns of non-negative floats order like the floats: one
    // warp-wide integer max gives the chunk's largest magnitude
    const uint32_t amax_bits = __reduce_max_sync(0xffffffffu, __float_as_uint(lmax));
    int e = 0;
    if (amax_bits != 0u) {
        // amax * 2^e in [2^29, 2^30): four balanced digits always suffice
        e = 29 - ((int)((amax_bits >> 23) & 255) - 127);
        e = e < -100 ? -100 : (e > 120 ? 120 : e);
    }
    const float sc = __uint_as_float((uint32_t)(127 + e) << 23);  // 2^e, a normal float for e in [-100, 120]
    uint32_t V[8];
    float fsum = 0.f;  // this lane's share of the sub-block / group sum, in units of 2^-e
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float y = v[i] * sc;  // exact scaling
        fsum += y;
        V[i] = digits_of(__float2int_rn(y));
    }
    uint32_t d03[4], d47[4];  // [digit position 0 = least significant]
    transpose4(V[0], V[1], V[2], V[3], d03);
    transpose4(V[4], V[5], V[6], V[7], d47);
    if constexpr (D == kQ4_K || D == kQ4_0 || D == kQ8_0) {
        const int s = lane >> 2, tt = lane & 3;  // sub-block (block) s, elements 8tt..
        if constexpr (D == kQ4_K) {
            uint2* xq = reinterpret_cast<uint2*>(base);
#pragma unroll
            for (int dg = 0; dg < 4; dg++)
                xq[(((s >> 1) * 4 + dg) * 4 + tt) * 2 + (s & 1)] = make_uint2(d03[3 - dg], d47[3 - dg]);
        } else {
            // elements 8tt..8tt+3 are k-slots of fragment lane 2 (tt & 1), half
            // tt >> 1 (b0 below 16, b1 from 16); 8tt+4.. those of the next lane
            uint32_t* xq = reinterpret_cast<uint32_t*>(base);
            const int f0 = 2 * (tt & 1), part = tt >> 1;
#pragma unroll
            for (int dg = 0; dg < 4; dg++) {
                xq[((((s >> 1) * 4 + dg) * 4 + f0) * 4) + (s & 1) * 2 + part] = d03[3 - dg];
                xq[((((s >> 1) * 4 + dg) * 4 + f0 + 1) * 4) + (s & 1) * 2 + part] = d47[3 - dg];
            }
        }
        fsum += __shfl_xor_sync(0xffffffffu, fsum, 1);
        fsum += __shfl_xor_sync(0xffffffffu, fsum, 2);  // lanes 4s..4s+3: S_s
        const float S = fsum * 4.76837158203125e-07f;  // 2^-21
        const float So = __shfl_down_sync(0xffffffffu, S, 4);  // S_{s+1}
        if ((lane & 7) == 0) {  // s even: the pair for k-slots 2t', 2t'+1, t' = s / 2
            uint32_t hi, lo;
            split2(S, So, hi, lo);
            uint32_t* sf = reinterpret_cast<uint32_t*>(base + 1024);
            sf[(lane >> 3) * 2] = hi;
            sf[(lane >> 3) * 2 + 1] = lo;
        }
    } else {
        // lane L: h = L / 16, grp = (L % 16) / 4, half = (L % 4) / 2, elements 8 (L % 2)..
        const int h = lane >> 4, grp = (lane >> 2) & 3, half = (lane >> 1) & 1, tt = 2 * (lane & 1);
        const int hh = 2 * h + half, j = hh * 4 + grp;
        uint32_t* xq = reinterpret_cast<uint32_t*>(base);
#pragma unroll
        for (int dg = 0; dg < 4; dg++) {
            xq[((hh * 4 + dg) * 4 + tt) * 4 + grp] = d03[3 - dg];
            xq[((hh * 4 + dg) * 4 + tt + 1) * 4 + grp] = d47[3 - dg];
        }
        fsum += __shfl_xor_sync(0xffffffffu, fsum, 1);  // lanes L, L^1: S_j
        const float S = fsum * 4.76837158203125e-07f;
        const float So = __shfl_down_sync(0xffffffffu, S, 4);  // group j + 1 (grp + 1)
        if ((lane & 1) == 0 && (grp & 1) == 0) {
            const int tp = (j & 7) >> 1, reg = j >> 3;  // pair (j, j+1) -> b0 (j < 8) or b1
            uint32_t hi, lo;
            split2(S, So, hi, lo);
            uint32_t* sf = reinterpret_cast<uint32_t*>(base + 1024);
            sf[(tp * 2) * 2 + reg] = hi;
            sf[(tp * 2 + 1) * 2 + reg] = lo;
        }
    }
    if (lane == 0) *reinterpret_cast<float*>(base + 1024 + I8Block<D>::sf) = __uint_as_float((uint32_t)(127 - e) << 23);
}

// AFTER_LOADS() runs once, after the first loads are issued and before any
// block is converted (a caller's hook to issue more copies behind them).
// XFORM may rewrite a lane's eight loaded activations of row U, columns COL..
// (a fused prologue) before they are converted: XFORM.load(u, col, aux) runs
// beside the activation loads (its own loads then share their round trip)
// and XFORM.apply(u, col, v, aux) after them; Xform::kBatch blocks are loaded
// per round trip.
struct NoHook {
    __device__ void operator()() const {}
};
struct NoXform {
    static constexpr int kBatch = 4;
    struct Aux {};
    __device__ void load(int, int64_t, Aux&) const {}
    __device__ void apply(int, int64_t, float (&)[8], const Aux&) const {}
};
template <int D, typename XT, int WARPS, typename Hook, typename Xform>
__device__ __forceinline__ void stage_x_i8_with(const void* xv, int64_t k, int x_aligned, int64_t c0, int pc,
                                                int ntok, unsigned char* stage, Hook after_loads, Xform& xform) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const XT* x = reinterpret_cast<const XT*>(xv);
    constexpr int TB = I8Block<D>::bytes;
    constexpr int B = Xform::kBatch;
    // warp w stages chunks w, w + WARPS, ... (all tokens of each), loading up to
    // B (chunk, token) blocks before converting any: one memory round trip per
    // B blocks
    const int per = warp < pc ? ((pc - warp + WARPS - 1) / WARPS) * ntok : 0;
    for (int b0 = 0; b0 < per; b0 += B) {
        float vb[B][8];
        typename Xform::Aux aux[B];
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int i = b0 + b, cc = warp + (i / ntok) * WARPS, u = i - (i / ntok) * ntok;
            const int64_t col = (c0 + cc) * 256 + 8 * lane;
            const XT* src = x + (int64_t)u * k + col;
            if (i >= per) {
#pragma unroll
                for (int e = 0; e < 8; e++) vb[b][e] = 0.f;
            } else {
                if (x_aligned) {
                    xload8(src, vb[b]);
                } else {
#pragma unroll
                    for (int e = 0; e < 8; e++) vb[b][e] = xload(src + e);
                }
                xform.load(u, col, aux[b]);
            }
        }
        if (b0 == 0) after_loads();
#pragma unroll
        for (int b = 0; b < B; b++) {
            const int i = b0 + b, cc = warp + (i / ntok) * WARPS, u = i - (i / ntok) * ntok;
            if (i < per) {
                xform.apply(u, (c0 + cc) * 256 + 8 * lane, vb[b], aux[b]);
                stage_block_i8<D>(vb[b], stage + (size_t)(cc * ntok + u) * TB);
            }
        }
    }
    if (per == 0) after_loads();
}

template <int D, typename XT, int WARPS, typename Hook = NoHook>
__device__ __forceinline__ void stage_x_i8(const void* xv, int64_t k, int x_aligned, int64_t c0, int pc, int ntok,
                                           unsigned char* stage, Hook after_loads = Hook()) {
    NoXform none;
    stage_x_i8_with<D, XT, WARPS>(xv, k, x_aligned, c0, pc, ntok, stage, after_loads, none);
}

// Per-lane constants of the i8 product.  Lane (g, t) reads B column g = token
// g / 4 (clamped to the staged tokens), digit g % 4; its accumulators are
// columns 2t, 2t+1 = token t / 2, digits (3, 2) or (1, 0); the correction MMA's
// columns 2t, 2t+1 are token t's hi and lo parts.  Tokens that do not exist
// read token 0's block and their results are dropped.
struct I8Lane {
    int t, g;
    float wa, wb;       // weights of the lane's two digit columns
    uint32_t m_sel;     // Q4_K: prmt selector of bytes (2t, 2t+1) of the 8 min bytes
    uint32_t s_sel;     // Q6_K: bytes t/2 and t/2 + 2 of a word, each under a magic byte
    int xb, xm;         // byte offsets of this lane's B column and correction column blocks
    int ua, um;         // byte offsets of the unscale of token t/2 and of token t
};

template <int D>
__device__ __forceinline__ I8Lane i8_lane(int ntok) {
    I8Lane L;
    const int lane = threadIdx.x & 31;
    constexpr int TB = I8Block<D>::bytes;
    L.t = lane & 3;
    L.g = lane >> 2;
    L.wa = (L.t & 1) ? 256.f : 16777216.f;
    L.wb = (L.t & 1) ? 1.f : 65536.f;
    L.m_sel = (uint32_t)(2 * L.t) | ((uint32_t)(2 * L.t + 1) << 4);
    const uint32_t b0 = (uint32_t)(L.t >> 1), b1 = b0 + 2;
    L.s_sel = b0 | (4u << 4) | (b1 << 8) | (4u << 12);
    const int tb = min(L.g >> 2, ntok - 1), tm = min(L.g >> 1, ntok - 1);
    const int dgt = L.g & 3, part = L.g & 1;
    L.xb = tb * TB + (dgt * 4 + L.t) * 16;  // + 256 bytes per sub-block pair (Q4_K) / (h, half) (Q6_K)
    if constexpr (D == kQ4_K) L.xm = tm * TB + 1024 + (L.t * 2 + part) * 4;
    else L.xm = tm * TB + 1024 + (L.t * 2 + part) * 8;
    L.ua = min(L.t >> 1, ntok - 1) * TB + 1024 + I8Block<D>::sf;
    L.um = min(L.t, ntok - 1) * TB + 1024 + I8Block<D>::sf;
    return L;
}

// Unsigned / sign-extended byte B of W, one permute each.
__device__ __forceinline__ int ubyte(uint32_t w, int b) { return (int)prmt(w, 0u, 0x4440u | (uint32_t)b); }
__device__ __forceinline__ int sbyte(uint32_t w, int b) {
    const uint32_t s = 8u | (uint32_t)b;
    return (int)prmt(w, 0u, (uint32_t)b | (s << 4) | (s << 8) | (s << 12));
}

// Q4_K, one chunk: HD[h] = 16-byte header of row g + 8h; CW[h][j] = bytes
// 8t..8t+7 of code group j; XS = the chunk's first staged block.  Adds to accm
// (digit-weighted, token t/2) and accn (min term of token t, to be subtracted).
// Low nibbles (sub-block 2j) enter the MMA as bytes 0..15; high nibbles
// (sub-block 2j+1) are only masked, entering as 16 q, and their sums go to a
// second accumulator: sum = 16 al + ah is 16x the scaled code sum (|.| < 2^30),
// and the factor 16 is taken out with the fp16 scale.
__device__ __forceinline__ void q4k_i8_chunk(const I8Lane& L, const uint32_t (&HD)[2][4], const uint2 (&CW)[2][4],
                                             const unsigned char* xs, float (&accm)[2], float (&accn)[2]) {
    const uint4* xb = reinterpret_cast<const uint4*>(xs + L.xb);
    uint32_t scw[2][2], m03[2], m47[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        scw[h][0] = HD[h][1] & 0x3F3F3F3Fu;                                        // sub-blocks 0..3
        scw[h][1] = (HD[h][3] & 0x0F0F0F0Fu) | ((HD[h][1] >> 2) & 0x30303030u);    // 4..7
        m03[h] = HD[h][2] & 0x3F3F3F3Fu;
        m47[h] = ((HD[h][3] >> 4) & 0x0F0F0F0Fu) | ((HD[h][2] >> 2) & 0x30303030u);
    }
    int al[4] = {0, 0, 0, 0}, ah[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint4 b = xb[16 * j];  // .xy: sub-block 2j, .zw: sub-block 2j + 1
        const uint32_t w0 = scw[0][j >> 1], w1 = scw[1][j >> 1];
        int c[4];
        imma_k32(c, CW[0][j].x & 0x0F0F0F0Fu, CW[1][j].x & 0x0F0F0F0Fu, CW[0][j].y & 0x0F0F0F0Fu,
                 CW[1][j].y & 0x0F0F0F0Fu, b.x, b.y);
        const int l0 = ubyte(w0, 2 * (j & 1)), l1 = ubyte(w1, 2 * (j & 1));
        al[0] += l0 * c[0];
        al[1] += l0 * c[1];
        al[2] += l1 * c[2];
        al[3] += l1 * c[3];
        imma_k32(c, CW[0][j].x & 0xF0F0F0F0u, CW[1][j].x & 0xF0F0F0F0u, CW[0][j].y & 0xF0F0F0F0u,
                 CW[1][j].y & 0xF0F0F0F0u, b.z, b.w);
        const int h0 = ubyte(w0, 2 * (j & 1) + 1), h1 = ubyte(w1, 2 * (j & 1) + 1);
        ah[0] += h0 * c[0];
        ah[1] += h0 * c[1];
        ah[2] += h1 * c[2];
        ah[3] += h1 * c[3];
    }
    // min term: A = (m_{2t}, m_{2t+1}) per row, k-slots 8.. are zero
    uint32_t am[2];
#pragma unroll
    for (int h = 0; h < 2; h++) am[h] = hsub2(prmt(prmt(m03[h], m47[h], L.m_sel), kMagic, kSelLo), kH1024);
    float cm[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816(cm, am[0], am[1], 0u, 0u, *reinterpret_cast<const uint32_t*>(xs + L.xm), 0u);
    const float ut = *reinterpret_cast<const float*>(xs + L.ua) * 0.0625f;  // and the 16 of the code sums
    const float umin = *reinterpret_cast<const float*>(xs + L.um) * 2097152.f;  // times 2^21
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const float d = lo_half(HD[h][0]), dm = hi_half(HD[h][0]);
        const int fa = al[2 * h] * 16 + ah[2 * h], fb = al[2 * h + 1] * 16 + ah[2 * h + 1];
        const float f = fmaf((float)fa, L.wa, (float)fb * L.wb);
        accm[h] = fmaf(d * ut, f, accm[h]);
        accn[h] = fmaf(dm * umin, cm[2 * h] + cm[2 * h + 1], accn[h]);
    }
}

// Q6_K, one chunk: QW[h][12] = this lane's 48 code bytes of row g + 8h (the
// lane-major plane: per (h, half) words ql lo, ql hi, qh); SW[h] = the 16 int8
// sub-scales; DB[h] = fp16 d bits.  Adds the main term to accm and the offset
// term 32 d sum_j sc_j S_j (to be subtracted) to accn.
__device__ __forceinline__ void q6k_i8_chunk(const I8Lane& L, const uint32_t (&QW)[2][12], const uint4 (&SW)[2],
                                             const uint32_t (&DB)[2], const unsigned char* xs, float (&accm)[2],
                                             float (&accn)[2]) {
    const uint4* xb = reinterpret_cast<const uint4*>(xs + L.xb);
    const uint32_t sw[2][4] = {{SW[0].x, SW[0].y, SW[0].z, SW[0].w}, {SW[1].x, SW[1].y, SW[1].z, SW[1].w}};
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int hh = 0; hh < 4; hh++) {  // (h, half)
        const int h6 = hh >> 1, half = hh & 1;
        uint32_t q[2][4];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint32_t W0 = QW[r][3 * hh], W1 = QW[r][3 * hh + 1], QH = QW[r][3 * hh + 2];
            q[r][0] = (W0 & 0x0F0F0F0Fu) | ((QH << 4) & 0x30303030u);
            q[r][1] = (W1 & 0x0F0F0F0Fu) | ((QH << 2) & 0x30303030u);
            q[r][2] = ((W0 >> 4) & 0x0F0F0F0Fu) | (QH & 0x30303030u);
            q[r][3] = ((W1 >> 4) & 0x0F0F0F0Fu) | ((QH >> 2) & 0x30303030u);
        }
        const uint4 bq = xb[16 * hh];
        const uint32_t bw[4] = {bq.x, bq.y, bq.z, bq.w};
#pragma unroll
        for (int grp = 0; grp < 4; grp++) {
            int c[4];
            imma_k16(c, q[0][grp], q[1][grp], bw[grp]);
            const int idx = 8 * h6 + 2 * grp + half;  // sub-scale of this group
            const int s0 = sbyte(sw[0][idx >> 2], idx & 3), s1 = sbyte(sw[1][idx >> 2], idx & 3);
            acc[0] += s0 * c[0];
            acc[1] += s0 * c[1];
            acc[2] += s1 * c[2];
            acc[3] += s1 * c[3];
        }
    }
    // offset term: A[row][j] = sc of group j; a0: j = 2t, 2t+1 -> bytes t/2, t/2 + 2 of
    // word t & 1; a2: j = 8 + 2t, 9 + 2t -> same bytes of word 2 + (t & 1)
    uint32_t a[2][2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const bool odd = (L.t & 1) != 0;  // a select, not an index: keeps sw in registers
        a[r][0] = hsub2(prmt((odd ? sw[r][1] : sw[r][0]) ^ 0x80808080u, kMagic, L.s_sel), kH1152);
        a[r][1] = hsub2(prmt((odd ? sw[r][3] : sw[r][2]) ^ 0x80808080u, kMagic, L.s_sel), kH1152);
    }
    const uint2 bs = *reinterpret_cast<const uint2*>(xs + L.xm);
    float co[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816(co, a[0][0], a[1][0], a[0][1], a[1][1], bs.x, bs.y);
    const float ut = *reinterpret_cast<const float*>(xs + L.ua);
    const float uo = *reinterpret_cast<const float*>(xs + L.um) * 67108864.f;  // times 32 * 2^21
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const float d = __half2float(__ushort_as_half((unsigned short)DB[h]));
        const float f = fmaf((float)acc[2 * h], L.wa, (float)acc[2 * h + 1] * L.wb);
        accm[h] = fmaf(d * ut, f, accm[h]);
        accn[h] = fmaf(d * uo, co[2 * h] + co[2 * h + 1], accn[h]);
    }
}

// End of a tile: lane (g, t) holds accm for token t/2 (its digit half) and
// accn for token t.  Returns the row g + 8h sum for token t/2 (lanes with even
// t hold it; odd lanes return the same value).
__device__ __forceinline__ float i8_finish(const I8Lane& L, float accm, float accn) {
    const float m = accm + __shfl_xor_sync(0xffffffffu, accm, 1);
    const int lane = threadIdx.x & 31;
    const float n = __shfl_sync(0xffffffffu, accn, (lane & ~3) | (L.t >> 1));
    return m - n;
}


// ---- several pairs of activation rows --------------------------------------
// The same product for NP pairs of activation rows (up to eight rows): the
// weight fragments of a unit are unpacked once and meet each pair's digit
// columns in its own MMA; the correction MMAs take four rows each.  Pair p's
// rows are 2p and 2p + 1 (lane (g, t): B column row 2p + g / 4; accumulator
// row 2p + t / 2), correction group q's rows 4q .. 4q + 3 (B column row
// 4q + g / 2, accumulator row 4q + t).  Rows past the staged ones read the
// last staged row, and their results are dropped.  At NP = 1 this is the
// single-pair product above.
template <int D, int NP>
struct I8LaneN {
    static constexpr int NQ = (NP + 1) / 2;
    int t, g;
    float wa, wb;
    uint32_t m_sel, s_sel;
    int xb[NP], ua[NP];  // B column block and unscale of pair p
    int xm[NQ], um[NQ];  // correction column block and unscale of group q
};

template <int D, int NP>
__device__ __forceinline__ I8LaneN<D, NP> i8_lane_n(int ntok) {
    I8LaneN<D, NP> L;
    const int lane = threadIdx.x & 31;
    constexpr int TB = I8Block<D>::bytes;
    L.t = lane & 3;
    L.g = lane >> 2;
    L.wa = (L.t & 1) ? 256.f : 16777216.f;
    L.wb = (L.t & 1) ? 1.f : 65536.f;
    L.m_sel = (uint32_t)(2 * L.t) | ((uint32_t)(2 * L.t + 1) << 4);
    const uint32_t b0 = (uint32_t)(L.t >> 1), b1 = b0 + 2;
    L.s_sel = b0 | (4u << 4) | (b1 << 8) | (4u << 12);
    const int dgt = L.g & 3, part = L.g & 1;
#pragma unroll
    for (int p = 0; p < NP; p++) {
        L.xb[p] = min(2 * p + (L.g >> 2), ntok - 1) * TB + (dgt * 4 + L.t) * 16;
        L.ua[p] = min(2 * p + (L.t >> 1), ntok - 1) * TB + 1024 + I8Block<D>::sf;
    }
#pragma unroll
    for (int q = 0; q < I8LaneN<D, NP>::NQ; q++) {
        const int tm = min(4 * q + (L.g >> 1), ntok - 1);
        L.xm[q] = tm * TB + 1024 + (L.t * 2 + part) * (D == kQ6_K ? 8 : 4);
        L.um[q] = min(4 * q + L.t, ntok - 1) * TB + 1024 + I8Block<D>::sf;
    }
    return L;
}

// Q4_K over NP pairs.  The low-nibble MMA's sums enter the accumulator times
// 16 (the sub-block scale is shifted instead), the high-nibble MMA's as they
// are: the accumulator is 16 al + ah of the single-pair form, |.| < 2^30 at
// the end (partial sums wrap harmlessly in two's complement).
template <int NP>
__device__ __forceinline__ void q4k_i8_chunk_n(const I8LaneN<kQ4_K, NP>& L, const uint32_t (&HD)[2][4],
                                               const uint2 (&CW)[2][4], const unsigned char* xs,
                                               float (&accm)[NP][2], float (&accn)[(NP + 1) / 2][2]) {
    constexpr int NQ = (NP + 1) / 2;
    uint32_t scw[2][2], m03[2], m47[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        scw[h][0] = HD[h][1] & 0x3F3F3F3Fu;
        scw[h][1] = (HD[h][3] & 0x0F0F0F0Fu) | ((HD[h][1] >> 2) & 0x30303030u);
        m03[h] = HD[h][2] & 0x3F3F3F3Fu;
        m47[h] = ((HD[h][3] >> 4) & 0x0F0F0F0Fu) | ((HD[h][2] >> 2) & 0x30303030u);
    }
    int acc[NP][4];
#pragma unroll
    for (int p = 0; p < NP; p++) acc[p][0] = acc[p][1] = acc[p][2] = acc[p][3] = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t w0 = scw[0][j >> 1], w1 = scw[1][j >> 1];
        const int l0 = ubyte(w0, 2 * (j & 1)) << 4, l1 = ubyte(w1, 2 * (j & 1)) << 4;
        const int h0 = ubyte(w0, 2 * (j & 1) + 1), h1 = ubyte(w1, 2 * (j & 1) + 1);
        const uint32_t lo0 = CW[0][j].x & 0x0F0F0F0Fu, lo1 = CW[1][j].x & 0x0F0F0F0Fu;
        const uint32_t lo2 = CW[0][j].y & 0x0F0F0F0Fu, lo3 = CW[1][j].y & 0x0F0F0F0Fu;
        const uint32_t hi0 = CW[0][j].x & 0xF0F0F0F0u, hi1 = CW[1][j].x & 0xF0F0F0F0u;
        const uint32_t hi2 = CW[0][j].y & 0xF0F0F0F0u, hi3 = CW[1][j].y & 0xF0F0F0F0u;
#pragma unroll
        for (int p = 0; p < NP; p++) {
            const uint4 b = reinterpret_cast<const uint4*>(xs + L.xb[p])[16 * j];
            int c[4];
            imma_k32(c, lo0, lo1, lo2, lo3, b.x, b.y);
            acc[p][0] += l0 * c[0];
            acc[p][1] += l0 * c[1];
            acc[p][2] += l1 * c[2];
            acc[p][3] += l1 * c[3];
            imma_k32(c, hi0, hi1, hi2, hi3, b.z, b.w);
            acc[p][0] += h0 * c[0];
            acc[p][1] += h0 * c[1];
            acc[p][2] += h1 * c[2];
            acc[p][3] += h1 * c[3];
        }
    }
    uint32_t am[2];
#pragma unroll
    for (int h = 0; h < 2; h++) am[h] = hsub2(prmt(prmt(m03[h], m47[h], L.m_sel), kMagic, kSelLo), kH1024);
#pragma unroll
    for (int p = 0; p < NP; p++) {
        const float ut = *reinterpret_cast<const float*>(xs + L.ua[p]) * 0.0625f;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const float d = lo_half(HD[h][0]);
            const float f = fmaf((float)acc[p][2 * h], L.wa, (float)acc[p][2 * h + 1] * L.wb);
            accm[p][h] = fmaf(d * ut, f, accm[p][h]);
        }
    }
#pragma unroll
    for (int q = 0; q < NQ; q++) {
        float cm[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(cm, am[0], am[1], 0u, 0u, *reinterpret_cast<const uint32_t*>(xs + L.xm[q]), 0u);
        const float umin = *reinterpret_cast<const float*>(xs + L.um[q]) * 2097152.f;
#pragma unroll
        for (int h = 0; h < 2; h++) accn[q][h] = fmaf(hi_half(HD[h][0]) * umin, cm[2 * h] + cm[2 * h + 1], accn[q][h]);
    }
}

// Q6_K over NP pairs.
template <int NP>
__device__ __forceinline__ void q6k_i8_chunk_n(const I8LaneN<kQ6_K, NP>& L, const uint32_t (&QW)[2][12],
                                               const uint4 (&SW)[2], const uint32_t (&DB)[2],
                                               const unsigned char* xs, float (&accm)[NP][2],
                                               float (&accn)[(NP + 1) / 2][2]) {
    constexpr int NQ = (NP + 1) / 2;
    const uint32_t sw[2][4] = {{SW[0].x, SW[0].y, SW[0].z, SW[0].w}, {SW[1].x, SW[1].y, SW[1].z, SW[1].w}};
    int acc[NP][4];
#pragma unroll
    for (int p = 0; p < NP; p++) acc[p][0] = acc[p][1] = acc[p][2] = acc[p][3] = 0;
#pragma unroll
    for (int hh = 0; hh < 4; hh++) {
        const int h6 = hh >> 1, half = hh & 1;
        uint32_t q[2][4];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint32_t W0 = QW[r][3 * hh], W1 = QW[r][3 * hh + 1], QH = QW[r][3 * hh + 2];
            q[r][0] = (W0 & 0x0F0F0F0Fu) | ((QH << 4) & 0x30303030u);
            q[r][1] = (W1 & 0x0F0F0F0Fu) | ((QH << 2) & 0x30303030u);
            q[r][2] = ((W0 >> 4) & 0x0F0F0F0Fu) | (QH & 0x30303030u);
            q[r][3] = ((W1 >> 4) & 0x0F0F0F0Fu) | ((QH >> 2) & 0x30303030u);
        }
        uint32_t bw[NP][4];
#pragma unroll
        for (int p = 0; p < NP; p++) {
            const uint4 bq = reinterpret_cast<const uint4*>(xs + L.xb[p])[16 * hh];
            bw[p][0] = bq.x; bw[p][1] = bq.y; bw[p][2] = bq.z; bw[p][3] = bq.w;
        }
#pragma unroll
        for (int grp = 0; grp < 4; grp++) {
            const int idx = 8 * h6 + 2 * grp + half;
            const int s0 = sbyte(sw[0][idx >> 2], idx & 3), s1 = sbyte(sw[1][idx >> 2], idx & 3);
#pragma unroll
            for (int p = 0; p < NP; p++) {
                int c[4];
                imma_k16(c, q[0][grp], q[1][grp], bw[p][grp]);
                acc[p][0] += s0 * c[0];
                acc[p][1] += s0 * c[1];
                acc[p][2] += s1 * c[2];
                acc[p][3] += s1 * c[3];
            }
        }
    }
    uint32_t a[2][2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const bool odd = (L.t & 1) != 0;
        a[r][0] = hsub2(prmt((odd ? sw[r][1] : sw[r][0]) ^ 0x80808080u, kMagic, L.s_sel), kH1152);
        a[r][1] = hsub2(prmt((odd ? sw[r][3] : sw[r][2]) ^ 0x80808080u, kMagic, L.s_sel), kH1152);
    }
    float d[2];
#pragma unroll
    for (int h = 0; h < 2; h++) d[h] = __half2float(__ushort_as_half((unsigned short)DB[h]));
#pragma unroll
    for (int p = 0; p < NP; p++) {
        const float ut = *reinterpret_cast<const float*>(xs + L.ua[p]);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const float f = fmaf((float)acc[p][2 * h], L.wa, (float)acc[p][2 * h + 1] * L.wb);
            accm[p][h] = fmaf(d[h] * ut, f, accm[p][h]);
        }
    }
#pragma unroll
    for (int q = 0; q < NQ; q++) {
        const uint2 bs = *reinterpret_cast<const uint2*>(xs + L.xm[q]);
        float co[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(co, a[0][0], a[1][0], a[0][1], a[1][1], bs.x, bs.y);
        const float uo = *reinterpret_cast<const float*>(xs + L.um[q]) * 67108864.f;
#pragma unroll
        for (int h = 0; h < 2; h++) accn[q][h] = fmaf(d[h] * uo, co[2 * h] + co[2 * h + 1], accn[q][h]);
    }
}

// The fp16 scales of row g + 8h's eight blocks, DW[h] (16 bytes), as floats.
__device__ __forceinline__ void block_scales(const uint4 (&DW)[2], float (&dd)[2][8]) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint32_t w[4] = {DW[h].x, DW[h].y, DW[h].z, DW[h].w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            dd[h][2 * i] = lo_half(w[i]);
            dd[h][2 * i + 1] = hi_half(w[i]);
        }
    }
}

// One block's MMA result C (rows g, g + 8; this lane's digit columns) into
// the chunk's block-scaled sums ACCF: the two digit columns weigh 256 : 1
// (their common factor, L.wb, is applied with the chunk's unscale), so one
// integer multiply-add joins them (|C| < 2^19, the sum < 2^28).
__device__ __forceinline__ void block_sum(const int (&c)[4], float d0, float d1, float (&accf)[2]) {
    accf[0] = fmaf(d0, (float)(c[0] * 256 + c[1]), accf[0]);
    accf[1] = fmaf(d1, (float)(c[2] * 256 + c[3]), accf[1]);
}

// Q8_0 over NP pairs, one chunk (eight blocks): QV[h][i] = this lane's 16
// code bytes of blocks 2i, 2i + 1 in row g + 8h (per block: elements
// 4t..4t+3, then 16+4t..16+4t+3); DW[h] = the row's eight fp16 scales.
// Codes are signed bytes: one s8 x s8 MMA per block and pair, no offset term.
template <int NP>
__device__ __forceinline__ void q8_0_i8_chunk_n(const I8LaneN<kQ8_0, NP>& L, const uint4 (&QV)[2][4],
                                                const uint4 (&DW)[2], const unsigned char* xs,
                                                float (&accm)[NP][2]) {
    float dd[2][8];
    block_scales(DW, dd);
    float accf[NP][2];
#pragma unroll
    for (int p = 0; p < NP; p++) accf[p][0] = accf[p][1] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
#pragma unroll
        for (int p = 0; p < NP; p++) {
            const uint4 b = reinterpret_cast<const uint4*>(xs + L.xb[p])[16 * j];
            int c[4];
            imma_k32_ss(c, QV[0][j].x, QV[1][j].x, QV[0][j].y, QV[1][j].y, b.x, b.y);
            block_sum(c, dd[0][2 * j], dd[1][2 * j], accf[p]);
            imma_k32_ss(c, QV[0][j].z, QV[1][j].z, QV[0][j].w, QV[1][j].w, b.z, b.w);
            block_sum(c, dd[0][2 * j + 1], dd[1][2 * j + 1], accf[p]);
        }
    }
#pragma unroll
    for (int p = 0; p < NP; p++) {
        const float ut = *reinterpret_cast<const float*>(xs + L.ua[p]) * L.wb;
#pragma unroll
        for (int h = 0; h < 2; h++) accm[p][h] = fmaf(ut, accf[p][h], accm[p][h]);
    }
}

// Q4_0 over NP pairs, one chunk: QW[h][b] = this lane's code word of block b
// in row g + 8h (low nibbles elements 4t..4t+3, high nibbles 16+4t..);
// DW[h] = the row's eight fp16 scales.  Codes enter the u8 x s8 MMA as they
// are (0..15); the offset term 8 sum_b d_b S_b (to be subtracted) is one fp16
// MMA per chunk and group of four rows: A = the scales of blocks 2t, 2t + 1
// (fp16, exact), B = hi + lo halves of the block sums of X.
template <int NP>
__device__ __forceinline__ void q4_0_i8_chunk_n(const I8LaneN<kQ4_0, NP>& L, const uint32_t (&QW)[2][8],
                                                const uint4 (&DW)[2], const unsigned char* xs,
                                                float (&accm)[NP][2], float (&accn)[(NP + 1) / 2][2]) {
    constexpr int NQ = (NP + 1) / 2;
    float dd[2][8];
    block_scales(DW, dd);
    float accf[NP][2];
#pragma unroll
    for (int p = 0; p < NP; p++) accf[p][0] = accf[p][1] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int b = 2 * j + e;
            const uint32_t lo0 = QW[0][b] & 0x0F0F0F0Fu, lo1 = QW[1][b] & 0x0F0F0F0Fu;
            const uint32_t hi0 = (QW[0][b] >> 4) & 0x0F0F0F0Fu, hi1 = (QW[1][b] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int p = 0; p < NP; p++) {
                const uint4 bx = reinterpret_cast<const uint4*>(xs + L.xb[p])[16 * j];
                int c[4];
                imma_k32(c, lo0, lo1, hi0, hi1, e ? bx.z : bx.x, e ? bx.w : bx.y);
                block_sum(c, dd[0][b], dd[1][b], accf[p]);
            }
        }
    }
#pragma unroll
    for (int p = 0; p < NP; p++) {
        const float ut = *reinterpret_cast<const float*>(xs + L.ua[p]) * L.wb;
#pragma unroll
        for (int h = 0; h < 2; h++) accm[p][h] = fmaf(ut, accf[p][h], accm[p][h]);
    }
    // the scales of blocks 2t, 2t + 1: word t of each row's scales (selects,
    // not an index, so DW stays in registers)
    uint32_t am[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint32_t a01 = (L.t & 1) ? DW[h].y : DW[h].x, a23 = (L.t & 1) ? DW[h].w : DW[h].z;
        am[h] = (L.t & 2) ? a23 : a01;
    }
#pragma unroll
    for (int q = 0; q < NQ; q++) {
        float cm[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(cm, am[0], am[1], 0u, 0u, *reinterpret_cast<const uint32_t*>(xs + L.xm[q]), 0u);
        const float u8 = *reinterpret_cast<const float*>(xs + L.um[q]) * 16777216.f;  // times 8 * 2^21
#pragma unroll
        for (int h = 0; h < 2; h++) accn[q][h] = fmaf(u8, cm[2 * h] + cm[2 * h + 1], accn[q][h]);
    }
}

// End of a tile for pair P: ACCM = accm[P][h], ACCN = accn[P / 2][h].  Lanes
// with even t return row g + 8h of activation row 2P + t / 2.
template <int D, int NP>
__device__ __forceinline__ float i8_finish_n(const I8LaneN<D, NP>& L, int p, float accm, float accn) {
    const float m = accm + __shfl_xor_sync(0xffffffffu, accm, 1);
    const int lane = threadIdx.x & 31;
    const float n = __shfl_sync(0xffffffffu, accn, (lane & ~3) | (2 * (p & 1) + (L.t >> 1)));
    return m - n;
}

}  // namespace
}  // namespace clq
