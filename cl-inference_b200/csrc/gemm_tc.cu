// gemm_tc.cu -- prefill GEMM for packed weights on the 5th-generation tensor
// cores: tcgen05.mma (kind::f16, fp32 accumulator in tensor memory).
//
// out[t, r] = sum_k x[t, k] * W[r, k] for many activation rows t (prompt
// tokens).  One CTA computes a 128-row weight tile x TN-token tile over a range
// of K (split-K when the output has too few tiles for the machine):
//   prep kernel  x -> fp16 scaled by a per-token power of two, written to
//                scratch pre-swizzled (SWIZZLE_128B image of every 64-wide
//                K block), so a plain 1-D bulk copy lands a ready MMA operand;
//   warps 0-7    dequantize the weight tile (fp32 math, one rounding to fp16)
//                straight into the swizzled A stage, two threads per weight
//                row; later the epilogue;
//   warp 8       bulk-copies the activation stage (B), mbarrier tx-count;
//   warp 9       one thread issues the MMAs and commits stages back.
// The MMA operands are fp16 (weights rounded once; activations rounded once
// after the power-of-two scaling), products accumulate in fp32.
// Every mbarrier wait is bounded; on expiry the CTA records CLQ_ERR_TIMEOUT in
// the library's device status word (read by clq_device_status), stops
// issuing, drains what it issued and frees its tensor memory.
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/clq.h"
#include "clq_internal.h"
#include "layout.cuh"
#include "tma_host.h"

namespace clq {
namespace {

constexpr int kTM = 128;          // weight rows per CTA (the MMA's M)
constexpr int kKB = 64;           // K elements per stage (one 128-byte swizzle span of fp16)
constexpr int kStages = 4;
constexpr int kThreads = 320;     // warps 0-7 dequant/epilogue, 8 copy, 9 MMA
constexpr uint32_t kWaitLimit = 1u << 26;  // polls before a wait gives up

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with PARITY; false (and *err set) when it gives up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        if (mbar_test(bar, parity)) return true;
        if (*(volatile int*)err) return false;
        if (i > 64) __nanosleep(32);
    }
    atomicExch(err, CLQ_ERR_TIMEOUT);
    return false;
}
// Bounded wait that ignores the error flag: used before teardown so that copies
// and MMAs this CTA issued have finished before it exits.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 22); i++) {
        if (mbar_test(bar, parity)) return;
        if (i > 64) __nanosleep(64);
    }
}
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: fp16 A and B (K-major), fp32 D, M = 128, N = n.
__host__ __device__ constexpr uint32_t instr_desc(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// Byte offset of 16-byte chunk C of row R in a SWIZZLE_128B K-major tile.
__host__ __device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) { return r * 128 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// ---- activation prep ------------------------------------------------------

// One CTA per activation row: power-of-two scale putting max|x| in [2^14, 2^15),
// then the fp16 values in the swizzled tile image:
//   xs[((tt * KBt + kb) * TN + r) * 128 + swz]   (row t = tt * TN + r)
// and us[t] = 1 / scale.  Rows t in [m, m_pad) are written as zeros.
template <typename XT>
__global__ void prep_x_kernel(const XT* __restrict__ x, int64_t m, int64_t k, int tn, uint8_t* __restrict__ xs,
                              float* __restrict__ us, uint8_t* __restrict__ xs_lo) {
    const int64_t t = blockIdx.x;
    const int64_t tt = t / tn, r = t % tn;
    const int64_t kbt = k / kKB;
    __shared__ float red[32];
    float amax = 0.f;
    if (t < m)
        for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
            float v;
            if constexpr (sizeof(XT) == 4) v = (float)x[t * k + i];
            else if constexpr (std::is_same<XT, __half>::value) v = __half2float(x[t * k + i]);
            else v = __bfloat162float(x[t * k + i]);
            amax = fmaxf(amax, fabsf(v));
        }
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    amax = red[0];
    int sexp = 0;
    if (amax > 0.f) {
        int e = (int)((__float_as_uint(amax) >> 23) & 255) - 127;
        sexp = 14 - e;
        sexp = sexp < -120 ? -120 : (sexp > 120 ? 120 : sexp);
    }
    const float scale = __uint_as_float((uint32_t)(127 + sexp) << 23);
    if (threadIdx.x == 0) us[t] = __uint_as_float((uint32_t)(127 - sexp) << 23);
    // 16-byte chunks of 8 elements
    for (int64_t cidx = threadIdx.x; cidx < k / 8; cidx += blockDim.x) {
        const int64_t kb = cidx / 8;
        const int c = (int)(cidx % 8);
        uint4 v = make_uint4(0, 0, 0, 0), vl = make_uint4(0, 0, 0, 0);
        if (t < m) {
            float f[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int64_t i = cidx * 8 + j;
                if constexpr (sizeof(XT) == 4) f[j] = (float)x[t * k + i];
                else if constexpr (std::is_same<XT, __half>::value) f[j] = __half2float(x[t * k + i]);
                else f[j] = __bfloat162float(x[t * k + i]);
                f[j] *= scale;
            }
            v.x = pack_half2(f[0], f[1]);
            v.y = pack_half2(f[2], f[3]);
            v.z = pack_half2(f[4], f[5]);
            v.w = pack_half2(f[6], f[7]);
            if (xs_lo) {
                // the rest of each value, times 2^11 (back in the fp16 range
                // of the value itself), so that hi + lo / 2^11 carries ~22 bits
                float g[8];
                const uint32_t hv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&hv[j]));
                    g[2 * j] = (f[2 * j] - h.x) * 2048.f;
                    g[2 * j + 1] = (f[2 * j + 1] - h.y) * 2048.f;
                }
                vl.x = pack_half2(g[0], g[1]);
                vl.y = pack_half2(g[2], g[3]);
                vl.z = pack_half2(g[4], g[5]);
                vl.w = pack_half2(g[6], g[7]);
            }
        }
        const int64_t off = (tt * kbt + kb) * tn * 128 + swz((uint32_t)r, (uint32_t)c);
        *reinterpret_cast<uint4*>(xs + off) = v;
        if (xs_lo) *reinterpret_cast<uint4*>(xs_lo + off) = vl;
    }
}

// ---- weight dequantization into the swizzled A stage -----------------------
//
// Two threads per weight row of the tile, each converting half of a 64-wide K
// block (32 values, 4 swizzled 16-byte chunks).  load_raw fetches the
// quantized bytes into registers one stage ahead; convert_raw decodes them
// with exact fp16 integer tricks (code bits ORed into the mantissa of 1024.0,
// one fused multiply-add to remove the bias and apply a sub-scale) and rounds
// each weight to fp16 at most twice.

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
__device__ __forceinline__ uint32_t dup_half(float v) {  // (fp16(v), fp16(v))
    const uint32_t h = __half_as_ushort(__float2half_rn(v));
    return h | (h << 16);
}
constexpr uint32_t kMagic = 0x64646464u;
constexpr uint32_t kH1024 = 0x64006400u;
constexpr uint32_t kH1056 = 0x64206420u;  // 1024 + 32
constexpr uint32_t kHSixteenth = 0x2C002C00u;
constexpr uint32_t kHNeg1024 = 0xE400E400u;
constexpr uint32_t kHNeg64 = 0xD400D400u;
constexpr uint32_t kLoNib = 0x640F640Fu;
constexpr uint32_t kHiNib = 0x64F064F0u;
constexpr uint32_t kH1032 = 0x64086408u;   // 1024 + 8
constexpr uint32_t kH1152 = 0x64806480u;   // 1024 + 128
constexpr uint32_t kHNeg72 = 0xD480D480u;

template <int D> struct Raw;
template <> struct Raw<kQ4_K> { uint4 hd, cw; };                          // header, 16 code bytes
template <> struct Raw<kQ6_K> { uint32_t w[12]; uint4 sv; uint32_t d; };  // lane quads 2hv, 2hv+1: 6 words each
// Q4_0 / Q8_0: the K block's two 32-element blocks, lane-quad words 0..3 of
// each (Q4_0: all 16 code bytes; Q8_0: the half of the 32 this thread
// converts), and their two fp16 scales
template <> struct Raw<kQ4_0> { uint32_t w[2][4]; uint32_t d2; };
template <> struct Raw<kQ8_0> { uint32_t w[2][4]; uint32_t d2; };

// Q6_K block KB's code words for lane quads 2hv, 2hv + 1 (superblock BLK).
__device__ __forceinline__ void load_words_q6k(const Planes& p, int64_t blk, int64_t kb, int hv, Raw<kQ6_K>& r) {
    // lane-major plane (layout.cuh): lane quad t's words for (hh, half) sit at
    // t*48 + (2hh + half)*12; the 24 bytes of one hh start 16-byte aligned
    // when hh = 0 and 8 bytes past alignment when hh = 1 (warp-uniform).
    const int hh = (int)((kb & 3) >> 1);
#pragma unroll
    for (int tq = 0; tq < 2; tq++) {
        const uint8_t* q = p.q + blk * 192 + (2 * hv + tq) * 48 + 24 * hh;
        uint32_t* w = &r.w[6 * tq];
        if (hh == 0) {
            const uint4 a = *reinterpret_cast<const uint4*>(q);
            const uint2 b = *reinterpret_cast<const uint2*>(q + 16);
            w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y;
        } else {
            const uint2 a = *reinterpret_cast<const uint2*>(q);
            const uint4 b = *reinterpret_cast<const uint4*>(q + 8);
            w[0] = a.x; w[1] = a.y; w[2] = b.x; w[3] = b.y; w[4] = b.z; w[5] = b.w;
        }
    }
}

template <int D>
__device__ __forceinline__ void load_raw(const Planes& p, int64_t grow, int64_t kb, int hv, Raw<D>& r) {
    if constexpr (D == kQ4_K) {
        const uint8_t* b = p.q + (grow * p.nb + (kb >> 2)) * 144;
        const int qt = (int)(kb & 3);
        r.hd = *reinterpret_cast<const uint4*>(b);
        r.cw = *reinterpret_cast<const uint4*>(b + 16 + 32 * qt + 16 * hv);
    } else if constexpr (D == kQ6_K) {
        const int64_t blk = grow * p.nb + (kb >> 2);
        load_words_q6k(p, blk, kb, hv, r);
        r.sv = *reinterpret_cast<const uint4*>(p.s + blk * 16);
        r.d = *reinterpret_cast<const unsigned short*>(p.d + 2 * blk);
    } else {
        // lane-major chunks of 8 blocks (layout.cuh, chunk_code_offset): lane
        // quad t's words of blocks b, b+1 of chunk c; blocks 2kb, 2kb+1 share a chunk
        constexpr int CB = D == kQ4_0 ? 16 : 32, words = CB / 16;
        const int64_t j0 = 2 * kb, c = j0 / 8, b = j0 % 8;
        const int64_t nbc = p.nb - 8 * c < 8 ? p.nb - 8 * c : 8;
        const uint8_t* base = p.q + grow * p.nb * CB + c * 8 * CB;
        if (!(nbc & 1)) {  // blocks b, b + 1 adjacent and aligned: one load per lane quad
#pragma unroll
            for (int t = 0; t < 4; t++) {
                if constexpr (D == kQ4_0) {
                    const uint2 v = *reinterpret_cast<const uint2*>(base + (t * nbc + b) * 4);
                    r.w[0][t] = v.x;
                    r.w[1][t] = v.y;
                } else {
                    const uint4 v = *reinterpret_cast<const uint4*>(base + (t * nbc + b) * 8);
                    r.w[0][t] = hv ? v.y : v.x;
                    r.w[1][t] = hv ? v.w : v.z;
                }
            }
        } else {
#pragma unroll
            for (int jb = 0; jb < 2; jb++)
#pragma unroll
                for (int t = 0; t < 4; t++)
                    r.w[jb][t] = *reinterpret_cast<const uint32_t*>(base + (D == kQ8_0 ? 4 * hv : 0) +
                                                                    (t * nbc + b + jb) * 4 * words);
        }
        r.d2 = *reinterpret_cast<const uint32_t*>(p.d + 2 * (grow * p.nb + j0));
    }
}

// Q4_K block KB's codes only (its header is its superblock's first block's).
__device__ __forceinline__ void load_codes_q4k(const Planes& p, int64_t grow, int64_t kb, int hv, Raw<kQ4_K>& r) {
    const uint8_t* b = p.q + (grow * p.nb + (kb >> 2)) * 144;
    r.cw = *reinterpret_cast<const uint4*>(b + 16 + 32 * (int)(kb & 3) + 16 * hv);
}

// Half hv of row `row`: four of its eight 16-byte chunks -- {2hv, 2hv+1,
// 4+2hv, 5+2hv} for Q4_K/Q4_0/Q8_0 (elements 16hv..16hv+15 of each 32),
// {hv, 2+hv, 4+hv, 6+hv} for Q6_K (lane quads 2hv, 2hv+1).
template <int D>
__device__ __forceinline__ void convert_raw(const Planes& p, int64_t grow, int64_t kb, int hv, const Raw<D>& rw,
                                            uint32_t row, uint8_t* a) {
    uint4 ch[4];
    int ci[4] = {2 * hv, 2 * hv + 1, 4 + 2 * hv, 5 + 2 * hv};
    if constexpr (D == kQ4_K) {
        const int qt = (int)(kb & 3);
        auto sbyte = [&](int i) -> uint32_t {  // scale byte i of the 12, runtime index
            const int wsel = i >> 2;
            const uint32_t w = wsel == 0 ? rw.hd.y : wsel == 1 ? rw.hd.z : rw.hd.w;
            return (w >> (8 * (i & 3))) & 0xFF;
        };
        uint32_t sc[2], mn[2];
#pragma unroll
        for (int u = 0; u < 2; u++) {  // quant/packed.lisp:91-98
            const int g = 2 * qt + u;
            if (g < 4) {
                sc[u] = sbyte(g) & 63;
                mn[u] = sbyte(g + 4) & 63;
            } else {
                sc[u] = (sbyte(g + 4) & 15) | ((sbyte(g - 4) & 192) >> 2);
                mn[u] = (sbyte(g + 4) >> 4) | ((sbyte(g) & 192) >> 2);
            }
        }
        const float dmin = __half2float(__ushort_as_half((unsigned short)(rw.hd.x >> 16)));
        const uint32_t D2 = prmt(rw.hd.x, rw.hd.x, 0x1010);  // (d, d)
        const uint32_t SC0 = hsub2(prmt(sc[0], kMagic, 0x4040), kH1024), SC1 = hsub2(prmt(sc[1], kMagic, 0x4040), kH1024);
        const uint32_t N0 = hmul2(SC0, kHNeg1024), N1 = hmul2(SC1, kHNeg64), S1 = hmul2(SC1, kHSixteenth);
        const uint32_t M0 = dup_half(-dmin * (float)mn[0]), M1 = dup_half(-dmin * (float)mn[1]);
        const uint32_t cw[4] = {rw.cw.x, rw.cw.y, rw.cw.z, rw.cw.w};
        uint32_t g0[8], g1[8];
#pragma unroll
        for (int wi = 0; wi < 4; wi++) {
            const uint32_t p01 = prmt(cw[wi], kMagic, 0x4140), p23 = prmt(cw[wi], kMagic, 0x4342);
            // sc*q exact in fp16, then one fused d*(sc*q) - dmin*m
            g0[2 * wi] = hfma2(hfma2(p01 & kLoNib, SC0, N0), D2, M0);
            g0[2 * wi + 1] = hfma2(hfma2(p23 & kLoNib, SC0, N0), D2, M0);
            g1[2 * wi] = hfma2(hfma2(p01 & kHiNib, S1, N1), D2, M1);
            g1[2 * wi + 1] = hfma2(hfma2(p23 & kHiNib, S1, N1), D2, M1);
        }
        ch[0] = make_uint4(g0[0], g0[1], g0[2], g0[3]);
        ch[1] = make_uint4(g0[4], g0[5], g0[6], g0[7]);
        ch[2] = make_uint4(g1[0], g1[1], g1[2], g1[3]);
        ch[3] = make_uint4(g1[4], g1[5], g1[6], g1[7]);
    } else if constexpr (D == kQ6_K) {
        const int odd = (int)(kb & 1);  // group pair {2odd, 2odd+1} of the 128-element half hh
        const int hh = (int)((kb & 3) >> 1);
        const float d = __half2float(__ushort_as_half((unsigned short)rw.d));
        auto sc = [&](int i) -> int {
            const int wsel = i >> 2;
            const uint32_t w = wsel == 0 ? rw.sv.x : wsel == 1 ? rw.sv.y : wsel == 2 ? rw.sv.z : rw.sv.w;
            return (int)(int8_t)((w >> (8 * (i & 3))) & 0xFF);
        };
        // words of (t = 2hv + tq, half): wv[6 tq + 3 half + {0: ql p0, 1: ql p1, 2: qh}]
        const uint32_t* wv = rw.w;
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int grp = 2 * odd + u;
            const int lo_shift = 4 * (grp >> 1);  // low or high nibble of ql
            const int qsh = 2 * grp;              // qh bit position
#pragma unroll
            for (int half = 0; half < 2; half++) {
                // (d * sc) rounded to fp16 once; the product with (q - 32) rounds once more
                const uint32_t FS = dup_half(d * (float)sc(8 * hh + 2 * grp + half));
                uint32_t pr[4];
#pragma unroll
                for (int tq = 0; tq < 2; tq++) {
                    const uint32_t* w3 = &wv[6 * tq + 3 * half];
                    // four 6-bit codes (elements l = 16 half + 4 (2hv + tq) + 0..3), one per byte lane
                    const uint32_t q = ((w3[u] >> lo_shift) & 0x0F0F0F0Fu) | (((w3[2] >> qsh) & 0x03030303u) << 4);
                    pr[2 * tq] = hmul2(hsub2(prmt(q, kMagic, 0x4140), kH1056), FS);
                    pr[2 * tq + 1] = hmul2(hsub2(prmt(q, kMagic, 0x4342), kH1056), FS);
                }
                ch[2 * u + half] = make_uint4(pr[0], pr[1], pr[2], pr[3]);
                ci[2 * u + half] = 4 * u + 2 * half + hv;
            }
        }
    } else {
        // Q4_0 / Q8_0: chunk i holds elements 16hv + 8(i & 1) .. + 7 of block
        // i >> 1 -- words 2(i & 1) and 2(i & 1) + 1, four elements each.  The
        // code becomes an exact small integer in fp16 (Q4_0: nibble - 8, from
        // the low nibbles for hv = 0 and the high ones for hv = 1; Q8_0: the
        // signed byte), and one multiply by d rounds it once, as rounding the
        // exact fp32 product of quant/packed.lisp:89-90 / q8-0.lisp:115-117 does
        const uint32_t DD[2] = {prmt(rw.d2, rw.d2, 0x1010), prmt(rw.d2, rw.d2, 0x3232)};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t v[4];
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const uint32_t w = rw.w[i >> 1][2 * (i & 1) + (h >> 1)];
                const uint32_t sel = (h & 1) ? 0x4342u : 0x4140u;
                uint32_t q;
                if constexpr (D == kQ4_0) {
                    const uint32_t pq = prmt(w, kMagic, sel);
                    q = hv ? hfma2(pq & kHiNib, kHSixteenth, kHNeg72) : hsub2(pq & kLoNib, kH1032);
                } else {
                    q = hsub2(prmt(w ^ 0x80808080u, kMagic, sel), kH1152);
                }
                v[h] = hmul2(q, DD[i >> 1]);
            }
            ch[i] = make_uint4(v[0], v[1], v[2], v[3]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) *reinterpret_cast<uint4*>(a + swz(row, (uint32_t)ci[i])) = ch[i];
}

// The exact form of convert_raw: each element's fp32 value as the reference
// computes it (quant/packed.lisp:89-108, the oracle's element functions,
// operations in the same order), split into hi = fp16(w) and
// lo = fp16((w - hi) * 2^11), written to A (chunks as convert_raw's) and A_LO.
__device__ __forceinline__ void put_split(float w0, float w1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(w0, w1);
    const float2 hf = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = pack_half2(__fmul_rn(__fsub_rn(w0, hf.x), 2048.f), __fmul_rn(__fsub_rn(w1, hf.y), 2048.f));
}
__device__ __forceinline__ float u2f(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.f; }  // v < 2^23

template <int D>
__device__ __forceinline__ void convert_raw_exact(const Planes& p, int64_t grow, int64_t kb, int hv, const Raw<D>& rw,
                                                  uint32_t row, uint8_t* a, uint8_t* a_lo) {
    uint32_t hi[4][4], lo[4][4];
    int ci[4] = {2 * hv, 2 * hv + 1, 4 + 2 * hv, 5 + 2 * hv};
    if constexpr (D == kQ4_K) {
        const int qt = (int)(kb & 3);
        auto sbyte = [&](int i) -> uint32_t {
            const int wsel = i >> 2;
            const uint32_t w = wsel == 0 ? rw.hd.y : wsel == 1 ? rw.hd.z : rw.hd.w;
            return (w >> (8 * (i & 3))) & 0xFF;
        };
        float ds[2], dm[2];
        const float d = __half2float(__ushort_as_half((unsigned short)(rw.hd.x & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(rw.hd.x >> 16)));
#pragma unroll
        for (int u = 0; u < 2; u++) {  // quant/packed.lisp:91-98
            const int g = 2 * qt + u;
            uint32_t sc, mn;
            if (g < 4) {
                sc = sbyte(g) & 63;
                mn = sbyte(g + 4) & 63;
            } else {
                sc = (sbyte(g + 4) & 15) | ((sbyte(g - 4) & 192) >> 2);
                mn = (sbyte(g + 4) >> 4) | ((sbyte(g) & 192) >> 2);
            }
            ds[u] = __fmul_rn(d, u2f(sc));
            dm[u] = __fmul_rn(dmin, u2f(mn));
        }
        const uint32_t cw[4] = {rw.cw.x, rw.cw.y, rw.cw.z, rw.cw.w};
        // code byte j: element j of this half of sub-block 2qt (low nibble) and 2qt + 1 (high)
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const uint32_t b0 = (cw[j >> 2] >> (8 * (j & 3))) & 0xFF, b1 = (cw[j >> 2] >> (8 * ((j + 1) & 3))) & 0xFF;
            const float l0 = __fsub_rn(__fmul_rn(ds[0], u2f(b0 & 15)), dm[0]);
            const float l1 = __fsub_rn(__fmul_rn(ds[0], u2f(b1 & 15)), dm[0]);
            const float h0 = __fsub_rn(__fmul_rn(ds[1], u2f(b0 >> 4)), dm[1]);
            const float h1 = __fsub_rn(__fmul_rn(ds[1], u2f(b1 >> 4)), dm[1]);
            put_split(l0, l1, hi[j >> 3][(j & 7) >> 1], lo[j >> 3][(j & 7) >> 1]);
            put_split(h0, h1, hi[2 + (j >> 3)][(j & 7) >> 1], lo[2 + (j >> 3)][(j & 7) >> 1]);
        }
    } else if constexpr (D == kQ6_K) {
        const int odd = (int)(kb & 1);
        const int hh = (int)((kb & 3) >> 1);
        const float d = __half2float(__ushort_as_half((unsigned short)rw.d));
        auto sc = [&](int i) -> int {
            const int wsel = i >> 2;
            const uint32_t w = wsel == 0 ? rw.sv.x : wsel == 1 ? rw.sv.y : wsel == 2 ? rw.sv.z : rw.sv.w;
            return (int)(int8_t)((w >> (8 * (i & 3))) & 0xFF);
        };
        const uint32_t* wv = rw.w;
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int grp = 2 * odd + u;
            const int lo_shift = 4 * (grp >> 1), qsh = 2 * grp;
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const float ds = __fmul_rn(d, (float)sc(8 * hh + 2 * grp + half));  // quant/packed.lisp:107-108
#pragma unroll
                for (int tq = 0; tq < 2; tq++) {
                    const uint32_t* w3 = &wv[6 * tq + 3 * half];
                    const uint32_t q = ((w3[u] >> lo_shift) & 0x0F0F0F0Fu) | (((w3[2] >> qsh) & 0x03030303u) << 4);
                    float e[4];
#pragma unroll
                    for (int b = 0; b < 4; b++) e[b] = __fmul_rn(ds, (float)((int)((q >> (8 * b)) & 0xFF) - 32));
                    put_split(e[0], e[1], hi[2 * u + half][2 * tq], lo[2 * u + half][2 * tq]);
                    put_split(e[2], e[3], hi[2 * u + half][2 * tq + 1], lo[2 * u + half][2 * tq + 1]);
                }
                ci[2 * u + half] = 4 * u + 2 * half + hv;
            }
        }
    } else {
        // Q4_0 / Q8_0: chunk i as convert_raw's; w = d * code in fp32
        // (quant/packed.lisp:89-90, quant/q8-0.lisp:115-117)
        const float dd[2] = {__half2float(__ushort_as_half((unsigned short)(rw.d2 & 0xFFFF))),
                             __half2float(__ushort_as_half((unsigned short)(rw.d2 >> 16)))};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float e[8];
#pragma unroll
            for (int x = 0; x < 8; x++) {
                const uint32_t byte = (rw.w[i >> 1][2 * (i & 1) + (x >> 2)] >> (8 * (x & 3))) & 0xFF;
                const int code = D == kQ4_0 ? (int)(hv ? byte >> 4 : byte & 15) - 8 : (int)(int8_t)byte;
                e[x] = __fmul_rn(dd[i >> 1], (float)code);
            }
#pragma unroll
            for (int h = 0; h < 4; h++) put_split(e[2 * h], e[2 * h + 1], hi[i][h], lo[i][h]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        *reinterpret_cast<uint4*>(a + swz(row, (uint32_t)ci[i])) = make_uint4(hi[i][0], hi[i][1], hi[i][2], hi[i][3]);
        *reinterpret_cast<uint4*>(a_lo + swz(row, (uint32_t)ci[i])) = make_uint4(lo[i][0], lo[i][1], lo[i][2], lo[i][3]);
    }
}

struct GemmParams {
    Planes p;
    int64_t rows, k, m;
    const uint8_t* xs;  // swizzled fp16 activations
    const float* us;    // per-token unscale
    float* out;         // final output (splits == 1) or partials [split][m][rows]
    int64_t ldo;
    int tn;             // tokens per tile (power of two, 32..256)
    int kb_per_split;
    int stages;         // pipeline depth (2..4)
    const uint8_t* xs_lo;  // exact form: the activations' scaled low parts, or null
    int* err;           // the device status word
};

// EXACT: the weights as fp16 hi plus a low part times 2^11 (two A tiles per
// stage), and for fp32 activations (P.xs_lo set) the activations likewise
// (two B tiles).  The hi x hi products accumulate in tensor-memory columns
// [0, tn), the lo x hi and hi x lo ones in [tn, 2 tn), and the epilogue adds
// the second accumulator times 2^-11: fp32-class products (about 22 bits of
// each operand) from fp16 MMAs, three per K step instead of one.
template <int D, bool EXACT>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(GemmParams P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzle atoms
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    // the fp16-operand form always plans kStages stages: a compile-time depth
    const int tn = P.tn, NS = EXACT ? P.stages : kStages;
    const bool xlo = EXACT && P.xs_lo != nullptr;
    constexpr uint32_t kA = (EXACT ? 2u : 1u) * kTM * 128;  // per stage: hi (and lo) weight tiles
    const uint32_t kBt = (uint32_t)tn * 128, kB = (xlo ? 2u : 1u) * kBt;
    uint8_t* A = smem;                                   // NS x kA
    uint8_t* B = A + (size_t)NS * kA;                    // NS x kB
    uint64_t* full_a = reinterpret_cast<uint64_t*>(B + (size_t)NS * kB);
    uint64_t* full_b = full_a + kStages;
    uint64_t* empty = full_b + kStages;
    uint64_t* done = empty + kStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tt = blockIdx.x;                 // token tile
    const int64_t row0 = (int64_t)blockIdx.y * kTM;
    const int split = blockIdx.z;
    const int64_t kbt = P.k / kKB;
    const int64_t kb0 = (int64_t)split * P.kb_per_split;
    const int64_t kb1 = (kb0 + P.kb_per_split) < kbt ? (kb0 + P.kb_per_split) : kbt;
    const int nk = (int)(kb1 - kb0);
    const uint32_t cols = EXACT ? 2u * (uint32_t)tn : (uint32_t)tn;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full_a[s], 8);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // tensor memory: tn fp32 columns x 128 lanes (two accumulators when exact)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    int* err = P.err;

    if (warp < 8) {
        // ---- weight tiles: thread i converts half (i / 128) of row (i % 128) ----
        const uint32_t row = (uint32_t)(threadIdx.x & 127);
        const int hv = threadIdx.x >> 7;
        const int64_t grow_u = row0 + row;
        const int64_t grow = grow_u < P.rows ? grow_u : P.rows - 1;
        // Each packed word is loaded once: a Q4_K block after the first of its
        // superblock loads only its codes (the header is kept from the first);
        // an odd Q6_K block loads nothing (it reads the even block's words,
        // sub-scales and scale) and the third block of a superblock only its
        // words.  The kept parts are filled in when a block is converted, from
        // blocks already in registers, so no copy waits on a load in flight.
        Raw<D> r0, r1, r2;  // stages it, it+1, it+2
        Raw<D> even;        // Q6_K: the last even block converted
        uint4 hd_sb = {};   // Q4_K: the current superblock's header
        (void)even;
        (void)hd_sb;
        if (nk > 0) load_raw<D>(P.p, grow, kb0, hv, r0);
        if (nk > 1) load_raw<D>(P.p, grow, kb0 + 1, hv, r1);
        for (int it = 0; it < nk; it++) {
            const int s = it % NS;
            if (it + 2 < nk) {  // two stages in flight
                const int64_t kb = kb0 + it + 2;
                if constexpr (D == kQ6_K) {
                    if (!(kb & 1)) {
                        if (kb & 3) load_words_q6k(P.p, grow * P.p.nb + (kb >> 2), kb, hv, r2);
                        else load_raw<D>(P.p, grow, kb, hv, r2);
                    }
                } else if constexpr (D == kQ4_K) {
                    if (kb & 3) load_codes_q4k(P.p, grow, kb, hv, r2);
                    else load_raw<D>(P.p, grow, kb, hv, r2);
                } else {
                    load_raw<D>(P.p, grow, kb, hv, r2);
                }
            }
            const int64_t b = kb0 + it;
            if constexpr (D == kQ4_K) {  // the first two blocks were loaded whole
                if (it < 2 || !(b & 3)) hd_sb = r0.hd;
                else r0.hd = hd_sb;
            } else if constexpr (D == kQ6_K) {
                if (it >= 2 && (b & 1)) {
                    r0 = even;
                } else {
                    if (it >= 2 && (b & 3)) {
                        r0.sv = even.sv;
                        r0.d = even.d;
                    }
                    even = r0;
                }
            }
            if (it >= NS && !mbar_wait(&empty[s], ((it / NS) - 1) & 1, err)) break;
            if constexpr (EXACT)
                convert_raw_exact<D>(P.p, grow, kb0 + it, hv, r0, row, A + (size_t)s * kA, A + (size_t)s * kA + kTM * 128);
            else
                convert_raw<D>(P.p, grow, kb0 + it, hv, r0, row, A + (size_t)s * kA);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_a[s]);
            r0 = r1;
            r1 = r2;
        }
        // ---- epilogue: tensor memory -> out; warp w: lanes 32 (w % 4).., column half w / 4 ----
        const bool ok = mbar_wait(done, 0, err);
        tc_fence_after();
        if (ok) {
            const int q = warp & 3, ch = warp >> 2;
            const int64_t r = row0 + 32 * q + lane;
            const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16);
            const int cbeg = ch * (tn / 2), cend = cbeg + tn / 2;
            for (int c0 = cbeg; c0 < cend; c0 += 16) {
                uint32_t v[16], vc[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                    "[%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15])
                    : "r"(taddr + (uint32_t)c0));
                if constexpr (EXACT) {
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                        "[%16];"
                        : "=r"(vc[0]), "=r"(vc[1]), "=r"(vc[2]), "=r"(vc[3]), "=r"(vc[4]), "=r"(vc[5]), "=r"(vc[6]),
                          "=r"(vc[7]), "=r"(vc[8]), "=r"(vc[9]), "=r"(vc[10]), "=r"(vc[11]), "=r"(vc[12]), "=r"(vc[13]),
                          "=r"(vc[14]), "=r"(vc[15])
                        : "r"(taddr + (uint32_t)(tn + c0)));
                }
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (r < P.rows) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int64_t t = tt * tn + c0 + j;
                        if (t < P.m) {
                            float acc = __uint_as_float(v[j]);
                            if constexpr (EXACT) acc = fmaf(__uint_as_float(vc[j]), 4.8828125e-4f, acc);  // + 2^-11 corr
                            const float val = acc * P.us[t];
                            if (gridDim.z == 1) P.out[t * P.ldo + r] = val;
                            else P.out[((int64_t)split * P.m + t) * P.rows + r] = val;
                        }
                    }
                }
            }
        }
    } else if (warp == 8) {
        // ---- activation tiles: one bulk copy per stage ----
        if (lane == 0) {
            for (int it = 0; it < nk; it++) {
                const int s = it % NS;
                if (it >= NS && !mbar_wait(&empty[s], ((it / NS) - 1) & 1, err)) break;
                const int64_t off = ((tt * kbt + kb0 + it) * tn) * 128;
                mbar_arrive_tx(&full_b[s], kB);
                bulk_copy(B + (size_t)s * kB, P.xs + off, kBt, &full_b[s]);
                if (xlo) bulk_copy(B + (size_t)s * kB + kBt, P.xs_lo + off, kBt, &full_b[s]);
            }
        }
    } else {
        // ---- MMA issue ----
        if (lane == 0) {
            const uint32_t idesc = instr_desc(tn);
            int it = 0;
            for (; it < nk; it++) {
                const int s = it % NS;
                const uint32_t ph = (it / NS) & 1;
                if (!mbar_wait(&full_a[s], ph, err) || !mbar_wait(&full_b[s], ph, err)) break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(A + (size_t)s * kA), b_addr = smem_u32(B + (size_t)s * kB);
#pragma unroll
                for (int j = 0; j < kKB / 16; j++) {
                    const uint32_t acc = (it > 0 || j > 0) ? 1u : 0u;
                    mma_f16(tmem, smem_desc(a_addr + 32 * j), smem_desc(b_addr + 32 * j), idesc, acc);
                    if constexpr (EXACT) {
                        // lo(w) x hi(x), then hi(w) x lo(x), into the correction accumulator
                        mma_f16(tmem + (uint32_t)tn, smem_desc(a_addr + kTM * 128 + 32 * j), smem_desc(b_addr + 32 * j),
                                idesc, acc);
                        if (xlo)
                            mma_f16(tmem + (uint32_t)tn, smem_desc(a_addr + 32 * j), smem_desc(b_addr + kBt + 32 * j),
                                    idesc, 1u);
                    }
                }
                mma_commit(&empty[s]);
            }
            mma_commit(done);  // arrives once every MMA issued above has completed
            mbar_drain(done, 0);
        }
    }
    // Bulk copies in flight must land before the CTA exits.
    if (warp == 8 && lane == 0) {
        for (int it = nk - NS < 0 ? 0 : nk - NS; it < nk; it++) mbar_drain(&full_b[it % NS], (it / NS) & 1);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols) : "memory");
    }
}

// ---- Q4_K prefill GEMM: 256-row tiles, packed bytes staged by TMA ------------
//
// The Q4_K form of the GEMM above for weights of at least 256 rows.  One CTA
// computes 256 weight rows x TN tokens as two 128-row MMAs into two tensor-
// memory accumulators that read the same activation stage, so every
// activation byte staged from L2 serves twice the products of a 128-row tile.
// The packed bytes are staged a superblock column at a time (256 rows x 144
// bytes, four 64-wide K blocks) by a copy warp with one tensor-map box (this
// GPU's own store, one destination), two superblocks ahead.  Sixteen
// converting warps (two threads a row) dequantize from shared memory into
// the two swizzled A halves.  A, B and the packed superblocks each have their
// own ring:
//   warps 0-15  convert; later the epilogue (warp w: TMEM lanes 32 (w % 4)..,
//               accumulator (w / 8), half of its columns by (w / 4) % 2)
//   warp 16     bulk-copies the activation stages (B)
//   warp 17     one thread issues the MMAs, committing each stage back
//   warp 18     tensor-map copies of the packed superblocks
constexpr int kRT = 256;                     // weight rows per CTA
constexpr int kTConv = 16;                   // converting warps
constexpr int kTThreads = (kTConv + 3) * 32;
constexpr int kTMaxStages = 4, kTPD = 2;     // A / B ring depths at most; superblocks in flight
constexpr uint32_t kPackStage = kRT * 144;

struct GemmTmaParams {
    CUtensorMap qmap;  // q plane as [rows][nb * 144] bytes, box 144 x 256 (a superblock column)
    Planes p;          // the register-fed form reads the packed words directly
    int64_t rows, k, m;
    const uint8_t* xs;
    const float* us;
    float* out;
    int64_t ldo;
    int tn;            // tokens per tile: a multiple of 16, at most 256
    int na, nbs;       // A and B ring depths
    int kb_per_split;
    int* err;
};

__device__ __forceinline__ void tma_box(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Bounded wait that spins without sleeping (stages are a few hundred cycles).
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int* err) {
    for (uint32_t i = 0; i < kWaitLimit; i++) {
        if (mbar_test(bar, parity)) return true;
        if ((i & 1023) == 1023 && *(volatile int*)err) return false;
    }
    atomicExch(err, CLQ_ERR_TIMEOUT);
    return false;
}

// STAGED: the packed superblocks come through the tensor-map ring; otherwise
// each converting thread loads its packed words from global memory into
// registers two blocks ahead (as gemm_tc_kernel's converters do).
template <bool STAGED>
__global__ void __launch_bounds__(kTThreads, 1) gemm_q4k_tma_kernel(const __grid_constant__ GemmTmaParams P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int tn = P.tn, NA = P.na, NB = P.nbs;
    const uint32_t a_stage = 2u * kTM * 128, b_stage = (uint32_t)tn * 128;
    uint8_t* A = smem;                                // NA x 32 KB (two 128-row halves)
    uint8_t* B = A + (size_t)NA * a_stage;            // NB x tn * 128
    uint8_t* Pk = B + (size_t)NB * b_stage;           // kTPD x (headers, codes)
    Pk = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(Pk) + 127) & ~(uintptr_t)127);
    uint64_t* full_a = reinterpret_cast<uint64_t*>(Pk + (STAGED ? kTPD * kPackStage : 0u));
    uint64_t* empty_a = full_a + kTMaxStages;
    uint64_t* full_b = empty_a + kTMaxStages;
    uint64_t* empty_b = full_b + kTMaxStages;
    uint64_t* full_p = empty_b + kTMaxStages;
    uint64_t* empty_p = full_p + kTPD;
    uint64_t* done = empty_p + kTPD;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tt = blockIdx.x;
    const int64_t row0 = (int64_t)blockIdx.y * kRT;
    const int split = blockIdx.z;
    const int64_t kbt = P.k / kKB;
    const int64_t kb0 = (int64_t)split * P.kb_per_split;
    const int64_t kb1 = (kb0 + P.kb_per_split) < kbt ? (kb0 + P.kb_per_split) : kbt;
    const int nk = (int)(kb1 - kb0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < NA; s++) {
            mbar_init(&full_a[s], kTConv);
            mbar_init(&empty_a[s], 1);
        }
        for (int s = 0; s < NB; s++) {
            mbar_init(&full_b[s], 1);
            mbar_init(&empty_b[s], 1);
        }
        for (int s = 0; s < kTPD; s++) {
            mbar_init(&full_p[s], 1);
            mbar_init(&empty_p[s], kTConv);
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // two accumulators of up to 256 fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    int* err = P.err;

    if (warp < kTConv) {
        // ---- convert: thread i takes half (i / 256) of row (i % 256) ----
        const uint32_t row = (uint32_t)(threadIdx.x & 255);
        const int hv = threadIdx.x >> 8;
        const uint32_t half_row = row & 127;
        uint8_t* a_half = A + (row >> 7) * (kTM * 128);
        const Planes none{};
        // the split starts at block kb0: superblock kb0 / 4, quarter kb0 % 4
        const int q0 = (int)(kb0 & 3);
        if constexpr (!STAGED) {
            const int64_t grow_u = row0 + row;
            const int64_t grow = grow_u < P.rows ? grow_u : P.rows - 1;
            Raw<kQ4_K> r0, r1, r2;  // blocks it, it + 1, it + 2
            if (nk > 0) load_raw<kQ4_K>(P.p, grow, kb0, hv, r0);
            if (nk > 1) load_raw<kQ4_K>(P.p, grow, kb0 + 1, hv, r1);
            for (int it = 0; it < nk; it++) {
                if (it + 2 < nk) load_raw<kQ4_K>(P.p, grow, kb0 + it + 2, hv, r2);
                const int sa = it % NA;
                if (it >= NA && !mbar_wait_spin(&empty_a[sa], (uint32_t)((it / NA) - 1) & 1u, err)) break;
                convert_raw<kQ4_K>(none, 0, kb0 + it, hv, r0, half_row, a_half + sa * a_stage);
                fence_async_shared();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full_a[sa]);
                r0 = r1;
                r1 = r2;
            }
        }
        for (int it = 0; STAGED && it < nk; it++) {
            const int sbi = (q0 + it) >> 2, qt = (q0 + it) & 3;
            const int ps = sbi % kTPD;
            if ((qt == 0 || it == 0) && !mbar_wait_spin(&full_p[ps], (uint32_t)(sbi / kTPD) & 1u, err)) break;
            const int sa = it % NA;
            if (it >= NA && !mbar_wait_spin(&empty_a[sa], (uint32_t)((it / NA) - 1) & 1u, err)) break;
            const uint8_t* pk = Pk + ps * kPackStage + row * 144;
            Raw<kQ4_K> rw;
            rw.hd = *reinterpret_cast<const uint4*>(pk);
            rw.cw = *reinterpret_cast<const uint4*>(pk + 16 + 32 * qt + 16 * hv);
            convert_raw<kQ4_K>(none, 0, kb0 + it, hv, rw, half_row, a_half + sa * a_stage);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&full_a[sa]);
                if (qt == 3 || it == nk - 1) mbar_arrive(&empty_p[ps]);  // this warp is done with the superblock
            }
        }
        // ---- epilogue: tensor memory -> out ----
        const bool fin = mbar_wait(done, 0, err);
        tc_fence_after();
        if (fin) {
            const int lq = warp & 3, acc = warp >> 3, ch = (warp >> 2) & 1;
            const int64_t r = row0 + acc * kTM + 32 * lq + lane;
            const uint32_t taddr = tmem + ((uint32_t)(32 * lq) << 16) + (uint32_t)(acc * 256);
            const int cbeg = ch * (tn / 2), cend = cbeg + tn / 2;
            for (int c0 = cbeg; c0 < cend; c0 += 8) {
                uint32_t v[8];
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                             : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                               "=r"(v[7])
                             : "r"(taddr + (uint32_t)c0));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (r < P.rows) {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int64_t t = tt * tn + c0 + j;
                        if (t < P.m) {
                            const float val = __uint_as_float(v[j]) * P.us[t];
                            if (gridDim.z == 1) P.out[t * P.ldo + r] = val;
                            else P.out[((int64_t)split * P.m + t) * P.rows + r] = val;
                        }
                    }
                }
            }
        }
    } else if (warp == kTConv) {
        // ---- activation stages: one bulk copy each ----
        if (lane == 0) {
            int it = 0;
            for (; it < nk; it++) {
                const int s = it % NB;
                if (it >= NB && !mbar_wait(&empty_b[s], (uint32_t)((it / NB) - 1) & 1u, err)) break;
                mbar_arrive_tx(&full_b[s], b_stage);
                bulk_copy(B + (size_t)s * b_stage, P.xs + ((tt * kbt + kb0 + it) * tn) * 128, b_stage, &full_b[s]);
            }
            // copies in flight land before the CTA exits
            for (int v = it - NB < 0 ? 0 : it - NB; v < it; v++) mbar_drain(&full_b[v % NB], (uint32_t)(v / NB) & 1u);
        }
    } else if (warp == kTConv + 1) {
        // ---- MMA issue: both 128-row halves against the same activation stage ----
        if (lane == 0) {
            const uint32_t idesc = instr_desc(tn);
            for (int it = 0; it < nk; it++) {
                const int sa = it % NA, sbs = it % NB;
                if (!mbar_wait_spin(&full_a[sa], (uint32_t)(it / NA) & 1u, err) ||
                    !mbar_wait_spin(&full_b[sbs], (uint32_t)(it / NB) & 1u, err))
                    break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(A + (size_t)sa * a_stage), b_addr = smem_u32(B + (size_t)sbs * b_stage);
#pragma unroll
                for (int h = 0; h < 2; h++)
#pragma unroll
                    for (int kk = 0; kk < kKB / 16; kk++)
                        mma_f16(tmem + (uint32_t)(h * 256), smem_desc(a_addr + h * (kTM * 128) + 32 * kk),
                                smem_desc(b_addr + 32 * kk), idesc, (it > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&empty_a[sa]);
                mma_commit(&empty_b[sbs]);
            }
            mma_commit(done);  // arrives once every MMA issued above has completed
            mbar_drain(done, 0);
        }
    } else if (STAGED) {
        // ---- packed superblocks: one tensor-map box each ----
        if (lane == 0) {
            const int nsb = (int)(((kb1 + 3) >> 2) - (kb0 >> 2));
            int s = 0;
            for (; s < nsb; s++) {
                const int ps = s % kTPD;
                if (s >= kTPD && !mbar_wait(&empty_p[ps], (uint32_t)((s / kTPD) - 1) & 1u, err)) break;
                mbar_arrive_tx(&full_p[ps], kPackStage);
                tma_box(Pk + ps * kPackStage, &P.qmap, (int)(((kb0 >> 2) + s) * 144), (int)row0, &full_p[ps]);
            }
            for (int v = s - kTPD < 0 ? 0 : s - kTPD; v < s; v++) mbar_drain(&full_p[v % kTPD], (uint32_t)(v / kTPD) & 1u);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

// out[t * ldo + r] = sum over splits of part[split][t][r], fixed order.
// V = 4: four consecutive r per thread (rows, ldo and out 16-byte aligned);
// every split's load is issued before the sum, in batches of eight.
template <int V>
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int64_t m, int64_t rows,
                                     float* __restrict__ out, int64_t ldo) {
    using Vec = typename std::conditional<V == 4, float4, float>::type;
    const int64_t total = m * rows, rv = rows / V, nv = m * rv;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / rv, r = (i - t * rv) * V;
        const float* src = part + t * rows + r;
        float acc[V];
#pragma unroll
        for (int c = 0; c < V; c++) acc[c] = 0.f;
        for (int j0 = 0; j0 < splits; j0 += 8) {
            Vec v[8];
#pragma unroll
            for (int b = 0; b < 8; b++)
                if (j0 + b < splits) v[b] = *reinterpret_cast<const Vec*>(src + (int64_t)(j0 + b) * total);
#pragma unroll
            for (int b = 0; b < 8; b++) {
                if (j0 + b < splits) {
                    const float* f = reinterpret_cast<const float*>(&v[b]);
#pragma unroll
                    for (int c = 0; c < V; c++) acc[c] += f[c];
                }
            }
        }
        float* dst = out + t * ldo + r;
        if constexpr (V == 4) *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        else dst[0] = acc[0];
    }
}

// Which kernel takes Q4_K weights of at least 256 rows (CLQ_GEMM_TMA, a
// tuning knob): 0 the 128-row register-fed gemm_tc_kernel (the default, the
// fastest measured), 1 the 256-row kernel with tensor-map staged packed
// superblocks, 2 the 256-row kernel with register-fed packed words.
int gemm_q4k_mode() {
    static int mode = -1;
    if (mode < 0) {
        const char* e = getenv("CLQ_GEMM_TMA");
        mode = e ? atoi(e) : 0;
        if (mode < 0 || mode > 2) mode = 0;
    }
    return mode;
}
bool gemm_tma_enabled() { return gemm_q4k_mode() != 0; }

int sm_count_gemm() {
    static int count = 0;
    if (!count) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || count <= 0)
            count = 148;
    }
    return count;
}

}  // namespace

namespace {
bool takes_tma(int dtype, int64_t rows) { return gemm_tma_enabled() && rows >= kRT && dtype == kQ4_K; }

// Shared memory of the Q4_K kernel and its ring depths: B as deep as fits
// (at least two), then A (at least two).
size_t tma_smem(int tn, bool staged, int* na, int* nb) {
    const size_t fixed = 1024 + 128 + (staged ? (size_t)kTPD * kPackStage : 0) + 512, b_stage = (size_t)tn * 128;
    const size_t a_stage = 2 * (size_t)kTM * 128, limit = 227 * 1024;
    for (int b = kTMaxStages; b >= 2; b--)
        for (int a = 3; a >= 2; a--) {
            const size_t total = fixed + (size_t)a * a_stage + (size_t)b * b_stage;
            if (total <= limit) {
                *na = a;
                *nb = b;
                return total;
            }
        }
    *na = *nb = 2;
    return fixed + 2 * a_stage + 2 * b_stage;
}

int split_count(int64_t ctas, int64_t kbt) {
    int64_t splits = 1;
    const int64_t want = sm_count_gemm();
    while (ctas * splits < want && kbt / (splits * 2) >= 4) splits *= 2;
    while (splits > 1 && kbt % splits) splits /= 2;  // every split gets the same, non-zero K range
    return (int)splits;
}

// Tuning knob: CLQ_GEMM_TN fixes the Q4_K kernel's tokens per tile (a
// multiple of 16 up to 256); by default the plan picks it.
int env_tn() {
    static int v = -2;
    if (v == -2) {
        const char* e = getenv("CLQ_GEMM_TN");
        v = e ? atoi(e) : -1;
        if (v != -1 && (v < 16 || v > 256 || v % 16)) v = -1;
    }
    return v;
}
}  // namespace

GemmPlan plan_gemm_tc(int dtype, int64_t rows, int64_t k, int64_t m, bool exact, bool xlo) {
    GemmPlan g;
    g.exact = exact;
    g.xlo = exact && xlo;
    const int64_t kbt = k / kKB;
    if (!exact && takes_tma(dtype, rows)) {
        // 256-row tiles; tokens per tile chosen so the tiles fill whole waves:
        // a tile costs max(4 tn, 900) cycles per 64-wide K block (its MMAs,
        // or the dequantization of 256 rows), a wave costs its slowest tile
        g.row_tile = kRT;
        g.row_tiles = (rows + kRT - 1) / kRT;
        const int64_t sms = sm_count_gemm();
        int best_tn = 256;
        double best = 1e300;
        for (int tn = 256; tn >= 32; tn -= 16) {
            if (env_tn() > 0 && tn != env_tn()) continue;
            if (tn < 256 && (tn - 16) >= m) continue;  // a smaller tile than the tokens need
            const int64_t tiles = (m + tn - 1) / tn * g.row_tiles;
            const int sp = split_count(tiles, kbt);
            const double waves = (double)((tiles * sp + sms - 1) / sms);
            const double cost = waves * (4.0 * tn > 900.0 ? 4.0 * tn : 900.0) / sp;
            if (cost < best * 0.999) {
                best = cost;
                best_tn = tn;
            }
        }
        g.tn = best_tn;
    } else {
        g.row_tile = kTM;
        g.row_tiles = (rows + kTM - 1) / kTM;
        int tn = 32;
        // the exact form doubles the weight tiles (and activation tiles for
        // fp32 activations): at most 128 tokens a tile keeps three stages
        while (tn < (exact ? 128 : 256) && tn < m) tn *= 2;
        g.tn = tn;
    }
    g.token_tiles = (m + g.tn - 1) / g.tn;
    g.splits = split_count(g.token_tiles * g.row_tiles, kbt);
    g.kb_per_split = (int)((kbt + g.splits - 1) / g.splits);
    g.xs_bytes = (size_t)g.token_tiles * g.tn * k * 2 * (g.xlo ? 2 : 1);  // hi image, then lo
    g.us_bytes = (size_t)g.token_tiles * g.tn * sizeof(float);
    g.part_bytes = g.splits > 1 ? (size_t)g.splits * m * rows * sizeof(float) : 0;
    const size_t per_stage = (size_t)kTM * 128 * (exact ? 2 : 1) + (size_t)g.tn * 128 * (g.xlo ? 2 : 1);
    g.stages = kStages;
    while (exact && g.stages > 2 && 1024 + (size_t)g.stages * per_stage + 256 > 227 * 1024) g.stages--;
    g.smem = 1024 + (size_t)g.stages * per_stage + 256;
    return g;
}

GemmPlan plan_gemm_tc_capped(int dtype, int64_t rows, int64_t k, int64_t m, size_t cap) {
    GemmPlan g = plan_gemm_tc(dtype, rows, k, m, false, false);
    while (g.splits > 1 && gemm_tc_scratch_bytes(g) > cap) {
        g.splits /= 2;
        const int64_t kbt = k / kKB;
        g.kb_per_split = (int)((kbt + g.splits - 1) / g.splits);
        g.part_bytes = g.splits > 1 ? (size_t)g.splits * m * rows * sizeof(float) : 0;
    }
    if (gemm_tc_scratch_bytes(g) > cap) g.splits = 0;  // does not fit even unsplit
    return g;
}

size_t gemm_tc_scratch_bytes(const GemmPlan& g) {
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    return al(g.xs_bytes) + al(g.us_bytes) + al(g.part_bytes);
}

bool gemm_tc_supported(const WeightView& w, int64_t m) { return w.k > 0 && w.k % 256 == 0 && m > 0; }

cudaError_t launch_gemm_tc(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m, float* out,
                           int64_t ldo, uint8_t* scratch, const GemmPlan& g, cudaStream_t stream, bool prepped) {
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    // an expired wait is reported through the status word clq_device_status reads
    int* err = device_status_word();
    if (!err) return cudaErrorNotSupported;
    uint8_t* xs = scratch;
    uint8_t* xs_lo = g.xlo ? xs + g.xs_bytes / 2 : nullptr;
    float* us = reinterpret_cast<float*>(xs + al(g.xs_bytes));
    float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(us) + al(g.us_bytes));
    cudaError_t e = cudaSuccess;
    const unsigned prep_grid = (unsigned)(g.token_tiles * g.tn);
    switch (prepped ? -1 : xtype) {
    case -1: break;
    case CLQ_X_F32:
        prep_x_kernel<float><<<prep_grid, 256, 0, stream>>>((const float*)x, m, w.k, g.tn, xs, us, xs_lo);
        break;
    case CLQ_X_BF16:
        prep_x_kernel<__nv_bfloat16><<<prep_grid, 256, 0, stream>>>((const __nv_bfloat16*)x, m, w.k, g.tn, xs, us,
                                                                     xs_lo);
        break;
    case CLQ_X_F16:
        prep_x_kernel<__half><<<prep_grid, 256, 0, stream>>>((const __half*)x, m, w.k, g.tn, xs, us, xs_lo);
        break;
    default: return cudaErrorInvalidValue;
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    GemmParams P;
    P.p = Planes{w.q, w.s, w.d, w.nb};
    P.rows = rows;
    P.k = w.k;
    P.m = m;
    P.xs = xs;
    P.us = us;
    P.out = g.splits > 1 ? part : out;
    P.ldo = ldo;
    P.tn = g.tn;
    P.kb_per_split = g.kb_per_split;
    P.stages = g.stages;
    P.xs_lo = xs_lo;
    P.err = err;
    dim3 grid((unsigned)g.token_tiles, (unsigned)g.row_tiles, (unsigned)g.splits);
    auto launch = [&](auto kern) -> cudaError_t {
        cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
        if (r != cudaSuccess) return r;
        kern<<<grid, kThreads, g.smem, stream>>>(P);
        return cudaGetLastError();
    };
    // Q4_K of at least 256 rows: 256-row tiles with tensor-map staged packed bytes
    if (g.row_tile == kRT) {
        if (w.dtype != kQ4_K || rows < kRT) return cudaErrorInvalidValue;  // a plan made for another weight
        GemmTmaParams T;
        const int64_t row_bytes = w.nb * 144;
        const bool staged = gemm_q4k_mode() == 1;
        if (staged && !encode_rows(&T.qmap, w.q, rows, row_bytes, 144, kRT)) return cudaErrorNotSupported;
        T.p = P.p;
        T.rows = rows;
        T.k = w.k;
        T.m = m;
        T.xs = xs;
        T.us = us;
        T.out = P.out;
        T.ldo = ldo;
        T.tn = g.tn;
        T.kb_per_split = g.kb_per_split;
        T.err = err;
        const size_t smem = tma_smem(g.tn, staged, &T.na, &T.nbs);
        auto kern = staged ? gemm_q4k_tma_kernel<true> : gemm_q4k_tma_kernel<false>;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        dim3 tgrid((unsigned)g.token_tiles, (unsigned)g.row_tiles, (unsigned)g.splits);
        kern<<<tgrid, kTThreads, smem, stream>>>(T);
        e = cudaGetLastError();
    } else {
        switch (w.dtype) {
        case kQ4_K: e = g.exact ? launch(gemm_tc_kernel<kQ4_K, true>) : launch(gemm_tc_kernel<kQ4_K, false>); break;
        case kQ6_K: e = g.exact ? launch(gemm_tc_kernel<kQ6_K, true>) : launch(gemm_tc_kernel<kQ6_K, false>); break;
        case kQ4_0: e = g.exact ? launch(gemm_tc_kernel<kQ4_0, true>) : launch(gemm_tc_kernel<kQ4_0, false>); break;
        case kQ8_0: e = g.exact ? launch(gemm_tc_kernel<kQ8_0, true>) : launch(gemm_tc_kernel<kQ8_0, false>); break;
        default: return cudaErrorInvalidValue;
        }
    }
    if (e != cudaSuccess || g.splits == 1) return e;
    const bool vec = rows % 4 == 0 && ldo % 4 == 0 && (uintptr_t)out % 16 == 0;
    const int64_t items = m * rows / (vec ? 4 : 1);
    const int rb = (int)((items + 255) / 256 < 148 * 8 ? (items + 255) / 256 : 148 * 8);
    if (vec) splitk_reduce_kernel<4><<<rb, 256, 0, stream>>>(part, g.splits, m, rows, out, ldo);
    else splitk_reduce_kernel<1><<<rb, 256, 0, stream>>>(part, g.splits, m, rows, out, ldo);
    return cudaGetLastError();
}

}  // namespace clq
