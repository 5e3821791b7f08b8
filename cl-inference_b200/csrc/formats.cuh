// formats.cuh -- GGUF block layouts and the bit-exact element decode, device side.
//
// Layouts (little-endian, quant/packed.lisp:85-108, quant/q8-0.lisp:113-117):
//   Q8_0  34 B / 32:  [0:2] fp16 d, [2:34] int8 q[32];           v = d*q
//   Q4_0  18 B / 32:  [0:2] fp16 d, [2:18] qs; e<16 low nibble of qs[e],
//                     else high nibble of qs[e-16];              v = d*(nib-8)
//   Q4_K 144 B / 256: [0:2] d, [2:4] dmin, [4:16] 6-bit scales/mins,
//                     [16:144] qs (qs[32*(g/2)+l] >> 4*(g%2));  v = (d*sc)*q - dmin*m
//   Q6_K 210 B / 256: [0:128] ql, [128:192] qh, [192:208] int8 scales,
//                     [208:210] d;                               v = (d*sc)*(q-32)
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace clq {

enum Dtype : int { kQ4_0 = 2, kQ8_0 = 8, kQ4_K = 12, kQ6_K = 14 };

template <int D> struct Geometry;
template <> struct Geometry<kQ4_0> { static constexpr int kElems = 32, kBytes = 18; };
template <> struct Geometry<kQ8_0> { static constexpr int kElems = 32, kBytes = 34; };
template <> struct Geometry<kQ4_K> { static constexpr int kElems = 256, kBytes = 144; };
template <> struct Geometry<kQ6_K> { static constexpr int kElems = 256, kBytes = 210; };

// fp16 -> fp32 is exact for every finite half, subnormals included, so this is
// the value block-scale (quant/q8-0.lisp:89-96) computes for exponents 0..30.
__device__ __forceinline__ float half_at(const uint8_t* p) {
    uint16_t bits = (uint16_t)p[0] | ((uint16_t)p[1] << 8);
    return __half2float(__ushort_as_half(bits));
}

// Byte offsets of the fp16 scales a block decodes (checked at store creation:
// exponent 31 is "Quantized scale is not finite", quant/q8-0.lisp:95).
__host__ __device__ inline int scale_offsets(int dtype, int* off) {
    switch (dtype) {
    case kQ4_0: case kQ8_0: off[0] = 0; return 1;
    case kQ4_K: off[0] = 0; off[1] = 2; return 2;
    case kQ6_K: off[0] = 208; return 1;
    default: return 0;
    }
}

// Q4_K 6-bit scale and min of sub-block g (quant/packed.lisp:91-98).
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int g, int& sc, int& mn) {
    if (g < 4) {
        sc = s[g] & 63;
        mn = s[g + 4] & 63;
    } else {
        sc = (s[g + 4] & 15) | ((s[g - 4] & 192) >> 2);
        mn = (s[g + 4] >> 4) | ((s[g] & 192) >> 2);
    }
}

// Element e of the block at b, in the reference's fp32 operation order.
// __fmul_rn/__fsub_rn keep the compiler from contracting into an FMA.
template <int D> __device__ __forceinline__ float element_exact(const uint8_t* b, int e);

template <> __device__ __forceinline__ float element_exact<kQ8_0>(const uint8_t* b, int e) {
    return __fmul_rn(half_at(b), (float)(int8_t)b[2 + e]);
}
template <> __device__ __forceinline__ float element_exact<kQ4_0>(const uint8_t* b, int e) {
    int byte = b[2 + (e & 15)];
    int nib = e < 16 ? (byte & 15) : (byte >> 4);
    return __fmul_rn(half_at(b), (float)(nib - 8));
}
template <> __device__ __forceinline__ float element_exact<kQ4_K>(const uint8_t* b, int e) {
    int g = e >> 5, sc, mn;
    q4k_scale_min(b + 4, g, sc, mn);
    int q = (b[16 + 32 * (g >> 1) + (e & 31)] >> (4 * (g & 1))) & 15;
    float v = __fmul_rn(__fmul_rn(half_at(b), (float)sc), (float)q);
    return __fsub_rn(v, __fmul_rn(half_at(b + 2), (float)mn));
}
template <> __device__ __forceinline__ float element_exact<kQ6_K>(const uint8_t* b, int e) {
    int h = e >> 7, g = (e & 127) >> 5, l = e & 31;
    int lo = (b[h * 64 + (g & 1) * 32 + l] >> (4 * (g >> 1))) & 15;
    int hi = (b[128 + h * 32 + l] >> (2 * g)) & 3;
    int sc = (int8_t)b[192 + h * 8 + g * 2 + (l >> 4)];
    return __fmul_rn(__fmul_rn(half_at(b + 208), (float)sc), (float)((lo | (hi << 4)) - 32));
}

}  // namespace clq
