// layout.cuh -- the device layout of a packed weight ("planes") and its
// bit-exact element decode.
//
// A store keeps the weight re-tiled from GGUF's interleaved blocks into up to
// three planes so that each lane of the product kernels reads its bytes as
// aligned 16-byte runs.  Re-tiling only moves bytes: every decoded value is
// the one packed-element gives for the native block.
//
//   Q4_K  q: the native 144-byte superblocks (already 16-byte aligned).
//   Q4_0  q: 16 code bytes per block; within a row, each chunk of 8 blocks is
//            stored lane-major: lane t (0..3) holds code bytes [4t, 4t+4) of
//            blocks 0..7 of the chunk, 32 contiguous bytes.
//         d: fp16 scale per block.
//   Q8_0  q: 32 code bytes per block; chunk of 8 blocks lane-major: lane t
//            holds bytes [4t,4t+4) and [16+4t,16+4t+4) of blocks 0..7 (64 B).
//         d: fp16 scale per block.
//   Q6_K  q: ql+qh (192 B) per superblock, lane-major: lane t holds, for
//            (h, half) in (0,0),(0,1),(1,0),(1,1), the words
//            ql[64h+16half+4t], ql[64h+32+16half+4t], qh[32h+16half+4t] (48 B).
//         s: the 16 int8 sub-scales per superblock; d: fp16 scale per superblock.
// A partial chunk at the end of a row (fewer than 8 blocks, Q4_0/Q8_0 only)
// uses the same lane-major order over the blocks it has.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "formats.cuh"

namespace clq {

struct PlaneGeometry {
    int q_block;  // bytes per block in the q plane
    int s_block;  // bytes per block in the s plane (0 = none)
    int d_block;  // bytes per block in the d plane (0 = none)
};

__host__ __device__ inline PlaneGeometry plane_geometry(int dtype) {
    switch (dtype) {
    case kQ4_0: return {16, 0, 2};
    case kQ8_0: return {32, 0, 2};
    case kQ4_K: return {144, 0, 0};
    case kQ6_K: return {192, 16, 2};
    default: return {0, 0, 0};
    }
}

inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Offsets of the planes for NBLOCKS blocks; *total includes 256 B of zeroed tail.
inline void plane_offsets(int dtype, int64_t nblocks, size_t* s_off, size_t* d_off, size_t* total) {
    PlaneGeometry g = plane_geometry(dtype);
    size_t q = align256((size_t)nblocks * g.q_block);
    size_t s = align256((size_t)nblocks * g.s_block);
    size_t d = align256((size_t)nblocks * g.d_block);
    *s_off = q;
    *d_off = q + s;
    *total = q + s + d + 256;
}

struct Planes {
    const uint8_t* q;
    const uint8_t* s;
    const uint8_t* d;
    int64_t nb;  // blocks per row
};

__device__ __forceinline__ float half_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }

__device__ __forceinline__ float d_of(const Planes& p, int64_t blk) {
    return half_bits((uint16_t)p.d[2 * blk] | ((uint16_t)p.d[2 * blk + 1] << 8));
}

// Byte offset, inside a row's q plane, of code byte `byte` of block j, for the
// lane-major chunks of Q4_0 (16 code bytes) and Q8_0 (32 code bytes).
template <int CODE_BYTES>
__host__ __device__ __forceinline__ int64_t chunk_code_offset(int64_t nb, int64_t j, int byte) {
    const int64_t c = j / 8, b = j % 8;
    const int64_t nbc = (nb - 8 * c) < 8 ? (nb - 8 * c) : 8;  // blocks in this chunk
    const int half = byte / 16, t = (byte % 16) / 4, bw = byte % 4;
    constexpr int words = CODE_BYTES / 16;  // words per (lane, block): 1 (Q4_0) or 2 (Q8_0)
    return c * 8 * CODE_BYTES + (int64_t)t * (4 * words * nbc) + b * 4 * words + 4 * half + bw;
}

// Q6_K: offsets (inside the 192-byte q block) of the ql and qh bytes of element i.
__host__ __device__ __forceinline__ void q6k_offsets(int i, int& ql_off, int& qh_off, int& sc_idx,
                                                    int& lo_shift, int& hi_shift) {
    const int h = i >> 7, grp = (i & 127) >> 5, l = i & 31;
    const int half = l >> 4, t = (l & 15) >> 2, bw = l & 3;
    const int base = t * 48 + (h * 2 + half) * 12;
    ql_off = base + (grp & 1) * 4 + bw;
    qh_off = base + 8 + bw;
    sc_idx = 8 * h + 2 * grp + half;
    lo_shift = 4 * (grp >> 1);
    hi_shift = 2 * grp;
}

// Element e of row `row` in the reference's fp32 operation order (bit-exact).
template <int D> __device__ __forceinline__ float element_planar(const Planes& p, int64_t row, int64_t e);

template <> __device__ __forceinline__ float element_planar<kQ4_K>(const Planes& p, int64_t row, int64_t e) {
    return element_exact<kQ4_K>(p.q + (row * p.nb + e / 256) * 144, (int)(e % 256));
}

template <> __device__ __forceinline__ float element_planar<kQ4_0>(const Planes& p, int64_t row, int64_t e) {
    const int64_t j = e / 32;
    const int i = (int)(e % 32);
    const uint8_t byte = p.q[row * p.nb * 16 + chunk_code_offset<16>(p.nb, j, i & 15)];
    const int nib = i < 16 ? (byte & 15) : (byte >> 4);
    return __fmul_rn(d_of(p, row * p.nb + j), (float)(nib - 8));
}

template <> __device__ __forceinline__ float element_planar<kQ8_0>(const Planes& p, int64_t row, int64_t e) {
    const int64_t j = e / 32;
    const int i = (int)(e % 32);
    const int8_t q = (int8_t)p.q[row * p.nb * 32 + chunk_code_offset<32>(p.nb, j, i)];
    return __fmul_rn(d_of(p, row * p.nb + j), (float)q);
}

template <> __device__ __forceinline__ float element_planar<kQ6_K>(const Planes& p, int64_t row, int64_t e) {
    const int64_t blk = row * p.nb + e / 256;
    int ql, qh, sc_idx, ls, hs;
    q6k_offsets((int)(e % 256), ql, qh, sc_idx, ls, hs);
    const uint8_t* q = p.q + blk * 192;
    const int lo = (q[ql] >> ls) & 15, hi = (q[qh] >> hs) & 3;
    const int sc = (int8_t)p.s[blk * 16 + sc_idx];
    return __fmul_rn(__fmul_rn(d_of(p, blk), (float)sc), (float)((lo | (hi << 4)) - 32));
}

}  // namespace clq
