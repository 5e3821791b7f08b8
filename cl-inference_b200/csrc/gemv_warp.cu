// gemv_warp.cu -- decode GEMV (one to eight activation rows) for Q4_K, Q6_K,
// Q4_0 and Q8_0 with an independent weight stream per warp.
//
// One persistent CTA of 16 warps per SM owns a contiguous range of 16-row
// tiles.  Its (tile, chunk) units -- 16 rows x 256 columns, tile-major -- are
// cut into contiguous runs of equal length, one per warp.  Each warp streams
// its own run: one lane copies each unit as one box of a 2-D tensor map over
// the weight's q plane (16 rows x one chunk's bytes) into a ring of DEPTH
// slots in shared memory, with completion counted on one mbarrier per slot
// (rows past the weight's end read as zeros); the warp waits for a slot,
// reads its words, refills the
// slot with the unit DEPTH ahead and multiplies with the integer-MMA product
// of gemv_i8.cuh -- for several activation rows, one MMA per pair of rows on
// the same unpacked weight fragments (NP pairs, up to eight rows).  No warp
// waits for another except once, after the activations are staged, so a slow
// warp never stalls the others' streams.
//
// A tile's K range can be split between consecutive warps.  A tile inside one
// warp's run is finished by that warp from its registers.  For a tile shared
// by several warps, each leaves its partial sum (a "piece") in shared memory
// -- one slot per warp for the first tile of its run, one for the last -- and
// counts it on the tile's counter; the warp that completes the count adds the
// tile's pieces in warp order -- a fixed order, so results do not depend on
// timing.  Finished tiles are written out or, under tensor parallelism, sent
// to every rank.
//
// A CTA stages the activations of every chunk it reads (4 bytes per element
// and row).  When those of all of K do not fit beside the rings -- several
// activation rows, or long rows -- K is split between the KS CTAs of a tile
// group: each stages and reads only its split, leaves its tile sums in a
// global scratch and counts them on the tile's counter, and the split that
// completes the count adds the KS partials in split order (again a fixed
// order) and writes the outputs.
//
// The copies do not depend on the previous kernel (the weights are constant):
// under programmatic dependent launch each warp starts its ring before
// griddepcontrol.wait and fills it once its activation loads are out; only
// the activation staging waits for the previous kernel.  The weight stream is
// read with an L2 evict-first policy.  Every wait is bounded (pipeline.cuh); after an expired wait the
// warp stops, drains the copies it issued, and the status word reports it.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <unordered_map>
#include <vector>

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/clq.h"
#include "fusion.cuh"
#include "clq_internal.h"
#include "gemv_common.cuh"
#include "gemv_i8.cuh"
#include "pipeline.cuh"
#include "tma_host.h"

namespace clq {
namespace {

using namespace pipe;

constexpr int kWW = 16;  // warps per CTA
constexpr int kWThreads = kWW * 32;
constexpr int kWMaxDepth = 4;
// header: slot barriers, this call's epoch, the fused RMSNorm's row scales
// and per-warp sums of squares
constexpr int kWEpochOff = kWW * kWMaxDepth * 8, kWNormOff = kWEpochOff + 16, kWRedOff = kWEpochOff + 32;
constexpr int kWHeader = kWRedOff + kWW * 2 * 4;
constexpr int kWMaxDevices = 64;
constexpr size_t kWSmemLimit = 227 * 1024;
// Units each warp copies before waiting for the previous kernel (at most the
// ring's depth); the rest of its ring is filled after its activation loads
// are issued, so that those loads do not queue behind a full ring's worth of
// weight traffic.  Three measured slower (1.60 against 1.51 ms on the
// Llama-3-8B decode step).
constexpr int kWPreWait = 2;

// Bytes of one row of one unit in the q plane (the whole unit's data for Q4_K;
// Q6_K's sub-scales and scale, 9% of its bytes, and the fp16 block scales of
// Q4_0 / Q8_0, 11% and 6%, are read with plain loads).  SWZ: the unit lands
// in shared memory under the 128-byte swizzle (16-byte chunk c of 128-byte
// line l at chunk c ^ (l & 7)), so that the lanes' 16-byte reads of rows
// 256 or 128 bytes apart spread over all banks.
template <int D> struct WGeo;
template <> struct WGeo<kQ4_K> { static constexpr int q = 144; static constexpr bool swz = false; };
template <> struct WGeo<kQ6_K> { static constexpr int q = 192; static constexpr bool swz = false; };
template <> struct WGeo<kQ4_0> { static constexpr int q = 128; static constexpr bool swz = true; };
template <> struct WGeo<kQ8_0> { static constexpr int q = 256; static constexpr bool swz = true; };

// Offset of 16-byte chunk C of 128-byte line L in a swizzled slot.
__device__ __forceinline__ int swz_off(int l, int c) { return l * 128 + ((c ^ (l & 7)) << 4); }

struct WarpParams {
    CUtensorMap maps[kGroup];  // q plane of each member: [rows][K / 256 * Q] bytes, box 16 x Q
    Member mem[kGroup];
    int nmem;
    int tiles;
    int nchunks;  // K / 256
    int m;        // activation rows, 1 .. 8
    int ksplit;   // K splits: CTAs per tile group, one cluster (1: each CTA takes all of K)
    int64_t k;
    const void* x;
    int x_aligned;
    int depth;    // ring slots per warp
    uint32_t cnt_off, x_off, piece_off, tsum_off, ring_off;
    int* err;
    int tp_on;
    TpLink tp;
    // fused prologue / epilogue (the FUSE variant): see Fusion in clq_internal.h
    const float* norm_w;
    float norm_eps;
    const void* gate;
    int gate_aligned, norm_aligned;
    const float* res;
    int64_t ldr;
};

// Every thread of the cluster's CTAs arrives (its earlier shared-memory
// stores released) and waits for all of them.
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The float at LOCAL's offset in the shared memory of the cluster's CTA RANK.
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(local);
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
    return v;
}

// The warp whose run holds unit u: runs are [w U / W, (w+1) U / W) for the
// W = min(16, U) warps in use, all non-empty.
__device__ __forceinline__ int warp_of(int u, int U, int W) { return (W * (u + 1) + U - 1) / U - 1; }

// The product's input element from activation X and gate G (fusion.cuh).
__device__ __forceinline__ float swiglu_in(float x, float g) { return swiglu(g, x); }

// The fused prologue as a staging transform: the gate and norm-weight words
// are loaded beside the activations (one round trip for all three), then
// h = silu(gate) * x (when gated) is staged as h * norm_w, its squares summed
// per row for the RMSNorm scale the finisher applies.
template <typename XT>
struct FusedInput {
    static constexpr int kBatch = 2;
    struct Aux {
        float g[8], w[8];
    };
    const XT* gate = nullptr;
    const float* norm_w = nullptr;
    int64_t k = 0;
    int gate_aligned = 0, norm_aligned = 0;
    float ss0 = 0.f, ss1 = 0.f;
    __device__ __forceinline__ void load(int u, int64_t col, Aux& a) const {
        if (gate) {
            const XT* gp = gate + (int64_t)u * k + col;
            if (gate_aligned) {
                xload8(gp, a.g);
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) a.g[i] = xload(gp + i);
            }
        }
        if (norm_w) {
            if (norm_aligned) {
                xload8(norm_w + col, a.w);
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) a.w[i] = norm_w[col + i];
            }
        }
    }
    __device__ __forceinline__ void apply(int u, int64_t, float (&v)[8], const Aux& a) {
        if (gate) {
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = swiglu_in(v[i], a.g[i]);
        }
        if (norm_w) {
            float sq = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                sq = fmaf(v[i], v[i], sq);
                v[i] *= a.w[i];
            }
            if (u == 0) ss0 += sq;
            else ss1 += sq;
        }
    }
};

template <int D, typename XT, bool FUSE, int NP, bool SPLIT>
__global__ void __launch_bounds__(kWThreads, 1) gemv_warp_kernel(const __grid_constant__ WarpParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int Q = WGeo<D>::q;
    constexpr uint32_t kSlot = 16u * Q;
    constexpr int TB = I8Block<D>::bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    uint32_t* ep_sh = reinterpret_cast<uint32_t*>(smem + kWEpochOff);
    int* cnt = reinterpret_cast<int*>(smem + P.cnt_off);
    unsigned char* xstage = smem + P.x_off;
    float* piece = reinterpret_cast<float*>(smem + P.piece_off);  // [2 per warp][m][16]
    float* tsum = reinterpret_cast<float*>(smem + P.tsum_off);    // K split: [tiles][m][16]

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    // CTA b takes K split b % KS of tile group b / KS (KS = 1: all of K)
    const int KS = SPLIT ? P.ksplit : 1, groups = (int)gridDim.x / KS;
    const int grp = (int)blockIdx.x / KS, ks = (int)blockIdx.x - grp * KS;
    const int kc0 = (int)((int64_t)ks * P.nchunks / KS);
    const int nch = (int)((int64_t)(ks + 1) * P.nchunks / KS) - kc0, ntok = P.m, depth = P.depth;
    const int t_begin = (int)((int64_t)grp * P.tiles / groups);
    const int t_end = (int)(((int64_t)grp + 1) * P.tiles / groups);
    const int U = (t_end - t_begin) * nch;
    const int W = U < kWW ? U : kWW;
    const int u0 = warp < W ? warp * U / W : 0, u1 = warp < W ? (warp + 1) * U / W : 0;
    uint64_t* bar = bars + warp * kWMaxDepth;
    unsigned char* rings = smem + P.ring_off;
    // the swizzle pattern repeats every 1024 bytes of shared memory: swizzled
    // slots start on that boundary (the plan leaves room to round up)
    if constexpr (WGeo<D>::swz) rings += (1024u - (smem_u32(rings) & 1023u)) & 1023u;
    unsigned char* ring = rings + (size_t)warp * depth * kSlot;
    int* err = P.err;

    if (lane == 0) {
        for (int s = 0; s < depth; s++) mbar_init(&bar[s], 1);
        mbar_init_fence();
    }
    __syncwarp();
    allow_dependents();

    // ---- this warp's copies: unit (itile, ic) into slot islot ----
    const uint64_t policy = evict_first_policy();
    int issued = u0, itile = t_begin + (u0 / (nch > 0 ? nch : 1)), ic = u0 - (itile - t_begin) * nch, islot = 0;
    auto issue = [&]() {
        if (lane == 0) {
            const int mi = member_of(P, (int64_t)itile);
            mbar_arrive_tx(&bar[islot], kSlot);
            const int row0 = (itile - (int)P.mem[mi].tile_begin) * 16;
            if constexpr (D == kQ8_0) {
                // the 3-D map's box: two 128-byte halves of the chunk x 16 rows
                tensor_copy_3d_hint(ring + islot * kSlot, &P.maps[mi], 0, 2 * (kc0 + ic), row0, &bar[islot],
                                    policy);
            } else {
                tensor_copy_2d_hint(ring + islot * kSlot, &P.maps[mi], (kc0 + ic) * Q, row0, &bar[islot], policy);
            }
        }
        ++issued;
        if (++islot == depth) islot = 0;
        if (++ic == nch) {
            ic = 0;
            ++itile;
        }
    };
    // never more copies in flight than the ring has slots: each slot's barrier
    // counts one copy per phase
    const int prewait = kWPreWait < depth ? kWPreWait : depth;
    while (issued < u1 && issued < u0 + prewait) issue();

    grid_dependency_wait();  // the activations may come from the previous kernel
    // read through L2: an SM's L1 may hold a line of epochs from an earlier call
    if (threadIdx.x == 0 && P.tp_on) ep_sh[0] = __ldcg(&P.tp.epochs[blockIdx.x]) + 1u;
    for (int i = threadIdx.x; i < t_end - t_begin; i += kWThreads) cnt[i] = 0;
    auto top_up = [&]() {
        while (issued < u1 && issued < u0 + depth) issue();
    };
    float* red = reinterpret_cast<float*>(smem + kWRedOff);
    if constexpr (FUSE) {
        // h = silu(gate) * x (when gated), staged as h * norm_w; the RMSNorm
        // scale 1 / sqrt(mean(h^2) + eps) is a per-row factor of the product,
        // applied by the tile finisher.  Its sum of squares comes from the
        // staging pass itself (every CTA stages the whole row, in the same
        // partition: the same fixed order in every CTA, no second read of x)
        FusedInput<XT> fi;
        fi.gate = reinterpret_cast<const XT*>(P.gate);
        fi.norm_w = P.norm_w;
        fi.k = P.k;
        fi.gate_aligned = P.gate_aligned;
        fi.norm_aligned = P.norm_aligned;
        stage_x_i8_with<D, XT, kWW>(P.x, P.k, P.x_aligned, kc0, nch, ntok, xstage, top_up, fi);
        if (P.norm_w) {
            float ss0 = fi.ss0, ss1 = fi.ss1;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                ss0 += __shfl_xor_sync(0xffffffffu, ss0, off);
                ss1 += __shfl_xor_sync(0xffffffffu, ss1, off);
            }
            if (lane == 0) {
                red[warp * 2] = ss0;
                red[warp * 2 + 1] = ss1;
            }
        }
    } else {
        stage_x_i8<D, XT, kWW>(P.x, P.k, P.x_aligned, kc0, nch, ntok, xstage, top_up);
    }
    __syncthreads();
    float* rn = reinterpret_cast<float*>(smem + kWNormOff);  // the fused RMSNorm's scale of rows 0 and 1
    if constexpr (FUSE) {
        if (P.norm_w) {
            if (threadIdx.x < 2) {
                float tot = 0.f;
#pragma unroll
                for (int w = 0; w < kWW; w++) tot += red[w * 2 + threadIdx.x];
                rn[threadIdx.x] = 1.f / sqrtf(tot / (float)P.k + P.norm_eps);
            }
            __syncthreads();
        }
    }

    constexpr int NQ = (NP + 1) / 2;
    const I8LaneN<D, NP> L8 = i8_lane_n<D, NP>(ntok);
    float accm[NP][2], accn[NQ][2];
#pragma unroll
    for (int p = 0; p < NP; p++) accm[p][0] = accm[p][1] = 0.f;
#pragma unroll
    for (int q = 0; q < NQ; q++) accn[q][0] = accn[q][1] = 0.f;
    bool ok = true;
    int done = u0;

    // Q6_K sub-scales and scale of rows g, g + 8 for a unit, one unit ahead
    // (Q4_0 / Q8_0: the rows' eight block scales, 16 bytes each, in s_*)
    uint4 s_cur[2] = {}, s_nxt[2] = {};
    uint32_t d_cur[2] = {0u, 0u}, d_nxt[2] = {0u, 0u};
    auto side = [&](int tile, int c) {
        const Member& M = P.mem[member_of(P, (int64_t)tile)];
        int64_t r0 = (int64_t)(tile - (int)M.tile_begin) * 16 + g, r1 = r0 + 8;
        if (r0 >= M.rows) r0 = M.rows - 1;
        if (r1 >= M.rows) r1 = M.rows - 1;
        const int64_t cg = kc0 + c, nc = P.nchunks;
        if constexpr (D == kQ6_K) {
            s_nxt[0] = __ldg(reinterpret_cast<const uint4*>(M.p.s + (r0 * nc + cg) * 16));
            s_nxt[1] = __ldg(reinterpret_cast<const uint4*>(M.p.s + (r1 * nc + cg) * 16));
            d_nxt[0] = __ldg(reinterpret_cast<const unsigned short*>(M.p.d + (r0 * nc + cg) * 2));
            d_nxt[1] = __ldg(reinterpret_cast<const unsigned short*>(M.p.d + (r1 * nc + cg) * 2));
        } else {
            // block b of row r at (r * 8 nc + b) * 2 bytes: the chunk's eight are 16 aligned bytes
            s_nxt[0] = __ldg(reinterpret_cast<const uint4*>(M.p.d + (r0 * nc + cg) * 16));
            s_nxt[1] = __ldg(reinterpret_cast<const uint4*>(M.p.d + (r1 * nc + cg) * 16));
        }
    };

    int tl = u0 / (nch > 0 ? nch : 1), c = u0 - tl * nch, slot = 0;
    const int tl_first = tl;  // the first tile of this warp's run
    uint32_t phase = 0;
    if constexpr (D != kQ4_K) {
        if (u0 < u1) side(t_begin + tl, c);
    }
    for (int u = u0; u < u1; u++) {
        if constexpr (D != kQ4_K) {
            s_cur[0] = s_nxt[0]; s_cur[1] = s_nxt[1];
            d_cur[0] = d_nxt[0]; d_cur[1] = d_nxt[1];
            if (u + 1 < u1) {
                const bool wrap = c + 1 == nch;
                side(t_begin + tl + (wrap ? 1 : 0), wrap ? 0 : c + 1);
            }
        }
        if (!mbar_wait(&bar[slot], phase, err)) {
            ok = false;
            break;
        }
        const unsigned char* st = ring + slot * kSlot;
        const unsigned char* xs = xstage + (size_t)c * ntok * TB;
        if constexpr (D == kQ4_K) {
            uint32_t HD[2][4];
            uint2 CW[2][4];
            // MMA rows g and g + 8 are the tile's rows 2g and 2g + 1: lanes g
            // then read 288 bytes apart, and one 16-lane phase (g = 0..3) of
            // the 8-byte reads covers all 32 banks once
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const unsigned char* q = st + (2 * g + h) * Q;
                const uint4 hd = *reinterpret_cast<const uint4*>(q);
                HD[h][0] = hd.x; HD[h][1] = hd.y; HD[h][2] = hd.z; HD[h][3] = hd.w;
#pragma unroll
                for (int j = 0; j < 4; j++) CW[h][j] = *reinterpret_cast<const uint2*>(q + 16 + 32 * j + 8 * t);
            }
            __syncwarp();
            if (issued < u1) issue();  // the slot's words are in registers: refill it
            q4k_i8_chunk_n<NP>(L8, HD, CW, xs, accm, accn);
        } else if constexpr (D == kQ8_0) {
            // row g + 8h, this lane's 64 bytes: half t / 2 of the chunk,
            // chunks 4 (t & 1) .. + 3 of its 128-byte line 2 (g + 8h) + t / 2
            uint4 QV[2][4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int l = 2 * (g + 8 * h) + (t >> 1);
#pragma unroll
                for (int i = 0; i < 4; i++) QV[h][i] = *reinterpret_cast<const uint4*>(st + swz_off(l, 4 * (t & 1) + i));
            }
            __syncwarp();
            if (issued < u1) issue();
            q8_0_i8_chunk_n<NP>(L8, QV, s_cur, xs, accm);
        } else if constexpr (D == kQ4_0) {
            // row g + 8h, this lane's 32 bytes: chunks 2t, 2t + 1 of line g + 8h
            uint32_t QW[2][8];
#pragma unroll
            for (int h = 0; h < 2; h++) {
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const uint4 v = *reinterpret_cast<const uint4*>(st + swz_off(g + 8 * h, 2 * t + i));
                    QW[h][4 * i] = v.x; QW[h][4 * i + 1] = v.y; QW[h][4 * i + 2] = v.z; QW[h][4 * i + 3] = v.w;
                }
            }
            __syncwarp();
            if (issued < u1) issue();
            q4_0_i8_chunk_n<NP>(L8, QW, s_cur, xs, accm, accn);
        } else {
            uint32_t QW[2][12];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const unsigned char* q = st + (g + 8 * h) * Q + 48 * t;
#pragma unroll
                for (int i = 0; i < 3; i++) {
                    const uint4 v = *reinterpret_cast<const uint4*>(q + 16 * i);
                    QW[h][4 * i] = v.x; QW[h][4 * i + 1] = v.y; QW[h][4 * i + 2] = v.z; QW[h][4 * i + 3] = v.w;
                }
            }
            __syncwarp();
            if (issued < u1) issue();
            q6k_i8_chunk_n<NP>(L8, QW, s_cur, d_cur, xs, accm, accn);
        }
        done = u + 1;
        if (++slot == depth) {
            slot = 0;
            phase ^= 1u;
        }
        const bool tile_end = ++c == nch;
        if (tile_end || u + 1 == u1) {
            const int wf = warp_of(tl * nch, U, W), wl = warp_of(tl * nch + nch - 1, U, W);
            // this warp's piece of the tile goes to its slot for the run's
            // first tile or the one for any later tile (a later tile not
            // shared with other warps is finished by this warp at once)
            const int slot = 2 * warp + (tl == tl_first ? 0 : 1);
#pragma unroll
            for (int p = 0; p < NP; p++) {
                float v[2];
#pragma unroll
                for (int h = 0; h < 2; h++) v[h] = i8_finish_n(L8, p, accm[p][h], accn[p >> 1][h]);
                const int tok = 2 * p + (t >> 1);
                if ((t & 1) == 0 && tok < ntok) {
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        piece[(slot * ntok + tok) * 16 + (D == kQ4_K ? 2 * g + h : g + 8 * h)] = v[h];
                    }
                }
            }
#pragma unroll
            for (int p = 0; p < NP; p++) accm[p][0] = accm[p][1] = 0.f;
#pragma unroll
            for (int q = 0; q < NQ; q++) accn[q][0] = accn[q][1] = 0.f;
            __syncwarp();
            int old = 0;
            if (lane == 0) {
                __threadfence_block();
                old = atomicAdd(&cnt[tl], 1);
            }
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == wl - wf) {  // the tile's last piece: add them in warp order
                __threadfence_block();
                const int tile = t_begin + tl;
                const Member& M = P.mem[member_of(P, (int64_t)tile)];
                // one output of the tile: into the cluster's sums (K split), to
                // every rank (tensor parallel) or, after the fused epilogue, out
                auto emit = [&](int idx, float sum) {
                    if constexpr (SPLIT) {
                        tsum[tl * ntok * 16 + idx] = sum;
                        return;
                    }
                    const int64_t row = (int64_t)(tile - (int)M.tile_begin) * 16 + (idx & 15);
                    if (row >= M.rows) return;
                    if (P.tp_on) {
                        tp_put(P.tp, ep_sh[0], (int)blockIdx.x, tl, ntok, idx, sum);
                        return;
                    }
                    float o = sum;
                    if constexpr (FUSE) {
                        if (P.norm_w) o *= rn[idx >> 4];
                        if (P.res) o += P.res[(int64_t)(idx >> 4) * P.ldr + row];  // single weight only
                    }
                    M.out[(int64_t)(idx >> 4) * M.ldo + row] = o;
                };
                // the tile is the first of every later warp's run, and of
                // warp wf's when that run starts with the tile
                const int s_first = 2 * wf + (wf * U / W == tl * nch ? 0 : 1);
                for (int idx = lane; idx < ntok * 16; idx += 32) {
                    float sum = 0.f;
                    sum += piece[s_first * ntok * 16 + idx];
                    for (int w = wf + 1; w <= wl; w++) sum += piece[2 * w * ntok * 16 + idx];
                    emit(idx, sum);
                }
            }
            if (tile_end) {
                c = 0;
                ++tl;
            }
        }
    }

    // copies issued but not consumed (only after an expired wait) land before the CTA exits
    if (!ok && lane == 0) {
        for (int v = done; v < issued; v++) {
            const int k = v - u0;
            mbar_drain(&bar[k % depth], (uint32_t)(k / depth) & 1u);
        }
    }
    if constexpr (SPLIT) {
        // the cluster's KS CTAs hold the same tiles' sums over their K
        // splits: each adds a share of the outputs over the splits, in split
        // order, reading the others' shared memory; the second barrier keeps
        // every CTA's sums alive until all reads are done
        __syncwarp();
        cluster_barrier();
        const float* ts = reinterpret_cast<const float*>(smem + P.tsum_off);
        const int per_tile = ntok * 16, total = (t_end - t_begin) * per_tile;
        const int e0 = (int)((int64_t)ks * total / KS), e1 = (int)((int64_t)(ks + 1) * total / KS);
        for (int e = e0 + (int)threadIdx.x; e < e1; e += kWThreads) {
            float sum = 0.f;
            for (int k2 = 0; k2 < KS; k2++) sum += ld_cluster_f32(ts + e, (uint32_t)k2);
            const int tile = t_begin + e / per_tile, idx = e - (e / per_tile) * per_tile;
            const Member& M = P.mem[member_of(P, (int64_t)tile)];
            const int64_t row = (int64_t)(tile - (int)M.tile_begin) * 16 + (idx & 15);
            if (row < M.rows) M.out[(int64_t)(idx >> 4) * M.ldo + row] = sum;
        }
        __syncwarp();
        cluster_barrier();
    }
    if (P.tp_on) {
        // every rank partitions the tiles the same way, so this CTA's
        // counterparts produce the same outputs: wait for their words, sum
        __syncthreads();
        const uint32_t ep = ep_sh[0];
        tp_gather_sum(P.tp, P.mem[0], t_begin, t_end, ntok, ep, err);
        __syncthreads();  // every thread has its words before the epoch moves on
        if (threadIdx.x == 0) P.tp.epochs[blockIdx.x] = ep;
    }
}

// Encoded maps, per thread, by (base, rows, row bytes, box, dtype): a map is a
// pure function of these, so an entry never goes stale.  Decode calls one
// weight at a time, so the per-call encode is the common case to avoid.
struct MapKey {
    const void* base;
    int64_t rows, row_bytes;
    int box, dtype;
    bool operator==(const MapKey& o) const {
        return base == o.base && rows == o.rows && row_bytes == o.row_bytes && box == o.box && dtype == o.dtype;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        return std::hash<const void*>()(k.base) ^ (std::hash<int64_t>()(k.rows) * 31) ^
               (std::hash<int64_t>()(k.row_bytes) * 131) ^ (size_t)k.box ^ ((size_t)k.dtype << 20);
    }
};
bool encode_unit_map(CUtensorMap* map, int dtype, const void* base, int64_t rows, int64_t row_bytes, int box);
bool cached_encode_rows(CUtensorMap* map, int dtype, const void* base, int64_t rows, int64_t row_bytes, int box) {
    thread_local std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    const MapKey key{base, rows, row_bytes, box, dtype};
    auto it = cache.find(key);
    if (it != cache.end()) {
        *map = it->second;
        return true;
    }
    if (!encode_unit_map(map, dtype, base, rows, row_bytes, box)) return false;
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, *map);
    return true;
}

// Tuning knob CLQ_GEMV_WARP: 0 sends decode to the shared-ring bulk kernel
// (Q4_K / Q6_K) and the register-fed one; k keeps the per-warp kernel for the
// K formats only (Q4_0 / Q8_0 on the register-fed kernel).  1: all four.
int warp_mode() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("CLQ_GEMV_WARP");
        const char* i = getenv("CLQ_GEMV_I8");
        on = ((e && e[0] == '0') || (i && i[0] == '0')) ? 0 : (e && e[0] == 'k') ? 2 : 1;
    }
    return on;
}
bool warp_enabled() { return warp_mode() != 0; }

size_t al128(size_t v) { return (v + 127) & ~(size_t)127; }

// CTAs for TILES tiles: one per SM, or -- with CLQ_GEMV_WARP_GRID=balanced, a
// tuning knob -- the count in [3/4 of the SMs, all of them] that leaves the
// fewest idle tile slots (the busiest CTA sets the kernel's time).
int64_t warp_grid(int64_t tiles) {
    static int mode = -1;
    if (mode < 0) {
        const char* e = getenv("CLQ_GEMV_WARP_GRID");
        mode = (e && e[0] == 'b') ? 1 : 0;
    }
    const int64_t sms = sm_count();
    if (tiles <= sms) return tiles;
    if (!mode) return sms;
    int64_t best = sms, best_pad = (tiles + sms - 1) / sms * sms - tiles;
    for (int64_t g = sms - 1; g >= sms * 3 / 4; g--) {
        const int64_t pad = (tiles + g - 1) / g * g - tiles;
        if (pad < best_pad) {
            best = g;
            best_pad = pad;
        }
    }
    return best;
}

// Shared memory: header, tile counters, the staged activations of the CTA's
// K split (all of K at KS = 1), the pieces, the tile sums a cluster reduces
// (KS > 1), then 16 rings of DEPTH slots (4, else 3; 2 when K is split).
// False when the fewest slots do not fit.
template <int D>
bool wplan(WarpParams& P, int64_t groups, int ks, size_t* smem) {
    const int64_t tiles_cta = (P.tiles + groups - 1) / groups;
    const int64_t pc = (P.nchunks + ks - 1) / ks;
    P.cnt_off = kWHeader;
    P.x_off = (uint32_t)al128(P.cnt_off + (size_t)tiles_cta * 4);
    P.piece_off = (uint32_t)al128(P.x_off + (size_t)pc * P.m * I8Block<D>::bytes);
    P.tsum_off = (uint32_t)al128(P.piece_off + (size_t)2 * kWW * P.m * 16 * 4);
    P.ring_off = (uint32_t)al128(P.tsum_off + (ks > 1 ? (size_t)tiles_cta * P.m * 16 * 4 : 0));
    for (int depth = kWMaxDepth; depth >= (ks > 1 ? 2 : 3); depth--) {
        const size_t total = P.ring_off + (WGeo<D>::swz ? 1024 : 0) + (size_t)kWW * depth * 16 * WGeo<D>::q;
        if (total <= kWSmemLimit) {
            P.depth = depth;
            *smem = total;
            return true;
        }
    }
    return false;
}

constexpr int kWMaxSplit = 8;

// When to split K across a cluster (CLQ_GEMV_SPLIT, a tuning knob): 0 only
// when the activations of all of K do not fit one CTA (the default), 1 also
// when the estimate says it evens out the CTAs' work, 2 always when a split
// fits.  Measured on the Llama-3-8B decode step, 1 costs more than it saves
// (1.60 against 1.51 ms; 70B: 10.76 against 10.35 ms): the cluster barriers
// and cross-CTA sums outweigh the better balance.
int split_mode() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("CLQ_GEMV_SPLIT");
        v = e ? atoi(e) : 0;
        if (v < 0 || v > 2) v = 0;
    }
    return v;
}
// The fixed cost of a split (two cluster barriers, the cross-CTA sums), in
// units of one 16-row x 256-column weight block (CLQ_GEMV_SPLIT_COST).
double split_cost() {
    static double v = -1.0;
    if (v < 0) {
        const char* e = getenv("CLQ_GEMV_SPLIT_COST");
        v = e ? atof(e) : 4.0;
        if (v < 0) v = 0;
    }
    return v;
}

// Raises the kernel's dynamic shared-memory limit on the current device to
// SMEM once (per instance and device).
template <typename Kern>
cudaError_t ensure_smem(Kern kern, std::atomic<int> (&set_for)[kWMaxDevices], size_t smem) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kWMaxDevices) return cudaErrorInvalidDevice;
    if ((int)smem > set_for[dev].load(std::memory_order_relaxed)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        int seen = set_for[dev].load(std::memory_order_relaxed);
        while ((int)smem > seen && !set_for[dev].compare_exchange_weak(seen, (int)smem)) {
        }
    }
    return cudaSuccess;
}

// Clusters of KS CTAs of SMEM bytes each that the current device holds at
// once (a cluster's CTAs wait for one another, so the launch must be one
// wave), cached per (device, KS, SMEM); 0 when the query fails.
template <typename Kern>
int64_t max_clusters(Kern kern, std::atomic<int> (&set_for)[kWMaxDevices], int ks, size_t smem) {
    static std::mutex mu;
    static std::unordered_map<uint64_t, int> seen;
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t key = ((uint64_t)dev << 40) | ((uint64_t)ks << 32) | (uint64_t)smem;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = seen.find(key);
        if (it != seen.end()) return it->second;
    }
    if (ensure_smem(kern, set_for, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(sm_count() / ks * ks));
    cfg.blockDim = dim3(kWThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ks;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    seen[key] = n;
    return n;
}

template <int D, typename XT, bool FUSE, int NP>
cudaError_t launch_warp(WarpParams P, cudaStream_t stream) {
    auto kern = gemv_warp_kernel<D, XT, FUSE, NP, false>;
    auto kern_split = gemv_warp_kernel<D, XT, false, NP, true>;
    static std::atomic<int> set_for[kWMaxDevices], set_for_split[kWMaxDevices];
    int64_t groups = warp_grid(P.tiles);
    if (P.tp_on && (groups > kMaxTpCtas || (P.tiles + groups - 1) / groups * 16 * P.m > P.tp.cap))
        return cudaErrorNotSupported;
    size_t smem = 0;
    int ks = 1;
    const bool whole = wplan<D>(P, groups, 1, &smem);
    // Not under tensor parallelism or a fused prologue, which need whole rows
    // in one CTA: K may be split between the CTAs of a cluster.  That is
    // needed when the activations of all of K do not fit beside the rings,
    // and it pays when whole tiles leave the CTAs unevenly loaded -- a CTA's
    // time is its units (tiles x chunks of its split), and fewer, larger tile
    // groups split K evenly (256 tiles over 148 CTAs: 2 against 1.73 on
    // average; over 37 clusters of 4: 7 against 6.9).
    if (!whole && (P.tp_on || FUSE)) return cudaErrorNotSupported;
    if (!P.tp_on && !FUSE) {
        const int mode = split_mode();
        auto units = [&](int64_t g, int k2) {
            return (double)((P.tiles + g - 1) / g) * (double)((P.nchunks + k2 - 1) / k2) + (k2 > 1 ? split_cost() : 0.0);
        };
        double best = whole && mode != 2 ? units(groups, 1) : 1e300;
        int best_ks = whole && mode != 2 ? 1 : 0;
        int64_t best_groups = groups;
        if (!whole || mode != 0) {
            const int64_t sms = sm_count();
            for (int k2 = 2; k2 <= kWMaxSplit && k2 <= P.nchunks; k2 *= 2) {
                int64_t g2 = sms / k2 < P.tiles ? sms / k2 : P.tiles;
                WarpParams Q = P;
                size_t s2 = 0;
                if (!wplan<D>(Q, g2, k2, &s2)) continue;
                const int64_t clusters = max_clusters(kern_split, set_for_split, k2, s2);
                if (clusters < 1) continue;
                if (clusters < g2) {  // fewer clusters fit than SMs / KS: more tiles each
                    g2 = clusters;
                    if (!wplan<D>(Q, g2, k2, &s2)) continue;
                }
                const double c = units(g2, k2);
                if (!best_ks || (!whole && best_ks == 1) || c < best) {
                    best = c;
                    best_ks = k2;
                    best_groups = g2;
                }
                if (!whole && mode == 0) break;  // the first split that fits, as needed
            }
        }
        if (!best_ks) return cudaErrorNotSupported;
        ks = best_ks;
        groups = best_groups;
        if (!wplan<D>(P, groups, ks, &smem)) return cudaErrorNotSupported;
    }
    P.ksplit = ks;
    cudaError_t e = ks > 1 ? ensure_smem(kern_split, set_for_split, smem) : ensure_smem(kern, set_for, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(groups * ks));
    cfg.blockDim = dim3(kWThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (gemv_pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na++].val.programmaticStreamSerializationAllowed = 1;
    }
    if (ks > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)ks;
        attr[na].val.clusterDim.y = 1;
        attr[na++].val.clusterDim.z = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return ks > 1 ? cudaLaunchKernelEx(&cfg, kern_split, P) : cudaLaunchKernelEx(&cfg, kern, P);
}

// One instance per pair count of activation rows; the fused prologue at one
// pair only, for Q4_K and Q6_K (fused Q4_0 / Q8_0 calls take the unfused
// product behind the fusion kernels).
template <int D, typename XT>
cudaError_t launch_warp_rows(const WarpParams& P, bool fuse, cudaStream_t s) {
    if constexpr (D == kQ4_K || D == kQ6_K) {
        if (fuse) return launch_warp<D, XT, true, 1>(P, s);
    } else {
        if (fuse) return cudaErrorNotSupported;
    }
    switch ((P.m + 1) / 2) {
    case 1: return launch_warp<D, XT, false, 1>(P, s);
    case 2: return launch_warp<D, XT, false, 2>(P, s);
    case 3: return launch_warp<D, XT, false, 3>(P, s);
    case 4: return launch_warp<D, XT, false, 4>(P, s);
    default: return cudaErrorNotSupported;
    }
}

template <typename XT>
cudaError_t launch_warp_dtype(const WarpParams& P, int dtype, bool fuse, cudaStream_t s) {
    switch (dtype) {
    case kQ4_K: return launch_warp_rows<kQ4_K, XT>(P, fuse, s);
    case kQ6_K: return launch_warp_rows<kQ6_K, XT>(P, fuse, s);
    case kQ4_0: return launch_warp_rows<kQ4_0, XT>(P, fuse, s);
    case kQ8_0: return launch_warp_rows<kQ8_0, XT>(P, fuse, s);
    default: return cudaErrorNotSupported;
    }
}

}  // namespace

static PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool encode_rows(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int box, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_tiled();
    if (!fn || (uintptr_t)base % 16 || row_bytes % 16 || box % 16 || box > 256 || box_rows < 1 || box_rows > 256)
        return false;
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t boxd[2] = {(cuuint32_t)box, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, boxd, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {
// The per-warp kernel's map over a weight's q plane (ROWS rows of ROW_BYTES),
// one box per unit of 16 rows x BOX bytes: Q4_K / Q6_K plain; Q4_0 (128-byte
// units) under the 128-byte swizzle; Q8_0 (256-byte units) as a 3-D map of
// 128-byte halves, {128, 2, 16} per box, so that a unit row's two halves are
// consecutive swizzled lines.
bool encode_unit_map(CUtensorMap* map, int dtype, const void* base, int64_t rows, int64_t row_bytes, int box) {
    if (dtype == kQ4_K || dtype == kQ6_K) return encode_rows(map, base, rows, row_bytes, box, 16);
    PFN_cuTensorMapEncodeTiled_v12000 fn = encode_tiled();
    if (!fn || (uintptr_t)base % 16 || row_bytes % 256) return false;
    const cuuint64_t dims2[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    const cuuint64_t strides2[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box2[2] = {128u, 16u};
    const cuuint64_t dims3[3] = {128u, (cuuint64_t)(row_bytes / 128), (cuuint64_t)rows};
    const cuuint64_t strides3[2] = {128u, (cuuint64_t)row_bytes};
    const cuuint32_t box3[3] = {128u, 2u, 16u};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    if (dtype == kQ4_0 && box == 128)
        return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims2, strides2, box2, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    if (dtype == kQ8_0 && box == 256)
        return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims3, strides3, box3, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    return false;
}
}  // namespace

cudaError_t launch_gemv_warp(const WeightView* const* w, const int64_t* rows, int count, const void* x, int xtype,
                             int64_t m, float* const* out, const int64_t* ldo, const TpLink* tp,
                             cudaStream_t stream, const Fusion* fuse) {
    if (!warp_enabled() || m < 1 || m > 8 || count < 1 || count > kGroup) return cudaErrorNotSupported;
    const bool fused = fuse && fuse->any();
    if (fused && (m > 2 || tp || (fuse->res && count != 1))) return cudaErrorNotSupported;
    const int dtype = w[0]->dtype;
    const bool kfmt = dtype == kQ4_K || dtype == kQ6_K;
    // Q4_0 / Q8_0: plain products, at eight rows or rows of at least 4096
    // (tensor-parallel ones take the other kernels).  Measured per launch, the
    // register-fed kernel is faster on 512-8192 x 2048 weights at one to four
    // rows (Q4_0 2048 x 2048, one row: 2.8 against 4.0 us); from K = 4096, or
    // at eight rows, this kernel is (Q4_0 2048 x 8192, one row: 6.5 against
    // 8.8 us; Q8_0 4096 x 14336, eight rows: 25.6 against 65.3 us).
    const bool small_k = !kfmt && m < 8 && w[0]->k < 4096;
    if (!(kfmt || ((dtype == kQ4_0 || dtype == kQ8_0) && !tp && !fused && warp_mode() == 1 && !small_k)) ||
        w[0]->k < 256)
        return cudaErrorNotSupported;
    int* err = device_status_word();
    if (!err) return cudaErrorNotSupported;
    WarpParams P = {};
    P.nmem = count;
    int64_t tiles = 0;
    for (int i = 0; i < count; i++) {
        if (w[i]->dtype != dtype || w[i]->k != w[0]->k || w[i]->k % 256 || rows[i] < 1) return cudaErrorNotSupported;
        P.mem[i].p = Planes{w[i]->q, w[i]->s, w[i]->d, w[i]->nb};
        P.mem[i].rows = rows[i];
        P.mem[i].out = out[i];
        P.mem[i].ldo = ldo[i];
        P.mem[i].tile_begin = tiles;
        tiles += (rows[i] + 15) / 16;
    }
    // unit counts per CTA stay far below 2^31 / 16
    if (tiles > (1 << 24) || w[0]->k / 256 > (1 << 16)) return cudaErrorNotSupported;
    P.tiles = (int)tiles;
    P.k = w[0]->k;
    P.nchunks = (int)(w[0]->k / 256);
    P.m = (int)m;
    P.x = x;
    P.err = err;
    const int qb = dtype == kQ4_K ? WGeo<kQ4_K>::q
                 : dtype == kQ6_K ? WGeo<kQ6_K>::q
                 : dtype == kQ4_0 ? WGeo<kQ4_0>::q
                                  : WGeo<kQ8_0>::q;
    for (int i = 0; i < count; i++)
        if (!cached_encode_rows(&P.maps[i], dtype, w[i]->q, rows[i], (int64_t)P.nchunks * qb, qb))
            return cudaErrorNotSupported;
    if (tp) {
        P.tp_on = 1;
        P.tp = *tp;
    }
    const int esize = xtype == CLQ_X_F32 ? 4 : 2;
    P.x_aligned = ((uintptr_t)x % 16 == 0) && ((P.k * esize) % 16 == 0);
    if (fused) {
        P.norm_w = fuse->norm_w;
        P.norm_eps = fuse->norm_eps;
        P.gate = fuse->gate;
        P.gate_aligned = ((uintptr_t)fuse->gate % 16 == 0) && ((P.k * esize) % 16 == 0);
        P.norm_aligned = (uintptr_t)fuse->norm_w % 16 == 0;
        P.res = fuse->res;
        P.ldr = fuse->ldr;
    }
    switch (xtype) {
    case CLQ_X_F32: return launch_warp_dtype<float>(P, dtype, fused, stream);
    case CLQ_X_BF16: return launch_warp_dtype<__nv_bfloat16>(P, dtype, fused, stream);
    case CLQ_X_F16: return launch_warp_dtype<__half>(P, dtype, fused, stream);
    default: return cudaErrorNotSupported;
    }
}

}  // namespace clq
