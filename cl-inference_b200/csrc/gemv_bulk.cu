// gemv_bulk.cu -- decode GEMV (up to 8 activation rows) with the weight stream
// fed by the bulk-copy engine.
//
// One persistent CTA per SM owns a contiguous range of 16-row tiles, walked as
// (tile, K-stage) units.  Per unit, warp 0 issues 16 row copies -- 16 rows x
// up to 16 chunks of the packed q plane, plus the d plane for Q4_0 / Q8_0 --
// with cp.async.bulk into a ring of shared-memory stages: it fills the ring
// before anything else and refills one stage after each unit it computes.
// Warps 0-15 each take one 256-column chunk of a stage,
// read their words from shared memory, release the stage, and run the product:
// for Q4_K and Q6_K at one or two activation rows the integer-MMA product of
// gemv_i8.cuh, otherwise the exact fp16 product of gemv_common.cuh.  Q6_K's
// sub-scales and scales (9% of its bytes) are not staged: each consumer loads
// its own with plain loads one unit ahead.  Per-warp sums meet in shared memory
// at the end of a tile.
//
// The copies do not depend on the previous kernel (the weights are constant),
// so under programmatic dependent launch the ring fills while the previous
// kernel drains; only the activation staging waits for it.  The
// activations are staged once per SM (all of K when it fits, else in passes).
//
// Shared-memory rows are padded so that the consumers' reads of rows g and
// g + 1 fall in different banks.  Every wait is bounded (see pipeline.cuh); on
// expiry the kernel stops issuing, the consumers skip their work but still meet
// at every barrier, and the CTA drains the copies in flight before it exits.
#include <atomic>
#include <cstdlib>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/clq.h"
#include "clq_internal.h"
#include "gemv_common.cuh"
#include "gemv_i8.cuh"
#include "pipeline.cuh"

namespace clq {
namespace {

using namespace pipe;

constexpr int kCW = 16;                // warps = chunks per stage; warp 0 also issues the copies
constexpr int kBulkThreads = kCW * 32;
constexpr int kMaxStages = 8;
constexpr int kHeader = 256;           // barriers, issued count, epoch
constexpr int kMaxDevices = 64;

// Bytes per row per chunk of the staged planes, and the row padding that keeps
// the consumers' reads of rows g and g + 1 in different banks (the int8 Q4_K
// path reads 8-byte pieces, the fp16 path 16-byte ones).  Q6_K's s and d
// planes are read from global memory by the consumers.
template <int D, bool I8> struct Geo;
template <bool I8> struct Geo<kQ4_K, I8> { static constexpr int q = 144, d = 0, qpad = I8 ? 32 : 16; };
template <bool I8> struct Geo<kQ6_K, I8> { static constexpr int q = 192, d = 0, qpad = 64; };
template <bool I8> struct Geo<kQ4_0, I8> { static constexpr int q = 128, d = 16, qpad = 16; };
template <bool I8> struct Geo<kQ8_0, I8> { static constexpr int q = 256, d = 16, qpad = 16; };

struct BulkParams {
    Member mem[kGroup];
    int nmem;
    int tiles;
    int nchunks;       // K / 256
    int m;
    int64_t k;
    const void* x;
    int x_aligned;
    int pc;            // chunks of x staged per pass
    int stages;
    uint32_t stage_bytes, qs, ds, d_off;          // one stage: row strides and d-region offset
    uint32_t x_off, part_off, acc_off, ring_off;  // shared-memory regions
    int* err;
    int tp_on;         // all-reduce the output over the ranks of tp (single weight only)
    TpLink tp;
};

template <int D>
__device__ __forceinline__ void stage_words(const unsigned char* st, const BulkParams& P, int r, int ci, int t,
                                            uint32_t (&w)[Words<D>::n]) {
    const unsigned char* q = st + r * P.qs + ci * Geo<D, false>::q;
    auto ld = [](const unsigned char* p) { return *reinterpret_cast<const uint4*>(p); };
    if constexpr (D == kQ4_K) {
        uint4 v0 = ld(q), v1 = ld(q + 16 + 32 * t), v2 = ld(q + 32 + 32 * t);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2);
    } else if constexpr (D == kQ6_K) {
        q += 48 * t;
        uint4 v0 = ld(q), v1 = ld(q + 16), v2 = ld(q + 32);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2);
    } else if constexpr (D == kQ4_0) {
        q += 32 * t;
        uint4 v0 = ld(q), v1 = ld(q + 16), v2 = ld(st + P.d_off + r * P.ds + ci * 16);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2);
    } else {
        q += 64 * t;
        uint4 v0 = ld(q), v1 = ld(q + 16), v2 = ld(q + 32), v3 = ld(q + 48),
              v4 = ld(st + P.d_off + r * P.ds + ci * 16);
        CLQ_PUT4(w, 0, v0); CLQ_PUT4(w, 4, v1); CLQ_PUT4(w, 8, v2); CLQ_PUT4(w, 12, v3); CLQ_PUT4(w, 16, v4);
    }
}

// Starts of the Q6_K s and d plane rows g and g + 8 of TILE (clamped to the
// member's last row).
__device__ __forceinline__ void tile_rows(const BulkParams& P, int tile, int g, const unsigned char*& s0,
                                          const unsigned char*& s1, const unsigned char*& d0,
                                          const unsigned char*& d1) {
    const Member& M = P.mem[member_of(P, (int64_t)tile)];
    int64_t r0 = (int64_t)(tile - (int)M.tile_begin) * 16 + g, r1 = r0 + 8;
    if (r0 >= M.rows) r0 = M.rows - 1;
    if (r1 >= M.rows) r1 = M.rows - 1;
    s0 = M.p.s + r0 * P.nchunks * 16;
    s1 = M.p.s + r1 * P.nchunks * 16;
    d0 = M.p.d + r0 * P.nchunks * 2;
    d1 = M.p.d + r1 * P.nchunks * 2;
}

// The copies of the CTA's units, issued in order by warp 0 (all lanes).
struct Producer {
    int u = 0, slot = 0, pass = 0, tile = 0, ks = 0;
    uint32_t phase = 0;
    bool ok = true;
};

template <int D, bool I8>
__device__ __forceinline__ void produce(const BulkParams& P, Producer& pr, int units, int t_begin, int t_end,
                                        uint64_t* full, uint64_t* empty, unsigned char* ring) {
    using G = Geo<D, I8>;
    if (!pr.ok || pr.u >= units) return;
    const int S = P.stages, lane = threadIdx.x & 31;
    if (pr.u >= S && !mbar_wait(&empty[pr.slot], pr.phase ^ 1u, P.err)) {
        pr.ok = false;
        return;
    }
    const int c0 = pr.pass * P.pc;
    const int pcn = min(P.pc, P.nchunks - c0);
    const int cs = c0 + pr.ks * kCW;
    const int kc = min(kCW, c0 + pcn - cs);
    const Member& M = P.mem[member_of(P, (int64_t)pr.tile)];
    int64_t row = (int64_t)(pr.tile - (int)M.tile_begin) * 16 + (lane & 15);
    if (row >= M.rows) row = M.rows - 1;  // ragged last tile: repeat a row, drop its output
    if (lane == 0) mbar_arrive_tx(&full[pr.slot], 16u * kc * (G::q + G::d));
    __syncwarp();
    unsigned char* st = ring + (size_t)pr.slot * P.stage_bytes;
    const int r = lane & 15;
    const int64_t cell = row * P.nchunks + cs;
    if (lane < 16) bulk_copy(st + r * P.qs, M.p.q + cell * G::q, kc * G::q, &full[pr.slot]);
    else if (G::d) bulk_copy(st + P.d_off + r * P.ds, M.p.d + cell * G::d, kc * G::d, &full[pr.slot]);
    // advance to the next unit
    ++pr.u;
    if (++pr.slot == S) {
        pr.slot = 0;
        pr.phase ^= 1u;
    }
    if (++pr.ks == (pcn + kCW - 1) / kCW) {
        pr.ks = 0;
        if (++pr.tile == t_end) {
            pr.tile = t_begin;
            ++pr.pass;
        }
    }
}

template <int D, typename XT, int MT, bool I8>
__global__ void __launch_bounds__(kBulkThreads, 1) gemv_bulk_kernel(const __grid_constant__ BulkParams P) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int NW = Words<D>::n;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    int* issued_sh = reinterpret_cast<int*>(empty + kMaxStages);
    uint32_t* tp_sh = reinterpret_cast<uint32_t*>(issued_sh + 1);  // this CTA's epoch for the call
    unsigned char* ring = smem + P.ring_off;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int S = P.stages;
    const int nchunks = P.nchunks;
    const int ntok = P.m;
    const int t_begin = (int)((int64_t)blockIdx.x * P.tiles / gridDim.x);
    const int t_end = (int)(((int64_t)blockIdx.x + 1) * P.tiles / gridDim.x);
    const int npass = (nchunks + P.pc - 1) / P.pc;
    int* err = P.err;
    int units = 0;
    for (int ps = 0; ps < npass; ps++) units += (t_end - t_begin) * ((min(P.pc, nchunks - ps * P.pc) + kCW - 1) / kCW);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        *issued_sh = 0;
        mbar_init_fence();
    }
    __syncthreads();
    allow_dependents();

    Producer pr;
    pr.tile = t_begin;
    if (warp == 0)
        for (int i = 0; i < S; i++) produce<D, I8>(P, pr, units, t_begin, t_end, full, empty, ring);

    {
        // ---- consumers ----
        const int g = lane >> 2, t = lane & 3;
        unsigned char* xstage = smem + P.x_off;
        uint4* xf = reinterpret_cast<uint4*>(xstage);
        uint2* sxf = reinterpret_cast<uint2*>(xf + (size_t)P.pc * 64 * ntok);
        float* us = reinterpret_cast<float*>(sxf + (D == kQ4_K ? (size_t)P.pc * 4 * ntok : 0));
        float* part = reinterpret_cast<float*>(smem + P.part_off);  // [2][kCW][ntok][16]
        float* accs = reinterpret_cast<float*>(smem + P.acc_off);   // [tiles of this CTA][ntok][16]
        int xtok[MT], utok[MT];
#pragma unroll
        for (int n = 0; n < MT; n++) {
            xtok[n] = min(4 * n + (g >> 1), ntok - 1);
            utok[n] = min(4 * n + t, ntok - 1);
        }
        const int part_sel = g & 1;
        I8Lane L8 = {};
        if constexpr (I8) L8 = i8_lane<D>(ntok);
        constexpr int TB = I8 ? I8Block<(D == kQ6_K ? kQ6_K : kQ4_K)>::bytes : 0;

        // Q6_K side data (sub-scales, scale) of this warp's chunk, loaded one unit
        // ahead; the rows of the next tile are looked up once per tile.
        uint4 s_cur[2] = {}, s_nxt[2] = {};
        uint32_t d_cur[2] = {0u, 0u}, d_nxt[2] = {0u, 0u};
        const unsigned char *rs0 = nullptr, *rs1 = nullptr, *rd0 = nullptr, *rd1 = nullptr;  // current tile
        const unsigned char *ns0 = nullptr, *ns1 = nullptr, *nd0 = nullptr, *nd1 = nullptr;  // next unit's tile
#define CLQ_SIDE_FETCH(S0, S1, D0, D1, C)                                                    \
    do {                                                                                     \
        s_nxt[0] = __ldg(reinterpret_cast<const uint4*>((S0) + (size_t)(C) * 16));           \
        s_nxt[1] = __ldg(reinterpret_cast<const uint4*>((S1) + (size_t)(C) * 16));           \
        d_nxt[0] = __ldg(reinterpret_cast<const unsigned short*>((D0) + (size_t)(C) * 2));   \
        d_nxt[1] = __ldg(reinterpret_cast<const unsigned short*>((D1) + (size_t)(C) * 2));   \
    } while (0)
        if constexpr (D == kQ6_K) {
            if (t_begin < t_end) {
                tile_rows(P, t_begin, g, rs0, rs1, rd0, rd1);
                if (warp < min(P.pc, nchunks)) CLQ_SIDE_FETCH(rs0, rs1, rd0, rd1, warp);
            }
        }

        int u = 0, slot = 0, par = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int pass = 0; pass < npass; pass++) {
            const int c0 = pass * P.pc;
            const int pcn = min(P.pc, nchunks - c0);
            const int nks = (pcn + kCW - 1) / kCW;
            if (pass == 0) {
                grid_dependency_wait();  // activations may come from the previous kernel
                // read through L2: an SM's L1 may hold a line of epochs from an earlier call
                if (P.tp_on && threadIdx.x == 0) tp_sh[0] = __ldcg(&P.tp.epochs[blockIdx.x]) + 1u;
            }
            if constexpr (I8) {
                // each warp restages only its own chunks (after its own units of
                // the previous pass) and reads only those: no CTA barrier
                stage_x_i8<D, XT, kCW>(P.x, P.k, P.x_aligned, c0, pcn, ntok, xstage);
                __syncwarp();
            } else {
                if (pass > 0) __syncthreads();  // everyone is done with the previous pass's x
                stage_x<D, XT, kCW>(P.x, P.k, P.x_aligned, P.pc, c0, pcn, 0, ntok, xf, us, sxf);
                __syncthreads();
            }
            for (int tile = t_begin; tile < t_end; tile++) {
                float acc[MT][2], accm[2] = {0.f, 0.f}, accn[2] = {0.f, 0.f};
#pragma unroll
                for (int n = 0; n < MT; n++) acc[n][0] = acc[n][1] = 0.f;
                for (int ks = 0; ks < nks; ks++, u++) {
                    const int cc = ks * kCW + warp;  // chunk within the pass
                    if constexpr (D == kQ6_K) {      // side data of this warp's next unit
                        s_cur[0] = s_nxt[0]; s_cur[1] = s_nxt[1];
                        d_cur[0] = d_nxt[0]; d_cur[1] = d_nxt[1];
                        int ks2 = ks + 1, tile2 = tile, c02 = c0, pcn2 = pcn;
                        ns0 = rs0; ns1 = rs1; nd0 = rd0; nd1 = rd1;
                        if (ks2 == nks) {
                            ks2 = 0;
                            if (++tile2 == t_end) {
                                tile2 = t_begin;
                                c02 = c0 + P.pc;
                                pcn2 = min(P.pc, nchunks - c02);
                            }
                            if (c02 < nchunks) tile_rows(P, tile2, g, ns0, ns1, nd0, nd1);
                        }
                        const int cc2 = ks2 * kCW + warp;
                        if (c02 < nchunks && cc2 < pcn2) CLQ_SIDE_FETCH(ns0, ns1, nd0, nd1, c02 + cc2);
                    }
                    if (ok && !mbar_wait(&full[slot], phase, err)) ok = false;
                    const bool have = ok && cc < pcn;
                    const unsigned char* st = ring + (size_t)slot * P.stage_bytes;
                    if constexpr (I8 && D == kQ4_K) {
                        uint32_t HD[2][4];
                        uint2 CW[2][4];
                        if (have) {
#pragma unroll
                            for (int h = 0; h < 2; h++) {
                                const unsigned char* q = st + (g + 8 * h) * P.qs + warp * 144;
                                const uint4 hd = *reinterpret_cast<const uint4*>(q);
                                HD[h][0] = hd.x; HD[h][1] = hd.y; HD[h][2] = hd.z; HD[h][3] = hd.w;
#pragma unroll
                                for (int j = 0; j < 4; j++) CW[h][j] = *reinterpret_cast<const uint2*>(q + 16 + 32 * j + 8 * t);
                            }
                        }
                        __syncwarp();
                        if (ok && lane == 0) mbar_arrive(&empty[slot]);
                        if (have) q4k_i8_chunk(L8, HD, CW, xstage + (size_t)cc * ntok * TB, accm, accn);
                    } else if constexpr (I8 && D == kQ6_K) {
                        uint32_t QW[2][12];
                        if (have) {
#pragma unroll
                            for (int h = 0; h < 2; h++) {
                                const unsigned char* q = st + (g + 8 * h) * P.qs + warp * 192 + 48 * t;
#pragma unroll
                                for (int i = 0; i < 3; i++) {
                                    const uint4 v = *reinterpret_cast<const uint4*>(q + 16 * i);
                                    QW[h][4 * i] = v.x; QW[h][4 * i + 1] = v.y; QW[h][4 * i + 2] = v.z; QW[h][4 * i + 3] = v.w;
                                }
                            }
                        }
                        __syncwarp();
                        if (ok && lane == 0) mbar_arrive(&empty[slot]);
                        if (have) q6k_i8_chunk(L8, QW, s_cur, d_cur, xstage + (size_t)cc * ntok * TB, accm, accn);
                    } else {
                        uint32_t w[2][NW], db[2] = {0u, 0u};
                        if (have) {
                            stage_words<D>(st, P, g, warp, t, w[0]);
                            stage_words<D>(st, P, g + 8, warp, t, w[1]);
                            if constexpr (D == kQ6_K) {
#pragma unroll
                                for (int h = 0; h < 2; h++) {
                                    w[h][12] = s_cur[h].x; w[h][13] = s_cur[h].y; w[h][14] = s_cur[h].z; w[h][15] = s_cur[h].w;
                                    db[h] = d_cur[h];
                                }
                            }
                        }
                        __syncwarp();
                        if (ok && lane == 0) mbar_arrive(&empty[slot]);
                        if (have) {
                            const uint2* xq[MT];
                            const uint32_t* sq[MT];
                            float ut[MT];
#pragma unroll
                            for (int n = 0; n < MT; n++) {
                                xq[n] = reinterpret_cast<const uint2*>(xf + (xtok[n] * P.pc + cc) * 64 + t) + part_sel;
                                sq[n] = reinterpret_cast<const uint32_t*>(sxf + (xtok[n] * P.pc + cc) * 4 + t) + part_sel;
                                ut[n] = us[utok[n] * P.pc + cc];
                            }
                            compute_chunk<D, MT>(w, db, t, xq, sq, ut, acc);
                        }
                    }
                    if constexpr (D == kQ6_K) {
                        rs0 = ns0; rs1 = ns1; rd0 = nd0; rd1 = nd1;
                    }
                    if (warp == 0) produce<D, I8>(P, pr, units, t_begin, t_end, full, empty, ring);
                    if (++slot == S) {
                        slot = 0;
                        phase ^= 1u;
                    }
                }
                // ---- end of tile: per-warp sums -> shared -> one sum per (token, row) ----
                if constexpr (I8) {
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const float v = i8_finish(L8, accm[h], accn[h]);
                        const int tok = t >> 1;
                        if ((t & 1) == 0 && tok < ntok) part[((par * kCW + warp) * ntok + tok) * 16 + g + 8 * h] = v;
                    }
                } else {
#pragma unroll
                    for (int n = 0; n < MT; n++)
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int tok = 4 * n + t;
                            if (tok < ntok) part[((par * kCW + warp) * ntok + tok) * 16 + g + 8 * h] = acc[n][h];
                        }
                }
                __syncthreads();
                for (int idx = threadIdx.x; idx < ntok * 16; idx += kCW * 32) {
                    float sum = 0.f;
#pragma unroll
                    for (int wv = 0; wv < kCW; wv++) sum += part[(par * kCW + wv) * ntok * 16 + idx];
                    float* keep = &accs[(tile - t_begin) * ntok * 16 + idx];
                    if (pass > 0) sum += *keep;
                    if (pass + 1 < npass) {
                        *keep = sum;
                        continue;
                    }
                    const Member& M = P.mem[member_of(P, (int64_t)tile)];
                    const int64_t row = (int64_t)(tile - (int)M.tile_begin) * 16 + (idx & 15);
                    if (!ok || row >= M.rows) continue;
                    if (P.tp_on) {  // this rank's partial, into this CTA's region of every rank
                        tp_put(P.tp, tp_sh[0], (int)blockIdx.x, tile - t_begin, ntok, idx, sum);
                    } else {
                        M.out[(int64_t)(idx >> 4) * M.ldo + row] = sum;
                    }
                }
                par ^= 1;
            }
        }
    }

#undef CLQ_SIDE_FETCH
    if (P.tp_on) {
        // ---- all-reduce over the ranks: every rank partitions the tiles the
        // same way, so this CTA's counterparts on the other ranks produce the
        // same outputs; wait for their words (bounded) and sum in rank order ----
        __syncthreads();
        const uint32_t ep = tp_sh[0];
        tp_gather_sum(P.tp, P.mem[0], t_begin, t_end, ntok, ep, err);
        __syncthreads();  // every thread has its words before the epoch moves on
        if (threadIdx.x == 0) P.tp.epochs[blockIdx.x] = ep;
    }

    // copies still in flight (only after an expired wait) land before the CTA exits
    if (warp == 0 && lane == 0) *issued_sh = pr.u;
    __syncthreads();
    if (threadIdx.x == 0) {
        const int iss = *issued_sh;
        for (int v = iss > S ? iss - S : 0; v < iss; v++) mbar_drain(&full[v % S], (v / S) & 1);
    }
}

int bulk_sm_count() { return sm_count(); }

bool bulk_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("CLQ_GEMV_BULK");  // tuning knob: 0 sends decode to the register-fed kernel
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

int bulk_max_tiles() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("CLQ_GEMV_BULK_TILES");  // tuning knob: most 16-row tiles per SM for the bulk kernel
        v = e ? atoi(e) : 1 << 20;
        if (v < 1) v = 1;
    }
    return v;
}

bool i8_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("CLQ_GEMV_I8");  // tuning knob: 0 keeps one- and two-row decode on fp16 MMAs
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

size_t al128(size_t v) { return (v + 127) & ~(size_t)127; }

size_t smem_budget() {
    static long kb = -1;
    if (kb < 0) {
        const char* e = getenv("CLQ_GEMV_SMEM_KB");  // tuning knob: shared memory per CTA
        kb = e ? atol(e) : 0;
    }
    return kb > 0 ? (size_t)kb * 1024 : 200 * 1024;
}

// Shared-memory plan for DTYPE at K, NTOK tokens and TILES tiles over GRID CTAs
// within BUDGET bytes: activations staged in passes of pc chunks (all of K
// when that leaves room for the ring), then the ring.  False when fewer than
// two stages fit.
template <int D, bool I8>
bool plan(BulkParams& P, int ntok, int64_t tiles, int64_t grid, size_t budget, size_t* smem) {
    using Gm = Geo<D, I8>;
    const int nchunks = P.nchunks;
    P.qs = kCW * Gm::q + Gm::qpad;
    P.ds = Gm::d ? kCW * Gm::d + 16 : 0;
    P.d_off = 16 * P.qs;
    P.stage_bytes = (uint32_t)al128(16 * (size_t)(P.qs + P.ds));
    size_t per_chunk;
    if constexpr (I8) per_chunk = (size_t)ntok * I8Block<D>::bytes;
    else per_chunk = (size_t)ntok * (1024 + (D == kQ4_K ? 32 : 0) + 4);
    const int64_t tiles_per_cta = (tiles + grid - 1) / grid;
    auto layout = [&](int64_t pc) {
        const int64_t npass = (nchunks + pc - 1) / pc;
        P.pc = (int)pc;
        P.x_off = kHeader;
        P.part_off = (uint32_t)(P.x_off + al128((size_t)pc * per_chunk));
        P.acc_off = (uint32_t)(P.part_off + al128((size_t)2 * kCW * ntok * 16 * 4));
        P.ring_off = (uint32_t)(P.acc_off + (npass > 1 ? al128((size_t)tiles_per_cta * ntok * 16 * 4) : 0));
        return P.ring_off < budget ? (int64_t)(budget - P.ring_off) / P.stage_bytes : (int64_t)0;
    };
    // stage the activations in passes of whole stages only when all of K leaves
    // fewer than two stages or under 96 KB of weights in flight
    auto enough = [&](int64_t st) { return st >= 2 && st * P.stage_bytes >= 96 * 1024; };
    int64_t pc = nchunks;
    int64_t stages = layout(pc);
    while (!enough(stages) && pc > kCW) {
        int64_t next = ((pc + 1) / 2 + kCW - 1) / kCW * kCW;
        if (next >= pc) next = pc - kCW;
        pc = next;
        stages = layout(pc);
    }
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < 2) return false;
    P.stages = (int)stages;
    *smem = P.ring_off + (size_t)stages * P.stage_bytes;
    return true;
}

template <int D, typename XT, int MT, bool I8>
cudaError_t launch_bulk(BulkParams P, cudaStream_t stream) {
    const int64_t sms = bulk_sm_count();
    const int64_t grid = P.tiles < sms ? P.tiles : sms;
    if (P.tp_on && (grid > kMaxTpCtas || (P.tiles + grid - 1) / grid * 16 * P.m > P.tp.cap))
        return cudaErrorNotSupported;
    size_t smem = 0;
    if (!plan<D, I8>(P, P.m, P.tiles, grid, smem_budget(), &smem)) return cudaErrorNotSupported;
    auto kern = gemv_bulk_kernel<D, XT, MT, I8>;
    // the attribute is per device; the largest plan of this variant so far is kept
    static std::atomic<int> set_for[kMaxDevices];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if ((int)smem > set_for[dev].load(std::memory_order_relaxed)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        int seen = set_for[dev].load(std::memory_order_relaxed);
        while ((int)smem > seen && !set_for[dev].compare_exchange_weak(seen, (int)smem)) {
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kBulkThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = gemv_pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, P);
}

template <int D, typename XT>
cudaError_t launch_bulk_shape(const BulkParams& P, cudaStream_t s) {
    if constexpr (D == kQ4_K || D == kQ6_K) {
        if (P.m <= 2 && i8_enabled()) return launch_bulk<D, XT, 1, true>(P, s);
    }
    if (P.m <= 4) return launch_bulk<D, XT, 1, false>(P, s);
    return launch_bulk<D, XT, 2, false>(P, s);
}

template <typename XT>
cudaError_t launch_bulk_dtype(const BulkParams& P, int dtype, cudaStream_t s) {
    switch (dtype) {
    case kQ4_K: return launch_bulk_shape<kQ4_K, XT>(P, s);
    case kQ6_K: return launch_bulk_shape<kQ6_K, XT>(P, s);
    case kQ4_0: return launch_bulk_shape<kQ4_0, XT>(P, s);
    case kQ8_0: return launch_bulk_shape<kQ8_0, XT>(P, s);
    default: return cudaErrorNotSupported;
    }
}

}  // namespace

int sm_count() {
    static int count = 0;
    if (!count) {
        int dev = 0, c = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
        count = c;
    }
    return count;
}

cudaError_t launch_gemv_bulk_impl(const WeightView* const* w, const int64_t* rows, int count, const void* x,
                                  int xtype, int64_t m, float* const* out, const int64_t* ldo, const TpLink* tp,
                                  cudaStream_t stream);

cudaError_t launch_gemv_bulk_allreduce(const WeightView& w, int64_t rows, const void* x, int xtype, int64_t m,
                                       float* out, int64_t ldo, const TpLink& tp, cudaStream_t stream) {
    if (tp.world < 1 || tp.world > kMaxRanks) return cudaErrorNotSupported;
    const WeightView* wp = &w;
    return launch_gemv_bulk_impl(&wp, &rows, 1, x, xtype, m, &out, &ldo, &tp, stream);
}

cudaError_t launch_gemv_bulk_group(const WeightView* const* w, const int64_t* rows, int count, const void* x,
                                   int xtype, int64_t m, float* const* out, const int64_t* ldo,
                                   cudaStream_t stream) {
    return launch_gemv_bulk_impl(w, rows, count, x, xtype, m, out, ldo, nullptr, stream);
}

// Most activation rows the per-warp passes take (GEMM territory beyond).
constexpr int64_t kMaxPassRows = 32;

cudaError_t launch_gemv_bulk_impl(const WeightView* const* w, const int64_t* rows, int count, const void* x,
                                  int xtype, int64_t m, float* const* out, const int64_t* ldo, const TpLink* tp,
                                  cudaStream_t stream) {
    // Q4_K / Q6_K rows the per-warp streams do not take in one pass (9 to 32
    // rows; fewer when the plan of all of them does not fit, as on the
    // largest vocabulary heads): passes of STEP rows, each reading the
    // weights once at that row count's rate -- at 16 rows two passes of
    // eight take half the time of one 16-row pass of the other GEMVs.  A
    // later pass has no more rows than the first, so its plan fits when the
    // first one's does; nothing is launched when the first does not fit.
    auto passes = [&](int64_t step) -> cudaError_t {
        const size_t esize = xtype == CLQ_X_F32 ? 4 : 2;
        for (int64_t r0 = 0; r0 < m; r0 += step) {
            float* o[kGroup];
            for (int i = 0; i < count; i++) o[i] = out[i] + r0 * ldo[i];
            const void* xr = static_cast<const uint8_t*>(x) + (size_t)r0 * (size_t)w[0]->k * esize;
            const cudaError_t e = launch_gemv_warp(w, rows, count, xr, xtype, m - r0 < step ? m - r0 : step, o, ldo,
                                                   nullptr, stream);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    };
    if (!bulk_enabled() || m < 1 || m > kMaxPassRows || count < 1 || count > kGroup) return cudaErrorNotSupported;
    if (m <= 8) {
        // up to eight activation rows: the per-warp streams when their plan fits
        const cudaError_t ew = launch_gemv_warp(w, rows, count, x, xtype, m, out, ldo, tp, stream);
        if (ew != cudaErrorNotSupported) return ew;
    }
    // passes for the K formats; Q4_0 / Q8_0 beyond eight rows keep the register-fed kernel
    if (!tp && (w[0]->dtype == kQ4_K || w[0]->dtype == kQ6_K)) {
        for (int64_t step : {8, 4, 2}) {
            if (step >= m) continue;
            const cudaError_t e = passes(step);
            if (e != cudaErrorNotSupported) return e;
        }
    }
    if (m > 8) return cudaErrorNotSupported;
    int* err = device_status_word();
    if (!err) return cudaErrorNotSupported;
    BulkParams P = {};
    P.nmem = count;
    int64_t tiles = 0;
    for (int i = 0; i < count; i++) {
        if (w[i]->dtype != w[0]->dtype || w[i]->k != w[0]->k || w[i]->k % 256) return cudaErrorNotSupported;
        if (rows[i] < 1) return cudaErrorNotSupported;
        P.mem[i].p = Planes{w[i]->q, w[i]->s, w[i]->d, w[i]->nb};
        P.mem[i].rows = rows[i];
        P.mem[i].out = out[i];
        P.mem[i].ldo = ldo[i];
        P.mem[i].tile_begin = tiles;
        tiles += (rows[i] + 15) / 16;
    }
    if (tiles > (1 << 30) || w[0]->k / 256 > (1 << 20)) return cudaErrorNotSupported;
    // The register-fed kernel is faster on Q4_0 / Q8_0 and on launches with
    // more than bulk_max_tiles() tiles per SM.
    if (w[0]->dtype != kQ4_K && w[0]->dtype != kQ6_K) return cudaErrorNotSupported;
    if (tiles > (int64_t)bulk_max_tiles() * bulk_sm_count()) return cudaErrorNotSupported;
    P.tiles = (int)tiles;
    P.k = w[0]->k;
    P.nchunks = (int)(w[0]->k / 256);
    P.m = (int)m;
    P.x = x;
    P.err = err;
    if (tp) {
        P.tp_on = 1;
        P.tp = *tp;
    }
    const int esize = xtype == CLQ_X_F32 ? 4 : 2;
    P.x_aligned = ((uintptr_t)x % 16 == 0) && ((P.k * esize) % 16 == 0);
    switch (xtype) {
    case CLQ_X_F32: return launch_bulk_dtype<float>(P, w[0]->dtype, stream);
    case CLQ_X_BF16: return launch_bulk_dtype<__nv_bfloat16>(P, w[0]->dtype, stream);
    case CLQ_X_F16: return launch_bulk_dtype<__half>(P, w[0]->dtype, stream);
    default: return cudaErrorNotSupported;
    }
}

}  // namespace clq
