// gemv_mma.cu -- fused dequant + GEMV/skinny-GEMM for packed weights on the
// warp-level tensor-core MMA (mma.sync m16n8k16, fp16 operands, fp32 accumulate),
// with weights loaded straight into registers (double-buffered).  Used for the
// shapes the bulk-copy GEMV (gemv_bulk.cu) does not take: more than 8
// activation rows, or Q6_K rows whose length is not a multiple of 2048.
// The CTA splits K across warps and reduces through shared memory; activations
// are staged once per CTA into shared memory in MMA-fragment order.
#include <cstdlib>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/clq.h"
#include "clq_internal.h"
#include "gemv_common.cuh"

namespace clq {
namespace {

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


// Each CTA owns tiles_per_cta consecutive 16-row tiles for one slice of up to
// 8*MT activation rows.  The activations are staged once per pass over K; each
// warp then streams a flat list of (tile, chunk) units -- its chunks are
// warp, warp + WARPS, ... -- with the next unit's weights loaded while the
// current one is computed.  Per-(warp, tile) partial sums stay in shared
// memory and one barrier at the end precedes the cross-warp sum.
// Launched with programmatic dependent launch: weight loads do not depend on
// the previous kernel, so only the activation staging waits for it.
template <int D, typename XT, int MT, int WARPS>
// Four token tiles (9-16 activation rows) need more registers than two CTAs of
// 8 warps leave: one CTA per SM for them.
__global__ void __launch_bounds__(WARPS * 32, MT >= 4 ? 8 / WARPS : 16 / WARPS) gemv_mma_kernel(Params P) {
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
        stage_x<D, XT, WARPS>(P.x, P.k, P.x_aligned, P.part_chunks, c0, pc, tok0, ntok, xf, us, sxf);
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
    const int64_t slots = ((MT >= 4 ? 8 : 16) / WARPS) * (int64_t)sm_count();
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

bool gemv_pdl_enabled() { return pdl_enabled(); }

bool gemv_mma_supported(const WeightView& w, int64_t m) {
    return w.k > 0 && w.k % 256 == 0 && m > 0;
}

cudaError_t launch_gemv_mma_group(const WeightView* const* w, const int64_t* rows, int count, const void* x,
                                  int xtype, int64_t m, float* const* out, const int64_t* ldo,
                                  cudaStream_t stream) {
    if (count < 1 || count > kGroup) return cudaErrorInvalidValue;
    // decode shapes go to the bulk-copy kernel; it declines the rest
    const cudaError_t eb = launch_gemv_bulk_group(w, rows, count, x, xtype, m, out, ldo, stream);
    if (eb != cudaErrorNotSupported) return eb;
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
