// api.cu -- the C ABI of libclq (include/clq.h): status codes, the device
// store, the host-range weight cache behind the drop-in kernels, and the
// per-thread stream and staging buffers for host-pointer calls.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <map>
#include <memory>
#include <mutex>
#include <tuple>
#include <new>
#include <string>
#include <vector>

#include "../../include/clq.h"
#include "clq_internal.h"
#include "layout.cuh"

struct clq_store {
    int dtype = 0;
    int64_t n = 0, k = 0;
    size_t nbytes = 0;            // native GGUF bytes
    int device = -1;
    uint8_t* dev = nullptr;       // re-tiled planes (layout.cuh)
    size_t s_off = 0, d_off = 0;  // plane offsets inside dev
    int elems = 0, block_bytes = 0;
    int64_t row_bytes = 0, nb = 0;
};

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    if (e == cudaErrorMemoryAllocation)
        return fail(CLQ_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(e));
    return fail(CLQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

const char* dtype_name(int dtype) {
    switch (dtype) {
    case CLQ_Q4_0: return "Q4_0";
    case CLQ_Q8_0: return "Q8_0";
    case CLQ_Q4_K: return "Q4_K";
    case CLQ_Q6_K: return "Q6_K";
    default: return "?";
    }
}

// The current device, checked once per device to be an sm_100 part.
int current_device(int* dev) {
    static std::mutex mu;
    static std::vector<int> checked;  // 0 unknown, 1 ok, 2 bad
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return fail(CLQ_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lock(mu);
    if ((int)checked.size() <= *dev) checked.resize(*dev + 1, 0);
    if (checked[*dev] == 0) {
        cudaDeviceProp prop;
        e = cudaGetDeviceProperties(&prop, *dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
        checked[*dev] = prop.major == 10 ? 1 : 2;
    }
    if (checked[*dev] != 1)
        return fail(CLQ_ERR_NO_DEVICE, "device %d is not an sm_100 (B200-class) GPU", *dev);
    return CLQ_OK;
}

int check_shape(int dtype, int64_t n, int64_t k, int* elems, int* bb) {
    if (!clq::geometry(dtype, elems, bb)) return fail(CLQ_ERR_ARGUMENT, "unknown packed dtype %d", dtype);
    if (n < 0 || k < 0) return fail(CLQ_ERR_SHAPE, "negative shape (%lld %lld)", (long long)n, (long long)k);
    if (k % *elems)
        return fail(CLQ_ERR_SHAPE, "%s row length %lld is not a multiple of %d", dtype_name(dtype),
                    (long long)k, *elems);
    return CLQ_OK;
}

clq::WeightView view_of(const clq_store* s, int64_t row_begin) {
    clq::PlaneGeometry g = clq::plane_geometry(s->dtype);
    const int64_t blk = row_begin * s->nb;
    clq::WeightView v;
    v.dtype = s->dtype;
    v.rows = s->n - row_begin;
    v.k = s->k;
    v.nb = s->nb;
    v.q = s->dev + blk * g.q_block;
    v.s = s->dev + s->s_off + blk * g.s_block;
    v.d = s->dev + s->d_off + blk * g.d_block;
    return v;
}

void destroy_store(clq_store* s) {
    if (!s) return;
    if (s->dev) {
        int prev = -1;
        cudaGetDevice(&prev);
        if (prev != s->device) cudaSetDevice(s->device);
        cudaFree(s->dev);
        if (prev >= 0 && prev != s->device) cudaSetDevice(prev);
    }
    delete s;
}

// Copy the native blocks to the device (or use them in place when already
// there), check every scale is finite, re-tile into the planes.  Synchronous.
int make_store(int dtype, int64_t n, int64_t k, const void* src, bool src_on_device, size_t nbytes,
               cudaStream_t stream, clq_store** out) {
    int elems, bb, rc;
    if ((rc = check_shape(dtype, n, k, &elems, &bb))) return rc;
    if (nbytes % (size_t)bb)
        return fail(CLQ_ERR_BLOCKS, "%s data of %zu bytes is not a whole number of %d-byte blocks",
                    dtype_name(dtype), nbytes, bb);
    const int64_t row_bytes = k / elems * bb;
    if ((size_t)(n * row_bytes) != nbytes)
        return fail(CLQ_ERR_SHAPE, "%s weight (%lld %lld) needs %lld bytes, got %zu", dtype_name(dtype),
                    (long long)n, (long long)k, (long long)(n * row_bytes), nbytes);
    if (nbytes && !src) return fail(CLQ_ERR_ARGUMENT, "null weight bytes");
    int device;
    if ((rc = current_device(&device))) return rc;
    std::unique_ptr<clq_store, void (*)(clq_store*)> s(new clq_store, destroy_store);
    s->dtype = dtype; s->n = n; s->k = k; s->nbytes = nbytes; s->device = device;
    s->elems = elems; s->block_bytes = bb; s->row_bytes = row_bytes; s->nb = k / elems;
    const int64_t nblocks = n * s->nb;
    size_t total;
    clq::plane_offsets(dtype, nblocks, &s->s_off, &s->d_off, &total);
    cudaError_t e = cudaMalloc((void**)&s->dev, total);
    if (e != cudaSuccess) { s->dev = nullptr; return cuda_fail(e, "cudaMalloc(weight store)"); }
    uint8_t* native = nullptr;
    if (nbytes && !src_on_device) {
        e = cudaMalloc((void**)&native, nbytes);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(upload staging)");
    }
    unsigned long long* flag = nullptr;
    e = cudaMalloc((void**)&flag, sizeof *flag);
    if (e != cudaSuccess) { cudaFree(native); return cuda_fail(e, "cudaMalloc(flag)"); }
    const uint8_t* nat = src_on_device ? (const uint8_t*)src : native;
    unsigned long long first_bad = ~0ull;
    do {
        if ((e = cudaMemsetAsync(s->dev, 0, total, stream)) != cudaSuccess) break;
        if (nbytes && !src_on_device &&
            (e = cudaMemcpyAsync(native, src, nbytes, cudaMemcpyHostToDevice, stream)) != cudaSuccess)
            break;
        if ((e = cudaMemcpyAsync(flag, &first_bad, sizeof first_bad, cudaMemcpyHostToDevice, stream)) !=
            cudaSuccess)
            break;
        if ((e = clq::launch_validate_scales(nat, dtype, nblocks, flag, stream)) != cudaSuccess) break;
        if ((e = clq::launch_retile(nat, dtype, n, s->nb, s->dev, stream)) != cudaSuccess) break;
        if ((e = cudaMemcpyAsync(&first_bad, flag, sizeof first_bad, cudaMemcpyDeviceToHost, stream)) !=
            cudaSuccess)
            break;
        e = cudaStreamSynchronize(stream);
    } while (0);
    cudaFree(flag);
    if (native) cudaFree(native);
    if (e != cudaSuccess) return cuda_fail(e, "weight upload");
    if (first_bad != ~0ull)
        return fail(CLQ_ERR_NONFINITE_SCALE, "Non-finite %s scale at byte %llu", dtype_name(dtype),
                    first_bad * (unsigned long long)bb);
    *out = s.release();
    return CLQ_OK;
}

// ---- per-thread stream and staging for host-pointer calls -----------------

struct DeviceBuffer {
    void* ptr = nullptr;
    size_t cap = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap) return cudaSuccess;
        if (ptr) cudaFree(ptr);
        ptr = nullptr; cap = 0;
        size_t want = bytes < 4096 ? 4096 : bytes + bytes / 4;
        cudaError_t e = cudaMalloc(&ptr, want);
        if (e == cudaSuccess) cap = want;
        return e;
    }
};

// Page-locked host staging: pageable copies make the driver stage through its
// own buffer on every call, which dominates small decode-sized products.
// Page-locked host memory, mapped into the device's address space: kernels
// can store into it directly (dptr), with no copy back.
struct PinnedBuffer {
    void* ptr = nullptr;
    void* dptr = nullptr;
    size_t cap = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap) return cudaSuccess;
        if (ptr) cudaFreeHost(ptr);
        ptr = dptr = nullptr; cap = 0;
        size_t want = bytes < 65536 ? 65536 : bytes + bytes / 4;
        cudaError_t e = cudaHostAlloc(&ptr, want, cudaHostAllocMapped);
        if (e != cudaSuccess) return e;
        e = cudaHostGetDevicePointer(&dptr, ptr, 0);
        if (e != cudaSuccess) {
            cudaFreeHost(ptr);
            ptr = dptr = nullptr;
            return e;
        }
        cap = want;
        return cudaSuccess;
    }
};

// One host call's device work (the copy of x, the linear) as an instantiated
// CUDA graph, replayed by later calls with the same store, shape and staging
// buffers: one launch instead of two, with the kernels' parameters checked
// once.  The entry keeps its store alive; a thread drops its graphs (and its
// remembered lookups) when the weight cache changes (clq_forget,
// clq_clear_cache).
using GraphKey = std::tuple<const clq_store*, int64_t, int64_t, int64_t, int64_t, unsigned, void*, void*, void*>;
struct CallGraph {
    cudaGraphExec_t exec = nullptr;
    std::shared_ptr<clq_store> store;
};
std::atomic<uint64_t> g_cache_generation{0};

struct ThreadContext {
    int device = -1;
    cudaStream_t stream = nullptr;
    DeviceBuffer x, out, ids;
    PinnedBuffer hx, hout;  // host staging of x and out for small products
    std::map<GraphKey, CallGraph> graphs;
    void* graph_buffers[3] = {nullptr, nullptr, nullptr};  // x, hx, hout when the graphs were made
    // this thread's earlier lookups: (host address, n, k, dtype) -> (store, first row)
    std::map<std::tuple<const uint8_t*, int64_t, int64_t, int>, std::pair<std::shared_ptr<clq_store>, int64_t>> hits;
    uint64_t graph_generation = 0;
    void drop_graphs() {
        for (auto& kv : graphs)
            if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
        graphs.clear();
        hits.clear();
    }
    // Drops the graphs and lookups that predate a change of the weight cache.
    void sync_generation() {
        const uint64_t gen = g_cache_generation.load();
        if (gen != graph_generation) {
            drop_graphs();
            graph_generation = gen;
        }
    }
};

struct ThreadContexts {
    std::vector<ThreadContext*> per_device;
    ~ThreadContexts() {
        for (ThreadContext* c : per_device) {
            if (!c) continue;
            cudaSetDevice(c->device);
            c->drop_graphs();
            if (c->stream) cudaStreamDestroy(c->stream);
            if (c->x.ptr) cudaFree(c->x.ptr);
            if (c->out.ptr) cudaFree(c->out.ptr);
            if (c->ids.ptr) cudaFree(c->ids.ptr);
            if (c->hx.ptr) cudaFreeHost(c->hx.ptr);
            if (c->hout.ptr) cudaFreeHost(c->hout.ptr);
            delete c;
        }
    }
};
thread_local ThreadContexts t_contexts;

int thread_context(int device, ThreadContext** out) {
    auto& v = t_contexts.per_device;
    if ((int)v.size() <= device) v.resize(device + 1, nullptr);
    if (!v[device]) {
        auto* c = new ThreadContext;
        c->device = device;
        cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) { delete c; return cuda_fail(e, "cudaStreamCreate"); }
        v[device] = c;
    }
    *out = v[device];
    return CLQ_OK;
}

// ---- host-range weight cache ----------------------------------------------

struct CacheEntry {
    const uint8_t* host;
    size_t nbytes;
    std::shared_ptr<clq_store> store;
};
std::mutex g_cache_mu;
std::vector<CacheEntry> g_cache;

// Find or create the store holding N rows of the weight at host address BYTES.
int cached_store(int dtype, int64_t n, int64_t k, const uint8_t* bytes, int device, bool use_cache,
                 cudaStream_t stream, std::shared_ptr<clq_store>* out, int64_t* row_begin) {
    int elems, bb, rc;
    if ((rc = check_shape(dtype, n, k, &elems, &bb))) return rc;
    const int64_t row_bytes = k / elems * bb;
    const size_t need = (size_t)(n * row_bytes);
    if (use_cache) {
        std::lock_guard<std::mutex> lock(g_cache_mu);
        for (const CacheEntry& e : g_cache) {
            const clq_store* s = e.store.get();
            if (s->device != device || s->dtype != dtype || s->k != k) continue;
            if (bytes < e.host || bytes + need > e.host + e.nbytes) continue;
            size_t off = (size_t)(bytes - e.host);
            if (row_bytes == 0 || off % (size_t)row_bytes) continue;
            *out = e.store;
            *row_begin = (int64_t)(off / (size_t)row_bytes);
            return CLQ_OK;
        }
    }
    clq_store* raw = nullptr;
    if ((rc = make_store(dtype, n, k, bytes, false, need, stream, &raw))) return rc;
    std::shared_ptr<clq_store> s(raw, destroy_store);
    if (use_cache) {
        std::lock_guard<std::mutex> lock(g_cache_mu);
        g_cache.push_back({bytes, need, s});
    }
    *out = s;
    *row_begin = 0;
    return CLQ_OK;
}

}  // namespace

int clq::set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

// Sticky per-device status word: a kernel whose bounded wait expires records a
// CLQ_ERR_* code here and every later wait on the device falls through at once;
// clq_device_status reads and clears it.
static __device__ int g_device_status;

int* clq::device_status_word() {
    static std::mutex mu;
    static std::vector<int*> addr;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)addr.size() <= device) addr.resize(device + 1, nullptr);
    if (!addr[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
        addr[device] = static_cast<int*>(p);
    }
    return addr[device];
}

// ---------------------------------------------------------------------------

extern "C" {

int clq_device_status(int* status) {
    if (!status) return fail(CLQ_ERR_ARGUMENT, "null status pointer");
    *status = CLQ_OK;
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    int* word = clq::device_status_word();
    if (!word) return fail(CLQ_ERR_CUDA, "device status word not found on device %d", device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
    int v = 0;
    if ((e = cudaMemcpy(&v, word, sizeof v, cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(e, "reading the device status");
    if (v && (e = cudaMemset(word, 0, sizeof v)) != cudaSuccess) return cuda_fail(e, "clearing the device status");
    *status = v;
    return CLQ_OK;
}

int clq_abi_version(void) { return CLQ_ABI_VERSION; }

int clq_last_error(char* buf, size_t len) {
    if (!buf || !len) return CLQ_ERR_ARGUMENT;
    std::snprintf(buf, len, "%s", t_last_error.c_str());
    return CLQ_OK;
}

int clq_block_geometry(int dtype, int64_t* elements, int64_t* block_bytes) {
    int e, b;
    if (!clq::geometry(dtype, &e, &b)) return fail(CLQ_ERR_ARGUMENT, "unknown packed dtype %d", dtype);
    if (elements) *elements = e;
    if (block_bytes) *block_bytes = b;
    return CLQ_OK;
}

int clq_store_create(int dtype, int64_t n, int64_t k, const uint8_t* host_bytes, size_t nbytes,
                     unsigned flags, clq_store** out) {
    if (!out) return fail(CLQ_ERR_ARGUMENT, "null store result pointer");
    if (flags != CLQ_STORE_DEFAULT) return fail(CLQ_ERR_ARGUMENT, "unknown store flags 0x%x", flags);
    *out = nullptr;
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    ThreadContext* ctx;
    if ((rc = thread_context(device, &ctx))) return rc;
    return make_store(dtype, n, k, host_bytes, false, nbytes, ctx->stream, out);
}

int clq_store_create_device(int dtype, int64_t n, int64_t k, const void* device_bytes, size_t nbytes,
                            unsigned flags, void* stream, clq_store** out) {
    if (!out) return fail(CLQ_ERR_ARGUMENT, "null store result pointer");
    if (flags != CLQ_STORE_DEFAULT) return fail(CLQ_ERR_ARGUMENT, "unknown store flags 0x%x", flags);
    *out = nullptr;
    return make_store(dtype, n, k, device_bytes, true, nbytes, (cudaStream_t)stream, out);
}

int clq_store_free(clq_store* store) {
    destroy_store(store);
    return CLQ_OK;
}

int clq_store_info(const clq_store* s, int* dtype, int64_t* n, int64_t* k, size_t* nbytes,
                   const void** device_bytes, int* device) {
    if (!s) return fail(CLQ_ERR_ARGUMENT, "null store");
    if (dtype) *dtype = s->dtype;
    if (n) *n = s->n;
    if (k) *k = s->k;
    if (nbytes) *nbytes = s->nbytes;
    if (device_bytes) *device_bytes = s->dev;
    if (device) *device = s->device;
    return CLQ_OK;
}

int clq_linear_device(const clq_store* w, int64_t row_begin, int64_t rows, const void* x, int xtype,
                      int64_t m, float* out, int64_t ldo, unsigned flags, void* stream) {
    if (!w) return fail(CLQ_ERR_ARGUMENT, "null store");
    if (xtype != CLQ_X_F32 && xtype != CLQ_X_BF16 && xtype != CLQ_X_F16)
        return fail(CLQ_ERR_ARGUMENT, "unknown activation type %d", xtype);
    if (flags & ~(CLQ_MATH_FAST | CLQ_MATH_EXACT)) return fail(CLQ_ERR_ARGUMENT, "unknown product flags 0x%x", flags);
    if (row_begin < 0 || rows < 0 || row_begin + rows > w->n || m < 0)
        return fail(CLQ_ERR_SHAPE, "rows [%lld, %lld) / m %lld outside a (%lld %lld) weight",
                    (long long)row_begin, (long long)(row_begin + rows), (long long)m,
                    (long long)w->n, (long long)w->k);
    if (ldo < rows) return fail(CLQ_ERR_SHAPE, "output stride %lld < rows %lld", (long long)ldo, (long long)rows);
    if (m == 0 || rows == 0) return CLQ_OK;
    if (!x || !out) return fail(CLQ_ERR_ARGUMENT, "null activation or output pointer");
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    if (device != w->device)
        return fail(CLQ_ERR_ARGUMENT, "store lives on device %d, current device is %d", w->device, device);
    if (w->k == 0) {
        for (int64_t i = 0; i < m; i++) {
            cudaError_t e = cudaMemsetAsync(out + i * ldo, 0, rows * sizeof(float), (cudaStream_t)stream);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
        }
        return CLQ_OK;
    }
    cudaError_t e = clq::launch_linear(view_of(w, row_begin), rows, x, xtype, m, out, ldo, flags,
                                       (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "linear kernel launch");
    return CLQ_OK;
}

int clq_linear_group_device(const clq_store* const* w, const int64_t* row_begin, const int64_t* rows,
                            int count, const void* x, int xtype, int64_t m, float* const* out,
                            const int64_t* ldo, unsigned flags, void* stream) {
    if (count < 1 || count > 4) return fail(CLQ_ERR_ARGUMENT, "group of %d weights (1..4 allowed)", count);
    if (!w || !row_begin || !rows || !out || !ldo) return fail(CLQ_ERR_ARGUMENT, "null group array");
    for (int i = 0; i < count; i++) {
        if (!w[i]) return fail(CLQ_ERR_ARGUMENT, "null store %d in group", i);
        if (w[i]->dtype != w[0]->dtype || w[i]->k != w[0]->k)
            return fail(CLQ_ERR_SHAPE, "group members need one dtype and row length");
    }
    bool fused = m > 0 && w[0]->k > 0 && w[0]->k % 256 == 0 && !(flags & ~(CLQ_MATH_FAST | CLQ_MATH_EXACT)) &&
                 !clq::uses_gemm_tc(view_of(w[0], 0), xtype, m, flags);
    for (int i = 0; i < count && fused; i++)
        fused = row_begin[i] >= 0 && rows[i] > 0 && row_begin[i] + rows[i] <= w[i]->n && ldo[i] >= rows[i] && out[i];
    if (!fused) {
        // the tensor-core GEMM forms the shared activation image once
        bool gemm = m > 0 && w[0]->k > 0 && w[0]->k % 256 == 0 && x && !(flags & ~(CLQ_MATH_FAST | CLQ_MATH_EXACT)) &&
                    (xtype == CLQ_X_F32 || xtype == CLQ_X_BF16 || xtype == CLQ_X_F16) &&
                    clq::uses_gemm_tc(view_of(w[0], 0), xtype, m, flags);
        int device = -1;
        if (gemm && current_device(&device)) gemm = false;  // the calls below report it
        for (int i = 0; i < count && gemm; i++)
            gemm = row_begin[i] >= 0 && rows[i] > 0 && row_begin[i] + rows[i] <= w[i]->n && ldo[i] >= rows[i] &&
                   out[i] && w[i]->device == device;
        if (gemm) {
            clq::WeightView views[4];
            const clq::WeightView* vp[4];
            for (int i = 0; i < count; i++) {
                views[i] = view_of(w[i], row_begin[i]);
                vp[i] = &views[i];
            }
            const cudaError_t e =
                clq::launch_linear_group_gemm(vp, rows, count, x, xtype, m, out, ldo, flags, (cudaStream_t)stream);
            if (e == cudaSuccess) return CLQ_OK;
            if (e != cudaErrorNotSupported) return cuda_fail(e, "grouped GEMM launch");
        }
        // validation and any other shape, one call each
        for (int i = 0; i < count; i++) {
            int rc = clq_linear_device(w[i], row_begin[i], rows[i], x, xtype, m, out[i], ldo[i], flags, stream);
            if (rc) return rc;
        }
        return CLQ_OK;
    }
    if (!x) return fail(CLQ_ERR_ARGUMENT, "null activations");
    if (xtype != CLQ_X_F32 && xtype != CLQ_X_BF16 && xtype != CLQ_X_F16)
        return fail(CLQ_ERR_ARGUMENT, "unknown activation type %d", xtype);
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    clq::WeightView views[4];
    const clq::WeightView* vp[4];
    for (int i = 0; i < count; i++) {
        if (w[i]->device != device)
            return fail(CLQ_ERR_ARGUMENT, "store lives on device %d, current device is %d", w[i]->device, device);
        views[i] = view_of(w[i], row_begin[i]);
        vp[i] = &views[i];
    }
    cudaError_t e = clq::launch_gemv_mma_group(vp, rows, count, x, xtype, m, out, ldo, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "grouped linear kernel launch");
    return CLQ_OK;
}

int clq_linear_group_fused_device(const clq_store* const* w, const int64_t* row_begin, const int64_t* rows,
                                  int count, const void* x, int xtype, int64_t m, const clq_fusion* fusion,
                                  float* const* out, const int64_t* ldo, unsigned flags, void* stream) {
    if (!fusion || (!fusion->norm_weight && !fusion->gate && !fusion->residual)) {
        if (count == 1 && w && row_begin && rows && out && ldo)
            return clq_linear_device(w[0], row_begin[0], rows[0], x, xtype, m, out[0], ldo[0], flags, stream);
        return clq_linear_group_device(w, row_begin, rows, count, x, xtype, m, out, ldo, flags, stream);
    }
    if (count < 1 || count > 4) return fail(CLQ_ERR_ARGUMENT, "group of %d weights (1..4 allowed)", count);
    if (!w || !row_begin || !rows || !out || !ldo) return fail(CLQ_ERR_ARGUMENT, "null group array");
    if (xtype != CLQ_X_F32 && xtype != CLQ_X_BF16 && xtype != CLQ_X_F16)
        return fail(CLQ_ERR_ARGUMENT, "unknown activation type %d", xtype);
    if (flags & ~(CLQ_MATH_FAST | CLQ_MATH_EXACT)) return fail(CLQ_ERR_ARGUMENT, "unknown product flags 0x%x", flags);
    if (fusion->residual && count != 1) return fail(CLQ_ERR_ARGUMENT, "a residual needs a single weight");
    if (!(fusion->norm_epsilon >= 0.f) || fusion->norm_epsilon == INFINITY)
        return fail(CLQ_ERR_ARGUMENT, "RMSNorm epsilon must be finite and non-negative");
    for (int i = 0; i < count; i++) {
        if (!w[i]) return fail(CLQ_ERR_ARGUMENT, "null store %d in group", i);
        if (w[i]->dtype != w[0]->dtype || w[i]->k != w[0]->k)
            return fail(CLQ_ERR_SHAPE, "group members need one dtype and row length");
        if (row_begin[i] < 0 || rows[i] < 0 || row_begin[i] + rows[i] > w[i]->n || ldo[i] < rows[i])
            return fail(CLQ_ERR_SHAPE, "member %d: rows [%lld, %lld), output stride %lld for a (%lld %lld) weight", i,
                        (long long)row_begin[i], (long long)(row_begin[i] + rows[i]), (long long)ldo[i],
                        (long long)w[i]->n, (long long)w[i]->k);
    }
    if (fusion->residual && fusion->ldr < rows[0])
        return fail(CLQ_ERR_SHAPE, "residual stride %lld < rows %lld", (long long)fusion->ldr, (long long)rows[0]);
    if (m < 0) return fail(CLQ_ERR_SHAPE, "negative activation rows %lld", (long long)m);
    if (m == 0) return CLQ_OK;
    if (!x) return fail(CLQ_ERR_ARGUMENT, "null activations");
    for (int i = 0; i < count; i++)
        if (rows[i] && !out[i]) return fail(CLQ_ERR_ARGUMENT, "null output %d", i);
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    clq::WeightView views[4];
    const clq::WeightView* vp[4];
    for (int i = 0; i < count; i++) {
        if (w[i]->device != device)
            return fail(CLQ_ERR_ARGUMENT, "store lives on device %d, current device is %d", w[i]->device, device);
        views[i] = view_of(w[i], row_begin[i]);
        vp[i] = &views[i];
    }
    const int64_t k = w[0]->k;
    clq::Fusion f;
    f.norm_w = fusion->norm_weight;
    f.norm_eps = fusion->norm_epsilon;
    f.gate = fusion->gate;
    f.res = fusion->residual;
    f.ldr = fusion->ldr;
    cudaStream_t s = (cudaStream_t)stream;
    bool nonempty = true;
    for (int i = 0; i < count; i++) nonempty = nonempty && rows[i] > 0;
    // the decode kernel applies the fusion itself
    if (nonempty && k > 0 && k % 256 == 0 && !clq::uses_gemm_tc(views[0], xtype, m, flags)) {
        cudaError_t e = clq::launch_gemv_warp(vp, rows, count, x, xtype, m, out, ldo, nullptr, s, &f);
        if (e == cudaSuccess) return CLQ_OK;
        if (e != cudaErrorNotSupported) return cuda_fail(e, "fused linear kernel launch");
    }
    // every other path: the fused input (fp32) into scratch, the plain product,
    // the residual; a request that takes the tensor-core GEMM keeps it (its
    // fp32 input then goes through the GEMM's own fp16 staging)
    float* h = nullptr;
    float* part = nullptr;
    cudaError_t e = cudaSuccess;
    if ((f.norm_w || f.gate) && k > 0) e = cudaMallocAsync((void**)&h, (size_t)(m * k) * sizeof(float), s);
    if (e == cudaSuccess && f.res) e = cudaMallocAsync((void**)&part, (size_t)(m * rows[0]) * sizeof(float), s);
    if (e != cudaSuccess) {
        if (h) cudaFreeAsync(h, s);
        return cuda_fail(e, "fusion scratch");
    }
    if (h && (e = clq::launch_fuse_input(x, xtype, m, k, f, h, s)) != cudaSuccess) rc = cuda_fail(e, "fused input");
    const void* xin = h ? (const void*)h : x;
    const int xt = h ? CLQ_X_F32 : xtype;
    // the fused input is fp32; a 16-bit request keeps the GEMM form it would have had
    const unsigned pf = (h && xtype != CLQ_X_F32 && !(flags & CLQ_MATH_EXACT)) ? (flags | CLQ_MATH_FAST) : flags;
    if (!rc) {
        if (f.res) rc = clq_linear_device(w[0], row_begin[0], rows[0], xin, xt, m, part, rows[0], pf, stream);
        else rc = clq_linear_group_device(w, row_begin, rows, count, xin, xt, m, out, ldo, pf, stream);
    }
    if (!rc && f.res &&
        (e = clq::launch_add_residual(out[0], ldo[0], part, rows[0], f.res, f.ldr, m, rows[0], s)) != cudaSuccess)
        rc = cuda_fail(e, "residual add");
    if (h) cudaFreeAsync(h, s);
    if (part) cudaFreeAsync(part, s);
    return rc;
}

int clq_linear_fused_device(const clq_store* w, int64_t row_begin, int64_t rows, const void* x, int xtype, int64_t m,
                            const clq_fusion* fusion, float* out, int64_t ldo, unsigned flags, void* stream) {
    return clq_linear_group_fused_device(&w, &row_begin, &rows, 1, x, xtype, m, fusion, &out, &ldo, flags, stream);
}

int clq_dequantize_device(const clq_store* w, int64_t row_begin, int64_t rows, float* out,
                          int transposed, void* stream) {
    if (!w) return fail(CLQ_ERR_ARGUMENT, "null store");
    if (row_begin < 0 || rows < 0 || row_begin + rows > w->n)
        return fail(CLQ_ERR_SHAPE, "rows [%lld, %lld) outside %lld rows", (long long)row_begin,
                    (long long)(row_begin + rows), (long long)w->n);
    if (rows == 0 || w->k == 0) return CLQ_OK;
    if (!out) return fail(CLQ_ERR_ARGUMENT, "null output");
    clq::WeightView v = view_of(w, row_begin);
    cudaError_t e = clq::launch_dequantize(v, rows, out, transposed != 0, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "dequantize kernel launch");
    return CLQ_OK;
}

int clq_gather_device(const clq_store* w, const int32_t* ids, int64_t count, float* out, void* stream) {
    if (!w) return fail(CLQ_ERR_ARGUMENT, "null store");
    if (count < 0) return fail(CLQ_ERR_SHAPE, "negative id count");
    if (count == 0 || w->k == 0) return CLQ_OK;
    if (!ids || !out) return fail(CLQ_ERR_ARGUMENT, "null ids or output");
    cudaError_t e = clq::launch_gather(view_of(w, 0), ids, count, out, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "gather kernel launch");
    return CLQ_OK;
}

int clq_matmul(int dtype, float* out, const float* x, const uint8_t* bytes, int64_t m, int64_t n,
               int64_t k, unsigned flags) {
    int elems, bb, rc;
    if ((rc = check_shape(dtype, n, k, &elems, &bb))) return rc;
    if (m < 0) return fail(CLQ_ERR_SHAPE, "negative activation rows %lld", (long long)m);
    if (flags & ~(CLQ_MATH_FAST | CLQ_NO_CACHE | CLQ_MATH_EXACT)) return fail(CLQ_ERR_ARGUMENT, "unknown flags 0x%x", flags);
    if (m == 0 || n == 0) return CLQ_OK;
    if (!out || (k && (!x || !bytes))) return fail(CLQ_ERR_ARGUMENT, "null out, x or weight bytes");
    if (k == 0) {
        std::memset(out, 0, (size_t)(m * n) * sizeof(float));
        return CLQ_OK;
    }
    int device;
    if ((rc = current_device(&device))) return rc;
    ThreadContext* ctx;
    if ((rc = thread_context(device, &ctx))) return rc;
    std::shared_ptr<clq_store> store;
    int64_t row_begin = 0;
    const bool use_cache = !(flags & CLQ_NO_CACHE);
    ctx->sync_generation();
    const auto hit_key = std::make_tuple(bytes, n, k, dtype);
    const auto hit = use_cache ? ctx->hits.find(hit_key) : ctx->hits.end();
    if (hit != ctx->hits.end()) {
        store = hit->second.first;
        row_begin = hit->second.second;
    } else {
        if ((rc = cached_store(dtype, n, k, bytes, device, use_cache, ctx->stream, &store, &row_begin))) return rc;
        if (use_cache) ctx->hits[hit_key] = {store, row_begin};
    }
    const size_t xbytes = (size_t)(m * k) * sizeof(float), obytes = (size_t)(m * n) * sizeof(float);
    cudaError_t e;
    if ((e = ctx->x.ensure(xbytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc(x)");
    if ((e = ctx->out.ensure(obytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc(out)");
    // small products (decode): x goes through page-locked staging and the
    // kernel stores its outputs straight into mapped page-locked memory (no
    // copy back); large ones copy from and to the caller's memory
    const bool staged = xbytes + obytes <= ((size_t)8 << 20);
    if (staged) {
        if ((e = ctx->hx.ensure(xbytes)) != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(x)");
        if ((e = ctx->hout.ensure(obytes)) != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(out)");
        std::memcpy(ctx->hx.ptr, x, xbytes);
    }
    float* dout = staged ? (float*)ctx->hout.dptr : (float*)ctx->out.ptr;
    const unsigned lflags = flags & (CLQ_MATH_FAST | CLQ_MATH_EXACT);
    // staged: a copy kernel reads x from the mapped staging buffer, and the
    // linear's kernel, launched behind it, prefetches its weights meanwhile
    const bool copy_kernel = staged && xbytes % 16 == 0;
    auto enqueue = [&]() -> cudaError_t {
        cudaError_t r = copy_kernel ? clq::launch_copy_in(ctx->x.ptr, ctx->hx.dptr, xbytes, ctx->stream)
                                    : cudaMemcpyAsync(ctx->x.ptr, staged ? ctx->hx.ptr : x, xbytes,
                                                      cudaMemcpyHostToDevice, ctx->stream);
        if (r != cudaSuccess) return r;
        return clq::launch_linear(view_of(store.get(), row_begin), n, ctx->x.ptr, CLQ_X_F32, m, dout, n, lflags,
                                  ctx->stream);
    };
    // decode-sized calls on cached weights replay a graph of the same work
    cudaGraphExec_t exec = nullptr;
    if (copy_kernel && m <= 8 && use_cache) {
        // staging that moved (a larger call reallocated it) orphans every graph
        void* const bufs[3] = {ctx->x.ptr, ctx->hx.dptr, ctx->hout.dptr};
        if (bufs[0] != ctx->graph_buffers[0] || bufs[1] != ctx->graph_buffers[1] || bufs[2] != ctx->graph_buffers[2]) {
            for (auto& kv : ctx->graphs)
                if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
            ctx->graphs.clear();
            for (int i = 0; i < 3; i++) ctx->graph_buffers[i] = bufs[i];
        }
        const GraphKey key{store.get(), row_begin, n, k, m, lflags, ctx->x.ptr, ctx->hx.dptr, ctx->hout.dptr};
        auto it = ctx->graphs.find(key);
        if (it != ctx->graphs.end()) {
            exec = it->second.exec;
        } else if (cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const cudaError_t le = enqueue();
            cudaGraph_t graph = nullptr;
            const cudaError_t ce = cudaStreamEndCapture(ctx->stream, &graph);
            if (le == cudaSuccess && ce == cudaSuccess && graph &&
                cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
                ctx->graphs[key] = CallGraph{exec, store};
            } else {
                exec = nullptr;  // not capturable: this call runs eagerly
            }
            if (graph) cudaGraphDestroy(graph);
            cudaGetLastError();
        } else {
            cudaGetLastError();
        }
    }
    e = exec ? cudaGraphLaunch(exec, ctx->stream) : enqueue();
    if (e != cudaSuccess) return cuda_fail(e, "linear kernel launch");
    if (!staged && (e = cudaMemcpyAsync(out, ctx->out.ptr, obytes, cudaMemcpyDeviceToHost, ctx->stream)) !=
                       cudaSuccess)
        return cuda_fail(e, "copy out to host");
    if ((e = cudaStreamSynchronize(ctx->stream)) != cudaSuccess) return cuda_fail(e, "linear");
    if (staged) std::memcpy(out, ctx->hout.ptr, obytes);
    return CLQ_OK;
}

int clq_q8_0_matmul(float* out, const float* x, const uint8_t* bytes, int64_t m, int64_t n, int64_t k) {
    return clq_matmul(CLQ_Q8_0, out, x, bytes, m, n, k, 0);
}
int clq_q4_0_matmul(float* out, const float* x, const uint8_t* bytes, int64_t m, int64_t n, int64_t k) {
    return clq_matmul(CLQ_Q4_0, out, x, bytes, m, n, k, 0);
}
int clq_q4_k_matmul(float* out, const float* x, const uint8_t* bytes, int64_t m, int64_t n, int64_t k) {
    return clq_matmul(CLQ_Q4_K, out, x, bytes, m, n, k, 0);
}
int clq_q6_k_matmul(float* out, const float* x, const uint8_t* bytes, int64_t m, int64_t n, int64_t k) {
    return clq_matmul(CLQ_Q6_K, out, x, bytes, m, n, k, 0);
}

int clq_forget(const uint8_t* bytes, size_t nbytes) {
    std::vector<std::shared_ptr<clq_store>> dropped;  // freed outside the lock
    {
        std::lock_guard<std::mutex> lock(g_cache_mu);
        for (size_t i = 0; i < g_cache.size();) {
            const CacheEntry& e = g_cache[i];
            bool overlap = e.host < bytes + nbytes && bytes < e.host + e.nbytes;
            if (overlap) {
                dropped.push_back(e.store);
                g_cache.erase(g_cache.begin() + i);
                g_cache_generation.fetch_add(1);
            } else {
                i++;
            }
        }
    }
    return CLQ_OK;
}

int clq_clear_cache(void) {
    std::vector<CacheEntry> dropped;
    {
        std::lock_guard<std::mutex> lock(g_cache_mu);
        dropped.swap(g_cache);
        g_cache_generation.fetch_add(1);
    }
    return CLQ_OK;
}

int clq_cache_stats(int64_t* count, int64_t* device_bytes) {
    std::lock_guard<std::mutex> lock(g_cache_mu);
    int64_t bytes = 0;
    for (const CacheEntry& e : g_cache) bytes += (int64_t)e.store->nbytes;
    if (count) *count = (int64_t)g_cache.size();
    if (device_bytes) *device_bytes = bytes;
    return CLQ_OK;
}

int clq_dequantize(int dtype, const uint8_t* bytes, size_t nbytes, float* out) {
    int elems, bb, rc;
    if (!clq::geometry(dtype, &elems, &bb)) return fail(CLQ_ERR_ARGUMENT, "unknown packed dtype %d", dtype);
    if (nbytes % (size_t)bb)
        return fail(CLQ_ERR_BLOCKS, "%s data of %zu bytes is not a whole number of %d-byte blocks",
                    dtype_name(dtype), nbytes, bb);
    const int64_t nblocks = (int64_t)(nbytes / bb);
    if (nblocks == 0) return CLQ_OK;
    if (!bytes || !out) return fail(CLQ_ERR_ARGUMENT, "null bytes or output");
    int device;
    if ((rc = current_device(&device))) return rc;
    ThreadContext* ctx;
    if ((rc = thread_context(device, &ctx))) return rc;
    clq_store* raw = nullptr;
    // One row of nblocks blocks.
    if ((rc = make_store(dtype, 1, nblocks * elems, bytes, false, nbytes, ctx->stream, &raw))) return rc;
    std::unique_ptr<clq_store, void (*)(clq_store*)> s(raw, destroy_store);
    const size_t obytes = (size_t)(nblocks * elems) * sizeof(float);
    cudaError_t e;
    if ((e = ctx->out.ensure(obytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc(out)");
    if ((e = clq::launch_dequantize(view_of(s.get(), 0), 1, (float*)ctx->out.ptr, false, ctx->stream)) !=
        cudaSuccess)
        return cuda_fail(e, "dequantize kernel launch");
    if ((e = cudaMemcpyAsync(out, ctx->out.ptr, obytes, cudaMemcpyDeviceToHost, ctx->stream)) != cudaSuccess)
        return cuda_fail(e, "copy out to host");
    if ((e = cudaStreamSynchronize(ctx->stream)) != cudaSuccess) return cuda_fail(e, "dequantize");
    return CLQ_OK;
}

int clq_take(int dtype, const uint8_t* bytes, int64_t n, int64_t k, const int32_t* ids, int64_t count,
             float* out) {
    int elems, bb, rc;
    if ((rc = check_shape(dtype, n, k, &elems, &bb))) return rc;
    if (count < 0) return fail(CLQ_ERR_SHAPE, "negative id count");
    for (int64_t i = 0; i < count; i++)
        if (ids[i] < 0 || ids[i] >= n)
            return fail(CLQ_ERR_ARGUMENT, "row id %d outside [0, %lld)", ids[i], (long long)n);
    if (count == 0 || k == 0) return CLQ_OK;
    if (!bytes || !out) return fail(CLQ_ERR_ARGUMENT, "null bytes or output");
    int device;
    if ((rc = current_device(&device))) return rc;
    ThreadContext* ctx;
    if ((rc = thread_context(device, &ctx))) return rc;
    std::shared_ptr<clq_store> store;
    int64_t row_begin = 0;
    if ((rc = cached_store(dtype, n, k, bytes, device, true, ctx->stream, &store, &row_begin))) return rc;
    const size_t ibytes = (size_t)count * sizeof(int32_t), obytes = (size_t)(count * k) * sizeof(float);
    cudaError_t e;
    if ((e = ctx->ids.ensure(ibytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc(ids)");
    if ((e = ctx->out.ensure(obytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc(out)");
    if ((e = cudaMemcpyAsync(ctx->ids.ptr, ids, ibytes, cudaMemcpyHostToDevice, ctx->stream)) != cudaSuccess)
        return cuda_fail(e, "copy ids to device");
    clq::WeightView v = view_of(store.get(), row_begin);
    v.rows = n;
    if ((e = clq::launch_gather(v, (const int32_t*)ctx->ids.ptr, count, (float*)ctx->out.ptr, ctx->stream)) !=
        cudaSuccess)
        return cuda_fail(e, "gather kernel launch");
    if ((e = cudaMemcpyAsync(out, ctx->out.ptr, obytes, cudaMemcpyDeviceToHost, ctx->stream)) != cudaSuccess)
        return cuda_fail(e, "copy out to host");
    if ((e = cudaStreamSynchronize(ctx->stream)) != cudaSuccess) return cuda_fail(e, "take");
    return CLQ_OK;
}

}  // extern "C"

// ---- prefill GEMM on a fixed, preallocated scratch buffer ------------------
//
// Some callers cannot allocate device memory when they call in: a process
// whose device memory is reserved up front by another framework's allocator
// (a call-time cudaMalloc could fail at an unpredictable moment), or a
// latency-bound loop that cannot afford the device-wide synchronization that
// cudaMalloc/cudaFree may imply.  clq_linear_device_noalloc runs the same
// tensor-core GEMM as clq_linear_device's prefill path, but stages its
// activations and split-K partials in this file-scope device array, which
// every GPU that loads the library holds until the process exits.

static __device__ __align__(256) uint8_t g_noalloc_scratch[CLQ_NOALLOC_SCRATCH_BYTES];

namespace {

// The device address of g_noalloc_scratch for the current device, looked up
// once per device with that device current (in host code the symbol is only a
// host-side stand-in, never a device address).
int noalloc_scratch(int device, uint8_t** out) {
    static std::mutex mu;
    static std::vector<uint8_t*> addr;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)addr.size() <= device) addr.resize(device + 1, nullptr);
    if (!addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
        addr[device] = (uint8_t*)p;
    }
    *out = addr[device];
    return CLQ_OK;
}

}  // namespace

extern "C" int clq_linear_device_noalloc(const clq_store* w, int64_t row_begin, int64_t rows, const void* x,
                                         int xtype, int64_t m, float* out, int64_t ldo, void* stream) {
    if (!w) return fail(CLQ_ERR_ARGUMENT, "null store");
    if (xtype != CLQ_X_F32 && xtype != CLQ_X_BF16 && xtype != CLQ_X_F16)
        return fail(CLQ_ERR_ARGUMENT, "unknown activation type %d", xtype);
    if (row_begin < 0 || rows < 0 || row_begin + rows > w->n || m < 0)
        return fail(CLQ_ERR_SHAPE, "rows [%lld, %lld) / m %lld outside a (%lld %lld) weight",
                    (long long)row_begin, (long long)(row_begin + rows), (long long)m,
                    (long long)w->n, (long long)w->k);
    if (ldo < rows) return fail(CLQ_ERR_SHAPE, "output stride %lld < rows %lld", (long long)ldo, (long long)rows);
    if (m == 0 || rows == 0) return CLQ_OK;
    if (!x || !out) return fail(CLQ_ERR_ARGUMENT, "null activation or output pointer");
    if (w->k % 256) return fail(CLQ_ERR_UNSUPPORTED, "row length %lld is not a multiple of 256", (long long)w->k);
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    if (device != w->device)
        return fail(CLQ_ERR_ARGUMENT, "store lives on device %d, current device is %d", w->device, device);
    const clq::GemmPlan g = clq::plan_gemm_tc_capped(w->dtype, rows, w->k, m, CLQ_NOALLOC_SCRATCH_BYTES);
    if (g.splits == 0)
        return fail(CLQ_ERR_SHAPE,
                    "%lld activation rows x %lld columns need %zu bytes of staging; the fixed buffer holds %u",
                    (long long)m, (long long)w->k, clq::gemm_tc_scratch_bytes(clq::plan_gemm_tc_capped(w->dtype, rows, w->k, m, (size_t)-1)),
                    (unsigned)CLQ_NOALLOC_SCRATCH_BYTES);
    uint8_t* scratch = nullptr;
    if ((rc = noalloc_scratch(device, &scratch))) return rc;
    cudaError_t e = clq::launch_gemm_tc(view_of(w, row_begin), rows, x, xtype, m, out, ldo, scratch, g,
                                        (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "prefill kernel launch");
    return CLQ_OK;
}

// ---- tensor-parallel groups: GEMV with the all-reduce over peer memory ------

struct clq_tp {
    clq::TpLink link;
    int device;
};

namespace {

size_t tp_recv_bytes(int world, int64_t cap) { return (size_t)2 * world * clq::kMaxTpCtas * cap * sizeof(uint2); }
constexpr size_t kTpFlagBytes = clq::kMaxTpCtas * sizeof(uint32_t);  // per-CTA call epochs

}  // namespace

extern "C" {

int clq_tp_buffers(int world, int64_t cap, void** recv, void** flags) {
    if (!recv || !flags) return fail(CLQ_ERR_ARGUMENT, "null result pointer");
    *recv = *flags = nullptr;
    if (world < 1 || world > clq::kMaxRanks) return fail(CLQ_ERR_ARGUMENT, "world %d outside 1..%d", world, clq::kMaxRanks);
    if (cap < 1) return fail(CLQ_ERR_ARGUMENT, "capacity %lld", (long long)cap);
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    cudaError_t e = cudaMalloc(recv, tp_recv_bytes(world, cap));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(tensor-parallel recv)");
    if ((e = cudaMalloc(flags, kTpFlagBytes)) != cudaSuccess) {
        cudaFree(*recv);
        *recv = nullptr;
        return cuda_fail(e, "cudaMalloc(tensor-parallel flags)");
    }
    if ((e = cudaMemset(*recv, 0, tp_recv_bytes(world, cap))) != cudaSuccess ||
        (e = cudaMemset(*flags, 0, kTpFlagBytes)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess) {
        cudaFree(*recv);
        cudaFree(*flags);
        *recv = *flags = nullptr;
        return cuda_fail(e, "clearing tensor-parallel buffers");
    }
    return CLQ_OK;
}

int clq_tp_buffers_free(void* recv, void* flags) {
    cudaError_t e = cudaSuccess;
    if (recv) e = cudaFree(recv);
    if (flags && e == cudaSuccess) e = cudaFree(flags);
    return e == cudaSuccess ? CLQ_OK : cuda_fail(e, "cudaFree(tensor-parallel buffers)");
}

int clq_ipc_handle(const void* dev_ptr, uint8_t* handle) {
    if (!dev_ptr || !handle) return fail(CLQ_ERR_ARGUMENT, "null pointer");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == 64, "IPC handles are 64 bytes");
    std::memcpy(handle, &h, sizeof h);
    return CLQ_OK;
}

int clq_ipc_open(const uint8_t* handle, void** dev_ptr) {
    if (!dev_ptr || !handle) return fail(CLQ_ERR_ARGUMENT, "null pointer");
    *dev_ptr = nullptr;
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    return CLQ_OK;
}

int clq_ipc_close(void* dev_ptr) {
    if (!dev_ptr) return CLQ_OK;
    cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    return e == cudaSuccess ? CLQ_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int clq_tp_create(int rank, int world, int64_t cap, void* const* recv, void* const* flags, clq_tp** out) {
    if (!out || !recv || !flags) return fail(CLQ_ERR_ARGUMENT, "null pointer");
    *out = nullptr;
    if (world < 1 || world > clq::kMaxRanks || rank < 0 || rank >= world)
        return fail(CLQ_ERR_ARGUMENT, "rank %d of world %d (1..%d ranks)", rank, world, clq::kMaxRanks);
    if (cap < 1) return fail(CLQ_ERR_ARGUMENT, "capacity %lld", (long long)cap);
    for (int r = 0; r < world; r++)
        if (!recv[r] || !flags[r]) return fail(CLQ_ERR_ARGUMENT, "null buffer of rank %d", r);
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    clq_tp* t = new (std::nothrow) clq_tp();
    if (!t) return fail(CLQ_ERR_OUT_OF_MEMORY, "tensor-parallel group");
    t->device = device;
    clq::TpLink& L = t->link;
    L.rank = rank;
    L.world = world;
    L.cap = cap;
    for (int r = 0; r < world; r++) L.peer_recv[r] = static_cast<uint2*>(recv[r]);
    L.my_recv = L.peer_recv[rank];
    L.epochs = static_cast<uint32_t*>(flags[rank]);
    // polls of one peer word before a wait gives up (about 1 us each under
    // load, so seconds); CLQ_TP_WAIT_POLLS lowers it for tests that make the
    // wait run out on purpose
    L.wait_polls = 1u << 22;
    if (const char* e = getenv("CLQ_TP_WAIT_POLLS")) {
        const long long v = atoll(e);
        if (v >= 1 && v <= (1ll << 30)) L.wait_polls = (uint32_t)v;
    }
    *out = t;
    return CLQ_OK;
}

int clq_tp_free(clq_tp* tp) {
    delete tp;
    return CLQ_OK;
}

int clq_linear_allreduce_device(const clq_store* w, int64_t row_begin, int64_t rows, const void* x, int xtype,
                                int64_t m, float* out, int64_t ldo, clq_tp* tp, void* stream) {
    if (!w || !tp) return fail(CLQ_ERR_ARGUMENT, "null store or group");
    if (xtype != CLQ_X_F32 && xtype != CLQ_X_BF16 && xtype != CLQ_X_F16)
        return fail(CLQ_ERR_ARGUMENT, "unknown activation type %d", xtype);
    if (row_begin < 0 || rows < 1 || row_begin + rows > w->n || m < 1 || ldo < rows)
        return fail(CLQ_ERR_SHAPE, "rows [%lld, %lld), m %lld, ldo %lld for a (%lld %lld) weight", (long long)row_begin,
                    (long long)(row_begin + rows), (long long)m, (long long)ldo, (long long)w->n, (long long)w->k);
    if (!x || !out) return fail(CLQ_ERR_ARGUMENT, "null activation or output pointer");
    int device, rc;
    if ((rc = current_device(&device))) return rc;
    if (device != w->device || device != tp->device)
        return fail(CLQ_ERR_ARGUMENT, "store, group and current device differ");
    cudaError_t e = clq::launch_gemv_bulk_allreduce(view_of(w, row_begin), rows, x, xtype, m, out, ldo, tp->link,
                                                    (cudaStream_t)stream);
    if (e == cudaErrorNotSupported)
        return fail(CLQ_ERR_UNSUPPORTED,
                    "the fused all-reduce GEMV takes Q4_K / Q6_K, K %% 256 == 0, m <= 8, and at most CAP outputs per SM");
    if (e != cudaSuccess) return cuda_fail(e, "all-reduce linear kernel launch");
    return CLQ_OK;
}

}  // extern "C"
