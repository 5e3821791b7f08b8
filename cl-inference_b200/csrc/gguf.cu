// gguf.cu -- GGUF v3 files: a read-only mapping, the header parse with the
// reference reader's checks (gguf/reader.lisp), and the loader that streams a
// quantized tensor from the mapping into a device store.
//
// The parse follows parse-gguf (gguf/reader.lisp:167-196): magic and version,
// u64 counts bounded by the bytes left, UTF-8 strings, metadata values of
// types 0..12 nested at most 32 deep, booleans 0 or 1, no duplicate keys or
// tensor names, tensor ranks 1..4 of positive dimensions, known ggml types,
// rows (the first dimension) of whole blocks, general.alignment a power of two
// of at most 4096 (default 32), and tensors at aligned offsets that neither
// overlap nor run past the end of the file (validate-layout, :152-165).
//
// The loader (clq_gguf_store) never makes a pageable copy of a whole tensor:
// the bytes are read (pread, no faults on the mapping) into two page-locked
// staging buffers in turn while the previous chunk's asynchronous copy to the
// device runs, then the
// device bytes are checked for non-finite scales and re-tiled exactly as
// clq_store_create does (the load-time scan of mlx/gguf/weights.lisp:19-23).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/clq.h"
#include "clq_internal.h"

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF"
constexpr int kMaxDepth = 32;
constexpr uint64_t kDefaultAlignment = 32, kMaxAlignment = 4096;
constexpr uint64_t kMaxDim = (1ull << 62) - 1;  // the reference's fixnum bound on a dimension
constexpr size_t kChunk = (size_t)16 << 20;     // staging buffer size

// ggml type id -> (elements per block, bytes per block): the file format's
// table (gguf/reader.lisp:35-47); ids not listed are rejected.
struct TypeGeo {
    int id, block, bytes;
};
constexpr TypeGeo kTypes[] = {
    {0, 1, 4},      {1, 1, 2},      {2, 32, 18},    {3, 32, 20},    {6, 32, 22},    {7, 32, 24},
    {8, 32, 34},    {9, 32, 36},    {10, 256, 84},  {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
    {14, 256, 210}, {15, 256, 292}, {16, 256, 66},  {17, 256, 74},  {18, 256, 98},  {19, 256, 50},
    {20, 32, 18},   {21, 256, 110}, {22, 256, 82},  {23, 256, 136}, {24, 1, 1},     {25, 1, 2},
    {26, 1, 4},     {27, 1, 8},     {28, 1, 8},     {29, 256, 56},  {30, 1, 2},     {34, 256, 54},
    {35, 256, 66},  {39, 32, 17},   {40, 64, 36},   {41, 128, 18},  {42, 64, 18},
};

const TypeGeo* find_type(uint32_t id) {
    for (const TypeGeo& t : kTypes)
        if ((uint32_t)t.id == id) return &t;
    return nullptr;
}

struct Value {
    int type = 0;
    uint64_t u = 0;  // unsigned integers and bools
    int64_t i = 0;   // signed integers
    double f = 0.0;  // floats
    std::string s;   // strings
    int elem = -1;   // arrays: element type and count
    uint64_t count = 0;
};

struct Tensor {
    std::string name;
    int type = 0, rank = 0;
    int64_t dims[4] = {1, 1, 1, 1};
    uint64_t offset = 0, nbytes = 0;
};

template <typename... A>
int format_error(const char* fmt, A... args) {
    return clq::set_error(CLQ_ERR_FORMAT, fmt, args...);
}

struct Cursor {
    const uint8_t* base;
    uint64_t limit, pos;
};

// Reserves N bytes; their start in *at.
int advance(Cursor& c, uint64_t n, const char* what, uint64_t* at) {
    if (n > c.limit - c.pos)
        return format_error("Truncated GGUF: %s needs %llu bytes at offset %llu", what, (unsigned long long)n,
                            (unsigned long long)c.pos);
    *at = c.pos;
    c.pos += n;
    return CLQ_OK;
}

template <typename T>
int scalar(Cursor& c, const char* what, T* v) {
    uint64_t at = 0;
    int rc = advance(c, sizeof(T), what, &at);
    if (rc) return rc;
    std::memcpy(v, c.base + at, sizeof(T));  // the format is little-endian, as is this host
    return CLQ_OK;
}

// A u64 count that cannot exceed the bytes left: every item takes at least one.
int count(Cursor& c, const char* what, uint64_t* v) {
    int rc = scalar(c, what, v);
    if (rc) return rc;
    if (*v > c.limit - c.pos)
        return format_error("%s %llu exceeds the remaining file", what, (unsigned long long)*v);
    return CLQ_OK;
}

// Strict UTF-8: no overlong forms, surrogates or code points above U+10FFFF.
bool valid_utf8(const uint8_t* p, uint64_t n) {
    uint64_t i = 0;
    while (i < n) {
        const uint8_t b = p[i];
        int len;
        uint32_t cp;
        if (b < 0x80) {
            i++;
            continue;
        } else if ((b & 0xE0) == 0xC0) {
            len = 2; cp = b & 0x1F;
        } else if ((b & 0xF0) == 0xE0) {
            len = 3; cp = b & 0x0F;
        } else if ((b & 0xF8) == 0xF0) {
            len = 4; cp = b & 0x07;
        } else {
            return false;
        }
        if (n - i < (uint64_t)len) return false;
        for (int j = 1; j < len; j++) {
            if ((p[i + j] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (p[i + j] & 0x3F);
        }
        if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000)) return false;
        if (cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
        i += len;
    }
    return true;
}

int string(Cursor& c, std::string* s) {
    uint64_t n = 0, at = 0;
    int rc = count(c, "String length", &n);
    if (rc) return rc;
    if ((rc = advance(c, n, "string", &at))) return rc;
    if (!valid_utf8(c.base + at, n)) return format_error("Invalid UTF-8 string");
    s->assign(reinterpret_cast<const char*>(c.base + at), n);
    return CLQ_OK;
}

int value(Cursor& c, uint32_t type, int depth, Value* v) {
    if (depth > kMaxDepth) return format_error("Metadata nesting exceeds %d levels", kMaxDepth);
    v->type = (int)type;
    int rc = CLQ_OK;
    switch (type) {
    case 0: { uint8_t x = 0; rc = scalar(c, "u8", &x); v->u = x; break; }
    case 1: { int8_t x = 0; rc = scalar(c, "i8", &x); v->i = x; break; }
    case 2: { uint16_t x = 0; rc = scalar(c, "u16", &x); v->u = x; break; }
    case 3: { int16_t x = 0; rc = scalar(c, "i16", &x); v->i = x; break; }
    case 4: { uint32_t x = 0; rc = scalar(c, "u32", &x); v->u = x; break; }
    case 5: { int32_t x = 0; rc = scalar(c, "i32", &x); v->i = x; break; }
    case 6: { float x = 0; rc = scalar(c, "f32", &x); v->f = x; break; }
    case 7: {
        uint8_t x = 0;
        if ((rc = scalar(c, "bool", &x))) break;
        if (x > 1) return format_error("Invalid boolean");
        v->u = x;
        break;
    }
    case 8: rc = string(c, &v->s); break;
    case 9: {
        uint32_t et = 0;
        if ((rc = scalar(c, "array type", &et))) break;
        if (et > 12) return format_error("Unknown metadata type %u", et);
        uint64_t n = 0;
        if ((rc = count(c, "Array length", &n))) break;
        v->elem = (int)et;
        v->count = n;
        Value item;
        for (uint64_t j = 0; j < n && !rc; j++) rc = value(c, et, depth + 1, &item);
        break;
    }
    case 10: { uint64_t x = 0; rc = scalar(c, "u64", &x); v->u = x; break; }
    case 11: { int64_t x = 0; rc = scalar(c, "i64", &x); v->i = x; break; }
    case 12: { double x = 0; rc = scalar(c, "f64", &x); v->f = x; break; }
    default: return format_error("Unknown metadata type %u", type);
    }
    return rc;
}

bool is_integer(int type) { return type <= 5 || type == 10 || type == 11; }

}  // namespace

struct clq_gguf {
    int fd = -1;
    uint8_t* base = nullptr;
    size_t size = 0;
    uint64_t data_start = 0, alignment = kDefaultAlignment;
    std::vector<std::string> keys;
    std::unordered_map<std::string, Value> meta;
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, int64_t> index;
    // upload staging, made on the first clq_gguf_store
    void* stage[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    cudaStream_t stream = nullptr;
    int stage_device = -1;
    ~clq_gguf() {
        for (int i = 0; i < 2; i++) {
            if (stage[i]) cudaFreeHost(stage[i]);
            if (done[i]) cudaEventDestroy(done[i]);
        }
        if (stream) cudaStreamDestroy(stream);
        if (base) munmap(base, size);
        if (fd >= 0) close(fd);
    }
};

namespace {

int parse(clq_gguf* g) {
    Cursor c{g->base, g->size, 0};
    uint32_t magic, version;
    int rc;
    if ((rc = scalar(c, "magic", &magic))) return rc;
    if (magic != kMagic) return format_error("Invalid GGUF magic");
    if ((rc = scalar(c, "version", &version))) return rc;
    if (version != 3) return format_error("Only little-endian GGUF v3 is supported");
    uint64_t ntensors, nmeta;
    if ((rc = count(c, "Tensor count", &ntensors))) return rc;
    if ((rc = count(c, "Metadata count", &nmeta))) return rc;
    for (uint64_t j = 0; j < nmeta; j++) {
        std::string key;
        if ((rc = string(c, &key))) return rc;
        if (g->meta.count(key)) return format_error("Duplicate metadata key %s", key.c_str());
        uint32_t type;
        if ((rc = scalar(c, "value type", &type))) return rc;
        Value v;
        if ((rc = value(c, type, 0, &v))) return rc;
        g->meta.emplace(key, std::move(v));
        g->keys.push_back(key);
    }
    for (uint64_t j = 0; j < ntensors; j++) {
        Tensor t;
        if ((rc = string(c, &t.name))) return rc;
        uint32_t rank;
        if ((rc = scalar(c, "tensor rank", &rank))) return rc;
        if (rank < 1 || rank > 4) return format_error("Invalid rank %u for tensor %s", rank, t.name.c_str());
        t.rank = (int)rank;
        unsigned __int128 elements = 1;
        for (uint32_t d = 0; d < rank; d++) {
            uint64_t dim;
            if ((rc = scalar(c, "tensor dimension", &dim))) return rc;
            if (dim < 1 || dim > kMaxDim)
                return format_error("Invalid dimension %llu for tensor %s", (unsigned long long)dim, t.name.c_str());
            t.dims[d] = (int64_t)dim;
            elements *= dim;
        }
        uint32_t type;
        if ((rc = scalar(c, "tensor type", &type))) return rc;
        if ((rc = scalar(c, "tensor offset", &t.offset))) return rc;
        const TypeGeo* geo = find_type(type);
        if (!geo) return format_error("Unsupported ggml type %u for tensor %s", type, t.name.c_str());
        if (t.dims[0] % geo->block)
            return format_error("Tensor %s row length %llu is not a multiple of %llu", t.name.c_str(),
                                (unsigned long long)t.dims[0], (unsigned long long)geo->block);
        const unsigned __int128 bytes = elements / (unsigned)geo->block * (unsigned)geo->bytes;
        if (bytes > (unsigned __int128)UINT64_MAX / 2) return format_error("Tensor %s is too large", t.name.c_str());
        t.type = (int)type;
        t.nbytes = (uint64_t)bytes;
        if (g->index.count(t.name)) return format_error("Duplicate tensor %s", t.name.c_str());
        g->index.emplace(t.name, (int64_t)g->tensors.size());
        g->tensors.push_back(std::move(t));
    }
    auto al = g->meta.find("general.alignment");
    if (al != g->meta.end()) {
        const Value& v = al->second;
        const bool neg = (v.type == 1 || v.type == 3 || v.type == 5 || v.type == 11) && v.i < 0;
        const uint64_t a = (v.type == 1 || v.type == 3 || v.type == 5 || v.type == 11) ? (uint64_t)v.i : v.u;
        if (!is_integer(v.type) || neg || a < 1 || a > kMaxAlignment || (a & (a - 1)))
            return format_error("Invalid tensor alignment");
        g->alignment = a;
    }
    g->data_start = (c.pos + g->alignment - 1) / g->alignment * g->alignment;
    if (!g->tensors.empty() && g->data_start > g->size) return format_error("Missing tensor data section");
    std::vector<const Tensor*> order;
    for (const Tensor& t : g->tensors) order.push_back(&t);
    std::sort(order.begin(), order.end(), [](const Tensor* a, const Tensor* b) { return a->offset < b->offset; });
    uint64_t end = 0;
    for (const Tensor* t : order) {
        if (t->offset % g->alignment)
            return format_error("Tensor %s offset %llu is not aligned to %llu", t->name.c_str(),
                                (unsigned long long)t->offset, (unsigned long long)g->alignment);
        if (t->offset < end) return format_error("Tensor %s overlaps another tensor", t->name.c_str());
        // compared without sums that could wrap: data_start <= size holds here
        const uint64_t room = g->size - g->data_start;
        if (t->offset > room || t->nbytes > room - t->offset)
            return format_error("Tensor %s extends past the end of the file", t->name.c_str());
        end = t->offset + t->nbytes;
    }
    return CLQ_OK;
}

// The store dtype of a ggml type (the ids coincide), or -1.
int store_dtype(int ggml_type) {
    switch (ggml_type) {
    case CLQ_Q4_0: case CLQ_Q8_0: case CLQ_Q4_K: case CLQ_Q6_K: return ggml_type;
    default: return -1;
    }
}

}  // namespace

extern "C" {

int clq_gguf_open(const char* path, clq_gguf** out) {
    if (!path || !out) return clq::set_error(CLQ_ERR_ARGUMENT, "null path or result pointer");
    *out = nullptr;
    std::unique_ptr<clq_gguf> g(new clq_gguf);
    g->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (g->fd < 0) return clq::set_error(CLQ_ERR_IO, "cannot open %s: %s", path, std::strerror(errno));
    struct stat st;
    if (fstat(g->fd, &st) != 0) return clq::set_error(CLQ_ERR_IO, "cannot stat %s: %s", path, std::strerror(errno));
    g->size = (size_t)st.st_size;
    // the header's fixed part: magic, version, tensor count, metadata count
    if (g->size < 24) return format_error("Truncated GGUF: %s has %llu bytes", path, (unsigned long long)g->size);
    void* p = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (p == MAP_FAILED) return clq::set_error(CLQ_ERR_IO, "cannot map %s: %s", path, std::strerror(errno));
    g->base = static_cast<uint8_t*>(p);
    const int rc = parse(g.get());
    if (rc) return rc;
    *out = g.release();
    return CLQ_OK;
}

int clq_gguf_close(clq_gguf* file) {
    delete file;
    return CLQ_OK;
}

int clq_gguf_tensor_count(const clq_gguf* file, int64_t* count) {
    if (!file || !count) return clq::set_error(CLQ_ERR_ARGUMENT, "null file or result pointer");
    *count = (int64_t)file->tensors.size();
    return CLQ_OK;
}

int clq_gguf_tensor_info(const clq_gguf* file, int64_t index, const char** name, int* ggml_type, int* rank,
                         int64_t dims[4], uint64_t* offset, uint64_t* nbytes, const uint8_t** bytes) {
    if (!file) return clq::set_error(CLQ_ERR_ARGUMENT, "null file");
    if (index < 0 || index >= (int64_t)file->tensors.size())
        return clq::set_error(CLQ_ERR_ARGUMENT, "tensor index %lld out of range", (long long)index);
    const Tensor& t = file->tensors[(size_t)index];
    if (name) *name = t.name.c_str();
    if (ggml_type) *ggml_type = t.type;
    if (rank) *rank = t.rank;
    if (dims)
        for (int d = 0; d < 4; d++) dims[d] = t.dims[d];
    if (offset) *offset = t.offset;
    if (nbytes) *nbytes = t.nbytes;
    if (bytes) *bytes = file->base + file->data_start + t.offset;
    return CLQ_OK;
}

int clq_gguf_find_tensor(const clq_gguf* file, const char* name, int64_t* index) {
    if (!file || !name || !index) return clq::set_error(CLQ_ERR_ARGUMENT, "null argument");
    auto it = file->index.find(name);
    if (it == file->index.end()) return clq::set_error(CLQ_ERR_ARGUMENT, "no tensor named %s", name);
    *index = it->second;
    return CLQ_OK;
}

int clq_gguf_metadata_count(const clq_gguf* file, int64_t* count) {
    if (!file || !count) return clq::set_error(CLQ_ERR_ARGUMENT, "null file or result pointer");
    *count = (int64_t)file->keys.size();
    return CLQ_OK;
}

int clq_gguf_metadata_key(const clq_gguf* file, int64_t index, const char** key, int* type) {
    if (!file) return clq::set_error(CLQ_ERR_ARGUMENT, "null file");
    if (index < 0 || index >= (int64_t)file->keys.size())
        return clq::set_error(CLQ_ERR_ARGUMENT, "metadata index %lld out of range", (long long)index);
    const std::string& k = file->keys[(size_t)index];
    if (key) *key = k.c_str();
    if (type) *type = file->meta.at(k).type;
    return CLQ_OK;
}

int clq_gguf_metadata_value(const clq_gguf* file, const char* key, int* type, uint64_t* uvalue, int64_t* ivalue,
                            double* fvalue, const char** svalue, uint64_t* slen, int* elem_type, uint64_t* count) {
    if (!file || !key) return clq::set_error(CLQ_ERR_ARGUMENT, "null file or key");
    auto it = file->meta.find(key);
    if (it == file->meta.end()) return clq::set_error(CLQ_ERR_ARGUMENT, "no metadata key %s", key);
    const Value& v = it->second;
    if (type) *type = v.type;
    if (uvalue) *uvalue = v.u;
    if (ivalue) *ivalue = v.i;
    if (fvalue) *fvalue = v.f;
    if (svalue) *svalue = v.s.c_str();
    if (slen) *slen = v.s.size();
    if (elem_type) *elem_type = v.elem;
    if (count) *count = v.count;
    return CLQ_OK;
}

int clq_gguf_store(clq_gguf* file, int64_t index, clq_store** out) {
    if (!file || !out) return clq::set_error(CLQ_ERR_ARGUMENT, "null file or result pointer");
    *out = nullptr;
    if (index < 0 || index >= (int64_t)file->tensors.size())
        return clq::set_error(CLQ_ERR_ARGUMENT, "tensor index %lld out of range", (long long)index);
    const Tensor& t = file->tensors[(size_t)index];
    const int dtype = store_dtype(t.type);
    if (dtype < 0)
        return clq::set_error(CLQ_ERR_UNSUPPORTED, "tensor %s has ggml type %d; stores take Q4_0, Q8_0, Q4_K, Q6_K",
                              t.name.c_str(), t.type);
    const int64_t k = t.dims[0], n = t.dims[1] * t.dims[2] * t.dims[3];
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return clq::set_error(CLQ_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
    if (file->stage_device != device) {
        // staging belongs to one device: remake it when the current device changed
        for (int i = 0; i < 2; i++) {
            if (file->stage[i]) cudaFreeHost(file->stage[i]);
            if (file->done[i]) cudaEventDestroy(file->done[i]);
            file->stage[i] = nullptr;
            file->done[i] = nullptr;
        }
        if (file->stream) cudaStreamDestroy(file->stream);
        file->stream = nullptr;
        file->stage_device = -1;
        if ((e = cudaStreamCreateWithFlags(&file->stream, cudaStreamNonBlocking)) != cudaSuccess)
            return clq::set_error(CLQ_ERR_CUDA, "cudaStreamCreate: %s", cudaGetErrorString(e));
        for (int i = 0; i < 2; i++) {
            if ((e = cudaMallocHost(&file->stage[i], kChunk)) != cudaSuccess ||
                (e = cudaEventCreateWithFlags(&file->done[i], cudaEventDisableTiming)) != cudaSuccess)
                return clq::set_error(e == cudaErrorMemoryAllocation ? CLQ_ERR_OUT_OF_MEMORY : CLQ_ERR_CUDA,
                                      "upload staging: %s", cudaGetErrorString(e));
        }
        file->stage_device = device;
    }
    uint8_t* native = nullptr;
    if ((e = cudaMalloc((void**)&native, t.nbytes ? t.nbytes : 1)) != cudaSuccess)
        return clq::set_error(e == cudaErrorMemoryAllocation ? CLQ_ERR_OUT_OF_MEMORY : CLQ_ERR_CUDA,
                              "device copy of %s: %s", t.name.c_str(), cudaGetErrorString(e));
    int rc = CLQ_OK;
    for (uint64_t off = 0, i = 0; off < t.nbytes && !rc; off += kChunk, i++) {
        const size_t len = (size_t)std::min<uint64_t>(kChunk, t.nbytes - off);
        const int slot = (int)(i & 1);
        // the copy that last read this buffer must be done before it is refilled
        if (i >= 2 && (e = cudaEventSynchronize(file->done[slot])) != cudaSuccess) break;
        // pread copies from the page cache straight into the staging buffer:
        // no page faults on the mapping (one per 4 KB page)
        size_t got = 0;
        while (got < len) {
            const ssize_t r = pread(file->fd, (uint8_t*)file->stage[slot] + got, len - got,
                                    (off_t)(file->data_start + t.offset + off + got));
            if (r <= 0) break;
            got += (size_t)r;
        }
        if (got < len) {
            rc = clq::set_error(CLQ_ERR_IO, "reading %s: %s", t.name.c_str(), std::strerror(errno));
            break;
        }
        if ((e = cudaMemcpyAsync(native + off, file->stage[slot], len, cudaMemcpyHostToDevice, file->stream)) !=
                cudaSuccess ||
            (e = cudaEventRecord(file->done[slot], file->stream)) != cudaSuccess)
            break;
    }
    if (rc == CLQ_OK) {
        if (e == cudaSuccess) rc = clq_store_create_device(dtype, n, k, native, t.nbytes, CLQ_STORE_DEFAULT, file->stream, out);
        else rc = clq::set_error(CLQ_ERR_CUDA, "uploading %s: %s", t.name.c_str(), cudaGetErrorString(e));
    }
    cudaStreamSynchronize(file->stream);
    cudaFree(native);
    return rc;
}

}  // extern "C"
