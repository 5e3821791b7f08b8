/*
 * clq.h -- C ABI of libclq, the B200 (sm_100a) quantized-linear library for
 * cl-inference's packed GGUF weights (Q8_0, Q4_0, Q4_K, Q6_K).
 *
 * Plain pointers and sizes only; no CUDA or torch types.  A `stream` argument
 * is a cudaStream_t passed as void* (NULL = the library's per-thread stream for
 * host-pointer calls, the legacy default stream for device-pointer calls).
 *
 * Every function returns 0 (CLQ_OK) or a CLQ_ERR_* code; clq_last_error() gives
 * the calling thread's message for its most recent failure.  Reference paths
 * cited below are relative to the cl-inference project.
 */
#ifndef CLQ_H
#define CLQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CLQ_ABI_VERSION 1

/* Packed dtypes, numbered by their ggml type id (gguf/reader.lisp:37-52). */
enum clq_dtype {
    CLQ_Q4_0 = 2,  /*  32 elements,  18 bytes: quant/packed.lisp:156 */
    CLQ_Q8_0 = 8,  /*  32 elements,  34 bytes: quant/q8-0.lisp:5-6   */
    CLQ_Q4_K = 12, /* 256 elements, 144 bytes: quant/packed.lisp:157 */
    CLQ_Q6_K = 14  /* 256 elements, 210 bytes: quant/packed.lisp:158 */
};

/* Activation element types for the device-pointer products. */
enum clq_xtype { CLQ_X_F32 = 0, CLQ_X_BF16 = 1, CLQ_X_F16 = 2 };

enum clq_status {
    CLQ_OK = 0,
    CLQ_ERR_ARGUMENT = 1,       /* null pointer, unknown dtype, bad flag            */
    CLQ_ERR_SHAPE = 2,          /* shape mismatch; K not a multiple of the block    */
    CLQ_ERR_BLOCKS = 3,         /* byte count is not a whole number of blocks       */
    CLQ_ERR_NONFINITE_SCALE = 4,/* an fp16 scale has exponent 31 (quant/q8-0.lisp:95) */
    CLQ_ERR_CUDA = 5,           /* a CUDA runtime call failed                        */
    CLQ_ERR_NCCL = 6,           /* a collective failed                               */
    CLQ_ERR_TIMEOUT = 7,        /* a bounded wait ran out                            */
    CLQ_ERR_NO_DEVICE = 8,      /* no usable sm_100 device                           */
    CLQ_ERR_UNSUPPORTED = 9,    /* valid request this build does not implement       */
    CLQ_ERR_OUT_OF_MEMORY = 10,
    CLQ_ERR_FORMAT = 11,        /* malformed GGUF file (gguf/reader.lisp's gguf-error) */
    CLQ_ERR_IO = 12,            /* a file could not be opened or mapped              */
    CLQ_ERR_NONFINITE_VALUE = 13, /* a non-finite key or value into a Q8 cache
                                     (local/kv-cache.lisp:49, "Non-finite key or value") */
    CLQ_ERR_CONTEXT = 14        /* positions past the cache's context
                                   (local/kv-cache.lisp:94-96, context-overflow)      */
};

/* Store creation flags. */
#define CLQ_STORE_DEFAULT 0u

/* Product flags. */
#define CLQ_MATH_DEFAULT 0u   /* fp32-class results for fp32 activations (from 17 rows of
                                 Q4_0 / Q8_0 and 25 of Q4_K / Q6_K the
                                 tcgen05 GEMM in its exact form: weights and activations as
                                 fp16 hi + lo parts, three MMAs per K step)             */
#define CLQ_MATH_FAST 1u      /* prefill GEMM may round dequantized weights to fp16  */
#define CLQ_NO_CACHE 2u       /* host-pointer calls: upload, use and drop the weight */
#define CLQ_MATH_EXACT 4u     /* prefill GEMM with fp32-class results for 16-bit activations too */

/* ---- library ------------------------------------------------------------- */

int clq_abi_version(void);
/* Copies the calling thread's last error message (NUL-terminated, truncated). */
int clq_last_error(char *buf, size_t len);
/* Elements and bytes per block of DTYPE. */
int clq_block_geometry(int dtype, int64_t *elements, int64_t *block_bytes);
/* No counterpart in the reference (its kernels run on the calling thread).
 * Waits for all work on the current device, then stores in *STATUS the code a
 * kernel recorded since the last call -- CLQ_OK, or CLQ_ERR_TIMEOUT when a
 * pipeline wait inside a kernel expired (that launch's outputs are invalid, and
 * launches that run while the code is set may stop early) -- and clears it. */
int clq_device_status(int *status);

/* ---- drop-in kernels ------------------------------------------------------
 * Same arguments and meaning as the trivial-simd kernels the packed dtypes
 * bind: (kernel out x bytes M N K), called from packed-matmul-executor
 * (quant/packed.lisp:68-75, slots registered at :156-158) and from the Q8_0
 * matmul-executor (quant/q8-0.lisp:87-94).
 *   out   host f32 [M, N] row-major, written
 *   x     host f32 [M, K] row-major, contiguous
 *   bytes host packed weight, N rows of K/elements blocks (row-major (N K)),
 *         beginning at the weight view's whole-row offset (packed.lisp:60-66)
 * The weight is uploaded to the current device once and cached by host
 * address range (the identity of a mapped GGUF view, gguf/weights.lisp:68-78);
 * a pointer inside a cached range at a whole-row offset reuses it.  Calls are
 * synchronous: `out` is valid on return.  M = 0 is a no-op.
 */
int clq_q8_0_matmul(float *out, const float *x, const uint8_t *bytes, int64_t m, int64_t n,
                    int64_t k);
int clq_q4_0_matmul(float *out, const float *x, const uint8_t *bytes, int64_t m, int64_t n,
                    int64_t k);
int clq_q4_k_matmul(float *out, const float *x, const uint8_t *bytes, int64_t m, int64_t n,
                    int64_t k);
int clq_q6_k_matmul(float *out, const float *x, const uint8_t *bytes, int64_t m, int64_t n,
                    int64_t k);
/* The four above with the dtype as an argument and CLQ_* flags. */
int clq_matmul(int dtype, float *out, const float *x, const uint8_t *bytes, int64_t m, int64_t n,
               int64_t k, unsigned flags);

/* Drop cached weights whose host range overlaps [bytes, bytes + nbytes):
 * call before the mapping is released (close-weights, local/weights.lisp:84-89). */
int clq_forget(const uint8_t *bytes, size_t nbytes);
/* Drop every cached weight on every device. */
int clq_clear_cache(void);
/* Number of cached weights and their device bytes. */
int clq_cache_stats(int64_t *count, int64_t *device_bytes);

/* ---- device-resident packed-weight store ----------------------------------
 * Uploads N x K packed blocks (native GGUF byte layout) once to the current
 * device, checks that every fp16 scale is finite (the load-time check of
 * mlx/gguf/weights.lisp:19-23), and re-tiles them on the device into aligned
 * planes; re-tiling only moves bytes, so every decoded value is unchanged.  The
 * store owns the device copy.
 */
typedef struct clq_store clq_store;

int clq_store_create(int dtype, int64_t n, int64_t k, const uint8_t *host_bytes, size_t nbytes,
                     unsigned flags, clq_store **out);
/* Same from bytes already on the current device (copied; DEVICE_BYTES may be freed after). */
int clq_store_create_device(int dtype, int64_t n, int64_t k, const void *device_bytes,
                            size_t nbytes, unsigned flags, void *stream, clq_store **out);
int clq_store_free(clq_store *store);
int clq_store_info(const clq_store *store, int *dtype, int64_t *n, int64_t *k, size_t *nbytes,
                   const void **device_bytes, int *device);

/* ---- device-pointer products (activations stay resident) ------------------
 * out[i, j] (j < rows) = sum_c x[i, c] * W[row_begin + j, c] for i < m, with
 * out row stride LDO floats (>= rows).  X is [m, K] contiguous of XTYPE.
 * Asynchronous on STREAM.  This is the linear of local/blocks.lisp:106-113 for a
 * packed weight, over a row range of it (a column-parallel shard when
 * row_begin/rows select a rank's rows).
 */
int clq_linear_device(const clq_store *w, int64_t row_begin, int64_t rows, const void *x,
                      int xtype, int64_t m, float *out, int64_t ldo, unsigned flags,
                      void *stream);

/* Up to 4 weights of one dtype and K that read the same activations X (the
 * q/k/v projections of attention, local/blocks.lisp:334-336, or the gate/up
 * pair of the SwiGLU MLP, :151-154) in one launch: member i computes
 * out[i][r, j] for rows [row_begin[i], row_begin[i] + rows[i]) of w[i]. */
int clq_linear_group_device(const clq_store *const *w, const int64_t *row_begin, const int64_t *rows,
                            int count, const void *x, int xtype, int64_t m, float *const *out,
                            const int64_t *ldo, unsigned flags, void *stream);

/* No counterpart in the reference.  For callers that cannot allocate device
 * memory at call time -- a process whose device memory another framework's
 * allocator reserved up front, where a call-time cudaMalloc could fail, or a
 * latency-bound loop that cannot take the device synchronization cudaMalloc
 * and cudaFree may imply.  Same product as clq_linear_device's prefill path
 * (the tcgen05 GEMM; activations rounded to fp16 after a power-of-two scale,
 * weights dequantized to fp16), but it allocates nothing: its staging lives in
 * one fixed device buffer of CLQ_NOALLOC_SCRATCH_BYTES that every GPU loading
 * the library holds until exit.  Requests whose staging (about 2*m*K bytes
 * plus split-K partials) does not fit are rejected with CLQ_ERR_SHAPE; K must
 * be a multiple of 256.  The first call on a device looks up the buffer's
 * device address: make it before any stream capture.  All calls share the
 * buffer, so calls that overlap on the GPU (other streams, other threads)
 * race; serialize them on one stream. */
#define CLQ_NOALLOC_SCRATCH_BYTES (32u << 20)
int clq_linear_device_noalloc(const clq_store *w, int64_t row_begin, int64_t rows, const void *x,
                              int xtype, int64_t m, float *out, int64_t ldo, void *stream);

/* ---- tensor-parallel groups ----------------------------------------------
 * No counterpart in the reference (it has no multi-GPU path).  One process per
 * GPU; a group maps each rank's receive buffer into every rank through CUDA
 * IPC, and clq_linear_allreduce_device runs a row-parallel shard product whose
 * epilogue writes each output straight into every rank's buffer over NVLink
 * (plain peer stores of 8-byte (epoch, value) words, so no fences or flags),
 * then each CTA waits for its counterparts' words and sums the ranks in a
 * fixed order -- the GEMV and the all-reduce in one kernel.
 *
 * Set-up: each rank calls clq_tp_buffers (its receive buffer of 2 x world x
 * 160 x CAP words of 8 bytes, and a local block of per-CTA epochs), exports
 * the receive buffer with clq_ipc_handle, exchanges the 64-byte handles with
 * the other ranks, maps theirs with clq_ipc_open and calls clq_tp_create with
 * all ranks' receive buffers (its own as allocated) and its own epoch block
 * (other ranks' entries of FLAGS are not read).  Every rank must make the same
 * sequence of clq_linear_allreduce_device calls with the same shapes; a wait
 * that expires records CLQ_ERR_TIMEOUT in clq_device_status. */
typedef struct clq_tp clq_tp;
int clq_tp_buffers(int world, int64_t cap, void **recv, void **flags);
int clq_tp_buffers_free(void *recv, void *flags);
int clq_ipc_handle(const void *device_ptr, uint8_t handle[64]);
int clq_ipc_open(const uint8_t handle[64], void **device_ptr);
int clq_ipc_close(void *device_ptr);
int clq_tp_create(int rank, int world, int64_t cap, void *const *recv, void *const *flags, clq_tp **out);
int clq_tp_free(clq_tp *tp);
/* out[i, j] = sum over ranks r of rank r's clq_linear_device product for rows
 * [row_begin, row_begin + rows) of its store (each rank holds a K-slice of the
 * weight, a row-parallel shard).  Q4_K / Q6_K, K a multiple of 256, m <= 8,
 * and at most CAP outputs per SM; otherwise CLQ_ERR_UNSUPPORTED.  Asynchronous
 * on STREAM. */
int clq_linear_allreduce_device(const clq_store *w, int64_t row_begin, int64_t rows, const void *x, int xtype,
                                int64_t m, float *out, int64_t ldo, clq_tp *tp, void *stream);

/* ---- work fused around the linear -----------------------------------------
 * The product's input is h, derived from X per activation row; OUT = h W^T,
 * plus a residual (local/blocks.lisp: the RMSNorm of apply-rmsnorm :115-116,
 * run ahead of q/k/v, gate/up and the head; the SwiGLU product silu(gate) * up
 * fed to the down projection, :151-154; the residual add of layer-forward,
 * :387-392):
 *   gate        (optional, X's type and shape)  h = silu(gate) * x, silu(g) = g / (1 + e^-g);
 *   norm_weight (optional, fp32 [K])            h = h * norm_weight / sqrt(mean(h^2) + norm_epsilon);
 *   residual    (optional, fp32 [m, ldr])       OUT = residual + h W^T (single weight only; OUT may
 *                                               be the residual itself).
 * The decode GEMV (Q4_K / Q6_K, up to two activation rows) applies these in
 * its activation staging and tile epilogue, with no extra launch or round
 * trip; other shapes run the same arithmetic as separate kernels on the
 * stream (scratch from the stream-ordered pool).  Asynchronous on STREAM.
 */
typedef struct clq_fusion {
    const float *norm_weight;
    float norm_epsilon;
    const void *gate;
    const float *residual;
    int64_t ldr;
} clq_fusion;
int clq_linear_fused_device(const clq_store *w, int64_t row_begin, int64_t rows, const void *x, int xtype,
                            int64_t m, const clq_fusion *fusion, float *out, int64_t ldo, unsigned flags,
                            void *stream);
/* clq_linear_group_device with a fusion (no residual): q/k/v or gate/up from one normalized input. */
int clq_linear_group_fused_device(const clq_store *const *w, const int64_t *row_begin, const int64_t *rows,
                                  int count, const void *x, int xtype, int64_t m, const clq_fusion *fusion,
                                  float *const *out, const int64_t *ldo, unsigned flags, void *stream);

/* ---- dequantize and gather ------------------------------------------------
 * Bit-exact fp32 values of packed-element (quant/packed.lisp:85-108) and the
 * Q8_0 dequantize-executor (quant/q8-0.lisp:98-123).
 */
/* Rows [row_begin, row_begin + rows) into OUT (device, [rows, K] row-major, or
 * [K, rows] when TRANSPOSED is non-zero: the transposed-view astype). */
int clq_dequantize_device(const clq_store *w, int64_t row_begin, int64_t rows, float *out,
                          int transposed, void *stream);
/* ct:take + dequantize of local/blocks.lisp:136-138: OUT[i, :] = row IDS[i]
 * (device int32 ids, duplicates allowed).  An id outside [0, N) cannot be
 * reported by this asynchronous call: its output row is filled with quiet
 * NaNs.  clq_take checks the ids on the host and returns an error instead. */
int clq_gather_device(const clq_store *w, const int32_t *ids, int64_t count, float *out,
                      void *stream);
/* Host-pointer forms (synchronous; the bytes are uploaded for the call only). */
int clq_dequantize(int dtype, const uint8_t *bytes, size_t nbytes, float *out);
int clq_take(int dtype, const uint8_t *bytes, int64_t n, int64_t k, const int32_t *ids,
             int64_t count, float *out);

/* ---- GGUF files -> device stores ------------------------------------------
 * clq_gguf_open maps a little-endian GGUF v3 file read-only and parses its
 * header with the checks of gguf/reader.lisp (parse-gguf, :167-196; replaces
 * open-gguf of gguf/weights.lisp:18-30 for the packed weights): magic and
 * version, u64 counts bounded by the bytes left, UTF-8 strings, metadata types
 * 0..12 nested at most 32 deep, booleans 0 or 1, no duplicate keys or tensors,
 * ranks 1..4 of positive dimensions, known ggml types, rows of whole blocks, a
 * power-of-two general.alignment of at most 4096 (default 32), and aligned,
 * non-overlapping tensors inside the file.  Malformed files fail with
 * CLQ_ERR_FORMAT, unreadable ones with CLQ_ERR_IO.  Names, strings and tensor
 * bytes handed out point into FILE and stay valid until clq_gguf_close.
 */
typedef struct clq_gguf clq_gguf;
int clq_gguf_open(const char *path, clq_gguf **out);
int clq_gguf_close(clq_gguf *file);
int clq_gguf_tensor_count(const clq_gguf *file, int64_t *count);
/* Tensor INDEX in file order: name, ggml type id, rank, dimensions in the
 * file's order (dims[0] = row length; unused ones are 1), offset in the data
 * section, byte count, and its bytes in the mapping (the :u8 view of
 * weights-make-bytes, gguf/weights.lisp:71-74).  Any output may be NULL. */
int clq_gguf_tensor_info(const clq_gguf *file, int64_t index, const char **name, int *ggml_type,
                         int *rank, int64_t dims[4], uint64_t *offset, uint64_t *nbytes,
                         const uint8_t **bytes);
int clq_gguf_find_tensor(const clq_gguf *file, const char *name, int64_t *index);
/* Metadata keys in file order, with their value types (0..12). */
int clq_gguf_metadata_count(const clq_gguf *file, int64_t *count);
int clq_gguf_metadata_key(const clq_gguf *file, int64_t index, const char **key, int *type);
/* The value of KEY: unsigned integers and booleans in *uvalue, signed integers
 * in *ivalue, floats in *fvalue, strings as (*svalue, *slen); for an array
 * (type 9) its element type and length (elements are not kept).  Any output
 * may be NULL. */
int clq_gguf_metadata_value(const clq_gguf *file, const char *key, int *type, uint64_t *uvalue,
                            int64_t *ivalue, double *fvalue, const char **svalue, uint64_t *slen,
                            int *elem_type, uint64_t *count);
/* Tensor INDEX (Q4_0, Q8_0, Q4_K or Q6_K; N = dims[1] * dims[2] * dims[3]
 * rows of K = dims[0]) as a store on the current device: the bytes are read
 * from the file into two page-locked staging buffers in turn, one filled while
 * the other's asynchronous copy runs, and are then checked and re-tiled as
 * clq_store_create does (CLQ_ERR_NONFINITE_SCALE for an fp16 scale with
 * exponent 31).  Other types: CLQ_ERR_UNSUPPORTED. */
int clq_gguf_store(clq_gguf *file, int64_t index, clq_store **out);

/* ---- KV cache, RoPE and attention around the linears --------------------
 * The decode layer's work between the projections (local/blocks.lisp:327-353)
 * on device memory.  A cache holds every layer's keys and values, each
 * [n_ctx][kv_heads][head_dim]: f32, or the reference's Q8 codec -- int8
 * codes and one f32 scale per 32-element group, scale = max(FLT_MIN, peak /
 * 127) (1 for an all-zero group), code = clamp(round-half-even(value /
 * scale), -127, 127) (local/kv-cache.lisp:20-78).  Rows are f32 with element
 * stride 1 and the given position and head strides (in elements). */
enum clq_kv_type { CLQ_KV_F32 = 0, CLQ_KV_Q8 = 1 };
enum clq_rope_pairing { CLQ_ROPE_ADJACENT = 0, CLQ_ROPE_NEOX = 1 };
typedef struct clq_kv_cache clq_kv_cache;
/* make-kv-cache (local/kv-cache.lisp:17-19) for LAYERS layers on the current device. */
int clq_kv_cache_create(int64_t n_ctx, int layers, int kv_heads, int head_dim, int cache_type, clq_kv_cache **out);
int clq_kv_cache_destroy(clq_kv_cache *cache);
int clq_kv_cache_info(const clq_kv_cache *cache, int64_t *n_ctx, int *layers, int *kv_heads, int *head_dim,
                      int *cache_type);
/* The store half of kv-cache-update (local/kv-cache.lisp:92-110): COUNT rows of
 * K and V into LAYER at positions [START, START + COUNT); CLQ_ERR_CONTEXT past
 * n_ctx.  Asynchronous on STREAM: a non-finite value into a Q8 cache is
 * reported by clq_kv_cache_status (the rows are stored all the same). */
int clq_kv_cache_update(clq_kv_cache *cache, int layer, const float *k, const float *v, int64_t count,
                        int64_t pos_stride, int64_t head_stride, int64_t start, void *stream);
/* No counterpart in the reference (its stores fail on the calling thread).
 * Waits for the device and returns in *STATUS CLQ_ERR_NONFINITE_VALUE when a
 * Q8 store met a non-finite value since the last call (else CLQ_OK), and clears it. */
int clq_kv_cache_status(clq_kv_cache *cache, int *status);
/* The prefix half of kv-cache-update: LAYER's first END positions decoded to f32
 * [end][kv_heads][head_dim] (the f32 slice, or q8-prefix, local/kv-cache.lisp:62-78);
 * either output may be null. */
int clq_kv_cache_read(const clq_kv_cache *cache, int layer, int64_t end, float *keys, float *values, void *stream);
/* apply-rope with rope-tables (local/blocks.lisp:172-214), in place on COUNT rows
 * of HEADS heads at positions START..: frequency theta^(-2i/rope_dims) / factors[i]
 * (FACTORS null: 1; the Llama-3 factors of llama3-rope-factors, :230-252, are the
 * caller's), cos and sin in double rounded to f32; PAIRING adjacent (2i, 2i+1)
 * or neox (i, i + rope_dims/2). */
int clq_rope_device(float *x, int64_t count, int heads, int head_dim, int64_t pos_stride, int64_t head_stride,
                    int rope_dims, int64_t start, double theta, const float *factors, int pairing, void *stream);
/* attend with causal-mask (local/blocks.lisp:282-325) over LAYER's cached prefix
 * [0, END): query row t at position QUERY_START + t sees keys at positions <= it;
 * head h reads KV head h / (n_heads / kv_heads); scores scaled by 1/sqrt(head_dim);
 * OUT[t][h * head_dim + d] (row stride LDO) the softmax-weighted values. */
int clq_attend_device(const float *q, int64_t count, int n_heads, int64_t q_pos_stride, const clq_kv_cache *cache,
                      int layer, int64_t end, int64_t query_start, float *out, int64_t ldo, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* CLQ_H */
