/*
 * clq_oracle.h -- CPU restatement of cl-inference's packed-weight arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This oracle is the checker for the CUDA library
 * (libclq.so): tests, the smoke check and the CPU-baseline leg of the
 * benchmark call it to produce expected values.  The product never links it.
 *
 * What it restates (paths are relative to the cl-inference project):
 *   - fp16 scale decode ........... quant/q8-0.lisp:89-96   (block-scale)
 *   - Q8_0 element ................ quant/q8-0.lisp:113-117 (dequantize-executor)
 *   - Q4_0 / Q4_K / Q6_K element .. quant/packed.lisp:85-108 (packed-element)
 *   - matmul contract ............. quant/packed.lisp:68-75, quant/q8-0.lisp:87-94
 *                                   out[M,N] = x[M,K] . dequant(W[N,K])^T, f32
 *   - fp64 dequant-matmul check ... tests/local/packed.lisp:5-12 (packed-product-close-p)
 *
 * Pinned by the llama.cpp golden blocks of tests/local/quant-golden.lisp:3-17
 * and the Q8_0 golden of tests/mlx-gguf/kernels.lisp:9-21 (see tests/golden/).
 * Every fp32 operation is written out in the reference's order; build with
 * -ffp-contract=off so no multiply-add is fused.
 */
#ifndef CLQ_ORACLE_H
#define CLQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids, gguf/reader.lisp:37-52 */
enum { CLQO_Q4_0 = 2, CLQO_Q8_0 = 8, CLQO_Q4_K = 12, CLQO_Q6_K = 14 };

/* Status codes: 0 ok, 1 bad argument/geometry, 4 non-finite scale. */
enum { CLQO_OK = 0, CLQO_ERR_ARGUMENT = 1, CLQO_ERR_NONFINITE = 4 };

/* Elements and bytes per block; 0 on unknown dtype. */
int clqo_block_geometry(int dtype, int64_t *elements, int64_t *bytes);

/* block-scale: decode the little-endian fp16 (low, high).  Exponent 31 is
 * an error ("Quantized scale is not finite", quant/q8-0.lisp:95). */
int clqo_block_scale(uint8_t low, uint8_t high, float *out);

/* packed-element / Q8_0 element: element E (0 <= E < elements) of the block
 * starting at BLOCK. */
int clqo_element(int dtype, const uint8_t *block, int e, float *out);

/* Dequantize NBLOCKS consecutive blocks into OUT (elements * NBLOCKS floats).
 * On a non-finite scale returns CLQO_ERR_NONFINITE and stores the index of the
 * offending block in *bad_block (if non-NULL). */
int clqo_dequantize(int dtype, const uint8_t *bytes, int64_t nblocks, float *out,
                    int64_t *bad_block);

/* Gather rows IDS[0..count) of an N x K packed matrix, dequantized, into
 * OUT[count, K] (the ct:take + dequantize of local/blocks.lisp:136-138). */
int clqo_gather(int dtype, const uint8_t *bytes, int64_t n, int64_t k,
                const int32_t *ids, int64_t count, float *out);

/* fp64 oracle: OUT[m,n] = sum_k x[m,k]*w[n,k] in double over the fp32
 * dequantized weights, and MAG[m,n] = sum_k |x[m,k]*w[n,k]| (may be NULL).
 * THREADS <= 0 uses every OpenMP thread. */
int clqo_matmul_f64(int dtype, const float *x, const uint8_t *bytes, int64_t m, int64_t n,
                    int64_t k, double *out, double *mag, int threads);

/* fp32 port of the CPU kernel contract (decode a block, reuse it across the
 * activation rows, fp32 products and sums): the timed CPU baseline. */
int clqo_matmul_f32(int dtype, const float *x, const uint8_t *bytes, int64_t m, int64_t n,
                    int64_t k, float *out, int threads);

/* Threads OpenMP would use (omp_get_max_threads), 1 without OpenMP. */
int clqo_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
