/*
 * clq_oracle.c -- CPU restatement of cl-inference's packed-weight arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for libclq.so, never part of it.
 * Build: see oracle/Makefile (gcc -O3 -ffp-contract=off -fopenmp).
 * Each function names the reference lines it follows; paths are relative to
 * the cl-inference project.
 */
#include "clq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int clqo_block_geometry(int dtype, int64_t *elements, int64_t *bytes) {
    /* quant/q8-0.lisp:5-6 and the registrations at quant/packed.lisp:156-158 */
    int64_t e = 0, b = 0;
    switch (dtype) {
    case CLQO_Q4_0: e = 32; b = 18; break;
    case CLQO_Q8_0: e = 32; b = 34; break;
    case CLQO_Q4_K: e = 256; b = 144; break;
    case CLQO_Q6_K: e = 256; b = 210; break;
    default: return 0;
    }
    if (elements) *elements = e;
    if (bytes) *bytes = b;
    return 1;
}

/* quant/q8-0.lisp:89-96: sign * 2^-24 * fraction for exponent 0, an error for
 * exponent 31, otherwise sign * 2^(exponent-25) * (1024 + fraction). */
int clqo_block_scale(uint8_t low, uint8_t high, float *out) {
    unsigned bits = (unsigned)low | ((unsigned)high << 8);
    float sign = (bits & 0x8000u) ? -1.0f : 1.0f;
    int exponent = (int)((bits >> 10) & 31u);
    unsigned fraction = bits & 1023u;
    if (exponent == 0) {
        *out = sign * ldexpf((float)fraction, -24);
    } else if (exponent == 31) {
        return CLQO_ERR_NONFINITE;
    } else {
        *out = sign * ldexpf((float)(1024u + fraction), exponent - 25);
    }
    return CLQO_OK;
}

static int half_at(const uint8_t *block, int offset, float *out) {
    /* packed-half, quant/packed.lisp:82-83 */
    return clqo_block_scale(block[offset], block[offset + 1], out);
}

int clqo_element(int dtype, const uint8_t *b, int e, float *out) {
    float d, dmin;
    int rc;
    switch (dtype) {
    case CLQO_Q8_0: {
        /* quant/q8-0.lisp:113-117: scale * signed byte */
        if ((rc = half_at(b, 0, &d))) return rc;
        int q = b[2 + e];
        q = q < 128 ? q : q - 256;
        *out = d * (float)q;
        return CLQO_OK;
    }
    case CLQO_Q4_0: {
        /* quant/packed.lisp:87-88: low nibble of qs[e] for e < 16, high
         * nibble of qs[e-16] otherwise; value d * (nibble - 8) */
        if ((rc = half_at(b, 0, &d))) return rc;
        int byte = b[2 + (e % 16)];
        int nib = (e < 16) ? (byte & 15) : ((byte >> 4) & 15);
        *out = d * (float)(nib - 8);
        return CLQO_OK;
    }
    case CLQO_Q4_K: {
        /* quant/packed.lisp:89-100 */
        if ((rc = half_at(b, 0, &d))) return rc;
        if ((rc = half_at(b, 2, &dmin))) return rc;
        int group = e / 32;
        const uint8_t *s = b + 4;
        int scale, minimum;
        if (group < 4) {
            scale = s[group] & 63;
            minimum = s[group + 4] & 63;
        } else {
            scale = (s[group + 4] & 15) | ((s[group - 4] & 192) >> 2);
            minimum = (s[group + 4] >> 4) | ((s[group] & 192) >> 2);
        }
        int q = (b[16 + 32 * (group / 2) + (e % 32)] >> (4 * (group % 2))) & 15;
        float ds = d * (float)scale;
        float v = ds * (float)q;
        float mm = dmin * (float)minimum;
        *out = v - mm;
        return CLQO_OK;
    }
    case CLQO_Q6_K: {
        /* quant/packed.lisp:101-108 */
        if ((rc = half_at(b, 208, &d))) return rc;
        int half = e / 128, group = (e % 128) / 32, l = e % 32;
        int low = (b[half * 64 + (group % 2) * 32 + l] >> (4 * (group / 2))) & 15;
        int high = (b[128 + half * 32 + l] >> (group * 2)) & 3;
        int scale = b[192 + half * 8 + group * 2 + l / 16];
        scale = scale < 128 ? scale : scale - 256;
        float ds = d * (float)scale;
        *out = ds * (float)((low | (high << 4)) - 32);
        return CLQO_OK;
    }
    default:
        return CLQO_ERR_ARGUMENT;
    }
}

/* Scale offsets the reference decodes for every element of a block. */
static int block_scales_finite(int dtype, const uint8_t *b) {
    float tmp;
    switch (dtype) {
    case CLQO_Q4_0:
    case CLQO_Q8_0: return half_at(b, 0, &tmp) == CLQO_OK;
    case CLQO_Q4_K: return half_at(b, 0, &tmp) == CLQO_OK && half_at(b, 2, &tmp) == CLQO_OK;
    case CLQO_Q6_K: return half_at(b, 208, &tmp) == CLQO_OK;
    default: return 0;
    }
}

/* A whole block, scales decoded once; per element the same fp32 operations as
 * clqo_element (the tests check the two agree bit for bit).  Scales must have
 * been checked finite. */
static void dequant_block(int dtype, const uint8_t *b, int64_t elements, float *out) {
    float d, dmin;
    switch (dtype) {
    case CLQO_Q8_0:
        half_at(b, 0, &d);
        for (int e = 0; e < 32; e++) out[e] = d * (float)(int8_t)b[2 + e];
        return;
    case CLQO_Q4_0:
        half_at(b, 0, &d);
        for (int e = 0; e < 16; e++) {
            out[e] = d * (float)((b[2 + e] & 15) - 8);
            out[e + 16] = d * (float)((b[2 + e] >> 4) - 8);
        }
        return;
    case CLQO_Q4_K:
        half_at(b, 0, &d);
        half_at(b, 2, &dmin);
        for (int g = 0; g < 8; g++) {
            const uint8_t *s = b + 4;
            int scale, minimum;
            if (g < 4) {
                scale = s[g] & 63;
                minimum = s[g + 4] & 63;
            } else {
                scale = (s[g + 4] & 15) | ((s[g - 4] & 192) >> 2);
                minimum = (s[g + 4] >> 4) | ((s[g] & 192) >> 2);
            }
            float ds = d * (float)scale, mm = dmin * (float)minimum;
            const uint8_t *q = b + 16 + 32 * (g / 2);
            int shift = 4 * (g % 2);
            for (int l = 0; l < 32; l++) {
                float v = ds * (float)((q[l] >> shift) & 15);
                out[g * 32 + l] = v - mm;
            }
        }
        return;
    case CLQO_Q6_K:
        half_at(b, 208, &d);
        for (int e = 0; e < 256; e++) {
            int half = e / 128, group = (e % 128) / 32, l = e % 32;
            int low = (b[half * 64 + (group % 2) * 32 + l] >> (4 * (group / 2))) & 15;
            int high = (b[128 + half * 32 + l] >> (group * 2)) & 3;
            int scale = (int8_t)b[192 + half * 8 + group * 2 + l / 16];
            float ds = d * (float)scale;
            out[e] = ds * (float)((low | (high << 4)) - 32);
        }
        return;
    default:
        for (int64_t e = 0; e < elements; e++) clqo_element(dtype, b, (int)e, &out[e]);
    }
}

int clqo_dequantize(int dtype, const uint8_t *bytes, int64_t nblocks, float *out,
                    int64_t *bad_block) {
    /* packed-dequantize-executor, quant/packed.lisp:110-124, row-major walk */
    int64_t el, bb;
    if (!clqo_block_geometry(dtype, &el, &bb) || nblocks < 0) return CLQO_ERR_ARGUMENT;
    for (int64_t i = 0; i < nblocks; i++) {
        if (!block_scales_finite(dtype, bytes + i * bb)) {
            if (bad_block) *bad_block = i;
            return CLQO_ERR_NONFINITE;
        }
    }
    for (int64_t i = 0; i < nblocks; i++) dequant_block(dtype, bytes + i * bb, el, out + i * el);
    return CLQO_OK;
}

int clqo_gather(int dtype, const uint8_t *bytes, int64_t n, int64_t k, const int32_t *ids,
                int64_t count, float *out) {
    int64_t el, bb;
    if (!clqo_block_geometry(dtype, &el, &bb) || k % el) return CLQO_ERR_ARGUMENT;
    int64_t per_row = k / el;
    for (int64_t i = 0; i < count; i++) {
        if (ids[i] < 0 || ids[i] >= n) return CLQO_ERR_ARGUMENT;
        int rc = clqo_dequantize(dtype, bytes + (int64_t)ids[i] * per_row * bb, per_row,
                                 out + i * k, NULL);
        if (rc) return rc;
    }
    return CLQO_OK;
}

static int check_matmul(int dtype, int64_t m, int64_t n, int64_t k, int64_t *el, int64_t *bb) {
    if (!clqo_block_geometry(dtype, el, bb)) return CLQO_ERR_ARGUMENT;
    if (m < 0 || n < 0 || k < 0 || k % *el) return CLQO_ERR_ARGUMENT;
    return CLQO_OK;
}

static int scan_scales(int dtype, const uint8_t *bytes, int64_t nblocks, int64_t bb) {
    for (int64_t i = 0; i < nblocks; i++)
        if (!block_scales_finite(dtype, bytes + i * bb)) return CLQO_ERR_NONFINITE;
    return CLQO_OK;
}

int clqo_matmul_f64(int dtype, const float *x, const uint8_t *bytes, int64_t m, int64_t n,
                    int64_t k, double *out, double *mag, int threads) {
    /* The reference's test oracle: ref-dot over doubles (tests/local/fixtures.lisp:134)
     * and the magnitude term of packed-product-close-p (tests/local/packed.lisp:5-12). */
    int64_t el, bb;
    int rc = check_matmul(dtype, m, n, k, &el, &bb);
    if (rc) return rc;
    int64_t per_row = k / el;
    if ((rc = scan_scales(dtype, bytes, n * per_row, bb))) return rc;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        float *w = (float *)malloc((size_t)(k > 0 ? k : 1) * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int64_t r = 0; r < n; r++) {
            for (int64_t b = 0; b < per_row; b++)
                dequant_block(dtype, bytes + (r * per_row + b) * bb, el, w + b * el);
            for (int64_t i = 0; i < m; i++) {
                double sum = 0.0, magnitude = 0.0;
                const float *xr = x + i * k;
                for (int64_t c = 0; c < k; c++) {
                    double p = (double)xr[c] * (double)w[c];
                    sum += p;
                    magnitude += fabs(p);
                }
                out[i * n + r] = sum;
                if (mag) mag[i * n + r] = magnitude;
            }
        }
        free(w);
    }
    (void)threads;
    return CLQO_OK;
}

int clqo_matmul_f32(int dtype, const float *x, const uint8_t *bytes, int64_t m, int64_t n,
                    int64_t k, float *out, int threads) {
    /* Port of the packed kernel contract (docs/quant.md, "Execution and
     * accuracy"): decode one block at a time, reuse it across the activation
     * rows, fp32 products and fp32 sums (eight partial sums per output). */
    int64_t el, bb;
    int rc = check_matmul(dtype, m, n, k, &el, &bb);
    if (rc) return rc;
    int64_t per_row = k / el;
    if ((rc = scan_scales(dtype, bytes, n * per_row, bb))) return rc;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        float blockv[256];
        float *acc = (float *)malloc((size_t)(m > 0 ? m : 1) * 8 * sizeof(float));
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int64_t r = 0; r < n; r++) {
            memset(acc, 0, (size_t)(m > 0 ? m : 1) * 8 * sizeof(float));
            for (int64_t b = 0; b < per_row; b++) {
                dequant_block(dtype, bytes + (r * per_row + b) * bb, el, blockv);
                for (int64_t i = 0; i < m; i++) {
                    const float *xr = x + i * k + b * el;
                    float *a = acc + i * 8;
                    for (int64_t e = 0; e < el; e += 8)
                        for (int j = 0; j < 8; j++) a[j] += xr[e + j] * blockv[e + j];
                }
            }
            for (int64_t i = 0; i < m; i++) {
                float *a = acc + i * 8;
                out[i * n + r] = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
            }
        }
        free(acc);
    }
    (void)threads;
    return CLQO_OK;
}

int clqo_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
