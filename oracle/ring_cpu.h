/* Test infrastructure only (the oracle): CPU restatements of the byte-codec
 * K/V cache arithmetic of the reference's bounded cache. Included by the
 * oracle (qwen_oracle.c), by the CPU stand-ins of the session host
 * (host_cpu_fakes.c) and by the reference ring driver (ref_ring.c), so that
 * all three compute the same bits. Never part of the product.
 *
 *   orc_codec_row          src/byte_codec.h:5-9 (the reference's CPU codec):
 *                          s = max|x| / 127 (1 when the row is zero), code =
 *                          clamp(roundf(x / s), +-127); -1 on a non-finite row;
 *   orc_encode_rows        src/qwen_cache.inc:3-15 layout: the (kind, KV head)
 *                          rows of the current token into slot `position`;
 *   orc_ring_attention_cpu src/qwen_cache.inc:31-43 (ring_decode, the QK^T
 *                          GEMM, ring_bias, softmax_kernel of
 *                          src/qwen_cuda.cu:65-71, the PV GEMM) as sequential
 *                          FP32 loops: rows taken in `order`, dequantised as
 *                          (float)code * scale, score = K.q (+ weight * sqrt(128)
 *                          when weighted), softmax of score / sqrt(128) with the
 *                          maximum subtracted, out = sum_i p_i V_i.
 * Geometry is the reference's: 12 query heads over 2 KV heads of 128.
 */
#ifndef TCM_ORACLE_RING_CPU_H
#define TCM_ORACLE_RING_CPU_H
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_RING_HEAD 128
#define ORC_RING_KV 2
#define ORC_RING_GROUP 6
#define ORC_RING_ROW_BYTES 528 /* 2 kinds x 2 heads x (128 codes) + 4 scales */

static int orc_codec_row(const float *x, int8_t *codes, float *scale) {
    float maximum = 0;
    for (int d = 0; d < ORC_RING_HEAD; d++) {
        if (!isfinite(x[d])) return -1;
        maximum = fmaxf(maximum, fabsf(x[d]));
    }
    float s = maximum > 0 ? maximum / 127.0f : 1.0f;
    if (!(s > 0) || !isfinite(s)) return -1;
    for (int d = 0; d < ORC_RING_HEAD; d++) {
        float value = roundf(x[d] / s);
        if (value > 127) value = 127;
        if (value < -127) value = -127;
        codes[d] = (int8_t)value;
    }
    *scale = s;
    return 0;
}

/* One layer's arena: K codes [2][capacity][128], V codes [2][capacity][128],
 * scales [kind * 2 + head][capacity]. */
static int orc_encode_rows(signed char *key, signed char *value, float *scales, const float *k, const float *v,
                           int capacity, int position) {
    for (int kind = 0; kind < 2; kind++)
        for (int h = 0; h < ORC_RING_KV; h++)
            if (orc_codec_row((kind ? v : k) + h * ORC_RING_HEAD,
                              (int8_t *)(kind ? value : key) + ((size_t)h * capacity + position) * ORC_RING_HEAD,
                              scales + (kind * 2 + h) * capacity + position))
                return -1;
    return 0;
}

static void orc_ring_attention_cpu(float *out, const float *q, const signed char *key, const signed char *value,
                                   const float *scales, const int *order, const float *weights, int capacity,
                                   int length, int weighted) {
    float *kd = malloc((size_t)length * ORC_RING_HEAD * sizeof(float));
    float *vd = malloc((size_t)length * ORC_RING_HEAD * sizeof(float));
    float *s = malloc((size_t)length * sizeof(float));
    if (!kd || !vd || !s) abort();
    const float scale = 1.0f / sqrtf((float)ORC_RING_HEAD), bias = sqrtf((float)ORC_RING_HEAD);
    for (int h = 0; h < ORC_RING_KV; h++) {
        for (int i = 0; i < length; i++) {
            const int slot = order[i];
            const float ks = scales[(0 * 2 + h) * capacity + slot], vs = scales[(1 * 2 + h) * capacity + slot];
            for (int d = 0; d < ORC_RING_HEAD; d++) {
                kd[(size_t)i * ORC_RING_HEAD + d] = (float)key[((size_t)h * capacity + slot) * ORC_RING_HEAD + d] * ks;
                vd[(size_t)i * ORC_RING_HEAD + d] = (float)value[((size_t)h * capacity + slot) * ORC_RING_HEAD + d] * vs;
            }
        }
        for (int g = 0; g < ORC_RING_GROUP; g++) {
            const float *qh = q + (size_t)(h * ORC_RING_GROUP + g) * ORC_RING_HEAD;
            float maximum = -INFINITY, sum = 0;
            for (int i = 0; i < length; i++) {
                float dot = 0;
                for (int d = 0; d < ORC_RING_HEAD; d++) dot += kd[(size_t)i * ORC_RING_HEAD + d] * qh[d];
                if (weighted) dot += weights[i] * bias;
                s[i] = dot;
                maximum = fmaxf(maximum, dot * scale);
            }
            for (int i = 0; i < length; i++) {
                float e = expf(s[i] * scale - maximum);
                s[i] = e;
                sum += e;
            }
            for (int i = 0; i < length; i++) s[i] /= sum;
            float *o = out + (size_t)(h * ORC_RING_GROUP + g) * ORC_RING_HEAD;
            for (int d = 0; d < ORC_RING_HEAD; d++) {
                float a = 0;
                for (int i = 0; i < length; i++) a += vd[(size_t)i * ORC_RING_HEAD + d] * s[i];
                o[d] = a;
            }
        }
    }
    free(kd);
    free(vd);
    free(s);
}
#endif
