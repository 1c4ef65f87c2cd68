/* Test infrastructure only: CPU stand-ins for the fused-decoder entry points
 * (include/qwen_b200.h) so that the session host (cmachine_b200/host) can be
 * linked with the reference's CPU primitive fake (tests/gpu_stub.c) into
 * _ref/libqwen_host_cpu.so. That library runs the host state machine -- cursor
 * checkpoints, the nested stack, token abort, reset, lineage, observer ports,
 * cache callbacks -- on the CPU, the way the reference's model-free lane does
 * (Makefile:58-83). No fused decoder exists there: models are built with
 * fused = 0 and every layer runs the primitive sequence. The byte-codec cache
 * entry points the CPU fake lacks are supplied as the reference's mechanics
 * test supplies them (tests/bounded_mechanics.c:7-12), with the oracle's codec
 * and ring attention (ring_cpu.h), plus a memcpy form of the token cut rows. */
#include "../include/qwen_b200.h"
#include "../include/tcm_seeded.h"
#include "ring_cpu.h"
#include <stdio.h>
#include <string.h>

void qwen_b200_seeded_fill(void *dst, int dtype, uint64_t seed, uint32_t id, size_t n, float offset, float scale) {
    TcmFill f = {offset, scale};
    uint64_t base = tcm_tensor_base(seed, id);
    for (size_t i = 0; i < n; i++) {
        float v = tcm_seeded_value(base, i, f);
        if (dtype == 2) ((uint16_t *)dst)[i] = tcm_bf16_rne(v);
        else ((float *)dst)[i] = v;
    }
}
void qwen_b200_register_matrix(const void *p, int rows, int columns, int encoded) { (void)p; (void)rows; (void)columns; (void)encoded; }
void qwen_b200_unregister_matrix(const void *p) { (void)p; }
QwenB200Decoder *qwen_b200_decoder_create(const QwenB200Shape *s, const float *e, const float *n,
                                          const QwenB200Layer *l, int d) {
    (void)s; (void)e; (void)n; (void)l; (void)d;
    return NULL;
}
void qwen_b200_decoder_free(QwenB200Decoder *d) { (void)d; }
QwenB200Runner *qwen_b200_runner_create(const QwenB200Decoder *d, const QwenB200Buffers *b) { (void)d; (void)b; return NULL; }
void qwen_b200_runner_free(QwenB200Runner *r) { (void)r; }
int qwen_b200_begin(QwenB200Runner *r, int t, int p) { (void)r; (void)t; (void)p; return -1; }
int qwen_b200_layer(QwenB200Runner *r, int l) { (void)r; (void)l; return -1; }
int qwen_b200_layer_qkv(QwenB200Runner *r, int l) { (void)r; (void)l; return -1; }
int qwen_b200_layer_mlp(QwenB200Runner *r, int l) { (void)r; (void)l; return -1; }
int qwen_b200_finish(QwenB200Runner *r, TcmTop2 *t) { (void)r; (void)t; return -1; }
int qwen_b200_token(QwenB200Runner *r, int t, int p, TcmTop2 *o) { (void)r; (void)t; (void)p; (void)o; return -1; }
int qwen_b200_generate(QwenB200Runner *r, int t, int p, int n, int *i, TcmTop2 *o) {
    (void)r; (void)t; (void)p; (void)n; (void)i; (void)o;
    return -1;
}

int qwen_b200_complete(QwenB200Runner *r, TcmTop2 *t) { (void)r; (void)t; return -1; }
int qwen_b200_can_complete(const QwenB200Runner *r) { (void)r; return 0; }
int qwen_b200_ring_attach(QwenB200Runner *r, const QwenB200Ring *g) { (void)r; (void)g; return -1; }
int qwen_b200_ring_stage(QwenB200Runner *r, const QwenB200RingStep *s) { (void)r; (void)s; return -1; }
int qwen_b200_ring_attention(QwenB200Runner *r, int l, const float *q, const float *k, const float *v, float *o) {
    (void)r; (void)l; (void)q; (void)k; (void)v; (void)o;
    return -1;
}
int qwen_b200_ring_status(QwenB200Runner *r) { (void)r; return -1; }

int gpu_encode_current(signed char *key, signed char *value, float *scales, const float *k, const float *v,
                       int capacity, int position, int *invalid) {
    *invalid = 0;
    return orc_encode_rows(key, value, scales, k, v, capacity, position);
}
void gpu_ring_attention(TcmGpu *g, float *out, const float *q, const signed char *key, const signed char *value,
                        const float *scales, float *scores, float *workspace, const int *order, const float *weights,
                        int capacity, int length, int weighted) {
    (void)g; (void)scores; (void)workspace;
    orc_ring_attention_cpu(out, q, key, value, scales, order, weights, capacity, length, weighted);
}
/* The token cut rows (528 bytes: 4 code segments of 128, then 4 scales). */
static void row_move(unsigned char *layer, int rows, int slot, unsigned char *buf, int to_buf) {
    for (int seg = 0; seg < 4; seg++) {
        unsigned char *a = layer + (size_t)(seg >> 1) * rows * 256 + ((size_t)(seg & 1) * rows + slot) * 128;
        if (to_buf) memcpy(buf + seg * 128, a, 128);
        else memcpy(a, buf + seg * 128, 128);
    }
    for (int j = 0; j < 4; j++) {
        unsigned char *a = layer + (size_t)rows * 512 + ((size_t)j * rows + slot) * 4;
        if (to_buf) memcpy(buf + 512 + j * 4, a, 4);
        else memcpy(a, buf + 512 + j * 4, 4);
    }
}
void qwen_b200_ring_rows(void *arena, int rows, int layers, void *save, int write_slot, int sample_slot, int mode) {
    for (int l = 0; l < layers; l++) {
        unsigned char *layer = (unsigned char *)arena + (size_t)l * rows * 528;
        unsigned char *s = (unsigned char *)save + (size_t)l * 2 * 528;
        if (mode == 0) {
            row_move(layer, rows, write_slot, s, 1);
            if (sample_slot >= 0) {
                row_move(layer, rows, sample_slot, s + 528, 1);
                row_move(layer, rows, sample_slot, s, 0);
            }
        } else {
            row_move(layer, rows, write_slot, s, 0);
            if (sample_slot >= 0) row_move(layer, rows, sample_slot, s + 528, 0);
        }
    }
}
QwenB200Batch *qwen_b200_batch_create(const QwenB200Decoder *d) { (void)d; return NULL; }
void qwen_b200_batch_free(QwenB200Batch *b) { (void)b; }
int qwen_b200_batch_max(void) { return 64; }
int qwen_b200_weight_dtype(const void *p) { (void)p; return 1; }
/* Weight profiles and allocation accounting have no CPU meaning. */
void gpu_weight_configure(int profile) { (void)profile; }
void gpu_weight_release(void) {}
size_t gpu_live_bytes(void) { return 0; }
int qwen_b200_batch_prefill(QwenB200Batch *b, const QwenB200BatchSession *s, const int *t, int n, int p, TcmTop2 *o) {
    (void)b; (void)s; (void)t; (void)n; (void)p; (void)o;
    return -1;
}
int qwen_b200_batch_step(QwenB200Batch *b, int n, const QwenB200BatchSession *s, const int *t, const int *p, TcmTop2 *o) {
    (void)b; (void)n; (void)s; (void)t; (void)p; (void)o;
    return -1;
}
int qwen_b200_tp_open(QwenB200Runner *r, int rank, int world, void *h) { (void)r; (void)rank; (void)world; (void)h; return -1; }
int qwen_b200_tp_connect(QwenB200Runner *r, const void *h) { (void)r; (void)h; return -1; }
int qwen_b200_tp_close(QwenB200Runner *r) { (void)r; return -1; }
int qwen_b200_tp_world(const QwenB200Runner *r) { (void)r; return 1; }
