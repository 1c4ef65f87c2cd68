/* Test infrastructure only: CPU stand-ins for the fused-decoder entry points
 * (include/qwen_b200.h) so that the session host (cmachine_b200/host) can be
 * linked with the reference's CPU primitive fake (tests/gpu_stub.c) into
 * _ref/libqwen_host_cpu.so. That library runs the host state machine -- cursor
 * checkpoints, the nested stack, token abort, reset, lineage, observer ports,
 * cache callbacks -- on the CPU, the way the reference's model-free lane does
 * (Makefile:58-83). No fused decoder exists there: models are built with
 * fused = 0 and every layer runs the primitive sequence. */
#include "../include/qwen_b200.h"
#include "../include/tcm_seeded.h"
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
