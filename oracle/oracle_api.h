/* Test infrastructure only: the C ABI shared by the two CPU checkers.
 *
 *   liboracle.so        -- this repository's C restatement of the reference's CPU
 *                          FP32 decode path (qwen_oracle.c);
 *   _ref/libref_cpu.so  -- the reference's own src/qwen.c + src/model.c +
 *                          tests/gpu_stub.c, built from the reference sources by
 *                          oracle/Makefile and driven through ref_driver.c.
 *
 * Both export the same orc_* symbols so tests can run them side by side. Nothing
 * in the product links against these libraries.
 */
#ifndef TCM_ORACLE_API_H
#define TCM_ORACLE_API_H
#include <stdint.h>
#include "../include/tcm_seeded.h"
#ifdef __cplusplus
extern "C" {
#endif
typedef struct {
    int hidden, layers, qheads, kvheads, head, intermediate, vocab, max_position;
    float epsilon, theta;
} OrcShape;
typedef struct { int first, second; float first_value, second_value; } OrcTop2;

/* weights: 0 = FP32 values, 1 = matrices (and embedding) rounded to BF16 and
 * consumed widened to FP32, as the reference's profile 0 / profile 2 do. */
void *orc_model_create(const OrcShape *shape, uint64_t seed, const TcmFillLaw *law, int bf16);
void orc_model_free(void *model);
void *orc_session_create(void *model, int capacity);
void orc_session_free(void *session);
/* One qwen_push: returns 0 on success; writes top-2 and, if logits != NULL,
 * all vocab logits of the readout that followed the token. The restatement
 * (liboracle.so) skips the readout when top == NULL (cheap prefill). */
int orc_push(void *session, int token, OrcTop2 *top, float *logits);
int orc_position(void *session);
/* K or V rows 0..position-1 of one layer: out[kvheads][position][head]. */
void orc_read_kv(void *session, int layer, int kind, float *out);
/* The final-norm input x of the last pushed token (hidden floats). */
void orc_read_hidden(void *session, float *out);
/* Context injection for long-context parity: write K (kind 0) or V (kind 1)
 * rows 0..rows-1 of one layer from in[kvheads][rows][head], and place the
 * cursor after `position` cached rows (the next push appends row `position`).
 * Both checkers accept the same calls, so seeded contexts of any length can be
 * compared without prefilling them token by token. */
void orc_write_kv(void *session, int layer, int kind, int rows, const float *in);
int orc_set_cursor(void *session, int position);
/* Bounded byte-codec ring sessions (liboracle.so only). */
typedef struct {
    int cursor;
    uint64_t population, rng;
    int write_slot, sample_slot, active, rows;
} OrcRingView;
void *orc_ring_session_create(void *model, int logical, int anchors, int recent, int sample);
/* View, slot positions [rows], order and weights [active], arena [layers][rows * 528]. */
int orc_ring_read(void *session, OrcRingView *view, int *positions, int *order, float *weights, void *arena);
/* The reference CPU codec for one row of 128 (src/byte_codec.h:5-9). */
int orc_codec(const float *x, int8_t *codes, float *scale);
/* Ring attention over int8 rows (src/qwen_cache.inc:31-43), 12 query / 2 KV heads of 128. */
void orc_ring_attention(float *out, const float *q, const signed char *key, const signed char *value,
                        const float *scales, const int *order, const float *weights, int capacity, int length,
                        int weighted);
/* Seeded weight element readback for generator pinning: tensor id, index. */
float orc_weight_value(void *model, uint32_t tensor, uint64_t index);
#ifdef __cplusplus
}
#endif
#endif
