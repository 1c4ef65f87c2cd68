/* Test infrastructure only: drives the reference's own bounded byte-codec
 * cache (src/bounded_cache.h) over the reference's C host (src/qwen.c) and CPU
 * primitives (tests/gpu_stub.c). oracle/Makefile builds _ref/libref_ring.so
 * from this file, ref_driver.c (the seeded model) and those sources where they
 * lie; nothing here is part of the product.
 *
 * The two device entry points the ring needs and the CPU stub lacks are
 * supplied as the reference's own mechanics test supplies them
 * (tests/bounded_mechanics.c:7-12): gpu_encode_current runs the reference's
 * CPU codec (src/byte_codec.h) row by row; gpu_ring_attention runs the CPU
 * restatement of src/qwen_cache.inc:31-43 (ring_cpu.h). The ring itself --
 * slot choice, reservoir sampling, order, cuts, guard, rewind, marks -- is the
 * reference's code, unchanged.
 */
#define _POSIX_C_SOURCE 200809L
#include <stdio.h>
#include <stdlib.h>
#define REQUIRE(x)                                                                  \
    do {                                                                            \
        if (!(x)) {                                                                 \
            fprintf(stderr, "reference ring %s:%d: %s\n", __FILE__, __LINE__, #x); \
            abort();                                                                \
        }                                                                           \
    } while (0)
#include "qwen.h"
#include "byte_codec.h"
#include "bounded_cache.h"
#include "ring_cpu.h"

int gpu_encode_current(signed char *k, signed char *v, float *s, const float *kr, const float *vr, int cap, int p,
                       int *invalid) {
    *invalid = 0;
    for (int kind = 0; kind < 2; kind++)
        for (int h = 0; h < 2; h++)
            if (codec_row((kind ? vr : kr) + h * 128, (int8_t *)(kind ? v : k) + ((size_t)h * cap + p) * 128,
                          s + (kind * 2 + h) * cap + p))
                return -1;
    return 0;
}
void gpu_ring_attention(TcmGpu *g, float *out, const float *q, const signed char *k, const signed char *v,
                        const float *s, float *scores, float *workspace, const int *order, const float *weights, int cap,
                        int n, int weighted) {
    (void)g; (void)scores; (void)workspace;
    orc_ring_attention_cpu(out, q, k, v, s, order, weights, cap, n, weighted);
}

/* The model comes from ref_driver.c (orc_model_create): a QwenModel first. */
typedef struct { QwenSession s; Ring c; } RefRing;

typedef struct {
    int cursor;
    uint64_t population, rng;
    int write_slot, sample_slot, active, capacity, transaction;
    unsigned long long calls, published, restores, main_tokens;
    int position, pending, delivered, phase, layer;
    unsigned depth;
    uint64_t epoch, lineage, session_id, top_frame;
    int top_first, top_second;
} RrState;

void *rr_open(void *model, int logical, int anchors, int recent, int sample, int full) {
    RefRing *r = calloc(1, sizeof(*r));
    if (!r) abort();
    ring_open(&r->c, &r->s, (const QwenModel *)model, logical, anchors, recent, sample, full);
    return r;
}
void rr_close(void *p) {
    RefRing *r = p;
    ring_close(&r->c);
    qwen_session_free(&r->s);
    free(r);
}
int rr_push(void *p, int token) { return ring_push(&((RefRing *)p)->c, token); }
int rr_begin(void *p, int token) { return ring_begin(&((RefRing *)p)->c, token); }
int rr_advance_layer(void *p) { return qwen_advance_layer(&((RefRing *)p)->s); }
int rr_finish(void *p) { return ring_finish(&((RefRing *)p)->c); }
int rr_abort(void *p) { return ring_abort(&((RefRing *)p)->c); }
int rr_mark(void *p, uint64_t *id) { return ring_mark(&((RefRing *)p)->c, id); }
int rr_rollback(void *p, uint64_t id) { return ring_rollback(&((RefRing *)p)->c, id); }
int rr_commit(void *p, uint64_t id) { return ring_commit(&((RefRing *)p)->c, id); }
/* The serve main's Z command (src/qwen_bounded_serve.c:58). */
int rr_reset(void *p) {
    RefRing *r = p;
    int e = qwen_reset(&r->s);
    if (!e) gpu_zero(r->s.logits, (size_t)r->s.model->vocab * 4);
    return e;
}
void rr_fail(void *p, int layer, int position) {
    RefRing *r = p;
    r->c.fail_layer = layer;
    r->c.fail_position = position;
}
void rr_state(void *p, RrState *o) {
    RefRing *r = p;
    const Ring *c = &r->c;
    const QwenSession *s = &r->s;
    memset(o, 0, sizeof(*o));
    o->cursor = c->view.cursor; o->population = c->view.population; o->rng = c->view.rng;
    o->write_slot = c->write_slot; o->sample_slot = c->sample_slot; o->active = c->active;
    o->capacity = c->capacity; o->transaction = c->transaction;
    o->calls = c->calls; o->published = c->published; o->restores = c->restores; o->main_tokens = c->main_tokens;
    o->position = s->position; o->pending = s->pending; o->delivered = s->delivered; o->phase = s->phase;
    o->layer = s->layer; o->depth = s->depth; o->epoch = s->epoch; o->lineage = s->lineage_id;
    o->session_id = s->session_id; o->top_frame = s->depth ? s->frames[s->depth - 1].id : 0;
    o->top_first = s->top.first; o->top_second = s->top.second;
}
void rr_positions(void *p, int *out) { RefRing *r = p; memcpy(out, r->c.positions, (size_t)r->c.capacity * 4); }
void rr_order(void *p, int *order, float *weights) {
    RefRing *r = p;
    memcpy(order, r->c.order, (size_t)r->c.active * 4);
    memcpy(weights, r->c.weights, (size_t)r->c.active * 4);
}
size_t rr_arena_bytes(void *p) { return ((RefRing *)p)->c.arena_bytes; }
void rr_arena(void *p, void *out) { RefRing *r = p; gpu_read(out, r->c.arena, r->c.arena_bytes); }
void rr_logits(void *p, float *out) { RefRing *r = p; gpu_read(out, r->s.logits, (size_t)r->s.model->vocab * 4); }
