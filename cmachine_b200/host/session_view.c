/* Flat accessors over QwenModel / QwenSession for foreign-function callers
 * (the Python mirror in cmachine_b200/__init__.py) that cannot lay out the C
 * structs themselves. Pure field reads and writes; no arithmetic. */
#include "../../include/qwen.h"
#include <string.h>

typedef struct {
    int position, capacity, pending, layer, phase, delivered, dense_layers, fused;
    unsigned depth;
    uint64_t session_id, epoch, lineage_id, checkpoint_serial, top_frame;
    TcmTop2 top;
    float *keys, *values, *x, *logits;
    size_t allocated_bytes;
    float *q, *k, *v, *attention;
} QwenSessionView;

size_t qwen_b200_model_size(void) { return sizeof(QwenModel); }
size_t qwen_b200_session_size(void) { return sizeof(QwenSession); }
size_t qwen_b200_checkpoint_size(void) { return sizeof(QwenCheckpoint); }

void qwen_b200_session_view(const QwenSession *s, QwenSessionView *v) {
    memset(v, 0, sizeof(*v));
    v->position = s->position; v->capacity = s->capacity; v->pending = s->pending; v->layer = s->layer;
    v->phase = s->phase; v->delivered = s->delivered; v->dense_layers = s->dense_layers; v->fused = s->runner != NULL;
    v->depth = s->depth; v->session_id = s->session_id; v->epoch = s->epoch; v->lineage_id = s->lineage_id;
    v->checkpoint_serial = s->checkpoint_serial; v->top_frame = s->depth ? s->frames[s->depth - 1].id : 0;
    v->top = s->top; v->keys = s->keys; v->values = s->values; v->x = s->x; v->logits = s->logits;
    v->allocated_bytes = s->allocated_bytes;
    v->q = s->q; v->k = s->k; v->v = s->v; v->attention = s->attention;
}

void qwen_b200_session_set_delivered(QwenSession *s, int delivered) { s->delivered = delivered; }

/* Benchmark aid: place a session's cursor after a context of `position` rows
 * whose K/V were written into the session's cache by other means (a seeded
 * fill), with `pending` as the next token. Only at a token boundary with no
 * stack frames; returns 0 or -1. */
int qwen_b200_session_set_cursor(QwenSession *s, int position, int pending) {
    if (s->phase == 2 || s->depth || position < 1 || position > s->capacity || pending < 0 ||
        pending >= s->model->vocab)
        return -1;
    s->position = position;
    s->pending = pending;
    s->phase = 1;
    return 0;
}

void qwen_b200_session_observe(QwenSession *s, QwenObserver observer, void *context, int position, int layer) {
    s->observer = observer;
    s->observer_context = context;
    s->observe_position = position;
    s->observe_layer = layer;
}

void qwen_b200_session_cache_guard(QwenSession *s, QwenCacheGuard guard) { s->cache_guard = guard; }

size_t qwen_b200_model_weight_bytes(const QwenModel *m) { return m->weight_bytes; }
const QwenB200Decoder *qwen_b200_model_decoder(const QwenModel *m) { return m->fused; }
/* Device pointer of a weight: layer -1 kind 0 the embedding, kind 1 the final
 * norm; layer >= 0 kinds 0..11 input norm, post norm, q, k, v, q bias, k bias,
 * v bias, o, gate, up, down. NULL when out of range. */
const void *qwen_b200_model_weight(const QwenModel *m, int layer, int kind) {
    if (layer == -1) return kind == 0 ? (const void *)m->embedding : kind == 1 ? (const void *)m->norm : NULL;
    if (layer < 0 || layer >= m->layers || kind < 0 || kind > 11) return NULL;
    const QwenLayer *L = &m->layer[layer];
    const float *all[12] = {L->input_norm, L->post_norm, L->q, L->k, L->v, L->qb, L->kb, L->vb, L->o, L->gate, L->up, L->down};
    return all[kind];
}
int qwen_b200_model_matrix_dtype(const QwenModel *m) { return m->matrix_dtype; }
QwenB200Runner *qwen_b200_session_runner(const QwenSession *s) { return s->runner; }

/* The bounded cache (include/bounded_cache.h), flattened. */
#include "../../include/bounded_cache.h"
typedef struct {
    int cursor;
    uint64_t population, rng;
    int write_slot, sample_slot, active, capacity, transaction, fused, layers, reservoir_count;
    unsigned long long calls, published, restores, main_tokens;
    size_t arena_bytes, gpu_bytes, host_bytes;
    void *arena;
    int *positions, *order;
    float *weights;
    int cut0_sample_position;  /* cuts[0].positions[sample_slot] (the slot's pre-token position), or -2 */
} QwenB200RingView;

size_t qwen_b200_ring_size(void) { return sizeof(Ring); }

void qwen_b200_ring_view(const Ring *c, QwenB200RingView *v) {
    memset(v, 0, sizeof(*v));
    v->cursor = c->view.cursor; v->population = c->view.population; v->rng = c->view.rng;
    v->write_slot = c->write_slot; v->sample_slot = c->sample_slot; v->active = c->active; v->capacity = c->capacity;
    v->transaction = c->transaction; v->fused = c->fused; v->layers = c->layers; v->reservoir_count = c->reservoir_count;
    v->calls = c->calls; v->published = c->published; v->restores = c->restores; v->main_tokens = c->main_tokens;
    v->arena_bytes = c->arena_bytes; v->gpu_bytes = c->gpu_bytes; v->host_bytes = c->host_bytes;
    v->arena = c->arena; v->positions = c->positions; v->order = c->order; v->weights = c->weights;
    v->cut0_sample_position = c->sample_slot >= 0 && c->cuts[0].positions ? c->cuts[0].positions[c->sample_slot] : -2;
}

void qwen_b200_ring_fail(Ring *c, int layer, int position) {
    c->fail_layer = layer;
    c->fail_position = position;
}
