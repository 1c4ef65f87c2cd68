/* Test infrastructure only (the oracle): a plain-C CPU restatement of the
 * reference's FP32 Qwen2.5 decode path. It is the checker for the CUDA path
 * and is never linked into, or called by, the product.
 *
 * What it restates, with the reference lines it follows:
 *   - matvec, rms, rope, cache append, GQA attention, swiglu, top-2 and BF16
 *     widening: the reference's CPU primitive set, tests/gpu_stub.c:139-177;
 *   - the dense decoder layer order: src/qwen.c:248-262 (input norm, q/k/v
 *     with bias, RoPE on q and k, cache append, attention), 275 (attention
 *     write added to x), 289 (post norm), 320 (gate/up), 329-330 (swiglu,
 *     down), 341 (residual add); qkv_apply src/qwen_operands.inc:71-84;
 *   - the readout: src/qwen.c:383-387 (final norm, tied-embedding logits,
 *     top-2, pending token, position advance).
 * Every loop keeps the reference's sequential FP32 order; built with
 * -ffp-contract=off (the reference's CFLAGS, Makefile:2) it reproduces the
 * reference CPU path bit for bit, which tests/test_oracle.py checks against
 * oracle/_ref and against the committed golden vectors. Matvec rows and
 * attention heads run in parallel (par.h); each keeps its own sequential sum,
 * so the bits do not depend on the thread count.
 */
#include "oracle_api.h"
#include "par.h"
#include "ring_cpu.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    float *input_norm, *post_norm, *q, *k, *v, *qb, *kb, *vb, *o, *gate, *up, *down;
} OrcLayer;
typedef struct {
    OrcShape shape;
    float *embedding, *norm;
    OrcLayer *layer;
} OrcModel;
/* Bounded anchors/recent/reservoir byte-codec cache (src/bounded_cache.h):
 * physical rows, the slot of each retained position (-1 empty), the view
 * (cursor, evictions, SplitMix64 state) and the arena in the reference layout,
 * per layer [K codes 2 x rows x 128][V codes][scales 4 x rows]. */
typedef struct {
    int anchors, recent, sample, rows, write_slot, sample_slot, active;
    int cursor;
    uint64_t population, rng;
    int *positions, *order;
    float *weights;
    unsigned char *arena;
} OrcRing;
typedef struct {
    const OrcModel *model;
    int position, capacity;
    float *keys, *values, *x, *norm, *q, *k, *v, *attention, *projected, *gate, *up, *logits, *scores;
    OrcRing *ring;
} OrcSession;

typedef struct { float *p; uint64_t base; TcmFill f; int bf16; } FillJob;
static void fill_body(void *c, size_t begin, size_t end) {
    FillJob *j = c;
    for (size_t i = begin; i < end; i++) {
        float value = tcm_seeded_value(j->base, i, j->f);
        j->p[i] = j->bf16 ? tcm_bf16_to_float(tcm_bf16_rne(value)) : value;
    }
}
static float *tensor(uint64_t seed, const TcmFillLaw *law, uint32_t id, size_t n, int bf16) {
    float *p = malloc(n * sizeof(float));
    if (!p) abort();
    FillJob job = {p, tcm_tensor_base(seed, id), tcm_tensor_fill(law, id), bf16};
    par_for(n, 1 << 16, fill_body, &job);
    return p;
}

void *orc_model_create(const OrcShape *shape, uint64_t seed, const TcmFillLaw *law, int bf16) {
    OrcModel *m = calloc(1, sizeof(*m));
    if (!m) abort();
    m->shape = *shape;
    int d = shape->hidden, qd = shape->qheads * shape->head, kv = shape->kvheads * shape->head, f = shape->intermediate;
    /* Matrices follow the requested storage; vectors stay FP32 (profile 2 keeps
     * vectors FP32, src/qwen_weights.inc:13). */
    m->embedding = tensor(seed, law, 0, (size_t)shape->vocab * d, bf16);
    m->norm = tensor(seed, law, 1, (size_t)d, 0);
    m->layer = calloc((size_t)shape->layers, sizeof(OrcLayer));
    if (!m->layer) abort();
    for (int l = 0; l < shape->layers; l++) {
        OrcLayer *L = &m->layer[l];
        L->input_norm = tensor(seed, law, tcm_layer_tensor(l, TCM_T_INPUT_NORM), (size_t)d, 0);
        L->post_norm = tensor(seed, law, tcm_layer_tensor(l, TCM_T_POST_NORM), (size_t)d, 0);
        L->q = tensor(seed, law, tcm_layer_tensor(l, TCM_T_Q), (size_t)qd * d, bf16);
        L->k = tensor(seed, law, tcm_layer_tensor(l, TCM_T_K), (size_t)kv * d, bf16);
        L->v = tensor(seed, law, tcm_layer_tensor(l, TCM_T_V), (size_t)kv * d, bf16);
        L->qb = tensor(seed, law, tcm_layer_tensor(l, TCM_T_QB), (size_t)qd, 0);
        L->kb = tensor(seed, law, tcm_layer_tensor(l, TCM_T_KB), (size_t)kv, 0);
        L->vb = tensor(seed, law, tcm_layer_tensor(l, TCM_T_VB), (size_t)kv, 0);
        L->o = tensor(seed, law, tcm_layer_tensor(l, TCM_T_O), (size_t)d * qd, bf16);
        L->gate = tensor(seed, law, tcm_layer_tensor(l, TCM_T_GATE), (size_t)f * d, bf16);
        L->up = tensor(seed, law, tcm_layer_tensor(l, TCM_T_UP), (size_t)f * d, bf16);
        L->down = tensor(seed, law, tcm_layer_tensor(l, TCM_T_DOWN), (size_t)d * f, bf16);
    }
    return m;
}

void orc_model_free(void *p) {
    OrcModel *m = p;
    if (!m) return;
    for (int l = 0; l < m->shape.layers; l++) {
        OrcLayer *L = &m->layer[l];
        float *all[] = {L->input_norm, L->post_norm, L->q, L->k, L->v, L->qb, L->kb, L->vb, L->o, L->gate, L->up, L->down};
        for (unsigned i = 0; i < sizeof(all) / sizeof(all[0]); i++) free(all[i]);
    }
    free(m->layer);
    free(m->embedding);
    free(m->norm);
    free(m);
}

float orc_weight_value(void *p, uint32_t id, uint64_t index) {
    OrcModel *m = p;
    if (id == 0) return m->embedding[index];
    if (id == 1) return m->norm[index];
    int l = (int)((id - 2) / TCM_T_PER_LAYER), kind = (int)((id - 2) % TCM_T_PER_LAYER);
    OrcLayer *L = &m->layer[l];
    float *all[] = {L->input_norm, L->post_norm, L->q, L->k, L->v, L->qb, L->kb, L->vb, L->o, L->gate, L->up, L->down};
    return all[kind][index];
}

void *orc_session_create(void *p, int capacity) {
    const OrcModel *m = p;
    OrcSession *s = calloc(1, sizeof(*s));
    if (!s) abort();
    const OrcShape *S = &m->shape;
    s->model = m;
    s->capacity = capacity;
    size_t kv = (size_t)S->layers * S->kvheads * capacity * S->head;
#define ORC_ALLOC(field, n) do { s->field = calloc((size_t)(n), sizeof(float)); if (!s->field) abort(); } while (0)
    ORC_ALLOC(keys, kv); ORC_ALLOC(values, kv); ORC_ALLOC(x, S->hidden); ORC_ALLOC(norm, S->hidden);
    ORC_ALLOC(q, S->qheads * S->head); ORC_ALLOC(k, S->kvheads * S->head); ORC_ALLOC(v, S->kvheads * S->head);
    ORC_ALLOC(attention, S->qheads * S->head); ORC_ALLOC(projected, S->hidden); ORC_ALLOC(gate, S->intermediate);
    ORC_ALLOC(up, S->intermediate); ORC_ALLOC(logits, S->vocab); ORC_ALLOC(scores, (size_t)S->qheads * capacity);
#undef ORC_ALLOC
    return s;
}

void orc_session_free(void *p) {
    OrcSession *s = p;
    if (!s) return;
    float *all[] = {s->keys, s->values, s->x, s->norm, s->q, s->k, s->v, s->attention, s->projected, s->gate, s->up, s->logits, s->scores};
    for (unsigned i = 0; i < sizeof(all) / sizeof(all[0]); i++) free(all[i]);
    if (s->ring) {
        free(s->ring->positions);
        free(s->ring->order);
        free(s->ring->weights);
        free(s->ring->arena);
        free(s->ring);
    }
    free(s);
}

/* tests/gpu_stub.c:143-145: one sequential FP32 dot product per output row. */
typedef struct { const float *w, *x; float *y; int in; } MatvecJob;
static void matvec_body(void *c, size_t begin, size_t end) {
    MatvecJob *m = c;
    for (size_t j = begin; j < end; j++) {
        const float *row = m->w + j * (size_t)m->in;
        float sum = 0;
        for (int i = 0; i < m->in; i++) sum += row[i] * m->x[i];
        m->y[j] = sum;
    }
}
static void matvec(const float *w, int in, int out, const float *x, float *y) {
    MatvecJob job = {w, x, y, in};
    par_for((size_t)out, 256, matvec_body, &job);
}
/* tests/gpu_stub.c:146-148: y = (x * r) * w with r = 1/sqrtf(mean(x^2) + eps). */
static void rms(float *y, const float *x, const float *w, int n, float eps) {
    float sum = 0;
    for (int i = 0; i < n; i++) sum += x[i] * x[i];
    float r = 1 / sqrtf(sum / n + eps);
    for (int i = 0; i < n; i++) y[i] = x[i] * r * w[i];
}
static void add(float *a, const float *b, int n) { for (int i = 0; i < n; i++) a[i] += b[i]; }
/* tests/gpu_stub.c:157-159: half-split rotation, angle = position / theta^(2i/d). */
static void rope(float *q, int heads, int d, int position, float theta) {
    for (int h = 0; h < heads; h++)
        for (int i = 0; i < d / 2; i++) {
            float angle = position / powf(theta, 2.0f * i / d);
            float a = q[h * d + i], b = q[h * d + i + d / 2];
            q[h * d + i] = a * cosf(angle) - b * sinf(angle);
            q[h * d + i + d / 2] = b * cosf(angle) + a * sinf(angle);
        }
}
/* tests/gpu_stub.c:160-162: row `position` of each head's [capacity][d] slab. */
static void cache_append(float *cache, const float *row, int heads, int d, int capacity, int position) {
    for (int h = 0; h < heads; h++) memcpy(cache + ((size_t)h * capacity + position) * d, row + h * d, (size_t)d * 4);
}
/* tests/gpu_stub.c:163-170: per query head h, K/V head h / (qheads/kvheads);
 * scores dot/sqrt(d); max-subtracted exp; out = sum_t (p_t / sum) * v_t. */
typedef struct { float *out; const float *q, *k, *v; float *scores; int qheads, kvheads, d, capacity, n; } AttnJob;
static void attention_body(void *c, size_t begin, size_t end) {
    AttnJob *J = c;
    float *out = J->out, *scores = J->scores;
    const float *q = J->q, *k = J->k, *v = J->v;
    int qheads = J->qheads, kvheads = J->kvheads, d = J->d, capacity = J->capacity, n = J->n;
    for (int h = (int)begin; h < (int)end; h++) {
        int group = h / (qheads / kvheads);
        float *p = scores + (size_t)h * capacity, max = -INFINITY, sum = 0;
        for (int t = 0; t < n; t++) {
            float dot = 0;
            for (int i = 0; i < d; i++) dot += q[h * d + i] * k[((size_t)group * capacity + t) * d + i];
            p[t] = dot / sqrtf((float)d);
            if (p[t] > max) max = p[t];
        }
        for (int t = 0; t < n; t++) { p[t] = expf(p[t] - max); sum += p[t]; }
        for (int i = 0; i < d; i++) {
            float a = 0;
            for (int t = 0; t < n; t++) a += p[t] / sum * v[((size_t)group * capacity + t) * d + i];
            out[h * d + i] = a;
        }
    }
}
static void attention(float *out, const float *q, const float *k, const float *v, float *scores,
                      int qheads, int kvheads, int d, int capacity, int n) {
    AttnJob job = {out, q, k, v, scores, qheads, kvheads, d, capacity, n};
    par_for((size_t)qheads, n >= 256 ? 1 : (size_t)qheads, attention_body, &job);
}
/* tests/gpu_stub.c:171. */
static void swiglu(float *gate, const float *up, int n) {
    for (int i = 0; i < n; i++) gate[i] = gate[i] / (1 + expf(-gate[i])) * up[i];
}
/* tests/gpu_stub.c:174-177: strict '>' scan, so the lower id wins ties. */
static OrcTop2 top2(const float *p, int n) {
    OrcTop2 r = {-1, -1, -INFINITY, -INFINITY};
    for (int i = 0; i < n; i++) {
        if (p[i] > r.first_value) { r.second = r.first; r.second_value = r.first_value; r.first = i; r.first_value = p[i]; }
        else if (p[i] > r.second_value) { r.second = i; r.second_value = p[i]; }
    }
    return r;
}

/* ------------------------------------------------------------------ bounded ring
 * The reference's retention policy, src/bounded_cache.h:
 *   ring_random / ring_draw  :24-25  SplitMix64 (state starts at 7) and an
 *                                     unbiased draw in [0, n) by rejection below
 *                                     (2^64 - n) mod n;
 *   ring_order               :51-57  retained slots sorted by position; reservoir
 *                                     slots weigh log(population / min(population,
 *                                     reservoir)), the others 0;
 *   ring_begin               :71-74  the write slot (anchors first, then the
 *                                     recent ring); overwriting a retained row is
 *                                     an eviction, offered to the reservoir
 *                                     (filled in order, then replaced with
 *                                     probability reservoir / evictions);
 *   ring_step / ring_copy_row :38-46,65  per layer: the sampled row copied from
 *                                     the evicted slot, the current K/V encoded
 *                                     into the write slot, ring attention. */
static uint64_t ring_next(OrcRing *r) {
    uint64_t z = (r->rng += UINT64_C(0x9e3779b97f4a7c15));
    z = (z ^ (z >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
    z = (z ^ (z >> 27)) * UINT64_C(0x94d049bb133111eb);
    return z ^ (z >> 31);
}
static uint64_t ring_draw(OrcRing *r, uint64_t n) {
    uint64_t x, t = (uint64_t)(-n) % n;
    do x = ring_next(r); while (x < t);
    return x % n;
}
static const int *sort_positions;
static int by_position(const void *a, const void *b) {
    int pa = sort_positions[*(const int *)a], pb = sort_positions[*(const int *)b];
    return (pa > pb) - (pa < pb);
}
static void ring_order(OrcRing *r) {
    r->active = 0;
    for (int i = 0; i < r->rows; i++)
        if (r->positions[i] >= 0) r->order[r->active++] = i;
    sort_positions = r->positions; /* positions are distinct: the order is unique */
    qsort(r->order, (size_t)r->active, sizeof(int), by_position);
    int m = r->population < (uint64_t)r->sample ? (int)r->population : r->sample;
    for (int i = 0; i < r->active; i++)
        r->weights[i] = (r->order[i] >= r->anchors + r->recent && m) ? logf((float)r->population / (float)m) : 0;
}
static void ring_begin(OrcRing *r, int p) {
    r->sample_slot = -1;
    r->write_slot = p < r->anchors ? p : r->anchors + (p - r->anchors) % r->recent;
    if (r->positions[r->write_slot] >= 0) {
        r->population++;
        if (r->sample) {
            uint64_t n = r->population, j = n <= (uint64_t)r->sample ? n - 1 : ring_draw(r, n);
            if (j < (uint64_t)r->sample) {
                r->sample_slot = r->anchors + r->recent + (int)j;
                r->positions[r->sample_slot] = r->positions[r->write_slot];
            }
        }
    }
    r->positions[r->write_slot] = p;
    r->cursor = p + 1;
    ring_order(r);
}
static unsigned char *ring_layer(OrcRing *r, int l) { return r->arena + (size_t)l * r->rows * ORC_RING_ROW_BYTES; }
/* ring_copy_row: the evicted row (still intact in this layer) into the sample slot. */
static void ring_copy_row(OrcRing *r, int l, int to, int from) {
    unsigned char *base = ring_layer(r, l);
    float *scales = (float *)(base + (size_t)r->rows * 512);
    for (int kind = 0; kind < 2; kind++)
        for (int h = 0; h < ORC_RING_KV; h++) {
            unsigned char *codes = base + (size_t)kind * r->rows * 256;
            memcpy(codes + ((size_t)h * r->rows + to) * 128, codes + ((size_t)h * r->rows + from) * 128, 128);
            scales[(kind * 2 + h) * r->rows + to] = scales[(kind * 2 + h) * r->rows + from];
        }
}
static int ring_layer_step(OrcSession *s, int l) {
    OrcRing *r = s->ring;
    unsigned char *base = ring_layer(r, l);
    if (r->sample_slot >= 0) ring_copy_row(r, l, r->sample_slot, r->write_slot);
    if (orc_encode_rows((signed char *)base, (signed char *)base + (size_t)r->rows * 256,
                        (float *)(base + (size_t)r->rows * 512), s->k, s->v, r->rows, r->write_slot))
        return -81;
    orc_ring_attention_cpu(s->attention, s->q, (const signed char *)base, (const signed char *)base + (size_t)r->rows * 256,
                           (const float *)(base + (size_t)r->rows * 512), r->order, r->weights, r->rows, r->active,
                           r->sample && r->population > 0);
    return 0;
}

void *orc_ring_session_create(void *model, int logical, int anchors, int recent, int sample) {
    const OrcModel *m = model;
    const OrcShape *S = &m->shape;
    if (recent < 1 || anchors < 0 || sample < 0 || anchors + recent + sample > logical || logical > S->max_position ||
        S->kvheads != ORC_RING_KV || S->head != ORC_RING_HEAD || S->qheads != ORC_RING_KV * ORC_RING_GROUP)
        return NULL;
    OrcSession *s = orc_session_create(model, 1);
    free(s->keys);
    free(s->values);
    s->keys = s->values = NULL;
    s->capacity = logical;
    OrcRing *r = calloc(1, sizeof(*r));
    if (!r) abort();
    r->anchors = anchors; r->recent = recent; r->sample = sample; r->rows = anchors + recent + sample;
    r->rng = 7;
    r->positions = malloc((size_t)r->rows * sizeof(int));
    r->order = malloc((size_t)r->rows * sizeof(int));
    r->weights = malloc((size_t)r->rows * sizeof(float));
    r->arena = calloc((size_t)S->layers * r->rows, ORC_RING_ROW_BYTES);
    if (!r->positions || !r->order || !r->weights || !r->arena) abort();
    for (int i = 0; i < r->rows; i++) r->positions[i] = -1;
    s->ring = r;
    return s;
}

int orc_ring_read(void *session, OrcRingView *view, int *positions, int *order, float *weights, void *arena) {
    OrcSession *s = session;
    OrcRing *r = s->ring;
    if (!r) return -1;
    if (view) {
        view->cursor = r->cursor; view->population = r->population; view->rng = r->rng;
        view->write_slot = r->write_slot; view->sample_slot = r->sample_slot; view->active = r->active;
        view->rows = r->rows;
    }
    if (positions) memcpy(positions, r->positions, (size_t)r->rows * sizeof(int));
    if (order) memcpy(order, r->order, (size_t)r->active * sizeof(int));
    if (weights) memcpy(weights, r->weights, (size_t)r->active * sizeof(float));
    if (arena) memcpy(arena, r->arena, (size_t)s->model->shape.layers * r->rows * ORC_RING_ROW_BYTES);
    return 0;
}

int orc_codec(const float *x, int8_t *codes, float *scale) { return orc_codec_row(x, codes, scale); }

void orc_ring_attention(float *out, const float *q, const signed char *key, const signed char *value,
                        const float *scales, const int *order, const float *weights, int capacity, int length,
                        int weighted) {
    orc_ring_attention_cpu(out, q, key, value, scales, order, weights, capacity, length, weighted);
}

int orc_push(void *p, int token, OrcTop2 *top, float *logits) {
    OrcSession *s = p;
    const OrcModel *m = s->model;
    const OrcShape *S = &m->shape;
    if (token < 0 || token >= S->vocab || s->position >= s->capacity) return -1;
    int d = S->hidden, qd = S->qheads * S->head, kv = S->kvheads * S->head, f = S->intermediate;
    if (s->ring) ring_begin(s->ring, s->position);
    memcpy(s->x, m->embedding + (size_t)token * d, (size_t)d * 4);
    for (int l = 0; l < S->layers; l++) {
        const OrcLayer *L = &m->layer[l];
        rms(s->norm, s->x, L->input_norm, d, S->epsilon);
        matvec(L->q, d, qd, s->norm, s->q); add(s->q, L->qb, qd);
        matvec(L->k, d, kv, s->norm, s->k); add(s->k, L->kb, kv);
        matvec(L->v, d, kv, s->norm, s->v); add(s->v, L->vb, kv);
        rope(s->q, S->qheads, S->head, s->position, S->theta);
        rope(s->k, S->kvheads, S->head, s->position, S->theta);
        if (s->ring) {
            if (ring_layer_step(s, l)) return -81;
        } else {
            size_t base = (size_t)l * S->kvheads * s->capacity * S->head;
            cache_append(s->keys + base, s->k, S->kvheads, S->head, s->capacity, s->position);
            cache_append(s->values + base, s->v, S->kvheads, S->head, s->capacity, s->position);
            attention(s->attention, s->q, s->keys + base, s->values + base, s->scores, S->qheads, S->kvheads, S->head,
                      s->capacity, s->position + 1);
        }
        matvec(L->o, qd, d, s->attention, s->projected);
        add(s->x, s->projected, d);
        rms(s->norm, s->x, L->post_norm, d, S->epsilon);
        matvec(L->gate, d, f, s->norm, s->gate);
        matvec(L->up, d, f, s->norm, s->up);
        swiglu(s->gate, s->up, f);
        matvec(L->down, f, d, s->gate, s->projected);
        add(s->x, s->projected, d);
    }
    s->position++;
    if (!top) return 0; /* prefill without a readout: K/V and x only */
    rms(s->norm, s->x, m->norm, d, S->epsilon);
    matvec(m->embedding, d, S->vocab, s->norm, s->logits);
    *top = top2(s->logits, S->vocab);
    if (logits) memcpy(logits, s->logits, (size_t)S->vocab * 4);
    return 0;
}

int orc_position(void *p) { return ((OrcSession *)p)->position; }

void orc_read_kv(void *p, int layer, int kind, float *out) {
    OrcSession *s = p;
    const OrcShape *S = &s->model->shape;
    const float *src = (kind ? s->values : s->keys) + (size_t)layer * S->kvheads * s->capacity * S->head;
    for (int h = 0; h < S->kvheads; h++)
        memcpy(out + (size_t)h * s->position * S->head, src + (size_t)h * s->capacity * S->head,
               (size_t)s->position * S->head * 4);
}

void orc_read_hidden(void *p, float *out) {
    OrcSession *s = p;
    memcpy(out, s->x, (size_t)s->model->shape.hidden * 4);
}

void orc_write_kv(void *p, int layer, int kind, int rows, const float *in) {
    OrcSession *s = p;
    const OrcShape *S = &s->model->shape;
    float *dst = (kind ? s->values : s->keys) + (size_t)layer * S->kvheads * s->capacity * S->head;
    for (int h = 0; h < S->kvheads; h++)
        memcpy(dst + (size_t)h * s->capacity * S->head, in + (size_t)h * rows * S->head, (size_t)rows * S->head * 4);
}

int orc_set_cursor(void *p, int position) {
    OrcSession *s = p;
    if (s->ring || position < 0 || position >= s->capacity) return -1;
    s->position = position;
    return 0;
}
