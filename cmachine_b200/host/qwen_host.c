/* The Qwen2.5 session state machine over the B200 decoder (include/qwen.h).
 *
 * Host-side semantics restated from the reference (src/qwen.c):
 *   session allocation and cache layout        :50-60
 *   token begin guards and token-parent cut    :75-81
 *   the dense layer and its observer ports     :216-368 (dense path only)
 *   finish / push / advance                    :383-393
 *   cursor checkpoint, restore, abort          :394-415
 *   nested stack push / rollback / commit      :416-432
 *   reset                                      :433-437
 * Lineage, session and frame ids come from process-wide atomics as in the
 * reference (:11-19). The arithmetic runs on the fused B200 kernels; a layer
 * with an armed observer runs the primitive sequence so every port exists.
 */
#include "../../include/qwen.h"
#include <math.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static _Atomic uint64_t next_session_id = 1;
static _Atomic uint64_t next_frame_id = 1;
static _Atomic uint64_t next_lineage_id = 1;

/* A fresh id from a counter that refuses to wrap (src/qwen.c:15-19). */
static int take_id(_Atomic uint64_t *counter, uint64_t *id) {
    uint64_t next = atomic_load(counter);
    do {
        if (next == UINT64_MAX) return -1;
    } while (!atomic_compare_exchange_weak(counter, &next, next + 1));
    *id = next;
    return 0;
}

/* ------------------------------------------------------------------ model */

static float *model_tensor(QwenModel *m, uint64_t seed, const TcmFillLaw *law, uint32_t id, int rows, int cols,
                           int bf16) {
    const size_t n = (size_t)rows * (cols > 0 ? cols : 1);
    const int matrix = cols > 0;
    const int dtype = matrix && bf16 ? 2 : 1;
    float *p = gpu_alloc(n * (dtype == 2 ? 2 : 4));
    TcmFill f = tcm_tensor_fill(law, id);
    qwen_b200_seeded_fill(p, dtype, seed, id, n, f.offset, f.scale);
    if (matrix && bf16) qwen_b200_register_matrix(p, rows, cols, 1);
    m->allocations[m->allocation_count++] = p;
    m->weight_bytes += n * (dtype == 2 ? 2 : 4);
    return p;
}

int qwen_model_init_seeded(QwenModel *m, const QwenB200Shape *shape, uint64_t seed, const TcmFillLaw *law,
                           int weight_profile, int fused) {
    memset(m, 0, sizeof(*m));
    const QwenB200Shape *s = shape;
    if (s->hidden < 1 || s->layers < 1 || s->layers > 64 || s->qheads < 1 || s->kvheads < 1 ||
        s->qheads % s->kvheads || s->head < 2 || s->head % 2 || s->intermediate < 1 || s->vocab < 1 ||
        s->max_position < 1 || (weight_profile != 0 && weight_profile != 2))
        return -1;
    const int bf16 = weight_profile == 2;
    m->hidden = s->hidden; m->layers = s->layers; m->qheads = s->qheads; m->kvheads = s->kvheads;
    m->head = s->head; m->intermediate = s->intermediate; m->vocab = s->vocab; m->max_position = s->max_position;
    m->epsilon = s->epsilon; m->theta = s->theta; m->eos = -1; m->eos_extra = 0;
    snprintf(m->identity, sizeof(m->identity), "seeded-%016llx", (unsigned long long)seed);
    snprintf(m->digest, sizeof(m->digest), "seeded-%016llx-%08x-%08x-%d", (unsigned long long)seed,
             (unsigned)(law->matrix.scale * 1e6f), (unsigned)s->layers, weight_profile);
    m->allocations = calloc(2 + 12 * (size_t)s->layers, sizeof(float *));
    m->layer = calloc((size_t)s->layers, sizeof(QwenLayer));
    if (!m->allocations || !m->layer) { free(m->allocations); free(m->layer); memset(m, 0, sizeof(*m)); return -1; }
    m->gpu = gpu_open();
    m->matrix_dtype = bf16 ? 2 : 1;
    const int d = s->hidden, kv = s->kvheads * s->head, f = s->intermediate;
    m->embedding = model_tensor(m, seed, law, 0, s->vocab, d, bf16);
    m->norm = model_tensor(m, seed, law, 1, d, 0, bf16);
    for (int l = 0; l < s->layers; l++) {
        QwenLayer *L = &m->layer[l];
        L->input_norm = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_INPUT_NORM), d, 0, bf16);
        L->post_norm = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_POST_NORM), d, 0, bf16);
        L->q = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_Q), s->qheads * s->head, d, bf16);
        L->k = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_K), kv, d, bf16);
        L->v = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_V), kv, d, bf16);
        L->qb = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_QB), s->qheads * s->head, 0, bf16);
        L->kb = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_KB), kv, 0, bf16);
        L->vb = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_VB), kv, 0, bf16);
        L->o = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_O), d, s->qheads * s->head, bf16);
        L->gate = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_GATE), f, d, bf16);
        L->up = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_UP), f, d, bf16);
        L->down = model_tensor(m, seed, law, tcm_layer_tensor(l, TCM_T_DOWN), d, f, bf16);
    }
    if (fused) {
        QwenB200Layer *layers = calloc((size_t)s->layers, sizeof(QwenB200Layer));
        if (!layers) { qwen_model_free(m); return -1; }
        for (int l = 0; l < s->layers; l++) {
            const QwenLayer *L = &m->layer[l];
            QwenB200Layer b = {L->input_norm, L->post_norm, L->q, L->k, L->v, L->qb, L->kb, L->vb, L->o, L->gate, L->up, L->down};
            layers[l] = b;
        }
        m->fused = qwen_b200_decoder_create(s, m->embedding, m->norm, layers, m->matrix_dtype);
        free(layers);
        if (!m->fused) { qwen_model_free(m); return -1; }
    }
    gpu_sync();
    return 0;
}

/* One bundle tensor into device memory (the reference's loader helper,
 * src/qwen.c:21-24): the name must exist with the given rank and leading
 * dimensions in FP32 or BF16. */
static float *bundle_weight(QwenModel *m, const TcmModel *b, const char *name, int rank, int rows, int cols) {
    const TcmTensor *t = tcm_tensor(b, name);
    if (!t || t->rank != (uint32_t)rank || t->dim[0] != (uint64_t)rows || (rank == 2 && t->dim[1] != (uint64_t)cols) ||
        (t->dtype != TCM_F32 && t->dtype != TCM_BF16))
        return NULL;
    const size_t count = t->bytes / (t->dtype == TCM_F32 ? 4 : 2);
    float *p = gpu_owned_weight(m->gpu, t->data, t->dtype, count, rank, rows, cols);
    m->allocations[m->allocation_count++] = p;
    m->weight_bytes += gpu_owned_weight_bytes(p, count);
    return p;
}

int qwen_model_init(QwenModel *m, const TcmModel *b, char *error, size_t capacity) {
    memset(m, 0, sizeof(*m));
    const uint32_t *c = b->config;
    if (b->architecture != TCM_QWEN || b->count != 338 || c[0] != 1536 || c[1] != 28 || c[2] != 12 || c[3] != 2 ||
        c[4] != 128 || c[5] != 8960 || c[6] != 151936 || c[10] != 32768) {
        snprintf(error, capacity, "unsupported Qwen2.5-1.5B profile");
        return -1;
    }
    m->hidden = (int)c[0]; m->layers = (int)c[1]; m->qheads = (int)c[2]; m->kvheads = (int)c[3]; m->head = (int)c[4];
    m->intermediate = (int)c[5]; m->vocab = (int)c[6]; m->eos = (int)c[9]; m->max_position = (int)c[10];
    m->eos_extra = (int)c[12];
    memcpy(&m->epsilon, &c[7], 4);
    memcpy(&m->theta, &c[8], 4);
    memcpy(m->identity, b->identity, 65);
    memcpy(m->digest, b->digest, 65);
    if (m->epsilon != 1e-6f || m->theta != 1e6f || c[11] != 1) {
        snprintf(error, capacity, "Qwen numerical configuration differs");
        memset(m, 0, sizeof(*m));
        return -1;
    }
    m->allocations = calloc(b->count, sizeof(float *));
    m->layer = calloc((size_t)m->layers, sizeof(QwenLayer));
    if (!m->allocations || !m->layer) {
        snprintf(error, capacity, "Qwen descriptor allocation failed");
        qwen_model_free(m);
        return -1;
    }
    m->gpu = gpu_open();
    const int d = m->hidden, kv = m->kvheads * m->head, f = m->intermediate;
    int bad = 0;
    m->embedding = bundle_weight(m, b, "model.embed_tokens.weight", 2, m->vocab, d);
    m->norm = bundle_weight(m, b, "model.norm.weight", 1, d, 0);
    bad |= !m->embedding || !m->norm;
    for (int i = 0; i < m->layers; i++) {
        QwenLayer *L = &m->layer[i];
        struct { float **field; const char *suffix; int rank, rows, cols; } spec[] = {
            {&L->input_norm, "input_layernorm.weight", 1, d, 0}, {&L->post_norm, "post_attention_layernorm.weight", 1, d, 0},
            {&L->q, "self_attn.q_proj.weight", 2, d, d}, {&L->k, "self_attn.k_proj.weight", 2, kv, d},
            {&L->v, "self_attn.v_proj.weight", 2, kv, d}, {&L->qb, "self_attn.q_proj.bias", 1, d, 0},
            {&L->kb, "self_attn.k_proj.bias", 1, kv, 0}, {&L->vb, "self_attn.v_proj.bias", 1, kv, 0},
            {&L->o, "self_attn.o_proj.weight", 2, d, d}, {&L->gate, "mlp.gate_proj.weight", 2, f, d},
            {&L->up, "mlp.up_proj.weight", 2, f, d}, {&L->down, "mlp.down_proj.weight", 2, d, f}};
        for (size_t j = 0; j < sizeof(spec) / sizeof(spec[0]); j++) {
            char name[64];
            snprintf(name, sizeof(name), "model.layers.%d.%s", i, spec[j].suffix);
            *spec[j].field = bundle_weight(m, b, name, spec[j].rank, spec[j].rows, spec[j].cols);
            bad |= !*spec[j].field;
        }
    }
    if (bad || m->allocation_count != 338) {
        snprintf(error, capacity, "Qwen tensor names/shapes differ");
        qwen_model_free(m);
        return -1;
    }
    /* The fused decoder reads the matrices in their stored type. */
    QwenB200Shape shape = {m->hidden, m->layers, m->qheads, m->kvheads, m->head, m->intermediate, m->vocab,
                           m->max_position, m->epsilon, m->theta};
    QwenB200Layer *layers = calloc((size_t)m->layers, sizeof(QwenB200Layer));
    if (layers) {
        for (int l = 0; l < m->layers; l++) {
            const QwenLayer *L = &m->layer[l];
            QwenB200Layer one = {L->input_norm, L->post_norm, L->q, L->k, L->v, L->qb, L->kb, L->vb, L->o, L->gate, L->up, L->down};
            layers[l] = one;
        }
        m->fused = qwen_b200_decoder_create(&shape, m->embedding, m->norm, layers, 0);
        free(layers);
    }
    m->matrix_dtype = qwen_b200_weight_dtype(m->embedding);
    gpu_sync();
    return 0;
}

void qwen_model_free(QwenModel *m) {
    if (!m) return;
    qwen_b200_batch_free(m->batch);
    qwen_b200_decoder_free(m->fused);
    for (unsigned i = 0; i < m->allocation_count; i++) {
        qwen_b200_unregister_matrix(m->allocations[i]);
        gpu_free(m->allocations[i]);
    }
    free(m->allocations);
    free(m->layer);
    if (m->gpu) gpu_close(m->gpu);
    memset(m, 0, sizeof(*m));
}

/* ------------------------------------------------------------------ session */

int qwen_session_init(QwenSession *s, const QwenModel *m, int capacity) {
    return qwen_session_init_layout(s, m, capacity, 0, NULL, NULL, NULL);
}

/* src/qwen.c:50-60: dense layers own FP32 K/V slabs [slot][kvheads][capacity][head];
 * layers selected by `mask` are served by the cache callbacks instead. */
int qwen_session_init_layout(QwenSession *s, const QwenModel *m, int capacity, uint64_t mask, QwenCacheStep step,
                             QwenCacheRewind rewind, void *context) {
    memset(s, 0, sizeof(*s));
    uint64_t lineage;
    if (capacity < 1 || capacity > m->max_position || take_id(&next_lineage_id, &lineage)) return -1;
    if (m->layers < 1 || m->layers > 64 || (m->layers < 64 && (mask >> m->layers)) || (mask && (!step || !rewind)))
        return -1;
    s->model = m;
    s->capacity = capacity;
    s->pending = -1;
    s->session_id = atomic_fetch_add(&next_session_id, 1);
    s->epoch = 1;
    s->lineage_id = lineage;
    s->observe_position = s->observe_layer = -1;
    s->cache_mask = mask;
    s->cache_step = step;
    s->cache_rewind = rewind;
    s->cache_context = context;
    for (int i = 0; i < m->layers; i++) s->cache_slots[i] = (mask & (UINT64_C(1) << i)) ? -1 : s->dense_layers++;
    const size_t kv = (size_t)s->dense_layers * m->kvheads * capacity * m->head;
#define SESSION_ALLOC(field, n)                                                        \
    do {                                                                               \
        size_t count_ = (size_t)(n);                                                   \
        s->field = count_ ? gpu_alloc(count_ * sizeof(float)) : NULL;                  \
        s->allocated_bytes += count_ * sizeof(float);                                  \
    } while (0)
    SESSION_ALLOC(keys, kv); SESSION_ALLOC(values, kv); SESSION_ALLOC(x, m->hidden); SESSION_ALLOC(norm, m->hidden);
    SESSION_ALLOC(q, m->qheads * m->head); SESSION_ALLOC(k, m->kvheads * m->head); SESSION_ALLOC(v, m->kvheads * m->head);
    SESSION_ALLOC(attention, m->qheads * m->head); SESSION_ALLOC(projected, m->hidden);
    SESSION_ALLOC(gate, m->intermediate); SESSION_ALLOC(up, m->intermediate); SESSION_ALLOC(logits, m->vocab);
    SESSION_ALLOC(scores, (size_t)m->qheads * capacity);
#undef SESSION_ALLOC
    if (kv) { gpu_zero(s->keys, kv * 4); gpu_zero(s->values, kv * 4); }
    if (m->fused) {
        QwenB200Buffers b = {s->keys, s->values, capacity, s->cache_slots, s->x, s->q, s->k, s->v, s->attention,
                             s->gate, s->logits};
        s->runner = qwen_b200_runner_create(m->fused, &b);
    }
    return 0;
}

void qwen_session_free(QwenSession *s) {
    qwen_b200_runner_free(s->runner);
    float *all[] = {s->keys, s->values, s->x, s->norm, s->q, s->k, s->v, s->attention, s->projected, s->gate, s->up,
                    s->logits, s->scores};
    for (unsigned i = 0; i < sizeof(all) / sizeof(all[0]); i++) gpu_free(all[i]);
    memset(s, 0, sizeof(*s));
}

const char *qwen_port_name(QwenPort port) {
    static const char *names[] = {"input", "query", "key", "value", "attention", "mlp_input", "mlp_gate", "mlp_up",
                                  "mlp_return", "output", "attention_write", "raw_receiver",
                                  "consumed_attention_write", "consumed_mlp_write"};
    return port >= 0 && port < QWEN_PORT_COUNT ? names[port] : NULL;
}

static int observing(const QwenSession *s, int layer) {
    return s->observer && s->position == s->observe_position && layer == s->observe_layer;
}
static void observe(QwenSession *s, QwenPort port, const float *data, size_t count) {
    if (observing(s, s->layer)) s->observer(s->observer_context, s->position, s->layer, port, data, count);
}

/* src/qwen.c:389-392 snapshot: the cursor state, no K/V copy. */
static void snapshot(const QwenSession *s, QwenCheckpoint *c) {
    memset(c, 0, sizeof(*c));
    memcpy(c->model_digest, s->model->digest, 65);
    c->position = s->position; c->pending = s->pending; c->capacity = s->capacity; c->delivered = s->delivered;
    c->top = s->top; c->session_id = s->session_id; c->epoch = s->epoch; c->lineage_id = s->lineage_id;
}
/* src/qwen.c:398-402: the backend rewinds its bytes, then the cursor returns. */
static void restore(QwenSession *s, const QwenCheckpoint *c) {
    if (s->cache_rewind) s->cache_rewind(s->cache_context, c->position, s->session_id, s->epoch);
    s->token_parent_valid = 0;
    s->position = c->position; s->pending = c->pending; s->delivered = c->delivered; s->top = c->top;
    s->phase = 0; s->layer = 0; s->lineage_id = c->lineage_id;
}

/* Guards shared by begin_token and the fused push (src/qwen.c:76-78). */
static int begin_guards(QwenSession *s, int token) {
    const QwenModel *m = s->model;
    if (token < 0 || token >= m->vocab || s->position >= s->capacity || s->phase == 2) return -1;
    if (s->cache_guard && s->cache_guard(s->cache_context, 0, s->position, s->session_id, s->epoch, s->lineage_id))
        return -1;
    return 0;
}

int qwen_begin_token(QwenSession *s, int token) {
    if (begin_guards(s, token)) return -1;
    const QwenModel *m = s->model;
    snapshot(s, &s->token_parent);
    s->token_parent_valid = 1;
    s->phase = 2; s->layer = 0; s->current_token = token;
    gpu_owned_embedding(s->x, m->embedding, token, m->hidden);
    if (s->runner && qwen_b200_begin(s->runner, token, s->position)) return -1;
    return 0;
}

/* The reference's dense layer on the primitives, with every observer port
 * (src/qwen.c:248-262,275,289,320,329-330,341 and the observe calls between). */
static int primitive_layer(QwenSession *s, int i) {
    const QwenModel *m = s->model;
    const QwenLayer *l = &m->layer[i];
    const int d = m->hidden, k = m->kvheads * m->head, qd = m->qheads * m->head;
    observe(s, QWEN_INPUT, s->x, (size_t)d);
    gpu_rms(s->norm, s->x, l->input_norm, d, m->epsilon);
    gpu_matvec(m->gpu, l->q, d, qd, s->norm, s->q); gpu_bias(s->q, l->qb, qd);
    gpu_matvec(m->gpu, l->k, d, k, s->norm, s->k); gpu_bias(s->k, l->kb, k);
    gpu_matvec(m->gpu, l->v, d, k, s->norm, s->v); gpu_bias(s->v, l->vb, k);
    gpu_rope(s->q, m->qheads, m->head, s->position, m->theta);
    gpu_rope(s->k, m->kvheads, m->head, s->position, m->theta);
    observe(s, QWEN_QUERY, s->q, (size_t)qd);
    observe(s, QWEN_KEY, s->k, (size_t)k);
    observe(s, QWEN_VALUE, s->v, (size_t)k);
    if (s->cache_slots[i] < 0) {
        if (!s->cache_step) return -1;
        int error = s->cache_step(s->cache_context, i, s->position, s->q, s->k, s->v, s->attention, s->scores);
        if (error) return error;
    } else {
        size_t base = (size_t)s->cache_slots[i] * m->kvheads * s->capacity * m->head;
        gpu_cache(s->keys + base, s->k, m->kvheads, m->head, s->capacity, s->position);
        gpu_cache(s->values + base, s->v, m->kvheads, m->head, s->capacity, s->position);
        gpu_attention(m->gpu, s->attention, s->q, s->keys + base, s->values + base, s->scores, m->qheads, m->kvheads,
                      m->head, s->capacity, s->position + 1);
    }
    observe(s, QWEN_ATTENTION, s->attention, (size_t)qd);
    gpu_matvec(m->gpu, l->o, qd, d, s->attention, s->projected);
    observe(s, QWEN_ATTENTION_WRITE, s->projected, (size_t)d);
    observe(s, QWEN_CONSUMED_ATTENTION_WRITE, s->projected, (size_t)d);
    gpu_add(s->x, s->projected, d);
    observe(s, QWEN_RAW_RECEIVER, s->x, (size_t)d);
    gpu_rms(s->norm, s->x, l->post_norm, d, m->epsilon);
    observe(s, QWEN_MLP_INPUT, s->norm, (size_t)d);
    gpu_matvec(m->gpu, l->gate, d, m->intermediate, s->norm, s->gate);
    gpu_matvec(m->gpu, l->up, d, m->intermediate, s->norm, s->up);
    observe(s, QWEN_MLP_GATE, s->gate, (size_t)m->intermediate);
    observe(s, QWEN_MLP_UP, s->up, (size_t)m->intermediate);
    gpu_swiglu(s->gate, s->up, m->intermediate);
    gpu_matvec(m->gpu, l->down, m->intermediate, d, s->gate, s->projected);
    observe(s, QWEN_CONSUMED_MLP_WRITE, s->projected, (size_t)d);
    gpu_add(s->x, s->projected, d);
    observe(s, QWEN_MLP_RETURN, s->projected, (size_t)d);
    observe(s, QWEN_OUTPUT, s->x, (size_t)d);
    return 0;
}

/* One layer on the fused kernels; a cache-callback layer runs the callback
 * between the q/k/v stage and the MLP stages (src/qwen.c:253-255). */
static int fused_layer(QwenSession *s, int i) {
    if (s->cache_slots[i] >= 0) return qwen_b200_layer(s->runner, i) ? -1 : 0;
    if (!s->cache_step) return -1;
    if (qwen_b200_layer_qkv(s->runner, i)) return -1;
    int error = s->cache_step(s->cache_context, i, s->position, s->q, s->k, s->v, s->attention, s->scores);
    if (error) return error;
    return qwen_b200_layer_mlp(s->runner, i) ? -1 : 0;
}

int qwen_advance_layer(QwenSession *s) {
    const QwenModel *m = s->model;
    if (s->phase != 2 || s->layer >= m->layers) return -1;
    const int i = s->layer;
    /* A tensor-parallel group runs only its fused split layers. */
    if (s->runner && observing(s, i) && qwen_b200_tp_world(s->runner) > 1) return -1;
    int error = (s->runner && !observing(s, i)) ? fused_layer(s, i) : primitive_layer(s, i);
    if (error) return error;
    s->layer++;
    return 0;
}

/* src/qwen.c:383-387. Non-finite logits are fatal, as in gpu_top2. */
static void finish_bookkeeping(QwenSession *s, uint64_t lineage) {
    s->pending = s->top.first;
    s->delivered = 0;
    s->position++;
    s->layer = s->model->layers;
    s->phase = 1;
    s->lineage_id = lineage;
    s->token_parent_valid = 0;
}

int qwen_finish_token(QwenSession *s) {
    const QwenModel *m = s->model;
    uint64_t lineage;
    if (s->phase != 2 || s->layer != m->layers || take_id(&next_lineage_id, &lineage)) return -1;
    if (s->runner) {
        int status = qwen_b200_finish(s->runner, &s->top);
        if (status == -3) { fprintf(stderr, "non-finite Qwen logits\n"); exit(2); }
        if (status) return -1;
    } else {
        gpu_rms(s->norm, s->x, m->norm, m->hidden, m->epsilon);
        gpu_matvec(m->gpu, m->embedding, m->hidden, m->vocab, s->norm, s->logits);
        s->top = gpu_top2(m->gpu, s->logits, m->vocab);
    }
    finish_bookkeeping(s, lineage);
    return 0;
}

int qwen_complete_token(QwenSession *s) {
    const QwenModel *m = s->model;
    if (s->phase != 2 || s->layer != 0) return -1;
    const int observed = s->observer && s->observe_position == s->position;
    if (!s->runner || observed || !qwen_b200_can_complete(s->runner)) {
        while (s->layer < m->layers) {
            int error = qwen_advance_layer(s);
            if (error) return error;
        }
        return qwen_finish_token(s);
    }
    int status = qwen_b200_complete(s->runner, &s->top);
    if (status == -3) { fprintf(stderr, "non-finite Qwen logits\n"); exit(2); }
    if (status == -5) return -81;
    uint64_t lineage;
    if (status || take_id(&next_lineage_id, &lineage)) return -1;
    s->layer = m->layers;
    finish_bookkeeping(s, lineage);
    return 0;
}

/* The whole token is one fused graph when no port is observed at this
 * position and every layer keeps its K/V in the session. */
static int fused_token_ok(const QwenSession *s) {
    if (!s->runner || s->cache_mask) return 0;
    return !(s->observer && s->observe_position == s->position);
}

int qwen_push(QwenSession *s, int token) {
    if (!fused_token_ok(s)) {
        if (qwen_begin_token(s, token)) return -1;
        while (s->layer < s->model->layers)
            if (qwen_advance_layer(s)) return -1;
        return qwen_finish_token(s);
    }
    if (begin_guards(s, token)) return -1;
    uint64_t lineage;
    if (take_id(&next_lineage_id, &lineage)) return -1;
    snapshot(s, &s->token_parent);
    s->current_token = token;
    int status = qwen_b200_token(s->runner, token, s->position, &s->top);
    if (status == -3) { fprintf(stderr, "non-finite Qwen logits\n"); exit(2); }
    if (status) return -1;
    finish_bookkeeping(s, lineage);
    return 0;
}

int qwen_advance(QwenSession *s) { return qwen_push(s, s->pending); }

int qwen_generate(QwenSession *s, int n, int *ids) {
    if (n < 1 || !fused_token_ok(s) || s->phase == 2 || s->pending < 0 || s->position + n > s->capacity) return -1;
    if (s->observer && s->observe_position >= s->position && s->observe_position < s->position + n) return -1;
    if (begin_guards(s, s->pending)) return -1;
    TcmTop2 *tops = malloc((size_t)n * sizeof(TcmTop2));
    uint64_t *lineages = malloc((size_t)n * sizeof(uint64_t));
    if (!tops || !lineages) { free(tops); free(lineages); return -1; }
    for (int i = 0; i < n; i++)
        if (take_id(&next_lineage_id, &lineages[i])) { free(tops); free(lineages); return -1; }
    int status = qwen_b200_generate(s->runner, s->pending, s->position, n, ids, tops);
    if (status == -3) { fprintf(stderr, "non-finite Qwen logits\n"); exit(2); }
    if (status) { free(tops); free(lineages); return -1; }
    for (int i = 0; i < n; i++) {
        s->current_token = s->pending;
        s->top = tops[i];
        finish_bookkeeping(s, lineages[i]);
    }
    free(tops);
    free(lineages);
    return 0;
}

int qwen_push_batch(QwenSession **ss, int n, const int *tokens) {
    if (!ss || !tokens || n < 1 || n > qwen_b200_batch_max()) return -1;
    QwenModel *m = (QwenModel *)ss[0]->model;
    if (!m->fused || m->matrix_dtype != 2) return -1;
    for (int i = 0; i < n; i++) {
        QwenSession *s = ss[i];
        if (s->model != m || !fused_token_ok(s) || begin_guards(s, tokens[i]) || s->position >= 9216) return -1;
        for (int j = 0; j < i; j++)
            if (ss[j] == s) return -1;
    }
    if (!m->batch) m->batch = qwen_b200_batch_create(m->fused);
    if (!m->batch) return -1;
    QwenB200BatchSession *bs = malloc((size_t)n * sizeof(*bs));
    int *positions = malloc((size_t)n * sizeof(int));
    uint64_t *lineages = malloc((size_t)n * sizeof(uint64_t));
    TcmTop2 *tops = malloc((size_t)n * sizeof(TcmTop2));
    int status = -1;
    if (!bs || !positions || !lineages || !tops) goto done;
    for (int i = 0; i < n; i++) {
        QwenSession *s = ss[i];
        QwenB200BatchSession b = {s->keys, s->values, s->capacity, s->logits, s->x};
        bs[i] = b;
        positions[i] = s->position;
    }
    status = qwen_b200_batch_step(m->batch, n, bs, tokens, positions, tops);
    if (status == -3) { fprintf(stderr, "non-finite Qwen logits\n"); exit(2); }
    if (status) { status = -1; goto done; }
    for (int i = 0; i < n; i++)
        if (take_id(&next_lineage_id, &lineages[i])) { status = -1; goto done; }
    for (int i = 0; i < n; i++) {
        QwenSession *s = ss[i];
        snapshot(s, &s->token_parent);
        s->current_token = tokens[i];
        s->top = tops[i];
        finish_bookkeeping(s, lineages[i]);
    }
done:
    free(bs);
    free(positions);
    free(lineages);
    free(tops);
    return status;
}

int qwen_prefill(QwenSession *s, const int *tokens, int n) {
    if (!s || !tokens || n < 1 || s->phase == 2 || n > s->capacity - s->position) return -1;
    QwenModel *m = (QwenModel *)s->model;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= m->vocab) return -1;
    const int batched = m->fused && m->matrix_dtype == 2 && fused_token_ok(s) && !s->observer && !s->cache_guard &&
                        s->position + n <= 9216;
    if (batched && !m->batch) m->batch = qwen_b200_batch_create(m->fused);
    if (!batched || !m->batch) {
        for (int i = 0; i < n; i++)
            if (qwen_push(s, tokens[i])) return -1;
        return 0;
    }
    QwenB200BatchSession b = {s->keys, s->values, s->capacity, s->logits, s->x};
    for (int done = 0; done < n;) {
        const int c = n - done < qwen_b200_batch_max() ? n - done : qwen_b200_batch_max();
        TcmTop2 top;
        int status = qwen_b200_batch_prefill(m->batch, &b, tokens + done, c, s->position, &top);
        if (status == -3) { fprintf(stderr, "non-finite Qwen logits\n"); exit(2); }
        if (status) return -1;
        uint64_t lineage = 0;
        for (int i = 0; i < c; i++)
            if (take_id(&next_lineage_id, &lineage)) return -1;
        snapshot(s, &s->token_parent);
        s->current_token = tokens[done + c - 1];
        s->top = top;
        s->position += c - 1;
        finish_bookkeeping(s, lineage);
        done += c;
    }
    return 0;
}

/* ------------------------------------------------------------------ checkpoints */

static int at_boundary(const QwenSession *s) {
    return (s->phase == 0 || s->phase == 1) && s->position > 0 && s->pending >= 0;
}

int qwen_abort_token(QwenSession *s) {
    if (!s || s->phase != 2 || !s->token_parent_valid || s->token_parent.session_id != s->session_id ||
        s->token_parent.epoch != s->epoch)
        return -1;
    if (s->cache_guard && s->cache_guard(s->cache_context, 1, s->token_parent.position, s->session_id, s->epoch,
                                         s->token_parent.lineage_id))
        return -1;
    restore(s, &s->token_parent);
    return 0;
}

int qwen_checkpoint(QwenSession *s, QwenCheckpoint *c) {
    if (!at_boundary(s)) return -1;
    snapshot(s, c);
    c->serial = ++s->checkpoint_serial;
    s->checkpoint_position = s->position;
    return 0;
}

int qwen_restore(QwenSession *s, const QwenCheckpoint *c) {
    if (s->phase == 2 || s->depth || strcmp(c->model_digest, s->model->digest) || c->session_id != s->session_id ||
        c->epoch != s->epoch || c->capacity != s->capacity || c->serial != s->checkpoint_serial ||
        c->position != s->checkpoint_position || c->position < 1 || c->position > s->position || c->pending < 0 ||
        c->pending >= s->model->vocab)
        return -1;
    if (s->cache_guard && s->cache_guard(s->cache_context, 1, c->position, s->session_id, s->epoch, c->lineage_id))
        return -1;
    restore(s, c);
    return 0;
}

int qwen_stack_push(QwenSession *s, uint64_t *id) {
    if (!id || !at_boundary(s) || s->depth >= QWEN_STACK_LIMIT) return -1;
    uint64_t unique;
    if (take_id(&next_frame_id, &unique)) return -1;
    QwenFrame *f = &s->frames[s->depth++];
    snapshot(s, &f->state);
    f->id = unique;
    *id = unique;
    return 0;
}

static int valid_top(const QwenSession *s, uint64_t id) {
    return s->phase != 2 && s->depth && s->frames[s->depth - 1].id == id &&
           s->frames[s->depth - 1].state.epoch == s->epoch && s->frames[s->depth - 1].state.position <= s->position;
}

int qwen_stack_rollback(QwenSession *s, uint64_t id) {
    if (!valid_top(s, id)) return -1;
    const QwenCheckpoint *top = &s->frames[s->depth - 1].state;
    if (s->cache_guard && s->cache_guard(s->cache_context, 1, top->position, s->session_id, s->epoch, top->lineage_id))
        return -1;
    restore(s, &s->frames[--s->depth].state);
    s->checkpoint_serial++;
    s->checkpoint_position = 0;
    return 0;
}

int qwen_stack_commit(QwenSession *s, uint64_t id) {
    if (!valid_top(s, id)) return -1;
    s->depth--;
    return 0;
}

int qwen_reset(QwenSession *s) {
    uint64_t lineage;
    if (s->epoch == UINT64_MAX || take_id(&next_lineage_id, &lineage)) return -1;
    s->position = 0; s->pending = -1; s->delivered = 0; s->phase = 0; s->layer = 0; s->depth = 0;
    s->epoch++;
    s->checkpoint_serial++;
    s->checkpoint_position = 0;
    s->lineage_id = lineage;
    s->token_parent_valid = 0;
    if (s->cache_rewind) s->cache_rewind(s->cache_context, 0, s->session_id, s->epoch);
    return 0;
}

/* Tensor-parallel decode over several GPUs (include/qwen_b200.h). */
int qwen_session_tp_open(QwenSession *s, int rank, int world, void *handle) {
    if (!s || !s->runner || s->cache_mask || s->phase == 2) return -1;
    return qwen_b200_tp_open(s->runner, rank, world, handle);
}
int qwen_session_tp_connect(QwenSession *s, const void *handles) {
    if (!s || !s->runner || s->phase == 2) return -1;
    return qwen_b200_tp_connect(s->runner, handles);
}
int qwen_session_tp_close(QwenSession *s) {
    if (!s || !s->runner) return -1;
    return qwen_b200_tp_close(s->runner);
}
