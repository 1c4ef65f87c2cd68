/* Test infrastructure only: drives the reference's own C runtime.
 *
 * oracle/Makefile compiles this file against the reference's src/qwen.h and
 * links it with the reference's src/qwen.c + src/model.c, and then either
 *   - tests/gpu_stub.c (the reference's CPU FP32 primitives) -> _ref/libref_cpu.so,
 *     the reference CPU path that pins the oracle and times the CPU baseline; or
 *   - this repository's libcmachine_b200.so (-DREF_GPU) -> _ref/libref_gpuhost.so,
 *     the reference's unchanged C host running on the B200 primitives, which shows
 *     the drop-in boundary from the caller's side.
 * The model is built field by field, as the reference's model-free tests do
 * (tests/state_mechanics.c:16-22), because qwen_model_init only accepts
 * 28-layer bundle files (src/qwen.c:27,44). Tensors go through
 * gpu_owned_weight in the reference's load order (src/qwen.c:21-24,34-41).
 */
#include "qwen.h"
#include "oracle_api.h"
#include "par.h"
#include <stdlib.h>
#include <string.h>

typedef struct { QwenModel model; float *slots[4096]; unsigned count; } RefModel;

typedef struct { void *p; uint64_t base; TcmFill f; int bf16; } GenJob;
static void gen_body(void *c, size_t begin, size_t end) {
    GenJob *j = c;
    for (size_t i = begin; i < end; i++) {
        float value = tcm_seeded_value(j->base, i, j->f);
        if (j->bf16) ((uint16_t *)j->p)[i] = tcm_bf16_rne(value);
        else ((float *)j->p)[i] = value;
    }
}
static float *upload(RefModel *r, uint64_t seed, const TcmFillLaw *law, uint32_t id, int rank, int rows, int cols, int bf16) {
    size_t n = (size_t)rows * (rank == 2 ? cols : 1);
    TcmFill f = tcm_tensor_fill(law, id);
    uint64_t base = tcm_tensor_base(seed, id);
    float *p;
    void *h = malloc(n * (bf16 ? 2 : 4));
    if (!h) abort();
    GenJob job = {h, base, f, bf16};
    par_for(n, 1 << 16, gen_body, &job);
    p = gpu_owned_weight(r->model.gpu, h, bf16 ? TCM_BF16 : TCM_F32, n, rank, rows, cols);
    free(h);
    r->slots[r->count++] = p;
    return p;
}

#ifdef REF_GPU
void orc_configure_profile(int profile) { gpu_weight_configure(profile); }
void orc_release_profile(void) { gpu_weight_release(); }
#endif

void *orc_model_create(const OrcShape *S, uint64_t seed, const TcmFillLaw *law, int bf16) {
    RefModel *r = calloc(1, sizeof(*r));
    if (!r) abort();
    QwenModel *m = &r->model;
    m->gpu = gpu_open();
    m->hidden = S->hidden; m->layers = S->layers; m->qheads = S->qheads; m->kvheads = S->kvheads;
    m->head = S->head; m->intermediate = S->intermediate; m->vocab = S->vocab;
    m->max_position = S->max_position; m->epsilon = S->epsilon; m->theta = S->theta;
    m->eos = -1; m->eos_extra = 0;
    memset(m->digest, 'a', 64);
    memset(m->identity, 'b', 64);
    int d = S->hidden, qd = S->qheads * S->head, kv = S->kvheads * S->head, f = S->intermediate;
    m->embedding = upload(r, seed, law, 0, 2, S->vocab, d, bf16);
    m->norm = upload(r, seed, law, 1, 1, d, 0, 0);
    m->layer = calloc((size_t)S->layers, sizeof(QwenLayer));
    if (!m->layer) abort();
    for (int l = 0; l < S->layers; l++) {
        QwenLayer *L = &m->layer[l];
        L->input_norm = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_INPUT_NORM), 1, d, 0, 0);
        L->post_norm = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_POST_NORM), 1, d, 0, 0);
        L->q = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_Q), 2, qd, d, bf16);
        L->k = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_K), 2, kv, d, bf16);
        L->v = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_V), 2, kv, d, bf16);
        L->qb = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_QB), 1, qd, 0, 0);
        L->kb = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_KB), 1, kv, 0, 0);
        L->vb = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_VB), 1, kv, 0, 0);
        L->o = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_O), 2, d, qd, bf16);
        L->gate = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_GATE), 2, f, d, bf16);
        L->up = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_UP), 2, f, d, bf16);
        L->down = upload(r, seed, law, tcm_layer_tensor(l, TCM_T_DOWN), 2, d, f, bf16);
    }
    return r;
}

void orc_model_free(void *p) {
    RefModel *r = p;
    if (!r) return;
    for (unsigned i = 0; i < r->count; i++) gpu_free(r->slots[i]);
    free(r->model.layer);
    gpu_close(r->model.gpu);
    free(r);
}

float orc_weight_value(void *p, uint32_t id, uint64_t index) {
    RefModel *r = p;
    float v;
    gpu_read(&v, r->slots[id] + index, 4);
    return v;
}

void *orc_session_create(void *p, int capacity) {
    RefModel *r = p;
    QwenSession *s = calloc(1, sizeof(*s));
    if (!s) abort();
    if (qwen_session_init(s, &r->model, capacity)) { free(s); return NULL; }
    return s;
}

void orc_session_free(void *p) {
    QwenSession *s = p;
    if (!s) return;
    qwen_session_free(s);
    free(s);
}

int orc_push(void *p, int token, OrcTop2 *top, float *logits) {
    QwenSession *s = p;
    if (qwen_push(s, token)) return -1;
    top->first = s->top.first; top->second = s->top.second;
    top->first_value = s->top.first_value; top->second_value = s->top.second_value;
    if (logits) gpu_read(logits, s->logits, (size_t)s->model->vocab * 4);
    return 0;
}

int orc_position(void *p) { return ((QwenSession *)p)->position; }

void orc_read_kv(void *p, int layer, int kind, float *out) {
    QwenSession *s = p;
    const QwenModel *m = s->model;
    const float *src = (kind ? s->values : s->keys) + (size_t)layer * m->kvheads * s->capacity * m->head;
    for (int h = 0; h < m->kvheads; h++)
        gpu_read(out + (size_t)h * s->position * m->head, src + (size_t)h * s->capacity * m->head,
                 (size_t)s->position * m->head * 4);
}

void orc_read_hidden(void *p, float *out) {
    QwenSession *s = p;
    gpu_read(out, s->x, (size_t)s->model->hidden * 4);
}

void orc_write_kv(void *p, int layer, int kind, int rows, const float *in) {
    QwenSession *s = p;
    const QwenModel *m = s->model;
    float *dst = (kind ? s->values : s->keys) + (size_t)layer * m->kvheads * s->capacity * m->head;
    for (int h = 0; h < m->kvheads; h++)
        gpu_write(dst + (size_t)h * s->capacity * m->head, in + (size_t)h * rows * m->head, (size_t)rows * m->head * 4);
}

/* The reference keeps the cursor in QwenSession.position (src/qwen.h:72);
 * qwen_begin_token appends the next row there. */
int orc_set_cursor(void *p, int position) {
    QwenSession *s = p;
    if (s->phase == 2 || s->depth || position < 0 || position >= s->capacity) return -1;
    s->position = position;
    return 0;
}

/* The reference's nested stack (src/qwen.c:416-431), for replay checks of the
 * reference host over the B200 primitives. */
int orc_stack_push(void *p, uint64_t *id) { return qwen_stack_push((QwenSession *)p, id); }
int orc_stack_rollback(void *p, uint64_t id) { return qwen_stack_rollback((QwenSession *)p, id); }

/* The model as the reference's qwen_model_free expects it: the tensors listed
 * in allocations (the serve build takes ownership of the descriptor). */
QwenModel *orc_model_take(void *p) {
    RefModel *r = p;
    QwenModel *m = &r->model;
    m->allocations = calloc(r->count ? r->count : 1, sizeof(float *));
    if (!m->allocations) abort();
    for (unsigned i = 0; i < r->count; i++) m->allocations[i] = r->slots[i];
    m->allocation_count = r->count;
    return m;
}
