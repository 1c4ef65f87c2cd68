/* Test infrastructure only: drives the reference's experimental operand APIs
 * (src/qwen.h:20-45,106-183: QKV and lexical programs, receiver planes,
 * subspaces, writers, gate laws; src/qwen_operands.inc and the experimental
 * branches of src/qwen.c:216-368) through the reference's own host.
 *
 * Linked into _ref/libref_cpu.so (the reference's CPU primitives) and
 * _ref/libref_gpuhost.so (this repository's B200 primitives), so one scripted
 * scenario can run on both and its logits be compared: the operand programs are
 * served on the B200 by the reference's host over this library. The call
 * patterns follow the reference's own mechanics tests (tests/state_mechanics.c,
 * tests/gate_mechanics.h, tests/writer_mechanics.h, tests/operand_mechanics.c)
 * on a seeded model: begin a token, run layer 0, apply the operand at layer 1,
 * finish the token, and record the logits. */
#include "qwen.h"
#include "oracle_api.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    QwenSession *s;
    float *out;
    int *codes;
    int n, cap, ncodes;
} Run;

static void record(Run *r) {
    if (r->n < r->cap) gpu_read(r->out + (size_t)r->n * r->s->model->vocab, r->s->logits, (size_t)r->s->model->vocab * 4);
    r->n++;
}
static int code(Run *r, int c) {
    if (r->ncodes < 256) r->codes[r->ncodes] = c;
    r->ncodes++;
    return c;
}
static void prefix(Run *r) {
    code(r, qwen_reset(r->s));
    for (int t = 2; t <= 4; t++) code(r, qwen_push(r->s, t));
}
static void to_layer1(Run *r, int token) {
    code(r, qwen_begin_token(r->s, token));
    code(r, qwen_advance_layer(r->s));
}
static void complete(Run *r) {
    while (r->s->layer < r->s->model->layers)
        if (code(r, qwen_advance_layer(r->s))) return;
    code(r, qwen_finish_token(r->s));
    record(r);
}

typedef struct { QwenGateLaw *law; const QwenModel *model; } GateCapture;
static void gate_capture(void *context, int position, int layer, QwenPort port, const float *data, size_t count) {
    GateCapture *c = context;
    (void)count;
    if (port == QWEN_MLP_GATE && layer == 1) qwen_gate_law_init(c->law, c->model, layer, position, data);
}

/* One scenario; returns the number of logits snapshots (written to out, at
 * most cap of vocab floats) and every API return code in order (codes, 256). */
int orc_operand_run(void *model, int which, float *out, int cap, int *codes, int *ncodes) {
    QwenModel *m = (QwenModel *)model;  /* ref_driver's model starts with its QwenModel */
    QwenSession s;
    if (qwen_session_init(&s, m, 64)) return -1;
    Run r = {&s, out, codes, 0, cap, 0};
    QwenCheckpoint parent;
    int d = m->hidden;
    if (which == 0) { /* receiver plane: compile, dense and compiled doses, held write */
        QwenPlane p;
        QwenPlaneWork w;
        code(&r, qwen_plane_init(&p, m));
        prefix(&r);
        code(&r, qwen_checkpoint(&s, &parent));
        to_layer1(&r, 9);
        code(&r, qwen_advance_layer_compile(&s, &p, &w));
        complete(&r);
        const float doses[][2] = {{0, 0}, {.25f, 0}, {-.25f, 0}, {0, .25f}, {.5f, .5f}};
        for (unsigned j = 0; j < sizeof(doses) / sizeof(doses[0]); j++)
            for (int mode = QWEN_PLANE_DENSE; mode <= QWEN_PLANE_COMPILED; mode++) {
                code(&r, qwen_restore(&s, &parent));
                to_layer1(&r, 9);
                code(&r, qwen_advance_layer_plane(&s, &p, (QwenPlaneMode)mode, doses[j][0], doses[j][1], &w));
                complete(&r);
            }
        code(&r, qwen_restore(&s, &parent));
        to_layer1(&r, 9);
        code(&r, qwen_advance_layer_plane(&s, &p, QWEN_PLANE_HELD_WRITE, .25f, 0, &w));
        complete(&r);
        qwen_plane_free(&p);
    } else if (which == 1) { /* gate law captured from the live MLP gate, then native / polynomial / zero */
        QwenGateLaw law = {0};
        QwenGateWork w;
        prefix(&r);
        code(&r, qwen_checkpoint(&s, &parent));
        GateCapture capture = {&law, m};
        s.observer = gate_capture;
        s.observer_context = &capture;
        s.observe_position = s.position;
        s.observe_layer = 1;
        code(&r, qwen_push(&s, 9));
        s.observer = NULL;
        s.observer_context = NULL;
        code(&r, law.ready ? 0 : -1);
        record(&r);
        for (int mode = QWEN_GATE_NATIVE; mode <= QWEN_GATE_ZERO; mode++) {
            code(&r, qwen_restore(&s, &parent));
            to_layer1(&r, 9);
            code(&r, qwen_advance_layer_gate(&s, &law, (QwenGateMode)mode, s.lineage_id, &w));
            complete(&r);
        }
        qwen_gate_law_free(&law);
    } else if (which == 2) { /* subspace: compile, then its execution modes */
        QwenSubspace p;
        QwenSubspaceStats st;
        code(&r, qwen_subspace_init(&p, m));
        prefix(&r);
        to_layer1(&r, 9);
        code(&r, qwen_advance_layer_subspace(&s, &p, QWEN_SUBSPACE_COMPILE, &st));
        complete(&r);
        code(&r, qwen_checkpoint(&s, &parent));
        const QwenSubspaceMode modes[] = {QWEN_SUBSPACE_DENSE, QWEN_SUBSPACE_PROJECT, QWEN_SUBSPACE_CORRECT,
                                          QWEN_SUBSPACE_REASSOC, QWEN_SUBSPACE_HELD};
        for (unsigned j = 0; j < sizeof(modes) / sizeof(modes[0]); j++) {
            code(&r, qwen_restore(&s, &parent));
            to_layer1(&r, 10);
            code(&r, qwen_advance_layer_subspace(&s, &p, modes[j], &st));
            complete(&r);
        }
        qwen_subspace_free(&p);
    } else if (which == 3) { /* rank-16 QKV programs on layers 1 and 2 (q and k compiled, v native) */
        const int rank = 16, k = m->kvheads * m->head;
        float *basis = malloc((size_t)rank * d * 4), *q = malloc((size_t)rank * d * 4), *kk = malloc((size_t)rank * k * 4);
        if (!basis || !q || !kk) abort();
        for (size_t i = 0; i < (size_t)rank * d; i++) {
            basis[i] = (float)((int)(i * 2654435761u % 97) - 48) / 400.0f;
            q[i] = (float)((int)(i * 40503u % 89) - 44) / 300.0f;
        }
        for (size_t i = 0; i < (size_t)rank * k; i++) kk[i] = (float)((int)(i * 69069u % 83) - 41) / 300.0f;
        QwenQkvProgram p[2] = {{0}};
        for (int j = 0; j < 2; j++) {
            code(&r, qwen_qkv_program_init(p + j, m, j + 1, rank, 3, basis, q, kk, NULL));
            code(&r, qwen_qkv_bind(&s, j + 1, p + j));
        }
        for (int t = 0; t < 6; t++) {
            code(&r, qwen_push(&s, t < 3 ? t + 2 : s.pending));
            record(&r);
        }
        code(&r, qwen_reset(&s));
        for (int j = 0; j < 2; j++) {
            code(&r, qwen_qkv_bind(&s, j + 1, NULL));
            qwen_qkv_program_free(p + j);
        }
        free(basis);
        free(q);
        free(kk);
    } else if (which == 4) { /* lexical program over 8 token ids (layer-0 q/k/v from the program) */
        QwenLexicalProgram p = {0};
        const int ids[] = {2, 3, 4, 5, 9, 17, 100, 1000};
        code(&r, qwen_lexical_compile(&p, m, ids, 8));
        code(&r, qwen_lexical_bind(&s, &p));
        for (int t = 0; t < 8; t++) {
            code(&r, qwen_push(&s, ids[t]));
            record(&r);
        }
        code(&r, qwen_push(&s, 6)); /* not in the program: refused */
        code(&r, qwen_reset(&s));
        code(&r, qwen_lexical_bind(&s, NULL));
        qwen_lexical_free(&p);
    } else if (which == 5) { /* writer over a supplied rank-3 subspace, each writer mode */
        double *columns = calloc((size_t)3 * d, sizeof(double));
        if (!columns) abort();
        for (int j = 0; j < 3; j++) columns[j * d + 7 * j + 1] = 1;
        QwenSubspace supplied = {0};
        supplied.model = m;
        supplied.ready = 1;
        supplied.rank = 3;
        supplied.layer = 0;
        supplied.q0 = columns;
        supplied.q1 = columns + d;
        supplied.q2 = columns + 2 * d;
        prefix(&r);
        for (unsigned mode = QWEN_WRITER_NATIVE; mode <= QWEN_WRITER_BOTH; mode++) {
            QwenWriter w;
            code(&r, qwen_writer_init(&w, &s, &supplied, 1));
            uint64_t frame;
            code(&r, qwen_stack_push(&s, &frame));
            to_layer1(&r, 9);
            code(&r, qwen_advance_layer_writer(&s, &w, mode));
            complete(&r);
            code(&r, qwen_stack_rollback(&s, frame));
            qwen_writer_free(&w);
        }
        free(columns);
    } else {
        qwen_session_free(&s);
        return -1;
    }
    qwen_session_free(&s);
    *ncodes = r.ncodes;
    return r.n;
}
