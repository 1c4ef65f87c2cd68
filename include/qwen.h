/* The Qwen2.5 session API of cmachine, executed by the B200 decoder.
 *
 * Replaces the reference's src/qwen.h for the decode path: the same types,
 * field names and entry points (model, session, push / begin / advance_layer /
 * finish, token abort, cursor checkpoint, 64-frame nested stack, reset,
 * observer ports and cache-backend callbacks), so that callers written against
 * the reference compile against this header and link libcmachine_b200.so.
 * Return codes follow the reference: 0 success, -1 refused with the session
 * unchanged, -2 retryable, and backend codes from cache callbacks.
 *
 * Execution: a plain decode token (no armed observer, every layer on the owned
 * FP32 K/V) runs the fused B200 kernels as one CUDA-graph replay
 * (include/qwen_b200.h). A layer with an armed observer runs the primitive
 * sequence of the reference (src/qwen.c:248-341) so every port is
 * materialised; a layer owned by a cache callback runs fused stages around
 * the callback.
 *
 * Not part of this header: the experimental operand programs of the
 * reference (QKV programs, lexical programs, plane / subspace / writer /
 * gate-law layer variants, src/qwen.h:20-45,106-183). The reference's own
 * src/qwen.c still runs them on the B200 primitive library.
 */
#ifndef TCM_QWEN_H
#define TCM_QWEN_H
#include <stdint.h>
#include "gpu.h"
#include "qwen_b200.h"
#include "tcm_bundle.h"
#include "tcm_seeded.h"
#ifdef __cplusplus
extern "C" {
#endif

/* src/qwen.h:6-8 */
typedef struct {
    float *input_norm, *post_norm, *q, *k, *v, *qb, *kb, *vb, *o, *gate, *up, *down;
} QwenLayer;

/* src/qwen.h:9-19; `fused` and `matrix_dtype` are the B200 additions. */
typedef struct {
    TcmGpu *gpu;
    int hidden, layers, qheads, kvheads, head, intermediate, vocab, max_position, eos, eos_extra;
    float epsilon, theta;
    char identity[65], digest[65];
    float *embedding, *norm;
    QwenLayer *layer;
    float **allocations;
    unsigned allocation_count;
    size_t weight_bytes;
    QwenB200Decoder *fused;
    int matrix_dtype;
    QwenB200Batch *batch;  /* the batched engine, created on the first qwen_push_batch */
} QwenModel;

/* src/qwen.h:46-52 */
typedef struct {
    char model_digest[65];
    int position, pending, capacity, delivered;
    TcmTop2 top;
    uint64_t serial, session_id, epoch, lineage_id;
} QwenCheckpoint;
typedef struct { QwenCheckpoint state; uint64_t id; } QwenFrame;
#define QWEN_STACK_LIMIT 64

/* src/qwen.h:54-62 */
typedef enum {
    QWEN_INPUT, QWEN_QUERY, QWEN_KEY, QWEN_VALUE, QWEN_ATTENTION,
    QWEN_MLP_INPUT, QWEN_MLP_GATE, QWEN_MLP_UP, QWEN_MLP_RETURN, QWEN_OUTPUT,
    QWEN_ATTENTION_WRITE, QWEN_RAW_RECEIVER,
    QWEN_CONSUMED_ATTENTION_WRITE, QWEN_CONSUMED_MLP_WRITE,
    QWEN_PORT_COUNT
} QwenPort;
/* src/qwen.h:63-69: observer (borrowed device pointer, valid during the call)
 * and cache backend callbacks. */
typedef void (*QwenObserver)(void *, int, int, QwenPort, const float *, size_t);
typedef int (*QwenCacheStep)(void *, int, int, const float *, const float *, const float *, float *, float *);
typedef int (*QwenCacheGuard)(void *, int, int, uint64_t, uint64_t, uint64_t);
typedef void (*QwenCacheRewind)(void *, int, uint64_t, uint64_t);

/* src/qwen.h:70-100 (decode-path fields); `runner` is the B200 addition. */
typedef struct {
    const QwenModel *model;
    int position, capacity, pending, layer, phase, delivered;
    float *keys, *values, *x, *norm, *q, *k, *v, *attention, *projected, *gate, *up, *logits, *scores;
    size_t allocated_bytes;
    TcmTop2 top;
    uint64_t checkpoint_serial;
    uint64_t session_id;
    int checkpoint_position;
    uint64_t epoch;
    uint64_t lineage_id;
    unsigned depth;
    QwenFrame frames[QWEN_STACK_LIMIT];
    QwenObserver observer;
    void *observer_context;
    int observe_position, observe_layer;
    uint64_t cache_mask;
    int cache_slots[64], dense_layers;
    QwenCacheStep cache_step;
    QwenCacheRewind cache_rewind;
    QwenCacheGuard cache_guard;
    void *cache_context;
    QwenCheckpoint token_parent;
    int token_parent_valid;
    int current_token;
    QwenB200Runner *runner;
} QwenSession;

/* Model construction. qwen_model_init_seeded builds a random-init model of any
 * Qwen2.5-architecture shape directly in device memory (include/tcm_seeded.h);
 * weight_profile 0 keeps FP32 matrices, 2 keeps BF16 matrices (FP32 vectors).
 * fused = 0 leaves the model on the primitive path only. */
int qwen_model_init_seeded(QwenModel *, const QwenB200Shape *, uint64_t seed, const TcmFillLaw *law,
                           int weight_profile, int fused);
void qwen_model_free(QwenModel *);
/* src/qwen.h:184: a Qwen2.5-1.5B model from a TCM1LE bundle (architecture
 * TCM_QWEN, 338 tensors, the Qwen2.5-1.5B configuration, epsilon 1e-6, theta
 * 1e6), the reference's tensor names and shapes, matrices stored per the weight
 * profile set by gpu_weight_configure (0 FP32, 1 FP32 tiled, 2 source BF16;
 * vectors FP32). The fused decoder is built over them. 0, or -1 with a message
 * (the reference's) and *m cleared. */
int qwen_model_init(QwenModel *, const TcmModel *, char *error, size_t capacity);

/* Sessions and the decode state machine (src/qwen.h:186-204). */
int qwen_session_init(QwenSession *, const QwenModel *, int capacity);
int qwen_session_init_layout(QwenSession *, const QwenModel *, int capacity, uint64_t mask, QwenCacheStep,
                             QwenCacheRewind, void *context);
int qwen_abort_token(QwenSession *);
void qwen_session_free(QwenSession *);
int qwen_push(QwenSession *, int token);
int qwen_begin_token(QwenSession *, int token);
int qwen_advance_layer(QwenSession *);
int qwen_finish_token(QwenSession *);
int qwen_advance(QwenSession *);
int qwen_checkpoint(QwenSession *, QwenCheckpoint *);
int qwen_restore(QwenSession *, const QwenCheckpoint *);
int qwen_stack_push(QwenSession *, uint64_t *);
int qwen_stack_rollback(QwenSession *, uint64_t);
int qwen_stack_commit(QwenSession *, uint64_t);
int qwen_reset(QwenSession *);
const char *qwen_port_name(QwenPort);

/* B200 addition: n greedy decode steps (each = qwen_advance) with one host
 * synchronisation; ids[i] receives the pending token after step i. Requires the
 * fused path (no armed observer, owned K/V); returns -1 otherwise. */
int qwen_generate(QwenSession *, int n, int *ids);

/* B200 addition: the rest of the token opened by qwen_begin_token -- every layer
 * and the readout -- as one CUDA graph replay when the session's runner serves
 * every layer (owned K/V, or a cache backend that attached its arena to the
 * runner, whose per-layer step callback is then not called) and no port is
 * observed at this position; otherwise advance_layer until done, then
 * finish_token. Must start at layer 0. Returns 0, -1, a layer's cache error, or
 * -81 when a layer encoded a non-finite K/V row into its byte cache (the token
 * is left open for abort, as after a failed layer). */
int qwen_complete_token(QwenSession *);

/* B200 addition: qwen_push for n sessions of one model in one batched step
 * (include/qwen_b200.h, tcgen05 GEMMs): session i takes tokens[i]; every
 * session's K/V, logits, top-2, pending token, position and lineage end as n
 * separate qwen_push calls would leave them. All sessions must be distinct,
 * belong to a BF16 model with the fused decoder, keep their K/V in the session
 * (no cache callbacks), have no port observed at their position, and pass
 * qwen_push's guards; n <= 64, positions < 9216. Returns 0, or -1 with nothing
 * changed. */
int qwen_push_batch(QwenSession **sessions, int n, const int *tokens);

/* B200 addition: prefill -- the same session state as n qwen_push calls
 * (K/V rows, logits, top-2, pending token, position, n lineage ids taken, the
 * last one kept). For a session qwen_push_batch could serve (BF16 model, fused
 * decoder, K/V in the session, no observer armed, positions < 9216), the tokens
 * run as batched tensor-core steps of up to 64 tokens each, every step causal
 * over its chunk (values within the BF16 profile's tolerance of n pushes);
 * otherwise it is n qwen_push calls. Returns 0, or -1: refused with the session
 * unchanged when a token is out of range, the tokens do not fit the capacity or
 * a token is open; when a cache guard refuses a later token, the tokens before
 * it stay pushed. */
int qwen_prefill(QwenSession *, const int *tokens, int n);

/* B200 addition: a model from a TCM1LE bundle path (loaded in weight profile
 * `profile`, as qwen_model_init after tcm_load) or from a seeded specification
 * seeded:SHAPE:SEED:PROFILE (SHAPE "qwen2.5-1.5b", "qwen2.5-1.5b@LAYERS" or
 * HIDDENxLAYERSxQHEADSxKVHEADSxHEADxINTERMEDIATExVOCABxPOSITIONS; PROFILE 0
 * FP32 or 2 BF16 matrices; weights N(0, 0.02), norms 1, biases 0). 0, or -1
 * with a message in error. */
int qwen_model_open(QwenModel *, const char *spec, int profile, char *error, size_t capacity);

/* B200 addition: the reference's timed single-session run (src/qwen.c:438-503),
 * `tcm-cuda qwen MODEL --tokens-file F [--new-tokens N] [--context C]
 * [--output P] [--first-logits P] [--checkpoint-test] [--trace-prefix P
 * --trace-layer L [--trace-position T]]`, printing the tcm-qwen-run-v1 JSON. */
int qwen_main(int argc, char **argv);

/* B200 addition: tensor-parallel decode of one session over `world` GPUs (2, 4
 * or 8), one process per GPU, each with the whole model and its own copy of the
 * session (qwen_b200_tp_open/_connect/_close in include/qwen_b200.h, applied
 * to the session's runner). Open on every rank, gather the handles
 * (QWEN_B200_TP_HANDLE_BYTES each) in rank order, connect; then every rank
 * pushes the same tokens. While connected, a layer with an armed observer
 * (which would run the single-GPU primitive path) is refused. Requires the
 * fused decoder and every layer's K/V in the session. 0 or -1 (nothing
 * changed). */
int qwen_session_tp_open(QwenSession *, int rank, int world, void *handle);
int qwen_session_tp_connect(QwenSession *, const void *handles);
int qwen_session_tp_close(QwenSession *);

#ifdef __cplusplus
}
#endif
#endif
