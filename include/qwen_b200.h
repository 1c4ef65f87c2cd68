/* Fused B200 decode entry points (additive to the reference ABI).
 *
 * The reference runs one decode token as ~24 primitive calls per layer and two
 * blocking reads in gpu_top2 (src/qwen.c:216-387, src/qwen_cuda.cu:100-118).
 * These entry points run the same equations as five fused sm_100a kernels per
 * layer plus a fused vocabulary readout with greedy top-2, and replay a whole
 * token as one CUDA graph:
 *
 *   layer: [RMSNorm -> q/k/v GEMV -> bias -> RoPE -> K/V append]
 *          [split-K GQA attention]            (or the caller's cache step)
 *          [O GEMV -> residual]
 *          [RMSNorm -> gate/up GEMV -> SwiGLU]
 *          [down GEMV -> residual]
 *   token: [final RMSNorm -> tied-embedding GEMV -> logits + top-2 + finite check]
 *
 * They replace, in order, the reference's gpu_rms + qkv_apply + gpu_rope +
 * gpu_cache (src/qwen.c:249-258), gpu_attention (src/qwen.c:259), gpu_matvec +
 * gpu_add (src/qwen.c:262,275), gpu_rms + 2 gpu_matvec + gpu_swiglu
 * (src/qwen.c:289,320,329), gpu_matvec + gpu_add (src/qwen.c:330,341), and
 * gpu_rms + gpu_matvec + gpu_top2 (src/qwen.c:384). Weights and buffers are
 * device pointers owned by the caller; weights are all FP32 or all BF16
 * (source-BF16 residence); activations, K/V and accumulation are FP32.
 * Errors: functions return 0, -1 for an invalid argument (nothing ran), or
 * -3 when the logits held a non-finite value.
 */
#ifndef QWEN_B200_H
#define QWEN_B200_H
#include <stddef.h>
#include <stdint.h>
#include "gpu.h"
#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int hidden, layers, qheads, kvheads, head, intermediate, vocab, max_position;
    float epsilon, theta;
} QwenB200Shape;

/* One layer's tensors (device pointers), the reference's QwenLayer fields. */
typedef struct {
    const float *input_norm, *post_norm, *q, *k, *v, *qb, *kb, *vb, *o, *gate, *up, *down;
} QwenB200Layer;

/* A session's device buffers (the reference's QwenSession fields). keys and
 * values are [dense layer][kvheads][capacity][head]; cache_slots[l] is the
 * dense slot of layer l or -1 when a caller-supplied cache step owns it. */
typedef struct {
    float *keys, *values;
    int capacity;
    const int *cache_slots;
    float *x, *q, *k, *v, *attention, *gate, *logits;
} QwenB200Buffers;

typedef struct QwenB200Decoder QwenB200Decoder;
typedef struct QwenB200Runner QwenB200Runner;

/* matrix_dtype: 1 FP32, 2 BF16, 0 = look the embedding up in the weight
 * residence registry (gpu_owned_weight). Requires head == 128, qheads a
 * multiple of kvheads with at most 8 query heads per KV head, hidden a multiple
 * of 8. Returns NULL on an unsupported shape. */
QwenB200Decoder *qwen_b200_decoder_create(const QwenB200Shape *shape, const float *embedding,
                                          const float *final_norm, const QwenB200Layer *layers, int matrix_dtype);
void qwen_b200_decoder_free(QwenB200Decoder *);
/* HBM bytes one decode token streams for the weights (matrices + vectors). */
size_t qwen_b200_decoder_weight_bytes(const QwenB200Decoder *);

/* Per-session executor: scratch, device-resident token state, a CUDA graph of
 * one whole token. Scratch comes from gpu_alloc (tracked). */
QwenB200Runner *qwen_b200_runner_create(const QwenB200Decoder *, const QwenB200Buffers *);
void qwen_b200_runner_free(QwenB200Runner *);

/* Token-level steps, for callers that drive layers one by one
 * (qwen_begin_token / qwen_advance_layer / qwen_finish_token). */
int qwen_b200_begin(QwenB200Runner *, int token, int position);
int qwen_b200_layer(QwenB200Runner *, int layer);           /* all five stages (dense slot) */
int qwen_b200_layer_qkv(QwenB200Runner *, int layer);       /* stage 1 (appends when dense) */
int qwen_b200_layer_attention(QwenB200Runner *, int layer); /* stage 2 (dense slot) */
int qwen_b200_layer_mlp(QwenB200Runner *, int layer);       /* stages 3-5 */
int qwen_b200_finish(QwenB200Runner *, TcmTop2 *top);

/* One whole token (embedding through top-2) as one graph replay; all layers
 * must be dense. Same bits as begin + layers + finish. */
int qwen_b200_token(QwenB200Runner *, int token, int position, TcmTop2 *top);
/* n greedy tokens back to back: the device feeds each top-1 to the next step
 * and advances the position; one host synchronisation at the end. ids[i] and
 * tops[i] describe the readout after step i (ids may be NULL). */
int qwen_b200_generate(QwenB200Runner *, int token, int position, int n, int *ids, TcmTop2 *tops);
/* Enqueue n chained steps without waiting (timing and pipelining); the result
 * of the last step is read by qwen_b200_last. */
int qwen_b200_enqueue(QwenB200Runner *, int token, int position, int n);
int qwen_b200_last(QwenB200Runner *, TcmTop2 *top);

/* ---- Bounded byte-codec K/V (the ring of include/bounded_cache.h) ----
 * Layers whose cache slot is -1 keep their K/V in a ring arena in the
 * reference layout (src/bounded_cache.h:26-28): per layer K codes
 * [2][rows][128] int8, V codes [2][rows][128], scales [kind * 2 + head][rows]
 * FP32, 528 bytes a row. The ring module owns the arena and the bookkeeping;
 * the runner encodes the current rows and attends over the retained ones.
 * Requires 2 KV heads. */
typedef struct {
    void *arena;         /* layers x rows x 528 bytes */
    int rows;            /* physical rows: anchors + recent + reservoir */
    int anchors, recent, reservoir;
    void *save;          /* token cut row store: layers x 2 x 528 bytes */
    float *logits_save;  /* token cut logits: vocab floats */
    int positions;       /* logical capacity: the position limit of the runner */
} QwenB200Ring;
/* One token's ring bookkeeping, computed on the host. Retained rows are the
 * first anchors_n anchor slots, the first reservoir_n reservoir slots and the
 * first recent_n recent slots; reservoir rows add `bias` (the reference's
 * weight * sqrt(128), src/qwen_cache.inc:34) to their scores when weighted. */
typedef struct {
    int write_slot, sample_slot;  /* sample_slot -1: no reservoir copy this token */
    int anchors_n, reservoir_n, recent_n;
    int weighted;
    float bias;
    int pad;
} QwenB200RingStep;
int qwen_b200_ring_attach(QwenB200Runner *, const QwenB200Ring *);
/* The step the next qwen_b200_begin writes; begin then also takes the token cut
 * (old write and sample rows of every layer and the logits into the save
 * areas) and copies each layer's evicted row into the sample slot. */
int qwen_b200_ring_stage(QwenB200Runner *, const QwenB200RingStep *);
/* One layer's cache step: encode k, v (FP32 [2][128]) into the write slot and
 * attend q over the retained rows into out. Device pointers. */
int qwen_b200_ring_attention(QwenB200Runner *, int layer, const float *q, const float *k, const float *v, float *out);
/* Synchronises; -1 when a row encoded since the last begin was non-finite. */
int qwen_b200_ring_status(QwenB200Runner *);
/* Every layer and the readout of the token opened by qwen_b200_begin, as one
 * graph replay. 0; -3 non-finite logits; -4 a pipeline wait ran out; -5 a
 * non-finite K/V row in a ring layer (the token must be aborted). */
int qwen_b200_complete(QwenB200Runner *, TcmTop2 *top);
/* 1 when qwen_b200_complete can run this runner's layers (every layer dense or
 * served by an attached ring), else 0. */
int qwen_b200_can_complete(const QwenB200Runner *);
/* Token cut rows: mode 0 saves the write and sample rows of every layer into
 * `save` and copies the old write row into the sample slot; mode 1 puts both
 * saved rows back. Device pointers; sample_slot -1 skips the sample row. */
void qwen_b200_ring_rows(void *arena, int rows, int layers, void *save, int write_slot, int sample_slot, int mode);

/* ---- Batched decode of independent sessions (BF16 weights) ----
 * One step decodes one token for each of n <= qwen_b200_batch_max() sessions
 * sharing the decoder's weights: the q/k/v, O, gate/up, down and vocabulary
 * projections run as tcgen05 tensor-core GEMMs (BF16 weights x activations
 * split into two BF16 halves, FP32 accumulation in tensor memory), attention
 * runs per session over its own FP32 K/V. Requires a BF16 decoder of the
 * Qwen2.5-1.5B geometry; returns NULL otherwise. */
typedef struct QwenB200Batch QwenB200Batch;
/* Session i of a step: its K/V slabs ([layer][2][capacity][128] FP32, the
 * session layout of include/qwen.h), capacity, and its logits and x buffers,
 * which the step overwrites as a single-session token would. */
typedef struct {
    float *keys, *values;
    int capacity;
    float *logits, *x;
} QwenB200BatchSession;
QwenB200Batch *qwen_b200_batch_create(const QwenB200Decoder *);
void qwen_b200_batch_free(QwenB200Batch *);
int qwen_b200_batch_max(void);
int qwen_b200_batch_launches_per_step(const QwenB200Batch *);
/* One step: session i takes tokens[i] at positions[i] (position < 9216); tops[i]
 * receives its top-2. 0, -1 invalid arguments (nothing ran), -3 non-finite
 * logits, -4 a pipeline wait ran out. */
int qwen_b200_batch_step(QwenB200Batch *, int n, const QwenB200BatchSession *sessions, const int *tokens,
                         const int *positions, TcmTop2 *tops);
/* Prefill chunk of one session: tokens[0..n) (n <= qwen_b200_batch_max()) at
 * positions position..position+n-1 as one step whose slots share the session's
 * cache (causal: every slot's K/V row is appended before any slot attends).
 * The last token's logits and hidden state go to the session's buffers, its
 * top-2 to *top; the other tokens' logits go to engine scratch. Returns as
 * qwen_b200_batch_step. */
int qwen_b200_batch_prefill(QwenB200Batch *, const QwenB200BatchSession *session, const int *tokens, int n,
                            int position, TcmTop2 *top);
/* `steps` chained greedy steps (the device feeds every session's top-1 back and
 * advances its position) without waiting; qwen_b200_batch_read then returns the
 * last step's tops and, if history is set, history[t * n + i] for every step. */
int qwen_b200_batch_enqueue(QwenB200Batch *, int n, const QwenB200BatchSession *sessions, const int *tokens,
                            const int *positions, int steps);
int qwen_b200_batch_read(QwenB200Batch *, int n, int steps, TcmTop2 *tops, TcmTop2 *history);
/* y[i][r] = sum_k W[r][k] x[i][k] on the tensor cores for a BF16 matrix W
 * (rows a multiple of 128, in a multiple of 64) and n <= 64 FP32 rows x, with
 * `splits` K-splits. Synchronous; 0, -1 invalid, -4 wait ran out. */
int qwen_b200_batch_matmul(const void *w, int rows, int in, const float *x, int n, float *y, int splits);
/* Measurement aid: mean device time (ms) of one standalone launch of a step's
 * stage for these sessions: 0 q/k/v GEMM (appends this step's K/V rows), 1
 * attention, 2 O GEMM, 3 gate/up GEMM, 4 down GEMM, 5 vocabulary GEMM, 6
 * RMSNorm, of `layer`, over `reps` launches. */
float qwen_b200_batch_time_stage(QwenB200Batch *, int n, const QwenB200BatchSession *sessions, const int *tokens,
                                 const int *positions, int stage, int layer, int reps);
/* The same launch with a per-CTA timeline: host receives ctas x 8 global-timer
 * stamps (ns; GEMM: entry, producer released, first stage ready, last MMA
 * committed, epilogue released, first accumulator read, last tile stored,
 * exit; attention: entry, consumers released, first stage ready, done). */
int qwen_b200_batch_trace_stage(QwenB200Batch *, int n, const QwenB200BatchSession *sessions, const int *tokens,
                                const int *positions, int stage, int layer, unsigned long long *host, int ctas);
/* How many thread-block clusters of `size` GEMM CTAs the GPU holds at once, and
 * the split-K cluster sizes the engine chose (0: split through global memory). */
int qwen_b200_batch_cluster_capacity(int size);
/* Tuning: key 0 = cache rows per attention work item (a multiple of 32 in
 * [256, 2048]); key 1 = the attention kernel: 0 tensor-core fragments (the
 * default, items of 256 rows), 1 CUDA-core flash-decoding (items of 1024
 * rows); choosing a kernel resets the item size to its default; key 2 = where
 * the O and down projections' K splits are summed: 1 in the RMSNorm that reads
 * their output next (the default), 0 in a thread-block cluster fold inside the
 * GEMM. Returns 0, or -1 for an unknown key or value. */
int qwen_b200_batch_tune(QwenB200Batch *, int key, int value);
int qwen_b200_batch_clusters(const QwenB200Batch *, int *qkv, int *o, int *down);

/* ---- Tensor-parallel decode of one session over several GPUs ----
 * One process per GPU, each holding the whole model and its own copy of the
 * session (same prompt, same tokens). A connected group splits every MLP (each
 * rank computes 8960/world of the intermediate units: its rows of gate and up,
 * its columns of down) and the tied-embedding readout (rows
 * [rank*V/world, (rank+1)*V/world)), the work the reference does at
 * src/qwen.c:320,329-330,341 and 383-387. After each layer's down projection
 * the ranks exchange partial residual sums through each other's memory (peer
 * stores over NVLink, per-CTA flags) and add them in rank order, so every rank
 * keeps a bit-identical residual stream and K/V cache; after the readout they
 * exchange top-2s (ties to the lower id) and every rank's logits buffer
 * receives all ranks' logits. Numerically this changes only the order of the
 * down projection's sum. world is 2, 4 or 8; every layer must keep its K/V in
 * the session (no ring). Steps:
 *   1. qwen_b200_tp_open on every rank: allocates the rank's exchange area and
 *      writes QWEN_B200_TP_HANDLE_BYTES of handle (CUDA IPC handles of the area
 *      and of the session's logits buffer, which must be a whole allocation);
 *   2. the caller gathers the world's handles in rank order (any transport,
 *      e.g. torch.distributed all_gather) and calls qwen_b200_tp_connect;
 *   3. all ranks then run the same whole tokens (qwen_push, qwen_advance,
 *      qwen_generate, qwen_b200_enqueue) in lockstep, each starting a token
 *      within the 2 s wait limit of the others. The stage calls of a layer's
 *      MLP and the readout exchange too and must also be made by every rank.
 * Returns 0 or -1 (invalid arguments, a handle of another group, memory that
 * cannot be exported or mapped; nothing changed). A wait that runs out marks
 * the token's fault (-4 from the token calls); the group must then be closed
 * and rebuilt. qwen_b200_tp_close (also done by qwen_b200_runner_free) unmaps
 * the peers and frees the area: close on every rank after a final barrier. */
#define QWEN_B200_TP_HANDLE_BYTES 256
int qwen_b200_tp_open(QwenB200Runner *, int rank, int world, void *handle);
int qwen_b200_tp_connect(QwenB200Runner *, const void *handles);
int qwen_b200_tp_close(QwenB200Runner *);
/* The connected group's size, or 1. */
int qwen_b200_tp_world(const QwenB200Runner *);

/* ---- Bounded waits ----
 * Every wait inside the kernels (a pipeline stage, a grid barrier, a peer's
 * flag) gives up after a time limit, records a fault bit and lets its kernel
 * return; the token calls then report -4. qwen_b200_wait_limit sets that limit
 * for the current device (ns; 0 restores the default 2 s; 1 ms .. 60 s,
 * else -1). qwen_b200_pipeline_check runs the decode GEMVs' shared-memory ring
 * on one CTA: y[rows] = W[rows][1536] x (FP32 device pointers, rows <= 4096)
 * and returns the fault bits (0 when every wait completed; with starve != 0
 * the producer issues nothing, so the consumers' waits run out: bit 1), or -1
 * for invalid arguments. */
int qwen_b200_wait_limit(unsigned long long ns);
int qwen_b200_pipeline_check(const float *w, int rows, const float *x, float *y, int starve);

/* Kernel launches one token issues (for launch accounting). */
int qwen_b200_launches_per_token(const QwenB200Runner *);
/* Whole-token execution: 1 = one persistent cooperative launch per token (one
 * CTA per SM runs every layer and the readout, the weights streaming through
 * grid barriers; applies when every layer is dense and no ring is attached);
 * 0 = the token graph of per-stage kernels (the default: faster on B200 at the
 * measured contexts); -1 queries. Both give identical bits. Returns the mode in
 * force, or -1 (mode 1 where it does not apply). */
int qwen_b200_persistent(QwenB200Runner *, int mode);
/* Tuning of the persistent kernel: key 0 = how far (KB, 0..2048) each CTA's
 * producer prefetches its coming weight and cache rows into L2 ahead of its
 * shared-memory copies (default 0). Returns 0, or -1 for an unknown key or
 * value. */
int qwen_b200_persistent_tune(QwenB200Runner *, int key, int value);
/* Measurement aid: mean device time (ms, CUDA events) of one standalone launch
 * of fused stage `stage` of `layer` (0 q/k/v, 1 attention, 2 O projection,
 * 3 gate/up, 4 down, 5 readout) at `position`, over `reps` launches. On a ring
 * layer, stage 1 is the ring attention of the last token's step (it rewrites
 * that token's row of the layer with the session's current K/V). */
float qwen_b200_time_stage(QwenB200Runner *, int stage, int layer, int position, int reps);

/* Timeline trace for performance work: with tracing on, every launch of a token
 * stamps the GPU global timer per CTA at entry, dependency release, input ready
 * and done (the whole-token graph is re-captured). trace_read copies the last
 * token's stamps, 160 launches x 160 CTAs x 4 (zero where a CTA had no work),
 * and returns the number of launches recorded. Under the persistent kernel the
 * buffer's first SMs x 512 entries are per CTA: its start, then for each grid
 * barrier (six a layer: after q/k/v, attention, merge, O, gate/up, down) the
 * moments it arrived and passed, then the end of its readout rows. */
int qwen_b200_trace(QwenB200Runner *, int enable);
int qwen_b200_trace_read(QwenB200Runner *, unsigned long long *host, size_t count);

/* CUDA-event timing on the library stream: record marks 0..15, elapsed ms. */
void qwen_b200_mark(int index);
float qwen_b200_elapsed_ms(int from, int to);
void qwen_b200_set_device(int device);
int qwen_b200_sm_count(void);

/* Register a device-resident matrix (rows x columns, FP32 or BF16 when
 * encoded) with the weight residence registry, as gpu_owned_weight does for a
 * host upload, so gpu_matvec reads it in its stored type. */
void qwen_b200_register_matrix(const void *p, int rows, int columns, int encoded);
void qwen_b200_unregister_matrix(const void *p);
/* How a device weight is stored: 2 source BF16 (registered encoded), else 1 (FP32). */
int qwen_b200_weight_dtype(const void *p);

/* Seeded device fill (include/tcm_seeded.h): n values of tensor `id` under
 * model seed `seed` with value offset + N(0,1)*scale, stored as FP32
 * (dtype 1) or BF16 (dtype 2) at dst. */
void qwen_b200_seeded_fill(void *dst, int dtype, uint64_t seed, uint32_t id, size_t n, float offset, float scale);

#ifdef __cplusplus
}
#endif
#endif
