/* Bounded anchors / recent / reservoir K/V cache in the byte codec, for B200.
 *
 * Replaces the reference's src/bounded_cache.h (a header of static functions
 * included by src/qwen_bounded_serve.c and tests/bounded_*_mechanics.c): the
 * same types, field names, entry points, arena layout and return codes, so a
 * caller written against that header compiles against this one and links with
 * libcmachine_b200.so. Per entry point, the reference lines it replaces:
 *   ring_open      src/bounded_cache.h:66-70   ring_begin    :71-76
 *   ring_step      :64-65                      ring_abort    :77
 *   ring_finish    :78                         ring_push     :79
 *   ring_mark      :80                         ring_rollback :81-85
 *   ring_commit    :86                         ring_close    :87
 * Semantics kept: the retention policy (anchors first, then a ring of recent
 * rows; each overwritten recent row is an eviction offered to a reservoir of
 * `sample` rows by reservoir sampling with SplitMix64 from state 7), the
 * attention weights (reservoir rows carry log(evictions / min(evictions,
 * sample))), the per-layer arena [K codes 2 x rows x 128][V codes][scales
 * 4 x rows] (528 bytes a row), token transactions with abort, two nested marks
 * (depth <= 2) with rollback and commit, the guard and rewind callbacks that
 * tie the cache to the session's lineage and epoch, and the error codes (-1
 * refused with nothing changed, -77 injected layer failure, -80 out-of-order
 * step, -81 non-finite K/V row).
 *
 * What differs (B200 design):
 *   - the token cut (cuts[0]) keeps only the rows a token can change -- the
 *     old write row and the old sample row of every layer, 2 x 528 bytes a
 *     layer -- and the logits, instead of a copy of the whole arena per token;
 *     cuts[0].arena points at that row store. Marks (cuts[1], cuts[2]) still
 *     copy the whole arena, once per mark;
 *   - with the fused decoder, encoding the current row, the sample-row copy and
 *     the attention over the retained rows run inside the B200 decode kernels
 *     (one launch per layer, no host synchronisation), and ring_push runs a
 *     whole token as one CUDA graph; a token with an injected failure or a row
 *     dump armed runs layer by layer through ring_step, as the reference does;
 *   - any layer count up to 64 is accepted (the reference requires 28); KV
 *     heads 2, head size 128 and 12 query heads are required, as there.
 */
#ifndef TCM_BOUNDED_CACHE_H
#define TCM_BOUNDED_CACHE_H
#include <stdint.h>
#include <stdio.h>
#include "qwen.h"
#ifdef __cplusplus
extern "C" {
#endif

#define RING_LAYERS 28      /* the reference's layer count (src/bounded_cache.h:10) */
#define RING_ROW_BYTES 528  /* one row of one layer: 4 x 128 codes + 4 scales */
#define RING_CUTS 3         /* the token cut and two marks */

typedef struct { int cursor; uint64_t population, rng; } RingView;
typedef struct {
    RingView view;
    int *positions;   /* host copy of the slot positions */
    void *arena;      /* cuts[0]: the row store (layers x 2 x 528); marks: a whole arena */
    float *logits;
    uint64_t id, owner, epoch, lineage;
    int valid;
} RingCut;
typedef struct {
    QwenSession *session;
    int anchors, recent, sample, capacity, full, transaction, restore_slot, write_slot, sample_slot, active, fail_layer,
        fail_position;
    uint64_t owner, epoch;
    RingView view;
    int *positions, *order;
    float *weights;
    void *arena;
    float *workspace;
    int *invalid, *device_order;
    float *device_weights;
    RingCut cuts[RING_CUTS];
    size_t arena_bytes, gpu_bytes, host_bytes;
    unsigned long long calls, published, restores, main_tokens;
    FILE *rows;  /* when set, K/V rows of layers 0, 17, 27 are appended as FP32 (src/bounded_cache.h:64) */
    /* B200 additions */
    int layers;
    int fused;            /* the session's runner serves the ring layers */
    int *reservoir;       /* reservoir slots in position order (reservoir_count of them) */
    int reservoir_count;
} Ring;

/* Opens the ring over `s` (initialised here) for model `m`: logical capacity
 * `logical`, `anchors` + `recent` + `sample` physical rows. Returns 0, or -1
 * (nothing allocated) when the sizes or the model geometry are unsupported. */
int ring_open(Ring *c, QwenSession *s, const QwenModel *m, int logical, int anchors, int recent, int sample,
              int full);
int ring_begin(Ring *c, int token);
/* The session's cache step for one layer (QwenCacheStep). */
int ring_step(void *context, int layer, int position, const float *q, const float *k, const float *v, float *out,
              float *scores);
int ring_abort(Ring *c);
int ring_finish(Ring *c);
int ring_push(Ring *c, int token);
int ring_mark(Ring *c, uint64_t *id);
int ring_rollback(Ring *c, uint64_t id);
int ring_commit(Ring *c, uint64_t id);
void ring_close(Ring *c);

#ifdef __cplusplus
}
#endif
#endif
