/* Bounded anchors / recent / reservoir byte-codec K/V cache over the B200
 * session (include/bounded_cache.h).
 *
 * Host bookkeeping restated from the reference's src/bounded_cache.h:
 *   SplitMix64 state and the unbiased draw             :24-25
 *   token cut save / guard / rewind                    :29-37
 *   retained-row order and reservoir weights           :51-57
 *   cache step (row dump, encode, injected failure)    :58-65
 *   open, begin, abort, finish, push                   :66-79
 *   marks: push, rollback, commit; close               :80-87
 * The device work -- the token cut, encoding the current rows, the sample-row
 * copy and the attention over the retained rows -- runs in the fused B200
 * decode kernels when the session has a runner, and on the primitive ABI
 * (gpu_encode_current, gpu_ring_attention, qwen_b200_ring_rows) otherwise.
 */
#include "../../include/bounded_cache.h"
#include "../../include/qwen_b200.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

#define RING_REQUIRE(x)                                                                \
    do {                                                                               \
        if (!(x)) {                                                                    \
            fprintf(stderr, "bounded cache %s:%d: %s\n", __FILE__, __LINE__, #x);      \
            exit(2);                                                                   \
        }                                                                              \
    } while (0)

/* SplitMix64 (a published generator; src/bounded_cache.h:24). */
static uint64_t ring_random(Ring *c) {
    uint64_t z = (c->view.rng += UINT64_C(0x9e3779b97f4a7c15));
    z = (z ^ (z >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
    z = (z ^ (z >> 27)) * UINT64_C(0x94d049bb133111eb);
    return z ^ (z >> 31);
}
/* Uniform in [0, n): reject draws below (2^64 - n) mod n, then reduce. */
static uint64_t ring_draw(Ring *c, uint64_t n) {
    uint64_t x, t = (uint64_t)(-n) % n;
    do x = ring_random(c); while (x < t);
    return x % n;
}

static signed char *ring_keys(const Ring *c, int l) {
    return (signed char *)c->arena + (size_t)l * c->capacity * RING_ROW_BYTES;
}
static signed char *ring_values(const Ring *c, int l) { return ring_keys(c, l) + (size_t)c->capacity * 256; }
static float *ring_scales(const Ring *c, int l) { return (float *)(ring_keys(c, l) + (size_t)c->capacity * 512); }
static size_t cut_rows_bytes(const Ring *c) { return (size_t)c->layers * 2 * RING_ROW_BYTES; }

/* Retained rows per region: anchors hold positions 0..anchors-1, the recent
 * ring the last `recent` positions, the reservoir min(evictions, sample) rows
 * filled in slot order. Every retained reservoir position is older than every
 * recent one (it was evicted from the ring), so position order is anchors, then
 * the reservoir by position, then the recent rows by position. */
static void ring_counts(const Ring *c, int *na, int *nm, int *nr) {
    const int cursor = c->view.cursor;
    *na = cursor < c->anchors ? cursor : c->anchors;
    const int r = cursor - c->anchors;
    *nr = r < 0 ? 0 : (r > c->recent ? c->recent : r);
    *nm = c->view.population < (uint64_t)c->sample ? (int)c->view.population : c->sample;
}

/* The reservoir slots in position order, from the slot positions (after a
 * restore). */
static void reservoir_rebuild(Ring *c) {
    const int base = c->anchors + c->recent;
    c->reservoir_count = 0;
    for (int j = 0; j < c->sample; j++) {
        const int slot = base + j;
        if (c->positions[slot] < 0) continue;
        int k = c->reservoir_count++;
        while (k && c->positions[c->reservoir[k - 1]] > c->positions[slot]) {
            c->reservoir[k] = c->reservoir[k - 1];
            k--;
        }
        c->reservoir[k] = slot;
    }
}
/* A sampled slot now holds the newest evicted position: it moves to the end. */
static void reservoir_take(Ring *c, int slot) {
    int k = 0;
    while (k < c->reservoir_count && c->reservoir[k] != slot) k++;
    if (k < c->reservoir_count) {
        memmove(c->reservoir + k, c->reservoir + k + 1, (size_t)(c->reservoir_count - k - 1) * sizeof(int));
        c->reservoir_count--;
    }
    c->reservoir[c->reservoir_count++] = slot;
}

/* src/bounded_cache.h:51-57: retained slots in position order and their weights. */
static void ring_order(Ring *c) {
    int na, nm, nr, k = 0;
    ring_counts(c, &na, &nm, &nr);
    for (int i = 0; i < na; i++) c->order[k++] = i;
    for (int i = 0; i < c->reservoir_count; i++) c->order[k++] = c->reservoir[i];
    for (int p = c->view.cursor - nr; p < c->view.cursor; p++) c->order[k++] = c->anchors + (p - c->anchors) % c->recent;
    c->active = k;
    const int m = c->view.population < (uint64_t)c->sample ? (int)c->view.population : c->sample;
    const float w = m ? logf((float)c->view.population / (float)m) : 0.f;
    for (int i = 0; i < c->active; i++) c->weights[i] = (i >= na && i < na + nm) ? w : 0.f;
    if (!c->fused) {
        gpu_write(c->device_order, c->order, (size_t)c->active * 4);
        gpu_write(c->device_weights, c->weights, (size_t)c->active * 4);
    }
}

/* Host half of a cut; the token cut's device rows are taken at begin. */
static void save_cut_host(Ring *c, int slot, uint64_t id) {
    RingCut *p = &c->cuts[slot];
    p->view = c->view;
    memcpy(p->positions, c->positions, (size_t)c->capacity * 4);
    p->id = id;
    p->owner = c->owner;
    p->epoch = c->epoch;
    p->lineage = c->session->lineage_id;
    p->valid = 1;
}
static void save_mark(Ring *c, int slot, uint64_t id) {
    RingCut *p = &c->cuts[slot];
    save_cut_host(c, slot, id);
    gpu_copy(p->arena, c->arena, c->arena_bytes);
    gpu_copy(p->logits, c->session->logits, (size_t)c->session->model->vocab * 4);
}

/* src/bounded_cache.h:32-35: the session asks before a token (operation 0) and
 * before any restore (operation 1); 0 allows. */
static int ring_guard(void *context, int operation, int position, uint64_t owner, uint64_t epoch, uint64_t lineage) {
    Ring *c = context;
    if (owner != c->owner || epoch != c->epoch) return -1;
    if (!operation)
        return !(c->transaction && c->cuts[0].valid && c->cuts[0].view.cursor == position && c->cuts[0].lineage == lineage);
    int slot = c->restore_slot;
    if (slot < 0 || slot >= RING_CUTS) return -1;
    const RingCut *p = &c->cuts[slot];
    return !(p->valid && p->owner == owner && p->epoch == epoch && p->view.cursor == position && p->lineage == lineage);
}

/* src/bounded_cache.h:36-37: a new epoch empties the cache; otherwise the cut
 * chosen by restore_slot comes back (the token cut: two rows a layer). */
static void ring_rewind(void *context, int position, uint64_t owner, uint64_t epoch) {
    Ring *c = context;
    RING_REQUIRE(owner == c->owner);
    if (epoch != c->epoch) {
        RING_REQUIRE(epoch == c->epoch + 1 && position == 0);
        c->epoch = epoch;
        c->view = (RingView){.cursor = 0, .population = 0, .rng = 7};
        for (int i = 0; i < c->capacity; i++) c->positions[i] = -1;
        c->reservoir_count = 0;
        gpu_zero(c->arena, c->arena_bytes);
        for (int j = 0; j < RING_CUTS; j++) c->cuts[j].valid = 0;
        c->transaction = 0;
        c->restore_slot = -1;
        return;
    }
    RING_REQUIRE(c->restore_slot >= 0 && c->restore_slot < RING_CUTS);
    RING_REQUIRE(!ring_guard(c, 1, position, owner, epoch, c->cuts[c->restore_slot].lineage));
    RingCut *p = &c->cuts[c->restore_slot];
    const size_t logits = (size_t)c->session->model->vocab * 4;
    if (c->restore_slot == 0) {
        qwen_b200_ring_rows(c->arena, c->capacity, c->layers, p->arena, c->write_slot, c->sample_slot, 1);
    } else {
        gpu_copy(c->arena, p->arena, c->arena_bytes);
    }
    gpu_copy(c->session->logits, p->logits, logits);
    memcpy(c->positions, p->positions, (size_t)c->capacity * 4);
    c->view = p->view;
    reservoir_rebuild(c);
    c->restores++;
    c->transaction = 0;
}

int ring_step(void *context, int layer, int position, const float *q, const float *k, const float *v, float *out,
              float *scores) {
    Ring *c = context;
    QwenSession *s = c->session;
    (void)scores;
    if (!c->transaction || layer < 0 || layer >= c->layers || position != c->cuts[0].view.cursor ||
        s->position != position || s->phase != 2 || c->view.cursor != position + 1)
        return -80;
    c->calls++;
    if (c->rows && (layer == 0 || layer == 17 || layer == 27)) {
        float row[2][256];
        gpu_read(row[0], k, 1024);
        gpu_read(row[1], v, 1024);
        RING_REQUIRE(fwrite(row, 1, sizeof(row), c->rows) == sizeof(row));
    }
    if (c->fused) {
        /* One launch: encode the current rows into the write slot, attend. */
        RING_REQUIRE(!qwen_b200_ring_attention(s->runner, layer, q, k, v, out));
        if (qwen_b200_ring_status(s->runner)) return -81;
        if (c->fail_layer == layer && c->fail_position == position) {
            c->fail_layer = -1;
            return -77;
        }
        c->published++;
        return 0;
    }
    if (gpu_encode_current(ring_keys(c, layer), ring_values(c, layer), ring_scales(c, layer), k, v, c->capacity,
                           c->write_slot, c->invalid))
        return -81;
    if (c->fail_layer == layer && c->fail_position == position) {
        c->fail_layer = -1;
        return -77;
    }
    c->published++;
    gpu_ring_attention(s->model->gpu, out, q, ring_keys(c, layer), ring_values(c, layer), ring_scales(c, layer),
                       s->scores, c->workspace, c->device_order, c->device_weights, c->capacity, c->active,
                       c->sample && c->view.population > 0);
    return 0;
}

int ring_open(Ring *c, QwenSession *s, const QwenModel *m, int logical, int anchors, int recent, int sample, int full) {
    memset(c, 0, sizeof(*c));
    if (recent <= 0 || anchors < 0 || sample < 0 || anchors + recent + sample > logical || logical > m->max_position ||
        m->layers < 1 || m->layers > 64 || m->qheads != 12 || m->kvheads != 2 || m->head != 128)
        return -1;
    c->session = s;
    c->anchors = anchors;
    c->recent = recent;
    c->sample = sample;
    c->full = full;
    c->capacity = anchors + recent + sample;
    c->layers = m->layers;
    c->restore_slot = -1;
    c->fail_layer = -1;
    c->view.rng = 7;
    const uint64_t mask = m->layers == 64 ? ~UINT64_C(0) : (UINT64_C(1) << m->layers) - 1;
    if (qwen_session_init_layout(s, m, c->capacity, mask, ring_step, ring_rewind, c)) return -1;
    s->capacity = logical;
    s->cache_guard = ring_guard;
    c->owner = s->session_id;
    c->epoch = s->epoch;
    const size_t logits = (size_t)m->vocab * 4;
    gpu_zero(s->logits, logits);
    c->arena_bytes = (size_t)m->layers * c->capacity * RING_ROW_BYTES;
    c->arena = gpu_alloc(c->arena_bytes);
    gpu_zero(c->arena, c->arena_bytes);
    c->positions = malloc((size_t)c->capacity * 4);
    c->order = malloc((size_t)c->capacity * 4);
    c->weights = malloc((size_t)c->capacity * 4);
    c->reservoir = malloc((size_t)(sample ? sample : 1) * 4);
    RING_REQUIRE(c->positions && c->order && c->weights && c->reservoir);
    for (int i = 0; i < c->capacity; i++) c->positions[i] = -1;
    c->gpu_bytes = c->arena_bytes;
    c->host_bytes = sizeof(*c) + (size_t)c->capacity * 12 + (size_t)(sample ? sample : 1) * 4;
    for (int j = 0; j < RING_CUTS; j++) {
        const size_t bytes = j ? c->arena_bytes : cut_rows_bytes(c);
        c->cuts[j].arena = gpu_alloc(bytes);
        c->cuts[j].logits = gpu_alloc(logits);
        c->cuts[j].positions = malloc((size_t)c->capacity * 4);
        RING_REQUIRE(c->cuts[j].positions);
        c->gpu_bytes += bytes + logits;
        c->host_bytes += (size_t)c->capacity * 4;
    }
    if (s->runner) {
        QwenB200Ring g = {c->arena, c->capacity, anchors, recent, sample, c->cuts[0].arena, c->cuts[0].logits, logical};
        c->fused = !qwen_b200_ring_attach(s->runner, &g);
    }
    if (!c->fused) {
        c->workspace = gpu_alloc((size_t)2 * c->capacity * 128 * 4);
        c->invalid = gpu_alloc(4);
        c->device_order = gpu_alloc((size_t)c->capacity * 4);
        c->device_weights = gpu_alloc((size_t)c->capacity * 4);
        c->gpu_bytes += (size_t)c->capacity * (1024 + 8) + 4;
    }
    return 0;
}

int ring_begin(Ring *c, int token) {
    QwenSession *s = c->session;
    if (c->transaction || s->phase == 2 || s->position >= s->capacity || token < 0 || token >= s->model->vocab ||
        c->owner != s->session_id || c->epoch != s->epoch || c->view.cursor != s->position)
        return -1;
    save_cut_host(c, 0, 0);
    c->transaction = 1;
    const int p = s->position;
    c->sample_slot = -1;
    c->write_slot = p < c->anchors ? p : c->anchors + (p - c->anchors) % c->recent;
    if (c->positions[c->write_slot] >= 0) {
        c->view.population++;
        if (c->sample) {
            uint64_t n = c->view.population, j = n <= (uint64_t)c->sample ? n - 1 : ring_draw(c, n);
            if (j < (uint64_t)c->sample) {
                c->sample_slot = c->anchors + c->recent + (int)j;
                c->positions[c->sample_slot] = c->positions[c->write_slot];
                reservoir_take(c, c->sample_slot);
            }
        }
    }
    c->positions[c->write_slot] = p;
    c->view.cursor = p + 1;
    ring_order(c);
    if (c->fused) {
        int na, nm, nr;
        ring_counts(c, &na, &nm, &nr);
        const int weighted = c->sample && c->view.population > 0;
        QwenB200RingStep step = {c->write_slot, c->sample_slot, na, nm, nr, weighted,
                                 weighted ? c->weights[na] * sqrtf(128.0f) : 0.f, 0};
        RING_REQUIRE(!qwen_b200_ring_stage(s->runner, &step));
    } else {
        /* The token cut: this token's two rows of every layer and the logits,
         * then each layer's evicted row into the sample slot. */
        qwen_b200_ring_rows(c->arena, c->capacity, c->layers, c->cuts[0].arena, c->write_slot, c->sample_slot, 0);
        gpu_copy(c->cuts[0].logits, s->logits, (size_t)s->model->vocab * 4);
    }
    RING_REQUIRE(!qwen_begin_token(s, token));
    return 0;
}

int ring_abort(Ring *c) {
    c->restore_slot = 0;
    int e = qwen_abort_token(c->session);
    c->restore_slot = -1;
    if (!e) c->cuts[0].valid = 0;
    return e;
}

int ring_finish(Ring *c) {
    int e = qwen_finish_token(c->session);
    if (!e) {
        c->transaction = 0;
        c->cuts[0].valid = 0;
        c->main_tokens++;
    }
    return e;
}

int ring_push(Ring *c, int token) {
    if (ring_begin(c, token)) return -1;
    QwenSession *s = c->session;
    int e = 0;
    const int armed = c->fail_layer >= 0 && c->fail_position == s->position;
    if (c->fused && !c->rows && !armed && qwen_b200_can_complete(s->runner)) {
        /* The whole token as one graph: every layer's cache step runs inside it. */
        e = qwen_complete_token(s);
        if (!e) {
            c->calls += (unsigned long long)c->layers;
            c->published += (unsigned long long)c->layers;
            c->transaction = 0;
            c->cuts[0].valid = 0;
            c->main_tokens++;
            return 0;
        }
        RING_REQUIRE(!ring_abort(c));
        return e;
    }
    while (s->layer < c->layers && !e) e = qwen_advance_layer(s);
    if (e) {
        RING_REQUIRE(!ring_abort(c));
        return e;
    }
    return ring_finish(c);
}

int ring_mark(Ring *c, uint64_t *id) {
    if (c->transaction || c->session->depth >= 2) return -1;
    int slot = (int)c->session->depth + 1;
    if (qwen_stack_push(c->session, id)) return -1;
    save_mark(c, slot, *id);
    return 0;
}

int ring_rollback(Ring *c, uint64_t id) {
    QwenSession *s = c->session;
    if (c->transaction || !s->depth || s->depth > 2) return -1;
    int slot = (int)s->depth;
    RingCut *p = &c->cuts[slot];
    if (!p->valid || p->id != id || p->owner != s->session_id || p->epoch != s->epoch || s->frames[s->depth - 1].id != id)
        return -1;
    c->restore_slot = slot;
    int e = qwen_stack_rollback(s, id);
    c->restore_slot = -1;
    if (!e) p->valid = 0;
    return e;
}

int ring_commit(Ring *c, uint64_t id) {
    QwenSession *s = c->session;
    if (c->transaction || !s->depth || s->depth > 2) return -1;
    RingCut *p = &c->cuts[s->depth];
    if (!p->valid || p->id != id || qwen_stack_commit(s, id)) return -1;
    p->valid = 0;
    return 0;
}

void ring_close(Ring *c) {
    gpu_free(c->arena);
    if (!c->fused) {
        gpu_free(c->workspace);
        gpu_free(c->invalid);
        gpu_free(c->device_order);
        gpu_free(c->device_weights);
    }
    free(c->positions);
    free(c->order);
    free(c->weights);
    free(c->reservoir);
    for (int j = 0; j < RING_CUTS; j++) {
        gpu_free(c->cuts[j].arena);
        gpu_free(c->cuts[j].logits);
        free(c->cuts[j].positions);
    }
    memset(c, 0, sizeof(*c));
}
