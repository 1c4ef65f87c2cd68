/* Serving front-ends over the session API: the reference's line protocol
 * (src/qwen_serve.c:27-82 for a dense session, src/qwen_bounded_serve.c:23-61
 * for the byte-codec ring), same commands, replies and errors, so recorded
 * protocol replays run unchanged:
 *   A ids...  append prompt tokens     G n    generate up to n tokens
 *   S         state and SHA-256 of the cache and logits
 *   C / R     cursor checkpoint / restore (dense only)
 *   P / B id / K id   push / roll back / commit a stack frame
 *   Z         reset     Q   quit
 * B200 differences: A on a dense session runs through qwen_prefill (batched
 * causal tensor-core steps on a BF16 model), and MODEL may name a seeded
 * random-init model instead of a bundle: seeded:SHAPE:SEED:PROFILE with SHAPE
 * "qwen2.5-1.5b", "qwen2.5-1.5b@LAYERS" or HIDDENxLAYERSxQHEADSxKVHEADSxHEADx
 * INTERMEDIATExVOCABxPOSITIONS, PROFILE 0 (FP32) or 2 (BF16 matrices). */
#define _POSIX_C_SOURCE 200809L
#include "../../include/bounded_cache.h"
#include "../../include/qwen.h"

#include <errno.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

int qwen_bounded_serve_main(int argc, char **argv);

/* ------------------------------------------------------------------ argument helpers */

static int parse_int(const char *text, long lo, long hi, int *out) {
    char *end;
    errno = 0;
    const long v = strtol(text, &end, 10);
    if (errno || end == text || *end || v < lo || v > hi) return -1;
    *out = (int)v;
    return 0;
}
/* A positive frame id filling the rest of the line (after blanks). */
static int parse_frame(const char *p, uint64_t *id) {
    while (*p == ' ' || *p == '\t') p++;
    if (*p < '0' || *p > '9') return -1;
    char *end;
    errno = 0;
    const unsigned long long v = strtoull(p, &end, 10);
    while (*end == ' ' || *end == '\t' || *end == '\r' || *end == '\n') end++;
    if (errno || *end || !v) return -1;
    *id = (uint64_t)v;
    return 0;
}
/* Token ids after the command letter: count, or -1 on a bad id or overflow. */
static int parse_tokens(const char *p, int vocab, int limit, int *out) {
    int n = 0;
    while (*p) {
        while (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r') p++;
        if (!*p) break;
        char *end;
        errno = 0;
        const long v = strtol(p, &end, 10);
        if (errno || end == p || v < 0 || v >= vocab || n >= limit) return -1;
        out[n++] = (int)v;
        p = end;
    }
    return n;
}
/* G's budget: 1..4096 with nothing after it but blanks. */
static int parse_budget(const char *p, long *budget) {
    char *end;
    errno = 0;
    *budget = strtol(p, &end, 10);
    while (*end == ' ' || *end == '\t' || *end == '\n' || *end == '\r') end++;
    return errno || end == p || *end || *budget < 1 || *budget > 4096 ? -1 : 0;
}

/* ------------------------------------------------------------------ models */

static int seeded_shape(const char *text, QwenB200Shape *s) {
    const QwenB200Shape qwen = {1536, 28, 12, 2, 128, 8960, 151936, 32768, 1e-6f, 1e6f};
    *s = qwen;
    if (!strcmp(text, "qwen2.5-1.5b")) return 0;
    if (!strncmp(text, "qwen2.5-1.5b@", 13)) return parse_int(text + 13, 1, 64, &s->layers);
    int v[8], n = 0;
    const char *p = text;
    while (n < 8) {
        char *end;
        errno = 0;
        const long x = strtol(p, &end, 10);
        if (errno || end == p || x < 1 || x > 1 << 20) return -1;
        v[n++] = (int)x;
        if (*end == 'x' && n < 8) p = end + 1;
        else if (!*end && n == 8) break;
        else return -1;
    }
    QwenB200Shape custom = {v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], 1e-6f, 1e6f};
    *s = custom;
    return 0;
}

/* A bundle path, or seeded:SHAPE:SEED:PROFILE (weights N(0, 0.02), norms 1,
 * biases 0). `profile` is the bundle's weight profile. */
int qwen_model_open(QwenModel *m, const char *spec, int profile, char *error, size_t capacity) {
    if (!strncmp(spec, "seeded:", 7)) {
        char shape_text[128];
        const char *a = spec + 7, *b = strchr(a, ':');
        const char *c = b ? strchr(b + 1, ':') : NULL;
        QwenB200Shape shape;
        int seed, weights;
        if (!b || !c || (size_t)(b - a) >= sizeof(shape_text)) goto bad;
        memcpy(shape_text, a, (size_t)(b - a));
        shape_text[b - a] = 0;
        char seed_text[32];
        if ((size_t)(c - b - 1) >= sizeof(seed_text)) goto bad;
        memcpy(seed_text, b + 1, (size_t)(c - b - 1));
        seed_text[c - b - 1] = 0;
        if (seeded_shape(shape_text, &shape) || parse_int(seed_text, 0, 2147483647, &seed) ||
            parse_int(c + 1, 0, 2, &weights) || weights == 1)
            goto bad;
        const TcmFillLaw law = {{0.0f, 0.02f}, {1.0f, 0.0f}, {0.0f, 0.0f}};
        /* The fused decoder where the shape has one, else the primitive path. */
        if (qwen_model_init_seeded(m, &shape, (uint64_t)seed, &law, weights, 1) &&
            qwen_model_init_seeded(m, &shape, (uint64_t)seed, &law, weights, 0)) {
            snprintf(error, capacity, "seeded model refused");
            return -1;
        }
        return 0;
    bad:
        snprintf(error, capacity, "invalid seeded model specification");
        return -1;
    }
    gpu_weight_configure(profile);
    TcmModel bundle;
    if (tcm_load(&bundle, spec, error, capacity)) return -1;
    const int status = qwen_model_init(m, &bundle, error, capacity);
    tcm_unload(&bundle);
    return status;
}

/* ------------------------------------------------------------------ dense session */

static int is_eos(const QwenModel *m, int token) { return token == m->eos || (m->eos_extra > 0 && token == m->eos_extra); }

/* SHA-256 of the K/V rows [0, position) in (kind, layer, KV head) order and of
 * the logits (empty when no logits are valid). */
static void dense_hashes(const QwenSession *s, char cache[65], char logits[65]) {
    const QwenModel *m = s->model;
    const size_t row = (size_t)s->position * m->head, n = (size_t)2 * m->layers * m->kvheads * row;
    float *host = malloc((n ? n : 1) * sizeof(float));
    if (!host) exit(2);
    size_t off = 0;
    for (int kind = 0; kind < 2; kind++)
        for (int l = 0; l < m->layers; l++)
            for (int h = 0; h < m->kvheads; h++) {
                const size_t at = ((size_t)l * m->kvheads + h) * s->capacity * m->head;
                if (row) gpu_read(host + off, (kind ? s->values : s->keys) + at, row * sizeof(float));
                off += row;
            }
    unsigned char digest[32];
    tcm_sha256(host, n * sizeof(float), digest);
    tcm_hex(digest, 32, cache);
    free(host);
    if (s->phase != 1) {
        logits[0] = 0;
        return;
    }
    host = malloc((size_t)m->vocab * sizeof(float));
    if (!host) exit(2);
    gpu_read(host, s->logits, (size_t)m->vocab * sizeof(float));
    tcm_sha256(host, (size_t)m->vocab * sizeof(float), digest);
    tcm_hex(digest, 32, logits);
    free(host);
}

int qwen_serve_main(int argc, char **argv) {
    int explicit_policy = 0;
    for (int i = 3; i + 1 < argc; i += 2)
        if (!strcmp(argv[i], "--cache-policy")) {
            explicit_policy = 1;
            if (strcmp(argv[i + 1], "native")) return qwen_bounded_serve_main(argc, argv);
        }
    const char *base = strrchr(argv[0], '/');
    base = base ? base + 1 : argv[0];
    if (!explicit_policy && !strcmp(base, "tcm-bounded-chat")) return qwen_bounded_serve_main(argc, argv);
    if (argc < 3 || !(argc % 2)) {
        fprintf(stderr, "usage: tcm-cuda serve MODEL [--context N] [--cache-policy native|full-byte|bounded]\n");
        return 2;
    }
    int capacity = 4096;
    for (int i = 3; i < argc; i += 2) {
        if (!strcmp(argv[i], "--cache-policy") && !strcmp(argv[i + 1], "native")) continue;
        if (strcmp(argv[i], "--context") || parse_int(argv[i + 1], 1, 32768, &capacity)) return 2;
    }
    QwenModel model;
    QwenSession session;
    QwenCheckpoint checkpoint;
    int have_checkpoint = 0;
    char error[256];
    if (qwen_model_open(&model, argv[2], 0, error, sizeof(error))) {
        fprintf(stderr, "%s\n", error);
        return 2;
    }
    if (qwen_session_init(&session, &model, capacity)) return 2;
    int *tokens = malloc((size_t)capacity * sizeof(int));
    if (!tokens) return 2;
    printf("{\"event\":\"ready\",\"model_identity\":\"%s\",\"model_digest\":\"%s\",\"capacity\":%d,"
           "\"gpu_weight_bytes\":%zu,\"gpu_session_bytes\":%zu}\n",
           model.identity, model.digest, capacity, model.weight_bytes, session.allocated_bytes);
    fflush(stdout);
    char *line = NULL;
    size_t line_bytes = 0;
    while (getline(&line, &line_bytes, stdin) >= 0) {
        const char cmd = line[0];
        if (cmd == 'Q') break;
        if (cmd == 'A') {
            const int count = parse_tokens(line + 1, model.vocab, capacity, tokens);
            if (count < 1 || count > capacity - session.position) {
                puts("{\"error\":\"invalid append or context capacity\"}");
            } else {
                if (qwen_prefill(&session, tokens, count)) return 2;
                printf("{\"event\":\"appended\",\"count\":%d,\"position\":%d}\n", count, session.position);
            }
        } else if (cmd == 'G') {
            long budget;
            if (parse_budget(line + 1, &budget) || session.pending < 0 ||
                budget > capacity - session.position + (session.delivered ? 0 : 1)) {
                puts("{\"error\":\"invalid generation budget or state\"}");
            } else {
                printf("{\"event\":\"generated\",\"ids\":[");
                int count = 0;
                for (long i = 0; i < budget; i++) {
                    if (session.delivered) {
                        if (is_eos(&model, session.pending)) break;
                        if (qwen_advance(&session)) return 2;
                    }
                    if (count++) putchar(',');
                    printf("%d", session.pending);
                    session.delivered = 1;
                    if (is_eos(&model, session.pending)) break;
                }
                printf("],\"count\":%d,\"position\":%d,\"pending_token\":%d}\n", count, session.position, session.pending);
            }
        } else if (cmd == 'S') {
            char cache[65], logits[65];
            dense_hashes(&session, cache, logits);
            printf("{\"event\":\"state\",\"position\":%d,\"pending_token\":%d,\"delivered\":%d,\"checkpoint_serial\":%llu,"
                   "\"stack_depth\":%u,\"top_frame\":%llu,\"epoch\":%llu,\"cache_sha256\":\"%s\",\"logits_sha256\":\"%s\","
                   "\"logits_valid\":%s}\n",
                   session.position, session.pending, session.delivered, (unsigned long long)session.checkpoint_serial,
                   session.depth, (unsigned long long)(session.depth ? session.frames[session.depth - 1].id : 0),
                   (unsigned long long)session.epoch, cache, logits, session.phase == 1 ? "true" : "false");
        } else if (cmd == 'C') {
            if (qwen_checkpoint(&session, &checkpoint)) {
                puts("{\"error\":\"checkpoint requires a token boundary\"}");
            } else {
                have_checkpoint = 1;
                printf("{\"event\":\"checkpoint\",\"position\":%d,\"serial\":%llu}\n", session.position,
                       (unsigned long long)checkpoint.serial);
            }
        } else if (cmd == 'R') {
            if (!have_checkpoint || qwen_restore(&session, &checkpoint))
                puts("{\"error\":\"no compatible saved parent\"}");
            else
                printf("{\"event\":\"restored\",\"position\":%d,\"pending_token\":%d}\n", session.position, session.pending);
        } else if (cmd == 'P') {
            uint64_t id;
            if (qwen_stack_push(&session, &id))
                puts("{\"error\":\"push requires a token boundary and stack capacity\"}");
            else
                printf("{\"event\":\"pushed\",\"frame\":%llu,\"depth\":%u,\"position\":%d}\n", (unsigned long long)id,
                       session.depth, session.position);
        } else if (cmd == 'B' || cmd == 'K') {
            uint64_t id;
            const int back = cmd == 'B';
            if (parse_frame(line + 1, &id) || (back ? qwen_stack_rollback(&session, id) : qwen_stack_commit(&session, id))) {
                puts("{\"error\":\"no compatible top frame\"}");
            } else {
                if (back) have_checkpoint = 0;
                printf("{\"event\":\"%s\",\"frame\":%llu,\"depth\":%u,\"position\":%d,\"pending_token\":%d}\n",
                       back ? "rolled_back" : "committed", (unsigned long long)id, session.depth, session.position,
                       session.pending);
            }
        } else if (cmd == 'Z') {
            if (qwen_reset(&session)) {
                puts("{\"error\":\"reset epoch exhausted\"}");
            } else {
                have_checkpoint = 0;
                puts("{\"event\":\"reset\"}");
            }
        } else {
            puts("{\"error\":\"unknown command\"}");
        }
        fflush(stdout);
    }
    free(line);
    free(tokens);
    qwen_session_free(&session);
    qwen_model_free(&model);
    return 0;
}

/* ------------------------------------------------------------------ bounded session */

#define SERVE_REQUIRE(x)                                                                   \
    do {                                                                                   \
        if (!(x)) {                                                                        \
            fprintf(stderr, "bounded-chat %s:%d: %s\n", __FILE__, __LINE__, #x);           \
            exit(2);                                                                       \
        }                                                                                  \
    } while (0)

static void hex_digest(const void *p, size_t n, char out[65]) {
    unsigned char raw[32];
    tcm_sha256(p, n, raw);
    tcm_hex(raw, 32, out);
}

/* The arena, cursor, population, rng and slot positions hashed together; the
 * logits (which must be finite) separately. */
static void ring_hashes(Ring *c, char cache[65], char logits[65]) {
    const size_t n = c->arena_bytes + 20 + (size_t)c->capacity * 4;
    unsigned char *p = malloc(n);
    SERVE_REQUIRE(p);
    gpu_read(p, c->arena, c->arena_bytes);
    size_t off = c->arena_bytes;
    memcpy(p + off, &c->view.cursor, 4);
    off += 4;
    memcpy(p + off, &c->view.population, 8);
    off += 8;
    memcpy(p + off, &c->view.rng, 8);
    off += 8;
    memcpy(p + off, c->positions, (size_t)c->capacity * 4);
    hex_digest(p, n, cache);
    free(p);
    const size_t vocab = (size_t)c->session->model->vocab;
    float *y = malloc(vocab * sizeof(float));
    SERVE_REQUIRE(y);
    gpu_read(y, c->session->logits, vocab * sizeof(float));
    for (size_t i = 0; i < vocab; i++) SERVE_REQUIRE(isfinite(y[i]));
    hex_digest(y, vocab * sizeof(float), logits);
    free(y);
}

static void ring_state(Ring *c, const char *policy) {
    const QwenSession *s = c->session;
    char cache[65], logits[65];
    ring_hashes(c, cache, logits);
    int resident = 0;
    for (int i = 0; i < c->capacity; i++) resident += c->positions[i] >= 0;
    printf("{\"event\":\"state\",\"cache_policy\":\"%s\",\"position\":%d,\"pending_token\":%d,\"delivered\":%d,"
           "\"stack_depth\":%u,\"top_frame\":%llu,\"epoch\":%llu,\"logical_capacity\":%d,\"resident_capacity\":%d,"
           "\"resident_rows\":%d,\"evictions\":%llu,\"rng\":%llu,\"cache_sha256\":\"%s\",\"logits_sha256\":\"%s\","
           "\"gpu_state_bytes\":%zu,\"tracked_gpu_bytes\":%zu}\n",
           policy, s->position, s->pending, s->delivered, s->depth,
           (unsigned long long)(s->depth ? s->frames[s->depth - 1].id : 0), (unsigned long long)s->epoch, s->capacity,
           c->capacity, resident, (unsigned long long)c->view.population, (unsigned long long)c->view.rng, cache, logits,
           s->allocated_bytes + c->gpu_bytes, gpu_live_bytes());
}

int qwen_bounded_serve_main(int argc, char **argv) {
    if (argc < 3 || strcmp(argv[1], "serve")) {
        fprintf(stderr, "usage: tcm-cuda serve MODEL [--context N] [--cache-policy bounded|full-byte] "
                        "[--anchors N --recent N --reservoir N]\n");
        return 2;
    }
    int logical = 768, anchors = 16, recent = 64, reservoir = 32, profile = 2;
    const char *policy = "bounded";
    for (int i = 3; i < argc; i += 2) {
        if (i + 1 >= argc) return 2;
        const char *key = argv[i], *value = argv[i + 1];
        if (!strcmp(key, "--cache-policy")) {
            if (strcmp(value, "bounded") && strcmp(value, "full-byte")) return 2;
            policy = value;
        } else if (!strcmp(key, "--weight-profile")) {
            if (!strcmp(value, "tiled-fp32")) profile = 1;
            else if (strcmp(value, "source-bf16")) return 2;
        } else if (!strcmp(key, "--context")) {
            if (parse_int(value, 1, 32768, &logical)) return 2;
        } else if (!strcmp(key, "--anchors")) {
            if (parse_int(value, 0, 32768, &anchors)) return 2;
        } else if (!strcmp(key, "--recent")) {
            if (parse_int(value, 1, 32768, &recent)) return 2;
        } else if (!strcmp(key, "--reservoir")) {
            if (parse_int(value, 0, 32768, &reservoir)) return 2;
        } else {
            return 2;
        }
    }
    const int full = !strcmp(policy, "full-byte");
    if (full) {
        anchors = 0;
        recent = logical;
        reservoir = 0;
    }
    if (anchors + recent + reservoir > logical) {
        fprintf(stderr, "physical support exceeds logical capacity\n");
        return 2;
    }
    QwenModel model;
    QwenSession session;
    Ring cache;
    char error[256];
    if (qwen_model_open(&model, argv[2], profile, error, sizeof(error))) {
        fprintf(stderr, "%s\n", error);
        return 2;
    }
    SERVE_REQUIRE(!ring_open(&cache, &session, &model, logical, anchors, recent, reservoir, full));
    printf("{\"event\":\"ready\",\"model_identity\":\"%s\",\"model_digest\":\"%s\",\"capacity\":%d,\"cache_policy\":\"%s\","
           "\"anchors\":%d,\"recent\":%d,\"reservoir\":%d,\"resident_capacity\":%d,\"stack_limit\":2,"
           "\"legacy_checkpoint\":false,\"weight_storage\":\"%s\",\"weight_profile\":%d,\"gpu_weight_bytes\":%zu,"
           "\"gpu_session_bytes\":%zu,\"tracked_gpu_bytes\":%zu}\n",
           model.identity, model.digest, logical, policy, anchors, recent, reservoir, cache.capacity,
           model.matrix_dtype == 2 ? "source-BF16 matrices" : "FP32 matrices", model.matrix_dtype == 2 ? 2 : profile,
           model.weight_bytes, session.allocated_bytes + cache.gpu_bytes, gpu_live_bytes());
    fflush(stdout);
    int *tokens = malloc((size_t)logical * sizeof(int));
    SERVE_REQUIRE(tokens);
    char *line = NULL;
    size_t line_bytes = 0;
    while (getline(&line, &line_bytes, stdin) >= 0) {
        const char cmd = line[0];
        if (cmd == 'Q') break;
        if (cmd == 'A') {
            const int count = parse_tokens(line + 1, model.vocab, logical, tokens);
            if (count < 1 || count > logical - session.position) {
                puts("{\"error\":\"invalid append or context capacity\"}");
            } else {
                for (int i = 0; i < count; i++) SERVE_REQUIRE(!ring_push(&cache, tokens[i]));
                printf("{\"event\":\"appended\",\"count\":%d,\"position\":%d}\n", count, session.position);
            }
        } else if (cmd == 'G') {
            long budget;
            if (parse_budget(line + 1, &budget) || session.pending < 0 ||
                budget > logical - session.position + (session.delivered ? 0 : 1)) {
                puts("{\"error\":\"invalid generation budget or state\"}");
            } else {
                printf("{\"event\":\"generated\",\"ids\":[");
                int count = 0;
                for (long i = 0; i < budget; i++) {
                    if (session.delivered) {
                        if (is_eos(&model, session.pending)) break;
                        SERVE_REQUIRE(!ring_push(&cache, session.pending));
                    }
                    if (count++) putchar(',');
                    printf("%d", session.pending);
                    session.delivered = 1;
                    if (is_eos(&model, session.pending)) break;
                }
                printf("],\"count\":%d,\"position\":%d,\"pending_token\":%d}\n", count, session.position, session.pending);
            }
        } else if (cmd == 'S') {
            ring_state(&cache, policy);
        } else if (cmd == 'P') {
            uint64_t id;
            if (ring_mark(&cache, &id))
                puts("{\"error\":\"push requires a token boundary and one of two snapshot slots\"}");
            else
                printf("{\"event\":\"pushed\",\"frame\":%llu,\"depth\":%u,\"position\":%d}\n", (unsigned long long)id,
                       session.depth, session.position);
        } else if (cmd == 'B' || cmd == 'K') {
            uint64_t id;
            const int back = cmd == 'B';
            if (parse_frame(line + 1, &id) || (back ? ring_rollback(&cache, id) : ring_commit(&cache, id)))
                puts("{\"error\":\"no compatible top snapshot\"}");
            else
                printf("{\"event\":\"%s\",\"frame\":%llu,\"depth\":%u,\"position\":%d,\"pending_token\":%d}\n",
                       back ? "rolled_back" : "committed", (unsigned long long)id, session.depth, session.position,
                       session.pending);
        } else if (cmd == 'C' || cmd == 'R') {
            puts("{\"error\":\"legacy cursor checkpoints unavailable; use P and B/K\"}");
        } else if (cmd == 'Z') {
            SERVE_REQUIRE(!qwen_reset(&session));
            gpu_zero(session.logits, (size_t)model.vocab * sizeof(float));
            puts("{\"event\":\"reset\"}");
        } else {
            puts("{\"error\":\"unknown command\"}");
        }
        fflush(stdout);
    }
    free(line);
    free(tokens);
    ring_close(&cache);
    qwen_session_free(&session);
    qwen_model_free(&model);
    gpu_weight_release();
    SERVE_REQUIRE(!gpu_live_bytes());
    return 0;
}
