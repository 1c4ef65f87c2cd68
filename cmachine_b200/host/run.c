/* The timed single-session run of the reference's executable
 * (`tcm-cuda qwen MODEL ...`, src/qwen.c:438-503) over this repository's
 * session host: same options, the same tcm-qwen-run-v1 JSON fields, the same
 * first-logits dump, exact-replay checkpoint test and observer port traces
 * (one raw FP32 file per port occurrence plus a JSONL ledger).
 *
 * B200 differences: the prompt runs through qwen_prefill (batched causal
 * tensor-core steps on a BF16 model) unless a port trace is armed, in which case
 * the tokens are pushed one by one so the traced position runs the primitive
 * layer with every port; generation runs on the fused token graph; MODEL may be
 * a seeded specification (qwen_model_open). */
#define _POSIX_C_SOURCE 200809L
#include "../../include/qwen.h"

#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static double now(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + t.tv_nsec * 1e-9;
}
/* A non-negative integer up to 1,000,000 and nothing else (src/qwen.c:439). */
static int integer(const char *text, int *out) {
    char *end;
    errno = 0;
    const long x = strtol(text, &end, 10);
    if (errno || end == text || *end || x < 0 || x > 1000000) return -1;
    *out = (int)x;
    return 0;
}
static int write_floats(const char *path, const float *device, size_t n) {
    float *host = malloc(n * sizeof(float));
    if (!host) return -1;
    gpu_read(host, device, n * sizeof(float));
    FILE *f = fopen(path, "wb");
    int bad = !f || fwrite(host, sizeof(float), n, f) != n;
    if (f && fclose(f)) bad = 1;
    free(host);
    return bad ? -1 : 0;
}

typedef struct {
    const char *prefix, *digest;
    FILE *ledger;
    unsigned count;
    int failed;
} PortTrace;
/* Every observed port: PREFIX-OCCURRENCE-PORT.f32 and one ledger line. */
static void trace_port(void *context, int position, int layer, QwenPort port, const float *data, size_t count) {
    PortTrace *t = context;
    if (t->failed) return;
    char path[4096];
    const int n = snprintf(path, sizeof(path), "%s-%04u-%s.f32", t->prefix, t->count, qwen_port_name(port));
    if (n < 0 || (size_t)n >= sizeof(path) || write_floats(path, data, count)) {
        t->failed = 1;
        return;
    }
    if (fprintf(t->ledger,
                "{\"model_digest\":\"%s\",\"position\":%d,\"layer\":%d,\"port\":\"%s\",\"occurrence\":%u,\"count\":%zu,"
                "\"dtype\":\"float32\"}\n",
                t->digest, position, layer, qwen_port_name(port), t->count, count) < 0)
        t->failed = 1;
    t->count++;
}

static int usage(void) {
    fprintf(stderr, "usage: tcm-cuda qwen MODEL --tokens-file F [--new-tokens N] [--context C] [--output P]\n"
                    "       [--first-logits P] [--checkpoint-test] [--trace-prefix P --trace-layer L [--trace-position T]]\n");
    return 2;
}

int qwen_main(int argc, char **argv) {
    if (argc < 3) return usage();
    const char *tokens_path = NULL, *output_path = NULL, *logits_path = NULL, *trace_prefix = NULL;
    int budget = 32, capacity = 4096, checkpoint_test = 0, trace_layer = -1, trace_position = -1;
    for (int i = 3; i < argc; i++) {
        if (!strcmp(argv[i], "--checkpoint-test")) {
            checkpoint_test = 1;
            continue;
        }
        if (i + 1 >= argc) return usage();
        const char *key = argv[i], *value = argv[++i];
        if (!strcmp(key, "--tokens-file")) tokens_path = value;
        else if (!strcmp(key, "--output")) output_path = value;
        else if (!strcmp(key, "--first-logits")) logits_path = value;
        else if (!strcmp(key, "--new-tokens")) { if (integer(value, &budget)) return usage(); }
        else if (!strcmp(key, "--context")) { if (integer(value, &capacity)) return usage(); }
        else if (!strcmp(key, "--trace-prefix")) trace_prefix = value;
        else if (!strcmp(key, "--trace-layer")) { if (integer(value, &trace_layer)) return usage(); }
        else if (!strcmp(key, "--trace-position")) { if (integer(value, &trace_position)) return usage(); }
        else return usage();
    }
    if (!tokens_path || budget < 1 || budget > 4096 || capacity < 1 || capacity > 32768) return usage();
    FILE *input = fopen(tokens_path, "r");
    if (!input) {
        perror("tokens");
        return 2;
    }
    int *ids = malloc((size_t)capacity * sizeof(int)), count = 0, id;
    if (!ids) return 2;
    while (fscanf(input, "%d", &id) == 1) {
        if (count >= capacity) {
            fprintf(stderr, "prompt exceeds capacity\n");
            return 2;
        }
        ids[count++] = id;
    }
    if (!feof(input) || fclose(input) || !count || count + budget - 1 > capacity) {
        fprintf(stderr, "invalid token input or insufficient context\n");
        return 2;
    }
    QwenModel model;
    QwenSession session;
    char error[256];
    double start = now();
    if (qwen_model_open(&model, argv[2], 0, error, sizeof(error))) {
        fprintf(stderr, "%s\n", error);
        return 2;
    }
    if (qwen_session_init(&session, &model, capacity)) return 2;
    gpu_sync();
    const double load = now() - start;
    PortTrace trace = {0};
    if (trace_prefix) {
        if (trace_layer < 0 || trace_layer >= model.layers || trace_position >= count + budget - 1) return 2;
        char path[4096];
        const int n = snprintf(path, sizeof(path), "%s.jsonl", trace_prefix);
        if (n < 0 || (size_t)n >= sizeof(path)) return 2;
        trace.prefix = trace_prefix;
        trace.digest = model.digest;
        trace.ledger = fopen(path, "wb");
        if (!trace.ledger) return 2;
        session.observer = trace_port;
        session.observer_context = &trace;
        session.observe_layer = trace_layer;
        session.observe_position = trace_position < 0 ? count - 1 : trace_position;
    } else if (trace_layer >= 0 || trace_position >= 0) {
        return 2;
    }
    start = now();
    int status = 0;
    if (trace_prefix) {
        for (int i = 0; i < count && !status; i++) status = qwen_push(&session, ids[i]);
    } else {
        status = qwen_prefill(&session, ids, count);
    }
    if (status) {
        fprintf(stderr, "invalid token or failed transition\n");
        return 2;
    }
    gpu_sync();
    const double prefill = now() - start;
    if (logits_path && write_floats(logits_path, session.logits, (size_t)model.vocab)) return 2;
    /* Exact replay: advance, restore the checkpoint, advance again; the token and
     * every logit must repeat bit for bit (src/qwen.c:477-481). */
    int checkpoint_exact = 1, checkpoint_tested = 0;
    if (checkpoint_test && session.position < capacity) {
        QwenCheckpoint checkpoint;
        if (qwen_checkpoint(&session, &checkpoint)) return 2;
        checkpoint_tested = 1;
        if (qwen_advance(&session)) return 2;
        const int expected = session.pending;
        const size_t bytes = (size_t)model.vocab * sizeof(float);
        float *reference = malloc(bytes), *actual = malloc(bytes);
        if (!reference || !actual) return 2;
        gpu_read(reference, session.logits, bytes);
        if (qwen_restore(&session, &checkpoint) || qwen_advance(&session)) return 2;
        gpu_read(actual, session.logits, bytes);
        checkpoint_exact = expected == session.pending && !memcmp(reference, actual, bytes);
        free(reference);
        free(actual);
        if (qwen_restore(&session, &checkpoint)) return 2;
    }
    FILE *output = output_path ? fopen(output_path, "w") : stdout;
    if (!output) return 2;
    fprintf(output,
            "{\"schema\":\"tcm-qwen-run-v1\",\"model_identity\":\"%s\",\"model_digest\":\"%s\",\"arithmetic\":\"FP32 "
            "activations and accumulation; %s weights read in place; fused sm_100a kernels, fixed reduction order\","
            "\"prompt_tokens\":%d,\"capacity\":%d,\"source_bundle_bytes\":%zu,\"gpu_weight_bytes\":%zu,"
            "\"gpu_session_bytes\":%zu,\"load_seconds\":%.9g,\"prefill_seconds\":%.9g,\"tokens\":[",
            model.identity, model.digest, model.matrix_dtype == 2 ? "BF16" : "FP32", count, capacity, (size_t)0,
            model.weight_bytes, session.allocated_bytes, load, prefill);
    int generated = 0;
    start = now();
    for (int i = 0; i < budget; i++) {
        if (i) fputc(',', output);
        fprintf(output, "{\"id\":%d,\"position\":%d,\"logit\":%.9g,\"runner_up\":%d,\"margin\":%.9g}", session.pending,
                session.position, session.top.first_value, session.top.second,
                session.top.first_value - session.top.second_value);
        generated++;
        session.delivered = 1;
        if (session.pending == model.eos || (model.eos_extra > 0 && session.pending == model.eos_extra) || i + 1 == budget)
            break;
        if (qwen_advance(&session)) return 2;
    }
    gpu_sync();
    const double generation = now() - start;
    fprintf(output,
            "],\"generated_tokens\":%d,\"generation_forward_passes\":%d,\"kv_rows\":%d,\"pending_token\":%d,"
            "\"generation_seconds\":%.9g,\"checkpoint_tested\":%s,\"checkpoint_exact\":%s,\"trace_ports\":%u}\n",
            generated, generated - 1, session.position, session.pending, generation, checkpoint_tested ? "true" : "false",
            checkpoint_tested ? (checkpoint_exact ? "true" : "false") : "null", trace.count);
    if (output_path && fclose(output)) return 2;
    if (trace.ledger && fclose(trace.ledger)) trace.failed = 1;
    free(ids);
    qwen_session_free(&session);
    qwen_model_free(&model);
    return trace.failed ? 2 : checkpoint_exact ? 0 : 1;
}
