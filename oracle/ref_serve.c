/* Test infrastructure only: the reference's own serving loops on its CPU path.
 *
 * oracle/Makefile links the reference's src/qwen_serve.c and
 * src/qwen_bounded_serve.c, unchanged, with src/qwen.c, src/model.c and the
 * CPU primitives of tests/gpu_stub.c into _ref/ref-serve-cpu, so a scripted
 * protocol session can be replayed through the reference and through this
 * repository's tcm-cuda and the replies compared field by field.
 *
 * The reference's qwen_model_init only accepts 28-layer bundle files
 * (src/qwen.c:25-27), so the link wraps tcm_load, tcm_unload and
 * qwen_model_init (ld --wrap): a MODEL of the form seeded:SHAPE:SEED:PROFILE
 * builds the same seeded random-init model as this repository's serve
 * (weights N(0, 0.02) through include/tcm_seeded.h, norms 1, biases 0; model
 * identity and digest strings as qwen_model_init_seeded writes them), field by
 * field as ref_driver.c does; any other MODEL goes to the reference's loader.
 * gpu_weight_configure, gpu_weight_release and gpu_live_bytes, which the
 * bounded serve calls and the CPU stub lacks, are no-ops (0 live bytes). The
 * byte codec and ring attention come from ref_ring.c. */
#define _POSIX_C_SOURCE 200809L
#include "qwen.h"
#include "oracle_api.h"
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

int __real_tcm_load(TcmModel *, const char *, char *, size_t);
void __real_tcm_unload(TcmModel *);
int __real_qwen_model_init(QwenModel *, const TcmModel *, char *, size_t);
QwenModel *orc_model_take(void *model);

static int seeded, profile;
static OrcShape shape;
static uint64_t seed;

void gpu_weight_configure(int p) { (void)p; }
void gpu_weight_release(void) {}
size_t gpu_live_bytes(void) { return 0; }

static int number(const char *p, const char **end, long lo, long hi, long *out) {
    char *e;
    errno = 0;
    long v = strtol(p, &e, 10);
    if (errno || e == p || v < lo || v > hi) return -1;
    *out = v;
    *end = e;
    return 0;
}
/* qwen2.5-1.5b, qwen2.5-1.5b@LAYERS, or HIDDENxLAYERSxQHEADSxKVHEADSxHEADxINTERxVOCABxPOSITIONS. */
static int parse_shape(const char *text, size_t n, OrcShape *s) {
    const OrcShape qwen = {1536, 28, 12, 2, 128, 8960, 151936, 32768, 1e-6f, 1e6f};
    *s = qwen;
    char buf[128];
    if (n >= sizeof(buf)) return -1;
    memcpy(buf, text, n);
    buf[n] = 0;
    if (!strcmp(buf, "qwen2.5-1.5b")) return 0;
    const char *end;
    long v;
    if (!strncmp(buf, "qwen2.5-1.5b@", 13)) {
        if (number(buf + 13, &end, 1, 64, &v) || *end) return -1;
        s->layers = (int)v;
        return 0;
    }
    int dims[8];
    const char *p = buf;
    for (int i = 0; i < 8; i++) {
        if (number(p, &end, 1, 1 << 20, &v)) return -1;
        dims[i] = (int)v;
        if (i < 7 && *end != 'x') return -1;
        p = end + 1;
    }
    if (*end) return -1;
    OrcShape c = {dims[0], dims[1], dims[2], dims[3], dims[4], dims[5], dims[6], dims[7], 1e-6f, 1e6f};
    *s = c;
    return 0;
}

int __wrap_tcm_load(TcmModel *b, const char *path, char *error, size_t cap) {
    if (strncmp(path, "seeded:", 7)) return __real_tcm_load(b, path, error, cap);
    const char *a = path + 7, *c1 = strchr(a, ':'), *c2 = c1 ? strchr(c1 + 1, ':') : NULL, *end;
    long s, p;
    if (!c1 || !c2 || parse_shape(a, (size_t)(c1 - a), &shape) || number(c1 + 1, &end, 0, 2147483647, &s) ||
        end != c2 || number(c2 + 1, &end, 0, 2, &p) || *end || p == 1) {
        snprintf(error, cap, "invalid seeded model specification");
        return -1;
    }
    seed = (uint64_t)s;
    profile = (int)p;
    seeded = 1;
    memset(b, 0, sizeof(*b));
    return 0;
}

void __wrap_tcm_unload(TcmModel *b) {
    if (seeded) return;
    __real_tcm_unload(b);
}

int __wrap_qwen_model_init(QwenModel *m, const TcmModel *b, char *error, size_t cap) {
    if (!seeded) return __real_qwen_model_init(m, b, error, cap);
    const TcmFillLaw law = {{0.0f, 0.02f}, {1.0f, 0.0f}, {0.0f, 0.0f}};
    *m = *orc_model_take(orc_model_create(&shape, seed, &law, profile == 2));
    /* What the reference's loader adds up (src/qwen.c:22): the CPU stub holds
     * every tensor as FP32 (tests/gpu_stub.c gpu_owned_weight_bytes). */
    const size_t d = (size_t)shape.hidden, qd = (size_t)shape.qheads * shape.head, kv = (size_t)shape.kvheads * shape.head,
                 f = (size_t)shape.intermediate;
    const size_t per_layer = 2 * d + qd * d + 2 * kv * d + qd + 2 * kv + d * qd + 3 * f * d;
    m->weight_bytes = ((size_t)shape.vocab * d + d + per_layer * (size_t)shape.layers) * sizeof(float);
    snprintf(m->identity, sizeof(m->identity), "seeded-%016llx", (unsigned long long)seed);
    snprintf(m->digest, sizeof(m->digest), "seeded-%016llx-%08x-%08x-%d", (unsigned long long)seed,
             (unsigned)(law.matrix.scale * 1e6f), (unsigned)shape.layers, profile);
    return 0;
}

int main(int argc, char **argv) {
    if (argc >= 2 && !strcmp(argv[1], "serve")) return qwen_serve_main(argc, argv);
    fprintf(stderr, "usage: ref-serve-cpu serve MODEL [options]\n");
    return 2;
}
