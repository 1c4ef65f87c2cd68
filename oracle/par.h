/* Test infrastructure only: a static-partition parallel loop on pthreads (the
 * image's gcc has no OpenMP runtime). Each index runs exactly once and keeps
 * its own sequential arithmetic, so results never depend on the thread count.
 * ORACLE_THREADS caps the threads (default: online cores, at most 64). */
#ifndef TCM_ORACLE_PAR_H
#define TCM_ORACLE_PAR_H
#include <pthread.h>
#include <stdlib.h>
#include <unistd.h>

typedef void (*par_body)(void *ctx, size_t begin, size_t end);
typedef struct { par_body body; void *ctx; size_t begin, end; } par_slice;

static void *par_run(void *p) {
    par_slice *s = p;
    s->body(s->ctx, s->begin, s->end);
    return NULL;
}
static int par_threads(void) {
    const char *env = getenv("ORACLE_THREADS");
    long n = env ? atol(env) : sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 64) n = 64;
    return (int)n;
}
/* Runs body over [0, n) split into contiguous slices; small loops stay serial. */
static void par_for(size_t n, size_t min_per_thread, par_body body, void *ctx) {
    int t = par_threads();
    if ((size_t)t > n / (min_per_thread ? min_per_thread : 1)) t = (int)(n / (min_per_thread ? min_per_thread : 1));
    if (t <= 1) { body(ctx, 0, n); return; }
    pthread_t ids[64];
    par_slice slices[64];
    for (int i = 0; i < t; i++) {
        slices[i] = (par_slice){body, ctx, n * (size_t)i / (size_t)t, n * (size_t)(i + 1) / (size_t)t};
        if (pthread_create(&ids[i], NULL, par_run, &slices[i])) { par_run(&slices[i]); ids[i] = 0; }
    }
    for (int i = 0; i < t; i++) if (ids[i]) pthread_join(ids[i], NULL);
}
#endif
