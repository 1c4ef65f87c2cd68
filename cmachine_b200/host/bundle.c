/* TCM1LE bundle loader and SHA-256 (include/tcm_bundle.h), the drop-in for
 * the reference's src/model.c:49-97: the same checks, in the same order, with
 * the same messages, so a caller sees the same accept/reject decision and
 * digest for any file. */
#define _POSIX_C_SOURCE 200809L
#include "../../include/tcm_bundle.h"

#include <fcntl.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------------ SHA-256 (FIPS 180-4) */

/* The round constants are the first 32 fractional bits of the cube roots of
 * the first 64 primes and the initial hash the same bits of the square roots
 * of the first 8: floor(root(p) * 2^32) mod 2^32, computed here with exact
 * integer roots of p * 2^96 and p * 2^64. */
static uint32_t round_k[64], initial_h[8];
static pthread_once_t constants_once = PTHREAD_ONCE_INIT;

static uint64_t integer_root(unsigned __int128 x, int cube) {
    uint64_t lo = 0, hi = (uint64_t)1 << 40;  /* root < 2^36 for both uses */
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo + 1) / 2;
        unsigned __int128 p = (unsigned __int128)mid * mid;
        if (cube) p *= mid;
        if (p <= x) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}
static void derive_constants(void) {
    int found = 0;
    for (uint32_t n = 2; found < 64; n++) {
        int prime = 1;
        for (uint32_t d = 2; d * d <= n; d++)
            if (n % d == 0) { prime = 0; break; }
        if (!prime) continue;
        round_k[found] = (uint32_t)integer_root((unsigned __int128)n << 96, 1);
        if (found < 8) initial_h[found] = (uint32_t)integer_root((unsigned __int128)n << 64, 0);
        found++;
    }
}

static inline uint32_t ror(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static void compress(uint32_t state[8], const unsigned char block[64]) {
    uint32_t w[64];
    for (int t = 0; t < 16; t++)
        w[t] = (uint32_t)block[4 * t] << 24 | (uint32_t)block[4 * t + 1] << 16 | (uint32_t)block[4 * t + 2] << 8 |
               (uint32_t)block[4 * t + 3];
    for (int t = 16; t < 64; t++) {
        const uint32_t s0 = ror(w[t - 15], 7) ^ ror(w[t - 15], 18) ^ (w[t - 15] >> 3);
        const uint32_t s1 = ror(w[t - 2], 17) ^ ror(w[t - 2], 19) ^ (w[t - 2] >> 10);
        w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t r[8];
    memcpy(r, state, sizeof(r));
    for (int t = 0; t < 64; t++) {
        const uint32_t e = r[4], a = r[0];
        const uint32_t t1 = r[7] + (ror(e, 6) ^ ror(e, 11) ^ ror(e, 25)) + ((e & r[5]) ^ (~e & r[6])) + round_k[t] + w[t];
        const uint32_t t2 = (ror(a, 2) ^ ror(a, 13) ^ ror(a, 22)) + ((a & r[1]) ^ (a & r[2]) ^ (r[1] & r[2]));
        memmove(&r[1], &r[0], 7 * sizeof(uint32_t));
        r[4] += t1;
        r[0] = t1 + t2;
    }
    for (int i = 0; i < 8; i++) state[i] += r[i];
}

void tcm_sha256(const void *data, size_t n, unsigned char out[32]) {
    pthread_once(&constants_once, derive_constants);
    uint32_t state[8];
    memcpy(state, initial_h, sizeof(state));
    const unsigned char *p = (const unsigned char *)data;
    size_t whole = n / 64;
    for (size_t i = 0; i < whole; i++) compress(state, p + 64 * i);
    /* The tail, a 1 bit, zeros, then the message length in bits (big-endian). */
    unsigned char last[128];
    memset(last, 0, sizeof(last));
    const size_t rest = n - 64 * whole;
    if (rest) memcpy(last, p + 64 * whole, rest);
    last[rest] = 0x80;
    const size_t end = rest < 56 ? 64 : 128;
    const uint64_t bits = (uint64_t)n << 3;
    for (int i = 0; i < 8; i++) last[end - 1 - i] = (unsigned char)(bits >> (8 * i));
    for (size_t off = 0; off < end; off += 64) compress(state, last + off);
    for (int i = 0; i < 8; i++) {
        out[4 * i] = (unsigned char)(state[i] >> 24);
        out[4 * i + 1] = (unsigned char)(state[i] >> 16);
        out[4 * i + 2] = (unsigned char)(state[i] >> 8);
        out[4 * i + 3] = (unsigned char)state[i];
    }
}

void tcm_hex(const unsigned char *p, size_t n, char *out) {
    static const char digits[] = "0123456789abcdef";
    for (size_t i = 0; i < n; i++) {
        out[2 * i] = digits[p[i] >> 4];
        out[2 * i + 1] = digits[p[i] & 15];
    }
    out[2 * n] = 0;
}

/* ------------------------------------------------------------------ bundle */

static uint32_t le32(const unsigned char *p) {
    return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24;
}
static uint64_t le64(const unsigned char *p) { return (uint64_t)le32(p) | (uint64_t)le32(p + 4) << 32; }

static int refuse(TcmModel *m, char *error, size_t capacity, const char *why) {
    if (error && capacity) snprintf(error, capacity, "%s", why);
    tcm_unload(m);
    return -1;
}

enum { HEADER_BYTES = 176, RECORD_BYTES = 120, MAX_TENSORS = 4096 };

int tcm_load(TcmModel *m, const char *path, char *error, size_t capacity) {
    memset(m, 0, sizeof(*m));
    const uint32_t probe = 1;
    if (*(const unsigned char *)&probe != 1) return refuse(m, error, capacity, "little-endian host required");
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return refuse(m, error, capacity, "cannot open model bundle");
    struct stat st;
    if (fstat(fd, &st) || st.st_size < HEADER_BYTES) {
        close(fd);
        return refuse(m, error, capacity, "truncated model bundle");
    }
    m->mapping_bytes = (size_t)st.st_size;
    m->mapping = mmap(NULL, m->mapping_bytes, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m->mapping == MAP_FAILED) {
        m->mapping = NULL;
        return refuse(m, error, capacity, "model mmap failed");
    }
    const unsigned char *p = (const unsigned char *)m->mapping;
    if (memcmp(p, "TCM1LE\0\0", 8)) return refuse(m, error, capacity, "unsupported bundle magic");
    unsigned char digest[32];
    tcm_sha256(p + 40, m->mapping_bytes - 40, digest);
    if (memcmp(digest, p + 8, 32)) return refuse(m, error, capacity, "bundle SHA256 mismatch");
    tcm_hex(digest, 32, m->digest);
    m->architecture = le32(p + 40);
    m->count = le32(p + 44);
    if (m->count == 0 || m->count > MAX_TENSORS) return refuse(m, error, capacity, "invalid tensor count");
    for (int i = 0; i < 16; i++) m->config[i] = le32(p + 48 + 4 * i);
    memcpy(m->identity, p + 112, 64);
    m->identity[64] = 0;
    for (int i = 0; i < 64; i++) {
        const char c = m->identity[i];
        if (!((c >= '0' && c <= '9') || (c >= 'a' && c <= 'f'))) return refuse(m, error, capacity, "invalid model identity");
    }
    const size_t table_end = HEADER_BYTES + (size_t)m->count * RECORD_BYTES;
    if (table_end > m->mapping_bytes) return refuse(m, error, capacity, "truncated tensor table");
    m->tensor = (TcmTensor *)calloc(m->count, sizeof(TcmTensor));
    if (!m->tensor) return refuse(m, error, capacity, "tensor descriptor allocation failed");
    uint64_t end = table_end;
    for (uint32_t i = 0; i < m->count; i++) {
        const unsigned char *rec = p + HEADER_BYTES + (size_t)i * RECORD_BYTES;
        TcmTensor *t = &m->tensor[i];
        memcpy(t->name, rec, 64);
        t->name[64] = 0;
        t->rank = le32(rec + 64);
        t->dtype = le32(rec + 68);
        if (!memchr(rec, 0, 64) || !t->name[0] || t->rank > 4)
            return refuse(m, error, capacity, "invalid tensor descriptor");
        uint64_t elements = 1;
        for (uint32_t j = 0; j < 4; j++) {
            t->dim[j] = le64(rec + 72 + 8 * j);
            if (j >= t->rank) continue;
            if (!t->dim[j] || elements > UINT64_MAX / t->dim[j]) return refuse(m, error, capacity, "invalid tensor dimensions");
            elements *= t->dim[j];
        }
        const uint64_t offset = le64(rec + 104);
        t->bytes = le64(rec + 112);
        const uint64_t item = t->dtype == TCM_F32 ? 4 : t->dtype == TCM_BF16 ? 2 : t->dtype == TCM_F64 ? 8 : 0;
        if (!item || elements > UINT64_MAX / item || t->bytes != elements * item || offset % item || offset < end ||
            offset > m->mapping_bytes || t->bytes > m->mapping_bytes - offset)
            return refuse(m, error, capacity, "invalid tensor extent or dtype");
        for (uint32_t j = 0; j < i; j++)
            if (!strcmp(t->name, m->tensor[j].name)) return refuse(m, error, capacity, "duplicate tensor name");
        t->data = p + offset;
        end = offset + t->bytes;
    }
    if (end != m->mapping_bytes) return refuse(m, error, capacity, "trailing bundle bytes");
    return 0;
}

void tcm_unload(TcmModel *m) {
    if (m->mapping) munmap(m->mapping, m->mapping_bytes);
    free(m->tensor);
    memset(m, 0, sizeof(*m));
}

const TcmTensor *tcm_tensor(const TcmModel *m, const char *name) {
    for (uint32_t i = 0; i < m->count; i++)
        if (!strcmp(m->tensor[i].name, name)) return &m->tensor[i];
    return NULL;
}
