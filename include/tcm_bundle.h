/* TCM1LE model bundles: the reference loader's C ABI (src/machine.h:7-27,
 * implemented by src/model.c:49-97) for the format tools/bundle.py:22-58 writes.
 *
 * Layout, little-endian: 8-byte magic "TCM1LE\0\0"; the SHA-256 of every byte
 * after offset 40; architecture (u32) and tensor count (u32) at 40; config[16]
 * (u32) at 48; the model identity, 64 lowercase hex digits, at 112; from 176 a
 * table of `count` 120-byte records {name[64] (NUL-terminated), rank u32,
 * dtype u32, dim[4] u64, offset u64, bytes u64}; then the tensor payloads in
 * table order, each at an offset aligned to its element size, not before the
 * previous one's end, the last one ending at the end of the file.
 * tcm_load maps the file read-only; TcmTensor.data points into the mapping. */
#ifndef TCM_BUNDLE_H
#define TCM_BUNDLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { TCM_ISA = 1, TCM_QWEN = 2, TCM_ISA_LAW = 3, TCM_PROGRAM = 4 };
enum { TCM_F32 = 1, TCM_BF16 = 2, TCM_F64 = 3 };

typedef struct {
    char name[65];
    uint32_t rank, dtype;
    uint64_t dim[4], bytes;
    const void *data;
} TcmTensor;

typedef struct {
    uint32_t architecture, count, config[16];
    char identity[65], digest[65];
    TcmTensor *tensor;
    void *mapping;
    size_t mapping_bytes;
} TcmModel;

/* 0, or -1 with a message in error[0..capacity) and *m cleared. */
int tcm_load(TcmModel *m, const char *path, char *error, size_t capacity);
void tcm_unload(TcmModel *m);
const TcmTensor *tcm_tensor(const TcmModel *m, const char *name);
void tcm_sha256(const void *data, size_t n, unsigned char out[32]);
/* n bytes as 2n lowercase hex digits and a NUL. */
void tcm_hex(const unsigned char *p, size_t n, char *out);

#ifdef __cplusplus
}
#endif

#endif
