/* The device primitive ABI of cmachine's Qwen runtime, implemented for B200.
 *
 * This header replaces the reference's src/gpu.h: a C caller written against
 * that header (the reference's src/qwen.c, src/bounded_cache.h, tests) links
 * against libcmachine_b200.so unchanged. Every prototype keeps the reference's
 * name, argument order and meaning; the line after each group cites the
 * reference declaration it replaces. Semantics kept from the reference:
 *   - all pointers are device pointers owned by the caller; gpu_alloc'd blocks
 *     are tracked process-wide and gpu_free of an unknown pointer is fatal
 *     (src/qwen_cuda.cu:13-19);
 *   - any CUDA error is fatal: message on stderr, exit(2) (src/qwen_cuda.cu:8);
 *   - gpu_top2 exits(2) on non-finite input (src/qwen_cuda.cu:117);
 *   - work is ordered as one stream: gpu_read returns data written by every
 *     earlier call.
 * What differs: no cuBLAS (hand-written sm_100a kernels), BF16 matrices are
 * read directly (no FP32 tile), and matvec/attention use FP32 with fused
 * multiply-add in a fixed parallel order, so results match the reference to
 * tolerance rather than bit for bit. Every kernel is deterministic: the same
 * inputs give the same bits on every call.
 */
#ifndef TCM_GPU_H
#define TCM_GPU_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct TcmGpu TcmGpu;
/* Top-2 of a vector: ids and values; ties go to the lower id. (src/gpu.h:9) */
typedef struct { int first, second; float first_value, second_value; } TcmTop2;

/* Handle with per-caller scratch (top-2 partials, flags). (src/gpu.h:10-11) */
TcmGpu *gpu_open(void);
void gpu_close(TcmGpu *);

/* Tracked device memory and copies. (src/gpu.h:12-17, 38, 49-51) */
void *gpu_alloc(size_t bytes);
void gpu_free(void *);
void gpu_zero(void *, size_t bytes);
void gpu_copy(void *dst, const void *src, size_t bytes);   /* device -> device */
void gpu_read(void *host, const void *dev, size_t bytes);  /* device -> host, synchronous */
void gpu_write(void *dev, const void *host, size_t bytes); /* host -> device, synchronous */
void gpu_sync(void);
size_t gpu_live_bytes(void);
size_t gpu_peak_bytes(void);
size_t gpu_free_bytes(void);

/* Upload n host values of dtype 1 (FP32) or 2 (BF16, widened) as FP32. (src/gpu.h:18) */
float *gpu_weight(const void *host, uint32_t dtype, size_t n);

/* y[out] = W[out][in] x, W row-major. If W was registered by gpu_owned_weight
 * under profile 2 it holds BF16 and is read as such. (src/gpu.h:19) */
void gpu_matvec(TcmGpu *, const float *w, int in, int out, const float *x, float *y);
/* out = (x * r) * w, r = rsqrt(mean(x^2) + eps); _scale also stores r. (src/gpu.h:20-23) */
void gpu_rms(float *out, const float *x, const float *w, int n, float eps);
void gpu_rms_scale(float *out, const float *x, const float *w, int n, float eps, float *scale);
/* Experimental elementwise ops of the receiver-plane studies. (src/gpu.h:24-28) */
void gpu_multiply(float *out, const float *x, const float *y, int n);
void gpu_plane(float *out, const float *base, const float *a, const float *b, int n, float s, float t);
void gpu_plane_scaled(float *out, const float *base, const float *a, const float *b, int n, float s, float t,
                      const float *scale);
void gpu_linear2(float *out, const float *a, const float *b, int n, float ca, float cb, const float *scale);
/* 1 when a and b are bitwise equal and finite, else 0. (src/gpu.h:29) */
int gpu_identical_finite(TcmGpu *, const float *a, const float *b, int n);
/* x += y. (src/gpu.h:30-31) */
void gpu_add(float *x, const float *y, int n);
void gpu_bias(float *x, const float *y, int n);
/* Half-split RoPE of `heads` rows of `dim` at `position`. (src/gpu.h:32) */
void gpu_rope(float *x, int heads, int dim, int position, float theta);
/* Row `position` of each head's [capacity][dim] slab <- x. (src/gpu.h:33) */
void gpu_cache(float *cache, const float *x, int heads, int dim, int capacity, int position);
/* GQA attention of qheads query rows over `length` cached rows; query head h
 * reads K/V head h / (qheads / kvheads); scores is scratch. (src/gpu.h:34) */
void gpu_attention(TcmGpu *, float *out, const float *q, const float *keys, const float *values, float *scores,
                   int qheads, int kvheads, int dim, int capacity, int length);
/* gpu_attention for callers that may not allocate device memory while they run
 * (a host that owns all GPU memory through its own pool, a loop that cannot
 * take cudaFree's device-wide synchronisation). No counterpart in the
 * reference. Same result as gpu_attention for dim 128; no scores are written.
 * Its split-K scratch is a fixed 1.2 MB device array inside the library, held
 * by every GPU that loads it: limits are dim == 128, 1 <= kvheads <= 4, at most
 * 8 query heads per KV head, 1 <= length <= capacity; other sizes return -1
 * with a message on stderr and launch nothing. Returns 0 when launched. CUDA
 * errors are fatal (message, exit(2)) as everywhere in this ABI; only sizes and
 * alignment come back as -1. The first call on each device looks up the
 * array's device address, and under the runtime's lazy module loading that is
 * also when the device first holds the array's 1.2 MB: make that first call at
 * start-up, before handing device memory to a pool and before any stream
 * capture. Calls share the array: calls that overlap on the GPU race. */
int gpu_attention_static(float *out, const float *q, const float *keys, const float *values, int qheads,
                         int kvheads, int dim, int capacity, int length);
/* gate = silu(gate) * up. (src/gpu.h:35) */
void gpu_swiglu(float *gate, const float *up, int n);
/* Experimental polynomial gate law. (src/gpu.h:36-38) */
void gpu_gate_anchor(const float *g, float *p, float *first, float *second, float *s, int n);
void gpu_gate_swiglu(float *g, const float *u, const float *source, const float *p, const float *first,
                     const float *second, const float *s, int n);
/* Top-2 of x[0..n). (src/gpu.h:39) */
TcmTop2 gpu_top2(TcmGpu *, const float *x, int n);

/* Process-wide weight residence profile: 0 native FP32, 1 tiled FP32 (kept as
 * native FP32 here: no tile is needed), 2 source BF16 matrices. Choose before
 * load; release after the model is freed. (src/gpu.h:40-48) */
void gpu_weight_configure(int profile);
float *gpu_owned_weight(TcmGpu *, const void *host, uint32_t dtype, size_t count, int rank, int rows, int columns);
size_t gpu_owned_weight_bytes(const float *, size_t count);
void gpu_owned_embedding(float *out, const float *embedding, int token, int width);
void gpu_weight_release(void);
void gpu_weight_info(size_t *matrix, size_t *vectors, size_t *scratch, int *count, unsigned long long *matvecs,
                     unsigned long long *tiles, unsigned long long *embeddings);

/* Byte-codec K/V cache (src/qwen_cache.inc:13,20,35; declared by the reference
 * in src/bounded_cache.h:7-8). Per (kind, KV head) row: scale = max|x|/127 (1
 * when zero) and code = clamp(round(x/scale), +-127). Returns 0, or -1 when the
 * row holds a non-finite value. Layout per layer: K codes [2][capacity][128],
 * V codes [2][capacity][128], scales [kind*2+head][capacity]. */
int gpu_encode_current(signed char *key, signed char *value, float *scales, const float *k, const float *v,
                       int capacity, int position, int *invalid);
void gpu_byte_attention(TcmGpu *, float *out, const float *q, const signed char *key, const signed char *value,
                        const float *scales, float *scores, float *workspace, int capacity, int length);
void gpu_ring_attention(TcmGpu *, float *out, const float *q, const signed char *key, const signed char *value,
                        const float *scales, float *scores, float *workspace, const int *order,
                        const float *weights, int capacity, int length, int weighted);

#ifdef __cplusplus
}
#endif
#endif
