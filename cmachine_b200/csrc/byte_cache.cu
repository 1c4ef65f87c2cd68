// Byte-codec K/V cache primitives (drop-in for src/qwen_cache.inc).
//
// Codec (src/qwen_cache.inc:3-15, CPU twin src/byte_codec.h:5-9): one row of
// 128 values per (kind, KV head); scale = max|x| / 127 with IEEE division (1
// when the row is all zero); code = clamp(roundf(x / scale), -127, 127). The
// same division and rounding run here, so codes and scales are bit-identical
// to the CPU codec for identical FP32 rows.
//
// Attention over the codes no longer decodes a full FP32 workspace and calls
// cuBLAS (src/qwen_cache.inc:16-43): the split-K attention kernel stages the
// int8 rows (gathered through `order` for the ring) and dequantises them in
// shared memory. The `scores` and `workspace` arguments are kept for ABI
// compatibility and are not touched.
#include "common.cuh"
#include "kernels.h"
#include "../../include/gpu.h"

namespace tcm {

// Block b = kind * 2 + head, 128 threads, thread d owns element d.
__global__ void encode_current_kernel(int8_t *key, int8_t *value, float *scales, const float *k, const float *v,
                                      int capacity, int position, int *invalid) {
    __shared__ float red[4];
    const int kind = blockIdx.x / 2, head = blockIdx.x % 2, d = threadIdx.x;
    const float x = (kind ? v : k)[head * 128 + d];
    const bool finite = isfinite(x);
    if (!finite) atomicExch(invalid, 1);
    float m = warp_max(finite ? fabsf(x) : 0.f);
    if ((d & 31) == 0) red[d >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float scale = m > 0.f ? __fdiv_rn(m, 127.0f) : 1.0f;
    if (!(scale > 0.f) || !isfinite(scale)) {
        if (d == 0) atomicExch(invalid, 1);
        return;
    }
    float qv = finite ? roundf(__fdiv_rn(x, scale)) : 0.f;
    qv = fminf(127.f, fmaxf(-127.f, qv));
    (kind ? value : key)[((size_t)head * capacity + position) * 128 + d] = (int8_t)qv;
    if (d == 0) scales[(kind * 2 + head) * capacity + position] = scale;
}

void encode_current(int8_t *key, int8_t *value, float *scales, const float *k, const float *v, int capacity,
                    int position, int *invalid, cudaStream_t s) {
    encode_current_kernel<<<4, 128, 0, s>>>(key, value, scales, k, v, capacity, position, invalid);
    TCM_CUDA(cudaGetLastError());
}

}  // namespace tcm

using namespace tcm;

extern "C" {

int gpu_encode_current(signed char *key, signed char *value, float *scales, const float *k, const float *v,
                       int capacity, int position, int *invalid) {
    gpu_zero(invalid, 4);
    encode_current(reinterpret_cast<int8_t *>(key), reinterpret_cast<int8_t *>(value), scales, k, v, capacity,
                   position, invalid, stream());
    int status = 0;
    gpu_read(&status, invalid, 4);
    return status ? -1 : 0;
}

// src/qwen_cache.inc:20-29: 2 KV heads x 6 query heads, rows 0..length-1.
void gpu_byte_attention(TcmGpu *g, float *out, const float *q, const signed char *key, const signed char *value,
                        const float *scales, float *, float *, int capacity, int length) {
    if (length < 1 || length > capacity) TCM_FATAL("gpu_byte_attention: invalid length");
    AttnSource src = {};
    src.kcodes = reinterpret_cast<const int8_t *>(key);
    src.vcodes = reinterpret_cast<const int8_t *>(value);
    src.scales = scales;
    float *part;
    unsigned *counters;
    attention_scratch(g, 2, &part, &counters);
    attention_split(q, src, true, capacity, length, nullptr, 12, 2, kAttnSplits, part, counters, out, stream(),
                    false);
}

// src/qwen_cache.inc:35-43: rows gathered through order[0..length); with
// `weighted`, active row i adds weights[i] * sqrt(128) to its scores.
void gpu_ring_attention(TcmGpu *g, float *out, const float *q, const signed char *key, const signed char *value,
                        const float *scales, float *, float *, const int *order, const float *weights, int capacity,
                        int length, int weighted) {
    if (length < 1 || length > capacity) TCM_FATAL("gpu_ring_attention: invalid length");
    AttnSource src = {};
    src.kcodes = reinterpret_cast<const int8_t *>(key);
    src.vcodes = reinterpret_cast<const int8_t *>(value);
    src.scales = scales;
    src.order = order;
    src.weights = weighted ? weights : nullptr;
    float *part;
    unsigned *counters;
    attention_scratch(g, 2, &part, &counters);
    attention_split(q, src, true, capacity, length, nullptr, 12, 2, kAttnSplits, part, counters, out, stream(),
                    false);
}

}  // extern "C"
