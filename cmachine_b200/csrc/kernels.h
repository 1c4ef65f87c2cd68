// Host-side launchers shared between the primitive ABI, the weight-residence
// layer and the fused decoder. All launches go to tcm::stream().
#pragma once
#include "common.cuh"
#include "attention.cuh"

struct TcmGpu;
struct QwenB200Decoder;
#include "../../include/qwen_b200.h"

namespace tcm {

// y[out] = W x for FP32 (dtype 1) or BF16 (dtype 2) row-major W.
void matvec(const void *w, int dtype, int in, int out, const float *x, float *y, cudaStream_t s);
// out[i] = float(bf16 in[i]).
void widen_bf16(float *out, const uint16_t *in, size_t n, cudaStream_t s);
// Split-K GQA attention (head_dim 128, group <= 8) over FP32 rows or byte-codec
// rows (bytes); part/counters sized by the caller.
void attention_split(const float *q, const AttnSource &source, bool bytes, int capacity, int length,
                     const int *position, int qheads, int kvheads, int nsplit, float *part, unsigned *counters,
                     float *out, cudaStream_t s, bool pdl);
// Split-K scratch of a primitive handle (grown on demand, kAttnSplits slices).
void attention_scratch(TcmGpu *g, int kvheads, float **part, unsigned **counters);
// Generic attention for any head size (reference semantics, scores written).
void attention_generic(float *out, const float *q, const float *keys, const float *values, float *scores,
                       int qheads, int kvheads, int dim, int capacity, int length, cudaStream_t s);

// Device table of RoPE denominators theta^(2d/dim) for d < dim/2.
const float *rope_denominators(float theta, int dim);

// Weight registry of the residence profile: dtype of a matrix handle
// (1 FP32, 2 BF16) or 0 when the pointer is not a registered matrix.
int weight_dtype(const void *p);

// The fused decoder's shape, tensors and tables (for the batched engine).
int decoder_view(const QwenB200Decoder *d, QwenB200Shape *shape, const QwenB200Layer **layers, const void **embed,
                 const float **final_norm, const float **rope_den, int *dtype);

// The bound of every bounded wait in each kernel module, for the current
// device (qwen_b200_wait_limit sets them all).
void set_wait_limit_decode(unsigned long long ns);
void set_wait_limit_persistent(unsigned long long ns);
void set_wait_limit_batch(unsigned long long ns);

}  // namespace tcm
