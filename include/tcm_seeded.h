/* Seeded random-init weights for a Qwen2.5-architecture decoder.
 *
 * The reference ships no weight generator: its tests build a QwenModel by hand
 * (tests/state_mechanics.c:12-22) and real runs load pretrained bundles. This
 * header defines the one generator that every party here shares -- the CPU
 * oracle, the reference CPU driver and the GPU fill kernel -- so that all of
 * them consume bit-identical weights.
 *
 * Element i of tensor t under model seed S:
 *   base  = mix64(S ^ ((t + 1) * 0xD1B54A32D192ED03))
 *   u_j   = mix64(base + (3*i + j + 1) * 0x9E3779B97F4A7C15), j = 0, 1, 2
 *   sum   = the twelve 16-bit fields of u_0, u_1, u_2 added as integers
 *   value = offset + (float)(sum - 393210) * (scale * 2^-16)
 * mix64 is the SplitMix64 output function (Steele, Lea & Flood 2014; the same
 * mixer the reference uses for reservoir draws, src/bounded_cache.h:24). The
 * sum of twelve uniforms is the classical Irwin-Hall approximation of a normal
 * variate: mean 0 and standard deviation 65536 in integer units, so the value
 * has standard deviation `scale` and is bounded by +-6 scale.
 *
 * Every step is integer arithmetic followed by one exact conversion and one
 * IEEE multiply (plus one add when offset != 0), so CPU and GPU agree bit for
 * bit. BF16 storage rounds the FP32 value to nearest-even.
 *
 * Tensor ids follow the reference's load order (src/qwen.c:34-41):
 *   0 embedding [vocab][hidden], 1 final norm [hidden], then for layer l the
 *   ids 2 + 12 l + {0 input_norm, 1 post_norm, 2 q, 3 k, 4 v, 5 q bias,
 *   6 k bias, 7 v bias, 8 o, 9 gate, 10 up, 11 down}.
 */
#ifndef TCM_SEEDED_H
#define TCM_SEEDED_H
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define TCM_SEEDED_FN static __host__ __device__ __forceinline__
#else
#define TCM_SEEDED_FN static inline
#endif

enum {
    TCM_T_INPUT_NORM = 0, TCM_T_POST_NORM, TCM_T_Q, TCM_T_K, TCM_T_V, TCM_T_QB, TCM_T_KB,
    TCM_T_VB, TCM_T_O, TCM_T_GATE, TCM_T_UP, TCM_T_DOWN, TCM_T_PER_LAYER
};

/* How one tensor is filled: value = offset + normal * scale (scale 0: constant). */
typedef struct { float offset, scale; } TcmFill;

/* Fill laws for the seeded Qwen model. The benchmark law has linear and
 * embedding weights N(0, 0.02), biases 0 and norm weights 1. Parity tests use a
 * law with nonzero biases and non-unit norms so that those terms are exercised. */
typedef struct { TcmFill matrix, norm, bias; } TcmFillLaw;

TCM_SEEDED_FN uint64_t tcm_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
    z = (z ^ (z >> 27)) * UINT64_C(0x94d049bb133111eb);
    return z ^ (z >> 31);
}
TCM_SEEDED_FN uint64_t tcm_tensor_base(uint64_t seed, uint32_t tensor) {
    return tcm_mix64(seed ^ ((uint64_t)(tensor + 1) * UINT64_C(0xD1B54A32D192ED03)));
}
TCM_SEEDED_FN int32_t tcm_irwin12(uint64_t base, uint64_t i) {
    int32_t sum = 0;
    for (uint64_t j = 0; j < 3; j++) {
        uint64_t u = tcm_mix64(base + (3 * i + j + 1) * UINT64_C(0x9E3779B97F4A7C15));
        sum += (int32_t)(u & 0xffff) + (int32_t)((u >> 16) & 0xffff) +
               (int32_t)((u >> 32) & 0xffff) + (int32_t)(u >> 48);
    }
    return sum - 393210;
}
/* scale * 2^-16 is exact for any normal float scale. */
TCM_SEEDED_FN float tcm_fill_step(TcmFill f) { return f.scale * (1.0f / 65536.0f); }
TCM_SEEDED_FN float tcm_seeded_value(uint64_t base, uint64_t i, TcmFill f) {
    if (f.scale == 0.0f) return f.offset;
#if defined(__CUDA_ARCH__)
    float v = __fmul_rn((float)tcm_irwin12(base, i), tcm_fill_step(f));
    return f.offset != 0.0f ? __fadd_rn(f.offset, v) : v;
#else
    volatile float v = (float)tcm_irwin12(base, i) * tcm_fill_step(f);
    return f.offset != 0.0f ? f.offset + v : v;
#endif
}
TCM_SEEDED_FN uint16_t tcm_bf16_rne(float x) {
    uint32_t bits;
#if defined(__CUDA_ARCH__)
    bits = __float_as_uint(x);
#else
    memcpy(&bits, &x, 4);
#endif
    bits += 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)(bits >> 16);
}
TCM_SEEDED_FN float tcm_bf16_to_float(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
#if defined(__CUDA_ARCH__)
    return __uint_as_float(bits);
#else
    float x;
    memcpy(&x, &bits, 4);
    return x;
#endif
}
/* Which fill a tensor id gets under a law. */
TCM_SEEDED_FN TcmFill tcm_tensor_fill(const TcmFillLaw *law, uint32_t tensor) {
    if (tensor == 0) return law->matrix;
    if (tensor == 1) return law->norm;
    uint32_t kind = (tensor - 2) % TCM_T_PER_LAYER;
    if (kind == TCM_T_INPUT_NORM || kind == TCM_T_POST_NORM) return law->norm;
    if (kind == TCM_T_QB || kind == TCM_T_KB || kind == TCM_T_VB) return law->bias;
    return law->matrix;
}
TCM_SEEDED_FN uint32_t tcm_layer_tensor(int layer, int kind) {
    return 2u + (uint32_t)layer * TCM_T_PER_LAYER + (uint32_t)kind;
}
/* Uniform token ids in [0, vocab): stream `seed`, draw i (used for prompts). */
TCM_SEEDED_FN int tcm_seeded_token(uint64_t seed, uint64_t i, int vocab) {
    uint64_t u = tcm_mix64(tcm_mix64(seed ^ UINT64_C(0x5851F42D4C957F2D)) + (i + 1) * UINT64_C(0x9E3779B97F4A7C15));
    return (int)((u >> 11) % (uint64_t)vocab);
}
#endif
