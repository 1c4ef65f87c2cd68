// The reference's device primitive set (src/qwen_cuda.cu:25-118) as
// hand-written sm_100a kernels: no cuBLAS, every reduction in a fixed order.
#include "common.cuh"
#include "gemv.cuh"
#include "attention.cuh"
#include "kernels.h"
#include "../../include/gpu.h"
#include <math.h>
#include <mutex>

struct TcmGpu {
    float *part_values;  // top-2 partials [2 * kTopBlocks]
    int *part_ids;
    int *invalid;        // [0]: non-finite flag, [1]: last-block counter
    TcmTop2 *result;
    float *attn_part;    // split-K attention partials (grown on demand)
    unsigned *attn_counters;
    size_t attn_part_floats;
    int attn_kv;
};

namespace tcm {

constexpr int kTopBlocks = 1184;  // grid-stride top-2 blocks (148 SMs x 8)
constexpr int kThreads = 256;

// ---------------------------------------------------------------- widen / matvec
__global__ void widen_kernel(float *out, const uint16_t *in, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __uint_as_float((uint32_t)in[i] << 16);
}
void widen_bf16(float *out, const uint16_t *in, size_t n, cudaStream_t s) {
    if (!n) return;
    const size_t blocks = (n + kThreads - 1) / kThreads;
    widen_kernel<<<(unsigned)(blocks < 65535u * 16u ? blocks : 65535u * 16u), kThreads, 0, s>>>(out, in, n);
    TCM_CUDA(cudaGetLastError());
}

// Vector path: rows are 16-byte aligned (in * sizeof(WT) % 16 == 0).
template <typename WT, bool SMEM_X>
__global__ void __launch_bounds__(kThreads) matvec_kernel(const WT *__restrict__ w, int in, int out,
                                                          const float *__restrict__ x, float *__restrict__ y) {
    extern __shared__ __align__(16) float xs_dyn[];
    const float *xs = x;
    if (SMEM_X) {
        for (int i = threadIdx.x; i < in; i += blockDim.x) xs_dyn[i] = x[i];
        __syncthreads();
        xs = xs_dyn;
    }
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int nvec = in / WVec<WT>::kElems;
    for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < out; row += warps) {
        const WT *rows[1] = {w + (size_t)row * in};
        float acc[1];
        warp_rows_dot<WT, 1, 8>(rows, xs, nvec, lane, acc);
        if (lane == 0) y[row] = acc[0];
    }
}
// Scalar path for unaligned shapes (tiny test fixtures).
template <typename WT>
__global__ void matvec_scalar_kernel(const WT *__restrict__ w, int in, int out, const float *__restrict__ x,
                                     float *__restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < out; row += warps) {
        const WT *r = w + (size_t)row * in;
        float acc = 0.f;
        for (int i = lane; i < in; i += 32) {
            float wv;
            if constexpr (sizeof(WT) == 4) wv = r[i];
            else wv = __uint_as_float((uint32_t)r[i] << 16);
            acc = fmaf(wv, x[i], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[row] = acc;
    }
}

template <typename WT>
static void matvec_typed(const WT *w, int in, int out, const float *x, float *y, cudaStream_t s) {
    if (in <= 0 || out <= 0) return;
    const int max_blocks = sm_count() * 8;
    int blocks = (out + 7) / 8;
    if (blocks > max_blocks) blocks = max_blocks;
    const bool aligned = ((size_t)in * sizeof(WT)) % 16 == 0 && ((uintptr_t)w & 15) == 0 && ((uintptr_t)x & 15) == 0;
    if (!aligned) {
        matvec_scalar_kernel<WT><<<blocks, kThreads, 0, s>>>(w, in, out, x, y);
    } else if ((size_t)in * 4 <= 96 * 1024) {
        static PerDeviceOnce once;
        once.run([] {
            TCM_CUDA(cudaFuncSetAttribute(matvec_kernel<WT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          96 * 1024));
        });
        matvec_kernel<WT, true><<<blocks, kThreads, (size_t)in * 4, s>>>(w, in, out, x, y);
    } else {
        matvec_kernel<WT, false><<<blocks, kThreads, 0, s>>>(w, in, out, x, y);
    }
    TCM_CUDA(cudaGetLastError());
}

void matvec(const void *w, int dtype, int in, int out, const float *x, float *y, cudaStream_t s) {
    if (dtype == 2) matvec_typed(static_cast<const uint16_t *>(w), in, out, x, y, s);
    else matvec_typed(static_cast<const float *>(w), in, out, x, y, s);
}

// ---------------------------------------------------------------- rms
// One block; the sum of squares is a fixed-order block reduction, then
// out = (x * r) * w with r = 1 / sqrt(mean + eps) (src/qwen_cuda.cu:35-40).
__global__ void __launch_bounds__(1024) rms_kernel(float *out, const float *x, const float *w, int n, float eps,
                                                  float *scale_out) {
    __shared__ float red[32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    const float total = block_sum(ss, red);
    const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], r), w[i]);
    if (scale_out && threadIdx.x == 0) *scale_out = r;
}

// ---------------------------------------------------------------- elementwise
__global__ void multiply_kernel(float *out, const float *x, const float *y, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fmul_rn(x[i], y[i]);
}
// (base + s a) + t b, optionally times *scale (src/qwen_cuda.cu:45).
__global__ void plane_kernel(float *out, const float *base, const float *a, const float *b, int n, float s, float t,
                             const float *scale) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float v = __fadd_rn(__fadd_rn(base[i], __fmul_rn(s, a[i])), __fmul_rn(t, b[i]));
        out[i] = scale ? __fmul_rn(*scale, v) : v;
    }
}
// ca a (+ cb b), optionally times *scale (src/qwen_cuda.cu:48).
__global__ void linear2_kernel(float *out, const float *a, const float *b, int n, float ca, float cb,
                               const float *scale) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        float v = __fmul_rn(ca, a[i]);
        if (b) v = __fadd_rn(v, __fmul_rn(cb, b[i]));
        out[i] = scale ? __fmul_rn(*scale, v) : v;
    }
}
__global__ void identical_kernel(const float *a, const float *b, int n, int *invalid) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && (!isfinite(a[i]) || !isfinite(b[i]) || __float_as_uint(a[i]) != __float_as_uint(b[i])))
        atomicExch(invalid, 1);
}
__global__ void add_kernel(float *x, const float *y, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fadd_rn(x[i], y[i]);
}
// Half-split rotation. `denominator[d]` = theta^(2d/dim) computed on the host
// with the C library's powf, angle = position / denominator (the reference's
// CPU form, tests/gpu_stub.c:158), rotation without contraction.
__global__ void rope_kernel(float *x, int heads, int dim, int position, const float *denominator) {
    const int half = dim / 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= heads * half) return;
    const int h = i / half, d = i % half;
    const float angle = __fdiv_rn((float)position, denominator[d]);
    float sn, cs;
    sincosf(angle, &sn, &cs);
    const float a = x[h * dim + d], b = x[h * dim + d + half];
    x[h * dim + d] = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
    x[h * dim + d + half] = __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
}
__global__ void cache_kernel(float *cache, const float *x, int heads, int dim, int capacity, int position) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < heads * dim) cache[((size_t)(i / dim) * capacity + position) * dim + i % dim] = x[i];
}
// silu(g) * u as g / (1 + exp(-g)) * u (src/qwen_cuda.cu:79).
__global__ void swiglu_kernel(float *g, const float *u, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) g[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.f, expf(-g[i]))), u[i]);
}
// Polynomial gate law of the experimental gate studies (src/qwen_cuda.cu:81-98).
__global__ void gate_anchor_kernel(const float *g, float *p, float *first, float *second, float *s, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float den = __fadd_rn(1.f, expf(-g[i]));
        const float pi = __fdiv_rn(1.f, den);
        p[i] = pi;
        const float f = __fmul_rn(pi, __fsub_rn(1.f, pi));
        first[i] = f;
        second[i] = __fmul_rn(__fmul_rn(0.5f, f), __fsub_rn(1.f, __fmul_rn(2.f, pi)));
        s[i] = __fdiv_rn(g[i], den);
    }
}
__global__ void gate_swiglu_kernel(float *g, const float *u, const float *source, const float *p, const float *first,
                                   const float *second, const float *s, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float d = __fsub_rn(g[i], source[i]);
        const float sigma = __fadd_rn(__fadd_rn(p[i], __fmul_rn(first[i], d)), __fmul_rn(__fmul_rn(second[i], d), d));
        const float predicted = __fadd_rn(s[i], __fsub_rn(__fmul_rn(g[i], sigma), __fmul_rn(source[i], p[i])));
        g[i] = __fmul_rn(predicted, u[i]);
    }
}

// ---------------------------------------------------------------- top-2
// Grid-stride per-block top-2, then the last block merges the block results
// (replaces top_kernel + finish_top, src/qwen_cuda.cu:102-118).
__device__ __forceinline__ Top2 top2_block(Top2 t, float *sv, int *si) {
    top2_merge_warp(t);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    if (lane == 0) {
        sv[2 * warp] = t.a; sv[2 * warp + 1] = t.b;
        si[2 * warp] = t.ai; si[2 * warp + 1] = t.bi;
    }
    __syncthreads();
    if (warp == 0) {
        Top2 u = top2_empty();
        if (lane < warps) {
            top2_insert(u, sv[2 * lane], si[2 * lane]);
            top2_insert(u, sv[2 * lane + 1], si[2 * lane + 1]);
        }
        top2_merge_warp(u);
        t = u;
    }
    return t;  // valid in warp 0
}
__global__ void __launch_bounds__(kThreads) top2_kernel(const float *x, int n, float *pv, int *pi, int *flags,
                                                        TcmTop2 *result) {
    __shared__ float sv[64];
    __shared__ int si[64];
    __shared__ int last;
    Top2 t = top2_empty();
    bool bad = false;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = x[i];
        bad |= !isfinite(v);
        top2_insert(t, v, i);
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicExch(&flags[0], 1);
    t = top2_block(t, sv, si);
    if (threadIdx.x == 0) {
        pv[2 * blockIdx.x] = t.a; pv[2 * blockIdx.x + 1] = t.b;
        pi[2 * blockIdx.x] = t.ai; pi[2 * blockIdx.x + 1] = t.bi;
        __threadfence();
        last = atomicAdd((unsigned *)&flags[1], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    Top2 u = top2_empty();
    for (int i = threadIdx.x; i < 2 * (int)gridDim.x; i += blockDim.x) top2_insert(u, __ldcg(pv + i), __ldcg(pi + i));
    __syncthreads();
    u = top2_block(u, sv, si);
    if (threadIdx.x == 0) {
        result->first = u.ai; result->second = u.bi;
        result->first_value = u.a; result->second_value = u.b;
        flags[1] = 0;
    }
}

// ---------------------------------------------------------------- attention
// Reference-semantics attention for any head size: one block per query head,
// scores[h * length + t] hold the softmax probabilities (src/qwen_cuda.cu:65-78).
__global__ void __launch_bounds__(kThreads) attention_generic_kernel(float *out, const float *q, const float *keys,
                                                                     const float *values, float *scores, int qheads,
                                                                     int kvheads, int dim, int capacity, int length,
                                                                     float sqrt_dim) {
    __shared__ float red[32];
    const int h = blockIdx.x, g = h / (qheads / kvheads);
    const float *qh = q + (size_t)h * dim;
    const float *kb = keys + (size_t)g * capacity * dim, *vb = values + (size_t)g * capacity * dim;
    float *p = scores + (size_t)h * length;
    float mx = -INFINITY;
    for (int t = threadIdx.x; t < length; t += blockDim.x) {
        float d = 0.f;
        for (int i = 0; i < dim; i++) d = fmaf(qh[i], kb[(size_t)t * dim + i], d);
        d = __fdiv_rn(d, sqrt_dim);
        p[t] = d;
        mx = fmaxf(mx, d);
    }
    mx = warp_max(mx);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float sum = 0.f;
    for (int t = threadIdx.x; t < length; t += blockDim.x) {
        const float e = expf(p[t] - mx);
        p[t] = e;
        sum += e;
    }
    sum = block_sum(sum, red);
    for (int t = threadIdx.x; t < length; t += blockDim.x) p[t] = __fdiv_rn(p[t], sum);
    __syncthreads();
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float a = 0.f;
        for (int t = 0; t < length; t++) a = fmaf(p[t], vb[(size_t)t * dim + i], a);
        out[(size_t)h * dim + i] = a;
    }
}

// Device table theta^(2d/dim), d < dim/2, formed with the C library's powf as
// the reference's CPU path does; cached per device for the last (theta, dim).
const float *rope_denominators(float theta, int dim) {
    static std::mutex lock;
    static float *table[64];
    static float key_theta[64];
    static int key_dim[64];
    const int half = dim / 2;
    if (half > 1024) TCM_FATAL("RoPE head size %d exceeds 2048", dim);
    int dev = 0;
    TCM_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> hold(lock);
    if (!table[dev]) TCM_CUDA(cudaMalloc((void **)&table[dev], 1024 * sizeof(float)));
    if (key_dim[dev] != dim || key_theta[dev] != theta) {
        float host[1024];
        for (int d = 0; d < half; d++) host[d] = powf(theta, 2.0f * d / dim);
        TCM_CUDA(cudaMemcpyAsync(table[dev], host, half * sizeof(float), cudaMemcpyHostToDevice, stream()));
        TCM_CUDA(cudaStreamSynchronize(stream()));
        key_dim[dev] = dim;
        key_theta[dev] = theta;
    }
    return table[dev];
}

void attention_generic(float *out, const float *q, const float *keys, const float *values, float *scores, int qheads,
                       int kvheads, int dim, int capacity, int length, cudaStream_t s) {
    attention_generic_kernel<<<qheads, kThreads, 0, s>>>(out, q, keys, values, scores, qheads, kvheads, dim, capacity,
                                                         length, sqrtf((float)dim));
    TCM_CUDA(cudaGetLastError());
}

void attention_split(const float *q, const AttnSource &source, bool bytes, int capacity, int length,
                     const int *position, int qheads, int kvheads, int nsplit, float *part, unsigned *counters,
                     float *out, cudaStream_t s, bool pdl) {
    static PerDeviceOnce once;
    once.run([] {
        TCM_CUDA(cudaFuncSetAttribute(attn_split_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kAttnSmemBytes));
        TCM_CUDA(cudaFuncSetAttribute(attn_split_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kAttnSmemBytes));
    });
    const float sqrt_dim = sqrtf((float)kHeadDim);
    if (bytes)
        launch(attn_split_kernel<true>, dim3(nsplit, kvheads), dim3(kAttnThreads), kAttnSmemBytes, s, pdl, q, source,
               capacity, length, position, qheads / kvheads, sqrt_dim, part, counters, out);
    else
        launch(attn_split_kernel<false>, dim3(nsplit, kvheads), dim3(kAttnThreads), kAttnSmemBytes, s, pdl, q, source,
               capacity, length, position, qheads / kvheads, sqrt_dim, part, counters, out);
}

}  // namespace tcm

using namespace tcm;

static inline unsigned blocks_for(int n) { return (unsigned)((n + kThreads - 1) / kThreads); }

namespace tcm {
// Split-K partials of the primitive attention calls, owned by the handle.
void attention_scratch(TcmGpu *g, int kvheads, float **part, unsigned **counters) {
    const size_t need = (size_t)kvheads * kAttnSplits * kAttnPartialFloats;
    if (g->attn_part_floats < need || g->attn_kv < kvheads) {
        gpu_free(g->attn_part);
        gpu_free(g->attn_counters);
        g->attn_part = (float *)gpu_alloc(need * sizeof(float));
        g->attn_counters = (unsigned *)gpu_alloc((size_t)kvheads * sizeof(unsigned));
        gpu_zero(g->attn_counters, (size_t)kvheads * sizeof(unsigned));
        g->attn_part_floats = need;
        g->attn_kv = kvheads;
    }
    *part = g->attn_part;
    *counters = g->attn_counters;
}
}  // namespace tcm

extern "C" {

TcmGpu *gpu_open(void) {
    TcmGpu *g = (TcmGpu *)calloc(1, sizeof(TcmGpu));
    if (!g) exit(2);
    g->part_values = (float *)gpu_alloc(2 * kTopBlocks * sizeof(float));
    g->part_ids = (int *)gpu_alloc(2 * kTopBlocks * sizeof(int));
    g->invalid = (int *)gpu_alloc(2 * sizeof(int));
    g->result = (TcmTop2 *)gpu_alloc(sizeof(TcmTop2));
    gpu_zero(g->invalid, 2 * sizeof(int));
    return g;
}

void gpu_close(TcmGpu *g) {
    if (!g) return;
    gpu_free(g->part_values);
    gpu_free(g->part_ids);
    gpu_free(g->invalid);
    gpu_free(g->result);
    gpu_free(g->attn_part);
    gpu_free(g->attn_counters);
    free(g);
}

float *gpu_weight(const void *data, uint32_t dtype, size_t n) {
    float *out = (float *)gpu_alloc(n * sizeof(float));
    if (dtype == 1) {
        gpu_write(out, data, n * sizeof(float));
    } else if (dtype == 2) {
        uint16_t *raw = (uint16_t *)gpu_alloc(n * 2);
        gpu_write(raw, data, n * 2);
        widen_bf16(out, raw, n, stream());
        gpu_free(raw);
    } else {
        TCM_FATAL("unsupported GPU weight dtype");
    }
    return out;
}

void gpu_rms(float *out, const float *x, const float *w, int n, float eps) {
    rms_kernel<<<1, 1024, 0, stream()>>>(out, x, w, n, eps, nullptr);
    TCM_CUDA(cudaGetLastError());
}
void gpu_rms_scale(float *out, const float *x, const float *w, int n, float eps, float *scale) {
    rms_kernel<<<1, 1024, 0, stream()>>>(out, x, w, n, eps, scale);
    TCM_CUDA(cudaGetLastError());
}
void gpu_multiply(float *out, const float *x, const float *y, int n) {
    if (n <= 0) return;
    multiply_kernel<<<blocks_for(n), kThreads, 0, stream()>>>(out, x, y, n);
    TCM_CUDA(cudaGetLastError());
}
void gpu_plane(float *out, const float *base, const float *a, const float *b, int n, float s, float t) {
    if (n <= 0) return;
    plane_kernel<<<blocks_for(n), kThreads, 0, stream()>>>(out, base, a, b, n, s, t, nullptr);
    TCM_CUDA(cudaGetLastError());
}
void gpu_plane_scaled(float *out, const float *base, const float *a, const float *b, int n, float s, float t,
                      const float *scale) {
    if (n <= 0) return;
    plane_kernel<<<blocks_for(n), kThreads, 0, stream()>>>(out, base, a, b, n, s, t, scale);
    TCM_CUDA(cudaGetLastError());
}
void gpu_linear2(float *out, const float *a, const float *b, int n, float ca, float cb, const float *scale) {
    if (n <= 0) return;
    linear2_kernel<<<blocks_for(n), kThreads, 0, stream()>>>(out, a, b, n, ca, cb, scale);
    TCM_CUDA(cudaGetLastError());
}
int gpu_identical_finite(TcmGpu *g, const float *a, const float *b, int n) {
    gpu_zero(g->invalid, sizeof(int));
    if (n > 0) {
        identical_kernel<<<blocks_for(n), kThreads, 0, stream()>>>(a, b, n, g->invalid);
        TCM_CUDA(cudaGetLastError());
    }
    int invalid = 0;
    gpu_read(&invalid, g->invalid, sizeof(int));
    return !invalid;
}
void gpu_add(float *x, const float *y, int n) {
    if (n <= 0) return;
    add_kernel<<<blocks_for(n), kThreads, 0, stream()>>>(x, y, n);
    TCM_CUDA(cudaGetLastError());
}
void gpu_bias(float *x, const float *y, int n) { gpu_add(x, y, n); }

void gpu_rope(float *x, int heads, int dim, int position, float theta) {
    const int half = dim / 2;
    if (heads <= 0 || half <= 0) return;
    rope_kernel<<<blocks_for(heads * half), kThreads, 0, stream()>>>(x, heads, dim, position,
                                                                     rope_denominators(theta, dim));
    TCM_CUDA(cudaGetLastError());
}
void gpu_cache(float *cache, const float *x, int heads, int dim, int capacity, int position) {
    if (heads * dim <= 0) return;
    cache_kernel<<<blocks_for(heads * dim), kThreads, 0, stream()>>>(cache, x, heads, dim, capacity, position);
    TCM_CUDA(cudaGetLastError());
}
void gpu_attention(TcmGpu *g, float *out, const float *q, const float *keys, const float *values, float *scores,
                   int qheads, int kvheads, int dim, int capacity, int length) {
    if (length < 1 || kvheads < 1 || qheads % kvheads) TCM_FATAL("gpu_attention: invalid shape");
    const int group = qheads / kvheads;
    if (dim == kHeadDim && group <= kAttnMaxGroup && ((uintptr_t)keys & 15) == 0 && ((uintptr_t)values & 15) == 0) {
        AttnSource src = {};
        src.keys = keys;
        src.values = values;
        float *part = nullptr;
        unsigned *counters = nullptr;
        attention_scratch(g, kvheads, &part, &counters);
        attention_split(q, src, false, capacity, length, nullptr, qheads, kvheads, kAttnSplits, part, counters, out,
                        stream(), false);
    } else {
        attention_generic(out, q, keys, values, scores, qheads, kvheads, dim, capacity, length, stream());
    }
}
void gpu_swiglu(float *gate, const float *up, int n) {
    if (n <= 0) return;
    swiglu_kernel<<<blocks_for(n), kThreads, 0, stream()>>>(gate, up, n);
    TCM_CUDA(cudaGetLastError());
}
void gpu_gate_anchor(const float *g, float *p, float *first, float *second, float *s, int n) {
    if (n <= 0) return;
    gate_anchor_kernel<<<blocks_for(n), kThreads, 0, stream()>>>(g, p, first, second, s, n);
    TCM_CUDA(cudaGetLastError());
}
void gpu_gate_swiglu(float *g, const float *u, const float *source, const float *p, const float *first,
                     const float *second, const float *s, int n) {
    if (n <= 0) return;
    gate_swiglu_kernel<<<blocks_for(n), kThreads, 0, stream()>>>(g, u, source, p, first, second, s, n);
    TCM_CUDA(cudaGetLastError());
}
TcmTop2 gpu_top2(TcmGpu *g, const float *x, int n) {
    if (n < 1) TCM_FATAL("gpu_top2: empty input");
    int blocks = (n + kThreads - 1) / kThreads;
    if (blocks > kTopBlocks) blocks = kTopBlocks;
    gpu_zero(g->invalid, sizeof(int));
    top2_kernel<<<blocks, kThreads, 0, stream()>>>(x, n, g->part_values, g->part_ids, g->invalid, g->result);
    TCM_CUDA(cudaGetLastError());
    struct { TcmTop2 top; } r;
    int flags[1];
    gpu_read(&r.top, g->result, sizeof(TcmTop2));
    gpu_read(flags, g->invalid, sizeof(int));
    if (flags[0]) TCM_FATAL("non-finite Qwen logits");
    return r.top;
}

}  // extern "C"
