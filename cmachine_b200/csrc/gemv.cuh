// Batch-1 GEMV building blocks: y[row] = W[row][:] . x, W row-major, FP32 or
// BF16 weights, FP32 activations and accumulation.
//
// A warp owns whole rows. Each lane streams 16-byte weight vectors at a
// 512-byte warp stride (fully coalesced), UNROLL vectors per row in flight,
// and multiplies them with the activation vector staged in shared memory. The
// per-lane partial sums are combined with a fixed butterfly, so the result is
// deterministic. These are HBM-bound: one weight byte is read once per token.
#pragma once
#include "common.cuh"

namespace tcm {

// Weight element types: float (FP32) or uint16_t holding BF16 bits.
template <typename WT> struct WVec;
template <> struct WVec<float> { static constexpr int kElems = 4; };
template <> struct WVec<uint16_t> { static constexpr int kElems = 8; };

// acc += w(16 bytes at vector index vi) . xs[vi*kElems ...]
__device__ __forceinline__ float dot16(const uint4 &w, const float *xs, int vi, float acc, float) {
    const float4 x = reinterpret_cast<const float4 *>(xs)[vi];
    acc = fmaf(__uint_as_float(w.x), x.x, acc);
    acc = fmaf(__uint_as_float(w.y), x.y, acc);
    acc = fmaf(__uint_as_float(w.z), x.z, acc);
    acc = fmaf(__uint_as_float(w.w), x.w, acc);
    return acc;
}
__device__ __forceinline__ float dot16(const uint4 &w, const float *xs, int vi, float acc, uint16_t) {
    const float4 x0 = reinterpret_cast<const float4 *>(xs)[2 * vi];
    const float4 x1 = reinterpret_cast<const float4 *>(xs)[2 * vi + 1];
    acc = fmaf(bf16_lo(w.x), x0.x, acc);
    acc = fmaf(bf16_hi(w.x), x0.y, acc);
    acc = fmaf(bf16_lo(w.y), x0.z, acc);
    acc = fmaf(bf16_hi(w.y), x0.w, acc);
    acc = fmaf(bf16_lo(w.z), x1.x, acc);
    acc = fmaf(bf16_hi(w.z), x1.y, acc);
    acc = fmaf(bf16_lo(w.w), x1.z, acc);
    acc = fmaf(bf16_hi(w.w), x1.w, acc);
    return acc;
}

// NR rows of `nvec` 16-byte vectors each, dotted with xs; lane partials in acc.
template <typename WT, int NR, int UNROLL>
__device__ __forceinline__ void warp_rows_partial(const WT *const (&rows)[NR], const float *xs, int nvec, int lane,
                                                  float (&acc)[NR]) {
    constexpr int E = WVec<WT>::kElems;
    for (int base = lane; base < nvec; base += kWarp * UNROLL) {
        uint4 w[NR][UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int vi = base + kWarp * u;
#pragma unroll
            for (int r = 0; r < NR; r++)
                if (vi < nvec) w[r][u] = ld_stream16(rows[r] + (size_t)vi * E);
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int vi = base + kWarp * u;
#pragma unroll
            for (int r = 0; r < NR; r++)
                if (vi < nvec) acc[r] = dot16(w[r][u], xs, vi, acc[r], WT());
        }
    }
}

template <typename WT, int NR, int UNROLL>
__device__ __forceinline__ void warp_rows_dot(const WT *const (&rows)[NR], const float *xs, int nvec, int lane,
                                              float (&acc)[NR]) {
#pragma unroll
    for (int r = 0; r < NR; r++) acc[r] = 0.f;
    warp_rows_partial<WT, NR, UNROLL>(rows, xs, nvec, lane, acc);
#pragma unroll
    for (int r = 0; r < NR; r++) acc[r] = warp_sum(acc[r]);
}

// Issue L2 prefetches for `bytes` of a row (lane-strided 128-byte lines).
__device__ __forceinline__ void prefetch_row_l2(const void *row, size_t bytes, int lane) {
    const char *p = static_cast<const char *>(row);
    for (size_t off = (size_t)lane * 128; off < bytes; off += kWarp * 128) prefetch_l2(p + off);
}

// Block-wide sum over blockDim.x threads (<= 1024); result broadcast to all.
__device__ __forceinline__ float block_sum(float v, float *red /* >= 32 floats */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    if (warp == 0) {
        t = lane < warps ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    return red[0];
}

// Stage x[0..n) into shared memory and, if w != nullptr, replace it by its
// RMS norm (x * r) * w, r = 1 / sqrt(mean(x^2) + eps) (IEEE divide and square
// root, as the reference's CPU path forms it). Returns r. All threads.
__device__ __forceinline__ float stage_rms(float *xs, const float *x, const float *w, int n, float eps,
                                           float *red) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i];
        xs[i] = v;
        ss = fmaf(v, v, ss);
    }
    if (!w) {
        __syncthreads();
        return 1.f;
    }
    const float total = block_sum(ss, red);
    const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)n), eps)));
    for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], r), w[i]);
    __syncthreads();
    return r;
}

}  // namespace tcm
