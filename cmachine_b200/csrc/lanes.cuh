// Lane-resident vectors and streamed-row dot products shared by the batch-1
// decode kernels (the per-stage kernels of decode.cu and the persistent token
// kernel of persistent.cu), plus the device-resident token state.
#pragma once
#include "common.cuh"
#include "stream.cuh"
#include "../../include/qwen_b200.h"

namespace tcm {

// Device-resident token state: the host writes token/position before a token;
// the readout's last CTA publishes the top-2 and, for chained greedy decode,
// feeds top-1 back as the next token and advances the position. `fault`
// collects the bits of any pipeline wait that ran out.
// Bits of `invalid`: 1 non-finite logits, 2 a non-finite K/V row encoded into
// a ring arena. `ring` is the token's ring bookkeeping (ring layers only).
// bar, arrive and nonfinite are zero between tokens (the host's state write
// and the kernel that used them last both clear them).
struct DecodeState {
    int token, position, step, invalid;
    unsigned fault;
    unsigned bar, arrive, nonfinite;  // the persistent token kernel's grid barrier, readout arrivals, non-finite flag
    TcmTop2 top;
    QwenB200RingStep ring;
};
constexpr int kLogCap = 4096;
constexpr int kRingRowBytes = 528;  // one ring row: 4 x 128 codes + 4 FP32 scales

constexpr int kHidden = 1536;       // Qwen2.5-1.5B hidden size (the fused kernels' geometry)
constexpr int kInter = 8960;        // MLP width
constexpr int kMaxPairsPerCta = 64; // q/k/v row pairs one CTA may own
constexpr int kMaxRowsPerCta = 64;  // residual rows one O or down CTA may own (grids of at least 24 CTAs)

// Weight geometry: E elements per 16-byte vector; R rows of 1536 per stage
// (48 KB either way); RD rows of 8960 per down stage (35 KB).
template <typename WT> struct Geo;
template <> struct Geo<float> { static constexpr int E = 4, R = 8, RD = 1; };
template <> struct Geo<uint16_t> { static constexpr int E = 8, R = 16, RD = 2; };
template <typename WT> constexpr int kNV = kHidden / (32 * Geo<WT>::E);  // vectors per lane in a row of 1536
template <typename WT> constexpr uint32_t kRow = kHidden * sizeof(WT);
template <typename WT> constexpr uint32_t kStage = Geo<WT>::R * kRow<WT>;
template <typename WT> constexpr uint32_t kDownRow = kInter * sizeof(WT);
template <typename WT> constexpr uint32_t kDownStage = Geo<WT>::RD * kDownRow<WT>;
constexpr int kStages = 2, kDownStages = 3;
constexpr int kLaneX = 48;  // floats of a 1536-vector one lane holds

// ---------------------------------------------------------------- lane-resident vectors
// Lane layout of a 1536-vector: lane owns 16-byte weight vectors v = lane + 32k
// (k < kNV), i.e. elements E*v .. E*v+E-1, stored at xr[E*k ...].
// kCg reads through L2 only (data another CTA of the same launch wrote).
template <typename WT, bool kCg = false>
__device__ __forceinline__ void load_lane_vec(float (&xr)[kLaneX], const float *x, int lane) {
    constexpr int E = Geo<WT>::E;
#pragma unroll
    for (int k = 0; k < kNV<WT>; k++)
#pragma unroll
        for (int h = 0; h < E / 4; h++) {
            const float4 *p = reinterpret_cast<const float4 *>(x) + (E / 4) * (lane + 32 * k) + h;
            const float4 f = kCg ? __ldcg(p) : *p;
            xr[E * k + 4 * h] = f.x;
            xr[E * k + 4 * h + 1] = f.y;
            xr[E * k + 4 * h + 2] = f.z;
            xr[E * k + 4 * h + 3] = f.w;
        }
}
// A 1536-float vector from global memory into shared memory by the consumer
// threads, 16 bytes each per pass; the caller's next consumers_sync publishes
// it. Every warp of every CTA needs the whole vector: read per warp, each of
// its 48 lines would take 8 x 148 requests at one L2 slice right after the
// dependency wait; staged, it takes one per CTA.
__device__ __forceinline__ void copy_hidden(float *v_s, const float *v) {
    for (int i = threadIdx.x; i < kHidden / 4; i += kConsumerWarps * 32)
        reinterpret_cast<float4 *>(v_s)[i] = __ldcg(reinterpret_cast<const float4 *>(v) + i);
}
template <typename WT> __device__ __forceinline__ void store_lane_vec(float *x, const float (&xr)[kLaneX], int lane) {
    constexpr int E = Geo<WT>::E;
#pragma unroll
    for (int k = 0; k < kNV<WT>; k++)
#pragma unroll
        for (int h = 0; h < E / 4; h++)
            reinterpret_cast<float4 *>(x)[(E / 4) * (lane + 32 * k) + h] =
                make_float4(xr[E * k + 4 * h], xr[E * k + 4 * h + 1], xr[E * k + 4 * h + 2], xr[E * k + 4 * h + 3]);
}
// A weight row (FP32 or BF16) of 1536 into the lane layout, widened to FP32.
template <typename WT> __device__ __forceinline__ void load_lane_row(float (&xr)[kLaneX], const WT *row, int lane) {
    if constexpr (sizeof(WT) == 4) {
        load_lane_vec<float>(xr, reinterpret_cast<const float *>(row), lane);
    } else {
#pragma unroll
        for (int k = 0; k < kNV<WT>; k++) {
            const uint4 w = reinterpret_cast<const uint4 *>(row)[lane + 32 * k];
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                xr[8 * k + 2 * j] = bf16_lo(u[j]);
                xr[8 * k + 2 * j + 1] = bf16_hi(u[j]);
            }
        }
    }
}
// x <- (x * r) * w with r = 1 / sqrt(mean(x^2) + eps) over the whole warp's
// vector; w is the norm weight vector staged in shared memory.
template <typename WT> __device__ __forceinline__ void rms_lane(float (&xr)[kLaneX], const float *w_s, float eps, int lane) {
    constexpr int E = Geo<WT>::E;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kLaneX; i++) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHidden), eps)));
#pragma unroll
    for (int k = 0; k < kNV<WT>; k++)
#pragma unroll
        for (int j = 0; j < E; j++)
            xr[E * k + j] = __fmul_rn(__fmul_rn(xr[E * k + j], r), w_s[E * (lane + 32 * k) + j]);
}
// The norm weights into shared memory (consumer threads; before the wait).
__device__ __forceinline__ void stage_norm(float *w_s, const float *w) {
    for (int i = threadIdx.x; i < kHidden / 4; i += kConsumerWarps * 32)
        reinterpret_cast<float4 *>(w_s)[i] = reinterpret_cast<const float4 *>(w)[i];
}
__device__ __forceinline__ float dot_vec(const uint4 &w, const float *x, float acc, float) {
    acc = fmaf(__uint_as_float(w.x), x[0], acc);
    acc = fmaf(__uint_as_float(w.y), x[1], acc);
    acc = fmaf(__uint_as_float(w.z), x[2], acc);
    return fmaf(__uint_as_float(w.w), x[3], acc);
}
__device__ __forceinline__ float dot_vec(const uint4 &w, const float *x, float acc, uint16_t) {
    acc = fmaf(bf16_lo(w.x), x[0], acc);
    acc = fmaf(bf16_hi(w.x), x[1], acc);
    acc = fmaf(bf16_lo(w.y), x[2], acc);
    acc = fmaf(bf16_hi(w.y), x[3], acc);
    acc = fmaf(bf16_lo(w.z), x[4], acc);
    acc = fmaf(bf16_hi(w.z), x[5], acc);
    acc = fmaf(bf16_lo(w.w), x[6], acc);
    return fmaf(bf16_hi(w.w), x[7], acc);
}
// Warp dot product of a shared-memory row of 1536 with the lane-resident vector.
template <typename WT> __device__ __forceinline__ float row_dot(const unsigned char *srow, const float (&xr)[kLaneX], int lane) {
    const uint4 *v = reinterpret_cast<const uint4 *>(srow);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kNV<WT>; k++) acc = dot_vec(v[lane + 32 * k], &xr[Geo<WT>::E * k], acc, WT());
    return warp_sum(acc);
}


__host__ __device__ __forceinline__ int share_begin(int total, int part, int parts) { return (int)((long long)part * total / parts); }

}  // namespace tcm
