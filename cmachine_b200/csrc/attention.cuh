// Split-K GQA decode attention over an FP32 K/V cache (head_dim 128).
//
// Replaces the reference's two cublasSgemm + global-memory softmax
// (src/qwen_cuda.cu:65-78) and, for the byte-codec cache, the decode-to-FP32
// workspace + cuBLAS path (src/qwen_cache.inc:16-43): int8 codes are staged
// and dequantised (code * row scale) in shared memory. One CTA owns one KV head and one contiguous slice
// of cache rows; all query heads of the group (6 for Qwen2.5-1.5B) share each
// K/V tile, which cp.async stages into shared memory two tiles ahead. Scores
// use the reference's scaling (dot / sqrt(128)), softmax is online (running
// max, rescaled sums) and the last CTA of each KV head combines the slices in
// a fixed order, so the result is deterministic.
#pragma once
#include "common.cuh"

namespace tcm {

constexpr int kHeadDim = 128;
constexpr int kAttnTile = 32;      // cache rows per shared-memory tile
constexpr int kAttnThreads = 256;  // 8 warps
constexpr int kAttnMaxGroup = 8;   // query heads per KV head
constexpr int kAttnSplits = 74;    // slices per KV head: 2 KV heads x 74 = 148 CTAs, one per SM
constexpr int kAttnMinRows = 64;   // fewest cache rows per slice
static_assert(kAttnSplits * kAttnMaxGroup <= 2 * kAttnTile * kHeadDim, "slice weights must fit a tile buffer");
static_assert(kAttnSplits <= 96, "the decode combine holds at most three slices per lane");
constexpr int kAttnPerThread = kAttnMaxGroup * kHeadDim / kAttnThreads;

// Floats of one slice's partial result: m[8], l[8], acc[8][128].
constexpr int kAttnPartialFloats = 2 * kAttnMaxGroup + kAttnMaxGroup * kHeadDim;
constexpr size_t kAttnSmemBytes =
    (size_t)(2 * 2 * kAttnTile * kHeadDim + kAttnMaxGroup * kHeadDim + kAttnMaxGroup * kAttnTile + 4 * kAttnMaxGroup) *
    sizeof(float);

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;  // 0 source bytes: the 16 destination bytes are zero-filled
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Rows [t, t + kAttnTile) of one KV head into a [kAttnTile][128] FP32 tile; rows at
// or beyond `end` are zero-filled.
__device__ __forceinline__ void attn_load_tile(float *tile, const float *src, int t, int end) {
    // 32 rows x 32 16-byte chunks = 1024 chunks, 4 per thread.
#pragma unroll
    for (int i = 0; i < (kAttnTile * kHeadDim / 4) / kAttnThreads; i++) {
        const int c = threadIdx.x + i * kAttnThreads;
        const int row = c >> 5, col = (c & 31) * 4;
        const bool valid = t + row < end;
        const float *g = src + (size_t)(valid ? t + row : t) * kHeadDim + col;
        cp_async16(tile + row * kHeadDim + col, g, valid);
    }
}
// Byte-codec rows: 128 int8 codes per row (8 16-byte chunks), gathered through
// `order` when it is non-null; the per-row scale goes to scale_tile[row].
__device__ __forceinline__ void attn_load_tile_bytes(int8_t *tile, float *scale_tile, const int8_t *codes,
                                                     const float *scales, const int *order, int t, int end) {
    const int c = threadIdx.x;  // 32 rows x 8 chunks = 256 chunks, one per thread
    const int row = c >> 3, col = (c & 7) * 16;
    const bool valid = t + row < end;
    const int src = valid ? (order ? __ldg(order + t + row) : t + row) : 0;
    cp_async16(tile + row * kHeadDim + col, codes + (size_t)src * kHeadDim + col, valid);
    if (threadIdx.x < kAttnTile) {
        const int r = threadIdx.x;
        scale_tile[r] = t + r < end ? __ldg(scales + (order ? __ldg(order + t + r) : t + r)) : 0.f;
    }
}

// K/V source of one KV head: FP32 rows, or byte-codec codes with per-row scales,
// optionally gathered through `order` and biased by `weights` (ring cache).
struct AttnSource {
    const float *keys, *values;          // FP32 [kvheads][capacity][128]
    const int8_t *kcodes, *vcodes;       // int8 [kvheads][capacity][128]
    const float *scales;                 // [kind * kvheads + head][capacity]
    const int *order;                    // active row -> physical row, or null
    const float *weights;                // log-weight per active row, or null
};

// grid (nsplit, kvheads), block 256, dynamic smem kAttnSmemBytes.
// length < 0: the row count is *position + 1 (device-resident decode state).
// part: [kvheads][nsplit][kAttnPartialFloats]; counters: [kvheads], zero on entry
// and left zero on exit. out: [qheads][128].
template <bool BYTES>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(
    const float *__restrict__ q, AttnSource src, int capacity, int length, const int *__restrict__ position,
    int group, float sqrt_dim, float *__restrict__ part, unsigned *__restrict__ counters, float *__restrict__ out) {
    extern __shared__ __align__(16) float smem[];
    float *k_tile = smem;                                     // [2][32][128]
    float *v_tile = k_tile + 2 * kAttnTile * kHeadDim;        // [2][32][128]
    float *q_s = v_tile + 2 * kAttnTile * kHeadDim;           // [8][128]
    float *p_s = q_s + kAttnMaxGroup * kHeadDim;              // [8][32]
    float *m_s = p_s + kAttnMaxGroup * kAttnTile;             // [8] running max
    float *l_s = m_s + kAttnMaxGroup;                         // [8] running sum
    float *c_s = l_s + kAttnMaxGroup;                         // [8] rescale of this tile
    __shared__ float ks_s[2][kAttnTile], vs_s[2][kAttnTile];  // byte-codec row scales
    __shared__ int last_s;

    const int kvh = blockIdx.y, split = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kvheads = gridDim.y;
    pdl_wait();
    pdl_trigger();
    // Slices of at least kAttnMinRows rows: short caches use few CTAs (cheap
    // combine), long ones all of the grid. CTAs past the last slice leave.
    const int L = min(length >= 0 ? length : *position + 1, capacity);
    const int chunk = max((L + (int)gridDim.x - 1) / (int)gridDim.x, kAttnMinRows);
    const int nsplit = (L + chunk - 1) / chunk;
    if (split >= nsplit) return;
    const int t0 = split * chunk, t1 = min(L, t0 + chunk);
    const float *kbase = nullptr, *vbase = nullptr, *ksc = nullptr, *vsc = nullptr;
    const int8_t *kcb = nullptr, *vcb = nullptr;
    if (BYTES) {
        kcb = src.kcodes + (size_t)kvh * capacity * kHeadDim;
        vcb = src.vcodes + (size_t)kvh * capacity * kHeadDim;
        ksc = src.scales + (size_t)kvh * capacity;
        vsc = src.scales + (size_t)(kvheads + kvh) * capacity;
    } else {
        kbase = src.keys + (size_t)kvh * capacity * kHeadDim;
        vbase = src.values + (size_t)kvh * capacity * kHeadDim;
    }
    const int ntile = (t1 - t0 + kAttnTile - 1) / kAttnTile;
    auto load = [&](int stage, int t) {
        if (BYTES) {
            attn_load_tile_bytes(reinterpret_cast<int8_t *>(k_tile + stage * kAttnTile * kHeadDim), ks_s[stage], kcb,
                                 ksc, src.order, t, t1);
            attn_load_tile_bytes(reinterpret_cast<int8_t *>(v_tile + stage * kAttnTile * kHeadDim), vs_s[stage], vcb,
                                 vsc, src.order, t, t1);
        } else {
            attn_load_tile(k_tile + stage * kAttnTile * kHeadDim, kbase, t, t1);
            attn_load_tile(v_tile + stage * kAttnTile * kHeadDim, vbase, t, t1);
        }
        cp_async_commit();
    };

    if (ntile > 0) load(0, t0);
    for (int i = tid; i < group * kHeadDim; i += kAttnThreads) q_s[i] = q[(size_t)kvh * group * kHeadDim + i];
    if (tid < kAttnMaxGroup) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.f;
    }
    float acc[kAttnPerThread];
#pragma unroll
    for (int j = 0; j < kAttnPerThread; j++) acc[j] = 0.f;
    __syncthreads();
    float4 q4[kAttnMaxGroup];
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; g++)
        q4[g] = g < group ? reinterpret_cast<const float4 *>(q_s + g * kHeadDim)[lane] : make_float4(0, 0, 0, 0);

    for (int it = 0; it < ntile; it++) {
        const int stage = it & 1, t = t0 + it * kAttnTile;
        if (it + 1 < ntile) {
            load(stage ^ 1, t + kAttnTile);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *kt = k_tile + stage * kAttnTile * kHeadDim;
        const float *vt = v_tile + stage * kAttnTile * kHeadDim;
        const int8_t *kb8 = reinterpret_cast<const int8_t *>(kt), *vb8 = reinterpret_cast<const int8_t *>(vt);
        const int nt = min(kAttnTile, t1 - t);
        // Scores: warp w scores rows 4w..4w+3 for every query head of the group.
#pragma unroll
        for (int r = 0; r < kAttnTile / 8; r++) {
            const int row = warp * (kAttnTile / 8) + r;
            float4 k4;
            if (BYTES) {
                const char4 c = reinterpret_cast<const char4 *>(kb8 + row * kHeadDim)[lane];
                const float s = ks_s[stage][row];
                k4 = make_float4(__fmul_rn((float)c.x, s), __fmul_rn((float)c.y, s), __fmul_rn((float)c.z, s),
                                 __fmul_rn((float)c.w, s));
            } else {
                k4 = reinterpret_cast<const float4 *>(kt + row * kHeadDim)[lane];
            }
            float bias = 0.f;
            if (BYTES && src.weights && row < nt) bias = __fmul_rn(__ldg(src.weights + t + row), sqrt_dim);
#pragma unroll
            for (int g = 0; g < kAttnMaxGroup; g++) {
                if (g >= group) break;
                float d = q4[g].x * k4.x;
                d = fmaf(q4[g].y, k4.y, d);
                d = fmaf(q4[g].z, k4.z, d);
                d = fmaf(q4[g].w, k4.w, d);
                d = warp_sum(d);
                if (lane == 0)
                    p_s[g * kAttnTile + row] = row < nt ? __fdiv_rn(__fadd_rn(d, bias), sqrt_dim) : -INFINITY;
            }
        }
        __syncthreads();
        // Online softmax statistics: warp g owns query head g.
        if (warp < group) {
            const float s = p_s[warp * kAttnTile + lane];
            const float m_old = m_s[warp];
            const float m_new = fmaxf(m_old, warp_max(s));
            const float e = s == -INFINITY ? 0.f : expf(s - m_new);
            const float sum = warp_sum(e);
            p_s[warp * kAttnTile + lane] = e;
            if (lane == 0) {
                const float c = m_old == -INFINITY ? 0.f : expf(m_old - m_new);
                c_s[warp] = c;
                l_s[warp] = fmaf(l_s[warp], c, sum);
                m_s[warp] = m_new;
            }
        }
        __syncthreads();
        // P.V: thread owns (g, d) pairs g = 2j + tid/128, d = tid%128.
#pragma unroll
        for (int j = 0; j < kAttnPerThread; j++) {
            const int g = j * (kAttnThreads / kHeadDim) + tid / kHeadDim, d = tid % kHeadDim;
            if (g < group) {
                float a = acc[j] * c_s[g];
                if (BYTES) {
                    for (int row = 0; row < kAttnTile; row++)
                        a = fmaf(p_s[g * kAttnTile + row], __fmul_rn((float)vb8[row * kHeadDim + d], vs_s[stage][row]), a);
                } else {
                    for (int row = 0; row < kAttnTile; row++) a = fmaf(p_s[g * kAttnTile + row], vt[row * kHeadDim + d], a);
                }
                acc[j] = a;
            }
        }
        __syncthreads();
    }

    // Publish this slice's partial result.
    float *mine = part + ((size_t)kvh * nsplit + split) * kAttnPartialFloats;
    if (tid < kAttnMaxGroup) {
        mine[tid] = m_s[tid];
        mine[kAttnMaxGroup + tid] = l_s[tid];
    }
#pragma unroll
    for (int j = 0; j < kAttnPerThread; j++) {
        const int g = j * (kAttnThreads / kHeadDim) + tid / kHeadDim, d = tid % kHeadDim;
        if (g < group) mine[2 * kAttnMaxGroup + g * kHeadDim + d] = acc[j];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last_s = atomicAdd(&counters[kvh], 1u) == (unsigned)(nsplit - 1);
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    // Last CTA of this KV head: combine the slices in split order. Warp g finds
    // head g's global max and per-slice weights exp(m_s - M); then every
    // (head, dim) output sums its slices with independent loads.
    const float *all = part + (size_t)kvh * nsplit * kAttnPartialFloats;
    float *w_s = k_tile;  // [kAttnMaxSplits][8] slice weights (tiles are free now)
    if (warp < group) {
        float M = -INFINITY;
        for (int s = lane; s < nsplit; s += 32) M = fmaxf(M, __ldcg(all + (size_t)s * kAttnPartialFloats + warp));
        M = warp_max(M);
        float den = 0.f;
        for (int s = lane; s < nsplit; s += 32) {
            const float *p = all + (size_t)s * kAttnPartialFloats;
            const float m = __ldcg(p + warp);
            const float w = m == -INFINITY ? 0.f : expf(m - M);
            w_s[s * kAttnMaxGroup + warp] = w;
            den = fmaf(w, __ldcg(p + kAttnMaxGroup + warp), den);
        }
        den = warp_sum(den);
        if (lane == 0) c_s[warp] = den;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kAttnPerThread; j++) {
        const int g = j * (kAttnThreads / kHeadDim) + tid / kHeadDim, d = tid % kHeadDim;
        if (g >= group) continue;
        const float *p = all + 2 * kAttnMaxGroup + g * kHeadDim + d;
        float num = 0.f;
#pragma unroll 8
        for (int s = 0; s < nsplit; s++) num = fmaf(w_s[s * kAttnMaxGroup + g], __ldcg(p + (size_t)s * kAttnPartialFloats), num);
        out[((size_t)kvh * group + g) * kHeadDim + d] = __fdiv_rn(num, c_s[g]);
    }
    if (tid == 0) counters[kvh] = 0u;
}

}  // namespace tcm
