// Decode attention for the fused path: one thread-block cluster per KV head,
// flash-decoding in registers, the slices merged through distributed shared
// memory.
//
// The kCluster CTAs of a KV head split its cache rows; each CTA's eight warps
// split them again. A lane holds 4 of the 128 head dimensions: per step of
// four rows it loads the K and V rows (512-byte coalesced reads; the next
// step's rows are loaded before this step's arithmetic), forms the query
// heads' partial dots, reduces them across the warp and updates each head's
// running max, rescaled sum and accumulator. The warps merge in a fixed order
// into the CTA's partial in shared memory; after a cluster barrier every CTA
// reads all partials of the cluster (DSMEM) for its share of the outputs and
// folds them in rank order (deterministic), and a second barrier keeps the
// partials alive until all reads are done. No global atomics or fences.
// Scores are dot * (1 / sqrt(128)), the reference's GPU scaling
// (src/qwen_cuda.cu:70).
#pragma once
#include "common.cuh"
#include "attention.cuh"
#include <cooperative_groups.h>

namespace tcm {

__device__ __forceinline__ unsigned long long attn_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr int kDecodeAttnWarps = 8;
constexpr int kDecodeAttnThreads = kDecodeAttnWarps * 32;
constexpr int kDecodeMinRows = 32;  // fewest cache rows per CTA: one step of four rows per warp

constexpr int kCluster = 16;  // CTAs per KV head (non-portable cluster size)

// A warp's running softmax state per query head: max m, rescaled sum l, and
// the lane's four accumulator dimensions.
template <int G> __device__ __forceinline__ void state_reset(float (&m)[G], float (&l)[G], float4 (&acc)[G]) {
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = -INFINITY;
        l[g] = 0.f;
        acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
}
// Fold one published partial (m[8], l[8], acc[8][128]) into the warp state.
template <int G>
__device__ __forceinline__ void state_merge(float (&m)[G], float (&l)[G], float4 (&acc)[G], const float *p, int lane) {
    float mp[G], lp[G];
    float4 ap[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        mp[g] = __ldcg(p + g);
        lp[g] = __ldcg(p + kAttnMaxGroup + g);
        ap[g] = __ldcg(reinterpret_cast<const float4 *>(p + 2 * kAttnMaxGroup + g * kHeadDim) + lane);
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        if (mp[g] == -INFINITY) continue;
        const float M = fmaxf(m[g], mp[g]);
        const float cs = m[g] == -INFINITY ? 0.f : expf(m[g] - M), cp = expf(mp[g] - M);
        l[g] = fmaf(l[g], cs, lp[g] * cp);
        acc[g] = make_float4(fmaf(acc[g].x, cs, ap[g].x * cp), fmaf(acc[g].y, cs, ap[g].y * cp),
                             fmaf(acc[g].z, cs, ap[g].z * cp), fmaf(acc[g].w, cs, ap[g].w * cp));
        m[g] = M;
    }
}
// Merge the eight warps' states in warp order; write a partial (m, l, acc) to
// `partial`, or the normalised result acc / l to `out` ([G][128]).
template <int G>
__device__ __forceinline__ void cta_merge(const float (&m)[G], const float (&l)[G], const float4 (&acc)[G],
                                          float (*wm)[G], float (*wl)[G], float (*wacc)[G][kHeadDim], float *partial,
                                          float *out) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __syncthreads();  // the buffers may still be read by a previous merge
#pragma unroll
    for (int g = 0; g < G; g++) {
        reinterpret_cast<float4 *>(wacc[warp][g])[lane] = acc[g];
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
    }
    __syncthreads();
    for (int o = tid; o < G * kHeadDim; o += kDecodeAttnThreads) {
        const int g = o / kHeadDim, d = o % kHeadDim;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kDecodeAttnWarps; w++) M = fmaxf(M, wm[w][g]);
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < kDecodeAttnWarps; w++) {
            if (wm[w][g] == -INFINITY) continue;
            const float e = expf(wm[w][g] - M);
            den = fmaf(e, wl[w][g], den);
            num = fmaf(e, wacc[w][g][d], num);
        }
        if (out) {
            out[g * kHeadDim + d] = __fdiv_rn(num, den);
        } else {
            partial[2 * kAttnMaxGroup + g * kHeadDim + d] = num;
            if (d == 0) {
                partial[g] = M;
                partial[kAttnMaxGroup + g] = den;
            }
        }
    }
}
template <int G>
__global__ void __launch_bounds__(kDecodeAttnThreads, 1) attn_decode_kernel(
    const float *__restrict__ q, const float *__restrict__ keys, const float *__restrict__ values, int capacity,
    const int *__restrict__ position, float inv_sqrt_dim, float *__restrict__ out,
    unsigned long long *__restrict__ trace) {
    static_assert(G <= kDecodeAttnWarps, "one warp per query head in the combine");
    __shared__ float wm[kDecodeAttnWarps][G], wl[kDecodeAttnWarps][G];
    __shared__ __align__(16) float wacc[kDecodeAttnWarps][G][kHeadDim];
    __shared__ __align__(16) float cta_part[kAttnPartialFloats];
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int kvh = blockIdx.y, split = (int)cluster.block_rank();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // Timeline trace (optional): entry, wait released, slice done, CTA done.
    unsigned long long *mark = trace ? trace + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 4 : nullptr;
    if (mark && tid == 0) mark[0] = attn_clock();
    pdl_wait();
    if (mark && tid == 0) mark[1] = attn_clock();
    pdl_trigger();
    const int L = min(*position + 1, capacity);
    const int chunk = (L + kCluster - 1) / kCluster;
    const int t0 = min(L, split * chunk), t1 = min(L, t0 + chunk);
    const int per_warp = (t1 - t0 + kDecodeAttnWarps - 1) / kDecodeAttnWarps;
    const int r0 = min(t1, t0 + warp * per_warp), r1 = min(t1, r0 + per_warp);
    const float4 *kb = reinterpret_cast<const float4 *>(keys + (size_t)kvh * capacity * kHeadDim);
    const float4 *vb = reinterpret_cast<const float4 *>(values + (size_t)kvh * capacity * kHeadDim);

    float4 q4[G], acc[G];
    float m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        q4[g] = reinterpret_cast<const float4 *>(q + ((size_t)kvh * G + g) * kHeadDim)[lane];
        acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
        m[g] = -INFINITY;
        l[g] = 0.f;
    }
    // Rows in steps of four; the next step's K/V rows are loaded before this
    // step's arithmetic so their latency overlaps it.
    constexpr int kStep = 4;
    float4 k4[kStep], v4[kStep], nk4[kStep], nv4[kStep];
    auto load_rows = [&](int t, float4 (&kk)[kStep], float4 (&vv)[kStep]) {
#pragma unroll
        for (int i = 0; i < kStep; i++) {
            const bool ok = t + i < r1;
            kk[i] = ok ? __ldcg(kb + (size_t)(t + i) * (kHeadDim / 4) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
            vv[i] = ok ? __ldcg(vb + (size_t)(t + i) * (kHeadDim / 4) + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    if (r0 < r1) load_rows(r0, k4, v4);
    for (int t = r0; t < r1; t += kStep) {
        if (t + kStep < r1) load_rows(t + kStep, nk4, nv4);
        float s[kStep][G];
#pragma unroll
        for (int i = 0; i < kStep; i++)
#pragma unroll
            for (int g = 0; g < G; g++) {
                float d = q4[g].x * k4[i].x;
                d = fmaf(q4[g].y, k4[i].y, d);
                d = fmaf(q4[g].z, k4[i].z, d);
                s[i][g] = fmaf(q4[g].w, k4[i].w, d);
            }
#pragma unroll
        for (int o = 16; o; o >>= 1)
#pragma unroll
            for (int i = 0; i < kStep; i++)
#pragma unroll
                for (int g = 0; g < G; g++) s[i][g] += __shfl_xor_sync(0xffffffffu, s[i][g], o);
#pragma unroll
        for (int g = 0; g < G; g++) {
            float mx = m[g];
#pragma unroll
            for (int i = 0; i < kStep; i++) {
                s[i][g] = t + i < r1 ? s[i][g] * inv_sqrt_dim : -INFINITY;
                mx = fmaxf(mx, s[i][g]);
            }
            const float c = m[g] == -INFINITY ? 0.f : expf(m[g] - mx);
            float4 a = make_float4(acc[g].x * c, acc[g].y * c, acc[g].z * c, acc[g].w * c);
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < kStep; i++) {
                const float p = s[i][g] == -INFINITY ? 0.f : expf(s[i][g] - mx);
                sum += p;
                a.x = fmaf(p, v4[i].x, a.x);
                a.y = fmaf(p, v4[i].y, a.y);
                a.z = fmaf(p, v4[i].z, a.z);
                a.w = fmaf(p, v4[i].w, a.w);
            }
            acc[g] = a;
            l[g] = fmaf(l[g], c, sum);
            m[g] = mx;
        }
#pragma unroll
        for (int i = 0; i < kStep; i++) {
            k4[i] = nk4[i];
            v4[i] = nv4[i];
        }
    }
    if (mark && tid == 0) mark[2] = attn_clock();
    // This CTA's slice result into shared memory, then the cluster combine.
    cta_merge<G>(m, l, acc, wm, wl, wacc, cta_part, nullptr);
    cluster.sync();
    constexpr int kOutPer = G * kHeadDim / kCluster;
    static_assert(G * kHeadDim % kCluster == 0 && kOutPer <= kDecodeAttnThreads, "cluster output split");
    if (tid < kOutPer) {
        const int o = split * kOutPer + tid, g = o / kHeadDim, d = o % kHeadDim;
        float M = -INFINITY;
        for (int r = 0; r < kCluster; r++) M = fmaxf(M, cluster.map_shared_rank(cta_part, r)[g]);
        float num = 0.f, den = 0.f;
        for (int r = 0; r < kCluster; r++) {
            const float *p = cluster.map_shared_rank(cta_part, r);
            const float mr = p[g];
            if (mr == -INFINITY) continue;
            const float e = expf(mr - M);
            den = fmaf(e, p[kAttnMaxGroup + g], den);
            num = fmaf(e, p[2 * kAttnMaxGroup + g * kHeadDim + d], num);
        }
        out[((size_t)kvh * G + g) * kHeadDim + d] = __fdiv_rn(num, den);
    }
    cluster.sync();
    if (mark && tid == 0) mark[3] = attn_clock();
}

}  // namespace tcm
