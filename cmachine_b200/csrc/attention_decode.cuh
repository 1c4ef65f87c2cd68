// Decode attention for the fused path: split-K over the FP32 K/V cache with
// every warp doing flash-decoding in registers.
//
// CTA (split, kv head) owns rows [t0, t1) (at least kAttnMinRows of them); its
// eight warps split those rows again. A lane holds 4 of the 128 head
// dimensions: per step of four rows it loads the K and V rows (512-byte
// coalesced reads, nothing staged in shared memory), forms the query heads'
// partial dots, reduces them across the warp, and updates each head's running
// max, rescaled sum and accumulator. The warps merge in a fixed order and each
// CTA publishes (m, l, acc) per head. The slices then combine in two levels:
// the last CTA to finish in each group of eight slices merges that group, and
// the last group merges the groups, every merge loading one partial per warp
// and folding the warps in order (deterministic).
// Scores are dot * (1 / sqrt(128)), the reference's GPU scaling
// (src/qwen_cuda.cu:70).
#pragma once
#include "common.cuh"
#include "attention.cuh"

namespace tcm {

__device__ __forceinline__ unsigned long long attn_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr int kDecodeAttnWarps = 8;
constexpr int kDecodeAttnThreads = kDecodeAttnWarps * 32;
constexpr int kDecodeMinRows = 32;  // fewest cache rows per CTA: one step of four rows per warp

constexpr int kGroup = 8;       // slices merged by the first combine level
constexpr int kMaxGroups = 16;  // >= ceil(kAttnSplits / kGroup)
static_assert(kMaxGroups * kGroup >= kAttnSplits, "group table too small");

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
// Publish: fence, count this CTA in `counter`; true in the CTA that arrives last
// of `expected` (all threads), which also sees every earlier CTA's writes.
__device__ __forceinline__ bool last_arrival(unsigned *counter, int expected, int *flag) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *flag = atomicAdd(counter, 1u) == (unsigned)(expected - 1);
    __syncthreads();
    if (*flag) __threadfence();
    return *flag != 0;
}

template <int G>
__global__ void __launch_bounds__(kDecodeAttnThreads, 1) attn_decode_kernel(
    const float *__restrict__ q, const float *__restrict__ keys, const float *__restrict__ values, int capacity,
    const int *__restrict__ position, float inv_sqrt_dim, float *__restrict__ part, unsigned *__restrict__ counters,
    float *__restrict__ out, unsigned long long *__restrict__ trace) {
    static_assert(G <= kDecodeAttnWarps, "one warp per query head in the combine");
    __shared__ float wm[kDecodeAttnWarps][G], wl[kDecodeAttnWarps][G];
    __shared__ __align__(16) float wacc[kDecodeAttnWarps][G][kHeadDim];
    __shared__ int last_s;
    const int kvh = blockIdx.y, split = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // Timeline trace (optional): entry, wait released, slice done, CTA done.
    unsigned long long *mark = trace ? trace + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 4 : nullptr;
    if (mark && tid == 0) mark[0] = attn_clock();
    pdl_wait();
    if (mark && tid == 0) mark[1] = attn_clock();
    pdl_trigger();
    const int L = min(*position + 1, capacity);
    const int chunk = max((L + (int)gridDim.x - 1) / (int)gridDim.x, kDecodeMinRows);
    const int nsplit = (L + chunk - 1) / chunk;
    if (split >= nsplit) return;
    const int t0 = split * chunk, t1 = min(L, t0 + chunk);
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
    // This CTA's slice result, then a two-level combine: the last CTA of each
    // group of kGroup slices merges the group, the last group merges the groups.
    float *head_part = part + (size_t)kvh * (kAttnSplits + kMaxGroups) * kAttnPartialFloats;
    cta_merge<G>(m, l, acc, wm, wl, wacc, head_part + (size_t)split * kAttnPartialFloats, nullptr);
    const int ngroups = (nsplit + kGroup - 1) / kGroup, group = split / kGroup;
    const int gsize = min(kGroup, nsplit - group * kGroup);
    unsigned *head_counters = counters + (size_t)kvh * (kMaxGroups + 1);
    if (!last_arrival(head_counters + 1 + group, gsize, &last_s)) {
        if (mark && tid == 0) mark[3] = attn_clock();
        return;
    }
    // Level 1: merge this group's slices (warp w takes slice w of the group).
    state_reset<G>(m, l, acc);
    if (warp < gsize) state_merge<G>(m, l, acc, head_part + (size_t)(group * kGroup + warp) * kAttnPartialFloats, lane);
    if (ngroups == 1) {
        cta_merge<G>(m, l, acc, wm, wl, wacc, nullptr, out + (size_t)kvh * G * kHeadDim);
        if (tid == 0) head_counters[1 + group] = 0u;
        if (mark && tid == 0) mark[3] = attn_clock();
        return;
    }
    cta_merge<G>(m, l, acc, wm, wl, wacc, head_part + (size_t)(kAttnSplits + group) * kAttnPartialFloats, nullptr);
    if (tid == 0) head_counters[1 + group] = 0u;
    if (!last_arrival(head_counters, ngroups, &last_s)) {
        if (mark && tid == 0) mark[3] = attn_clock();
        return;
    }
    // Level 2: merge the group results (warp w takes groups w and w + 8).
    state_reset<G>(m, l, acc);
    for (int gi = warp; gi < ngroups; gi += kDecodeAttnWarps)
        state_merge<G>(m, l, acc, head_part + (size_t)(kAttnSplits + gi) * kAttnPartialFloats, lane);
    cta_merge<G>(m, l, acc, wm, wl, wacc, nullptr, out + (size_t)kvh * G * kHeadDim);
    if (tid == 0) head_counters[0] = 0u;
    if (mark && tid == 0) mark[3] = attn_clock();
}

}  // namespace tcm
