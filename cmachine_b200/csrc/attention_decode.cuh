// Decode attention for the fused path: thread-block clusters per KV head,
// flash-decoding in registers, the slices merged through distributed shared
// memory.
//
// The kCluster CTAs of a KV head split its cache rows (caches longer than
// kSingleClusterRows use kClustersPerHead clusters); each CTA's eight warps
// split them again. A lane holds 4 of the 128 head dimensions: per step of
// four rows it loads the K and V rows (512-byte coalesced reads; the next
// step's rows are loaded before this step's arithmetic), forms the partial
// dots of the 4 x 8 (row, head) pairs (heads padded to eight), and a
// reduce-scatter butterfly leaves one full score per lane; the online softmax
// then updates each head's running max and rescaled sum, and the accumulators
// take the probabilities by shuffle. The warps merge in a fixed order into the
// CTA's partial in shared memory; after a cluster barrier every CTA reads all
// partials of its cluster (DSMEM) for its share of the outputs and folds them
// in rank order (deterministic); a second barrier keeps the partials alive
// until all reads are done. With several clusters per head, their partials
// meet in global memory and the last CTA to arrive folds them in order.
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
// Cluster partials and the cross-cluster merge (long caches only).
constexpr int kClustersPerHead = 4;
constexpr int kSingleClusterRows = 1024;  // caches up to this length use one cluster per head

template <int G>
__global__ void __launch_bounds__(kDecodeAttnThreads, 2) attn_decode_kernel(
    const float *__restrict__ q, const float *__restrict__ keys, const float *__restrict__ values, int capacity,
    const int *__restrict__ position, float inv_sqrt_dim, float *__restrict__ part, unsigned *__restrict__ counters,
    float *__restrict__ out, unsigned long long *__restrict__ trace) {
    static_assert(G <= 8, "query heads per KV head are padded to eight");
    constexpr int GP = 8;       // padded heads: 4 rows x 8 heads = 32 scores, one per lane
    constexpr int kStep = 4;    // rows per step
    __shared__ float wm[kDecodeAttnWarps][G], wl[kDecodeAttnWarps][G];
    __shared__ __align__(16) float wacc[kDecodeAttnWarps][G][kHeadDim];
    __shared__ __align__(16) float cta_part[kAttnPartialFloats];
    __shared__ int last_s;
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int kvh = blockIdx.y, rank = (int)cluster.block_rank(), cid = blockIdx.x / kCluster;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned long long *mark = trace ? trace + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 4 : nullptr;
    if (mark && tid == 0) mark[0] = attn_clock();
    // The position is set before a token's first kernel and the cache rows
    // below it were written by earlier tokens, so the row split and an L2
    // prefetch of those rows need not wait for the q/k/v kernel; only q and the
    // newest row (written by it) are read after griddepcontrol.wait.
    const int L = min(*position + 1, capacity);
    const int clusters = (int)(gridDim.x / kCluster);
    const bool multi = L > kSingleClusterRows && clusters > 1;
    if (!multi && cid > 0) {  // whole clusters leave together
        pdl_trigger();
        if (mark && tid == 0) mark[0] = 0ull;  // no work: not part of the timeline
        return;
    }
    const int ctas = multi ? clusters * kCluster : kCluster, cta = multi ? cid * kCluster + rank : rank;
    const int chunk = (L + ctas - 1) / ctas;
    const int t0 = min(L, cta * chunk), t1 = min(L, t0 + chunk);
    const int per_warp = (t1 - t0 + kDecodeAttnWarps - 1) / kDecodeAttnWarps;
    const int r0 = min(t1, t0 + warp * per_warp), r1 = min(t1, r0 + per_warp);
    const float4 *kb = reinterpret_cast<const float4 *>(keys + (size_t)kvh * capacity * kHeadDim);
    const float4 *vb = reinterpret_cast<const float4 *>(values + (size_t)kvh * capacity * kHeadDim);
    for (int t = r0 + (lane >> 2); t < min(r1, L - 1); t += 8) {
        const int part = lane & 3;  // four 128-byte lines per 512-byte row
        prefetch_l2(reinterpret_cast<const char *>(kb + (size_t)t * (kHeadDim / 4)) + 128 * part);
        prefetch_l2(reinterpret_cast<const char *>(vb + (size_t)t * (kHeadDim / 4)) + 128 * part);
    }
    pdl_wait();
    if (mark && tid == 0) mark[1] = attn_clock();
    pdl_trigger();

    float4 q4[G], acc[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        q4[g] = reinterpret_cast<const float4 *>(q + ((size_t)kvh * G + g) * kHeadDim)[lane];
        acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // Lane (row i = lane / 8, head g = lane % 8) owns one score per step; the
    // running max and sum of head g are kept in the lanes with lane % 8 == g.
    const int my_row = lane >> 3, my_head = lane & 7;
    float m_run = -INFINITY, l_run = 0.f;
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
        // Partial dots for the 32 (row, head) pairs, then a reduce-scatter
        // butterfly: after the stage with offset o each lane keeps the half of
        // its values selected by bit o of its lane id, so 31 shuffles leave
        // lane j holding the full dot of pair j.
        float v[kStep * GP];
#pragma unroll
        for (int i = 0; i < kStep; i++)
#pragma unroll
            for (int g = 0; g < GP; g++) {
                if (g < G) {
                    float d = q4[g].x * k4[i].x;
                    d = fmaf(q4[g].y, k4[i].y, d);
                    d = fmaf(q4[g].z, k4[i].z, d);
                    v[GP * i + g] = fmaf(q4[g].w, k4[i].w, d);
                } else {
                    v[GP * i + g] = 0.f;
                }
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int j = 0; j < o; j++) {
                const float send = upper ? v[j] : v[j + o];
                const float keep = upper ? v[j + o] : v[j];
                v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        const bool valid = t + my_row < r1 && my_head < G;
        const float sc = valid ? v[0] * inv_sqrt_dim : -INFINITY;
        float mx = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run, mx);
        const float c = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
        const float p = sc == -INFINITY ? 0.f : expf(sc - m_new);
        float ps = p + __shfl_xor_sync(0xffffffffu, p, 8);
        ps += __shfl_xor_sync(0xffffffffu, ps, 16);
        l_run = fmaf(l_run, c, ps);
        m_run = m_new;
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float cg_ = __shfl_sync(0xffffffffu, c, g);
            float4 a = make_float4(acc[g].x * cg_, acc[g].y * cg_, acc[g].z * cg_, acc[g].w * cg_);
#pragma unroll
            for (int i = 0; i < kStep; i++) {
                const float pg = __shfl_sync(0xffffffffu, p, GP * i + g);
                a.x = fmaf(pg, v4[i].x, a.x);
                a.y = fmaf(pg, v4[i].y, a.y);
                a.z = fmaf(pg, v4[i].z, a.z);
                a.w = fmaf(pg, v4[i].w, a.w);
            }
            acc[g] = a;
        }
#pragma unroll
        for (int i = 0; i < kStep; i++) {
            k4[i] = nk4[i];
            v4[i] = nv4[i];
        }
    }
    float m[G], l[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = __shfl_sync(0xffffffffu, m_run, g);
        l[g] = __shfl_sync(0xffffffffu, l_run, g);
    }
    if (mark && tid == 0) mark[2] = attn_clock();
    // This CTA's slice result into shared memory, then the cluster combine:
    // rank r folds the cluster's partials for outputs [r * kOutPer, ...).
    cta_merge<G>(m, l, acc, wm, wl, wacc, cta_part, nullptr);
    cluster.sync();
    constexpr int kOutPer = G * kHeadDim / kCluster;
    static_assert(G * kHeadDim % kCluster == 0 && kOutPer <= kDecodeAttnThreads, "cluster output split");
    float *cpart = multi ? part + ((size_t)kvh * clusters + cid) * kAttnPartialFloats : nullptr;
    if (tid < kOutPer) {
        const int o = rank * kOutPer + tid, g = o / kHeadDim, d = o % kHeadDim;
        float mr[kCluster], lr[kCluster], ar[kCluster];
#pragma unroll
        for (int r = 0; r < kCluster; r++) {
            const float *pr = cluster.map_shared_rank(cta_part, r);
            mr[r] = pr[g];
            lr[r] = pr[kAttnMaxGroup + g];
            ar[r] = pr[2 * kAttnMaxGroup + g * kHeadDim + d];
        }
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kCluster; r++) M = fmaxf(M, mr[r]);
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int r = 0; r < kCluster; r++) {
            if (mr[r] == -INFINITY) continue;
            const float e = expf(mr[r] - M);
            den = fmaf(e, lr[r], den);
            num = fmaf(e, ar[r], num);
        }
        if (!multi) {
            out[((size_t)kvh * G + g) * kHeadDim + d] = __fdiv_rn(num, den);
        } else {
            cpart[2 * kAttnMaxGroup + g * kHeadDim + d] = num;
            cpart[g] = M;  // every rank touching head g writes the same values
            cpart[kAttnMaxGroup + g] = den;
        }
    }
    cluster.sync();  // no CTA leaves while another still reads its partial
    if (multi) {
        // The last CTA of the head to arrive merges the clusters' partials.
        __threadfence();
        __syncthreads();
        if (tid == 0) last_s = atomicAdd(&counters[kvh], 1u) == (unsigned)(clusters * kCluster - 1);
        __syncthreads();
        if (last_s) {
            __threadfence();
            const float *hp = part + (size_t)kvh * clusters * kAttnPartialFloats;
            for (int o = tid; o < G * kHeadDim; o += kDecodeAttnThreads) {
                const int g = o / kHeadDim, d = o % kHeadDim;
                float mc[kClustersPerHead], lc[kClustersPerHead], ac[kClustersPerHead];
#pragma unroll
                for (int c = 0; c < kClustersPerHead; c++) {
                    const float *pc = hp + (size_t)c * kAttnPartialFloats;
                    const bool ok = c < clusters;
                    mc[c] = ok ? __ldcg(pc + g) : -INFINITY;
                    lc[c] = ok ? __ldcg(pc + kAttnMaxGroup + g) : 0.f;
                    ac[c] = ok ? __ldcg(pc + 2 * kAttnMaxGroup + g * kHeadDim + d) : 0.f;
                }
                float M = -INFINITY;
#pragma unroll
                for (int c = 0; c < kClustersPerHead; c++) M = fmaxf(M, mc[c]);
                float num = 0.f, den = 0.f;
#pragma unroll
                for (int c = 0; c < kClustersPerHead; c++) {
                    if (mc[c] == -INFINITY) continue;
                    const float e = expf(mc[c] - M);
                    den = fmaf(e, lc[c], den);
                    num = fmaf(e, ac[c], num);
                }
                out[((size_t)kvh * G + g) * kHeadDim + d] = __fdiv_rn(num, den);
            }
            if (tid == 0) counters[kvh] = 0u;
        }
    }
    if (mark && tid == 0) mark[3] = attn_clock();
}

}  // namespace tcm
