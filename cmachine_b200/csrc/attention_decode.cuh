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
// CTA's partial in shared memory; every CTA then writes each rank the part of
// its partial that rank folds (distributed shared memory stores), and after one
// cluster barrier each rank folds its share of the outputs from its own shared
// memory in rank order (deterministic). With several clusters per head, their partials
// meet in global memory and the last CTA to arrive folds them in order.
// Scores are dot * (1 / sqrt(128)), the reference's GPU scaling
// (src/qwen_cuda.cu:70).
#pragma once
#include "common.cuh"
#include "attention.cuh"
#include "stream.cuh"
#include "../../include/qwen_b200.h"
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
// `sync` is a barrier over the eight warps (the CTA's, or a named barrier when
// the CTA has other warps).
template <int G, class Sync>
__device__ __forceinline__ void cta_merge(const float (&m)[G], const float (&l)[G], const float4 (&acc)[G],
                                          float (*wm)[G], float (*wl)[G], float (*wacc)[G][kHeadDim], float *partial,
                                          float *out, Sync sync) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    sync();  // the buffers may still be read by a previous merge
#pragma unroll
    for (int g = 0; g < G; g++) {
        reinterpret_cast<float4 *>(wacc[warp][g])[lane] = acc[g];
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
    }
    sync();
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

// ---------------------------------------------------------------- row sources
// The kernel reads rows through a source: rows t in [0, length()) of the KV
// head bound with bind(); load() gives the lane's four dimensions of K and V
// (FP32), bias() an additive score term, prefetch_line() warms one 128-byte
// line of row t in L2. current() runs after the dependency wait, before the
// first load.

// Cache rows a CTA stages in shared memory before its dependency wait.
constexpr int kStagedRows = 80;
constexpr unsigned kErrStaging = 0x20u;  // fault bit: launched without the staging buffer
constexpr uint32_t kStagedBytes = 2u * kStagedRows * kHeadDim * sizeof(float);

// Dense FP32 rows [kvheads][capacity][128]; rows 0..position. The rows of a
// CTA's slice below the newest (written by earlier tokens) are bulk-copied into
// shared memory before the dependency wait -- up to kStagedRows of them, rows
// [s0, s1) -- while the q/k/v kernel still runs; load() reads them there.
struct DenseRows {
    static constexpr bool kBias = false;
    static constexpr bool kStaged = true;
    static constexpr int kLines = 4;  // 128-byte lines per row and kind
    const float *keys, *values;
    int capacity;
    const int *position;
    unsigned *fault;                  // receives the bit of a staging wait that ran out
    const float4 *kb, *vb;
    const float4 *ks, *vs;            // staged rows (shared memory)
    int s0, s1;
    __device__ __forceinline__ void bind(int kvh) {
        kb = reinterpret_cast<const float4 *>(keys + (size_t)kvh * capacity * kHeadDim);
        vb = reinterpret_cast<const float4 *>(values + (size_t)kvh * capacity * kHeadDim);
    }
    __device__ __forceinline__ int length() const { return min(*position + 1, capacity); }
    // The newest row is written by the q/k/v kernel of this token: not prefetched.
    __device__ __forceinline__ int prefetch_limit() const { return length() - 1; }
    __device__ __forceinline__ void prefetch_line(int t, int part) const {
        prefetch_l2(reinterpret_cast<const char *>(kb + (size_t)t * (kHeadDim / 4)) + 128 * part);
        prefetch_l2(reinterpret_cast<const char *>(vb + (size_t)t * (kHeadDim / 4)) + 128 * part);
    }
    __device__ __forceinline__ void current(int, int, int) {}
    __device__ __forceinline__ void load(int t, int lane, float4 &k, float4 &v) const {
        if (t >= s0 && t < s1) {
            k = ks[(t - s0) * (kHeadDim / 4) + lane];
            v = vs[(t - s0) * (kHeadDim / 4) + lane];
            return;
        }
        k = __ldcg(kb + (size_t)t * (kHeadDim / 4) + lane);
        v = __ldcg(vb + (size_t)t * (kHeadDim / 4) + lane);
    }
    __device__ __forceinline__ float bias(int) const { return 0.f; }
};

// One (kind, KV head) row of the byte codec (src/qwen_cache.inc:3-15): s =
// max|x| / 127 (1 for a zero row), code = clamp(roundf(x / s), +-127), with
// IEEE division as the reference's encode_current; non-finite elements encode
// as 0 and flag the row. When `codes` is set the warp stores the row and its
// scale (unless the scale itself is unusable) and raises bit 2 of *invalid on
// a non-finite row. Returns the lane's dequantised dimensions (float)code * s.
__device__ __forceinline__ float4 encode_row(const float4 x, int lane, unsigned *codes, float *scale_out, int *invalid) {
    auto fin_abs = [](float v) { return isfinite(v) ? fabsf(v) : 0.f; };
    const bool fin = isfinite(x.x) && isfinite(x.y) && isfinite(x.z) && isfinite(x.w);
    const float m = warp_max(fmaxf(fmaxf(fin_abs(x.x), fin_abs(x.y)), fmaxf(fin_abs(x.z), fin_abs(x.w))));
    const bool all_fin = __all_sync(0xffffffffu, fin);
    const float s = m > 0.f ? __fdiv_rn(m, 127.f) : 1.f;
    const bool ok = s > 0.f && isfinite(s);
    auto code = [&](float v) {
        float c = isfinite(v) ? roundf(__fdiv_rn(v, s)) : 0.f;
        return (int)fminf(127.f, fmaxf(-127.f, c));
    };
    const int c0 = code(x.x), c1 = code(x.y), c2 = code(x.z), c3 = code(x.w);
    if (codes) {
        if (ok) {
            codes[lane] = (unsigned)(c0 & 0xff) | ((unsigned)(c1 & 0xff) << 8) | ((unsigned)(c2 & 0xff) << 16) |
                          ((unsigned)(c3 & 0xff) << 24);
            if (lane == 0) *scale_out = s;
        }
        if (lane == 0 && (!all_fin || !ok)) atomicOr(invalid, 2);
    }
    return make_float4(__fmul_rn((float)c0, s), __fmul_rn((float)c1, s), __fmul_rn((float)c2, s), __fmul_rn((float)c3, s));
}
__device__ __forceinline__ float4 dequant4(unsigned w, float s) {
    return make_float4(__fmul_rn((float)(signed char)(w & 0xffu), s), __fmul_rn((float)(signed char)((w >> 8) & 0xffu), s),
                       __fmul_rn((float)(signed char)((w >> 16) & 0xffu), s), __fmul_rn((float)(signed char)(w >> 24), s));
}

// Ring rows of one layer's byte-codec arena (per layer K codes [2][rows][128],
// V codes [2][rows][128], scales [kind * 2 + head][rows]). Logical rows are the
// retained anchor slots, then the retained reservoir slots, then the retained
// recent slots; the softmax does not depend on the order. The write slot's row
// is this token's K/V: every warp encodes it from the FP32 rows in registers
// (identical bits everywhere), and CTA 0 of the head also stores it.
struct ByteRows {
    static constexpr bool kBias = true;
    static constexpr bool kStaged = false;
    static constexpr int kLines = 1;
    const signed char *arena;  // this layer
    int rows, anchors, reservoir_base;  // reservoir_base = anchors + recent
    const QwenB200RingStep *step;
    const float *kcur, *vcur;           // this token's K, V rows [2][128] (FP32)
    int *invalid;
    // bound per CTA
    const unsigned *kc, *vc;
    const float *ks, *vs;
    int na, nm, nr, write_slot, kvh;
    bool weighted;
    float bias_v;
    float4 kq, vq;
    __device__ __forceinline__ void bind(int h) {
        kvh = h;
        kc = reinterpret_cast<const unsigned *>(arena + (size_t)h * rows * kHeadDim);
        vc = reinterpret_cast<const unsigned *>(arena + (size_t)rows * 2 * kHeadDim + (size_t)h * rows * kHeadDim);
        ks = reinterpret_cast<const float *>(arena + (size_t)rows * 4 * kHeadDim) + (size_t)h * rows;
        vs = reinterpret_cast<const float *>(arena + (size_t)rows * 4 * kHeadDim) + (size_t)(2 + h) * rows;
        na = step->anchors_n;
        nm = step->reservoir_n;
        nr = step->recent_n;
        write_slot = step->write_slot;
        weighted = step->weighted != 0;
        bias_v = step->bias;
    }
    __device__ __forceinline__ int length() const { return na + nm + nr; }
    __device__ __forceinline__ int prefetch_limit() const { return length(); }
    __device__ __forceinline__ int slot(int t) const {
        return t < na ? t : (t < na + nm ? reservoir_base + (t - na) : anchors + (t - na - nm));
    }
    __device__ __forceinline__ void prefetch_line(int t, int) const {
        const int s = slot(t);
        prefetch_l2(kc + (size_t)s * (kHeadDim / 4));
        prefetch_l2(vc + (size_t)s * (kHeadDim / 4));
    }
    __device__ __forceinline__ void current(int lane, int warp, int cta) {
        const float4 kx = reinterpret_cast<const float4 *>(kcur + (size_t)kvh * kHeadDim)[lane];
        const float4 vx = reinterpret_cast<const float4 *>(vcur + (size_t)kvh * kHeadDim)[lane];
        const bool store = cta == 0 && warp == 0;
        unsigned *kd = store ? const_cast<unsigned *>(kc) + (size_t)write_slot * (kHeadDim / 4) : nullptr;
        unsigned *vd = store ? const_cast<unsigned *>(vc) + (size_t)write_slot * (kHeadDim / 4) : nullptr;
        kq = encode_row(kx, lane, kd, const_cast<float *>(ks) + write_slot, invalid);
        vq = encode_row(vx, lane, vd, const_cast<float *>(vs) + write_slot, invalid);
    }
    __device__ __forceinline__ void load(int t, int lane, float4 &k, float4 &v) const {
        const int s = slot(t);
        if (s == write_slot) {
            k = kq;
            v = vq;
            return;
        }
        k = dequant4(__ldcg(kc + (size_t)s * (kHeadDim / 4) + lane), __ldcg(ks + s));
        v = dequant4(__ldcg(vc + (size_t)s * (kHeadDim / 4) + lane), __ldcg(vs + s));
    }
    __device__ __forceinline__ float bias(int t) const { return (weighted && t >= na && t < na + nm) ? bias_v : 0.f; }
};

// One flash-decoding step of a warp over four rows: k4[i], v4[i] hold the
// lane's four dimensions of row i, rows i >= nvalid are padding (K and V
// zero), bias(i) is row i's additive score term (kBias only). The partial dots
// of the 4 x 8 (row, head) pairs (heads padded to eight) go through a
// reduce-scatter butterfly: after the stage with offset o each lane keeps the
// half of its values selected by bit o of its lane id, so 31 shuffles leave
// lane j = 8 * row + head with the full dot of its pair. The lanes with
// lane % 8 == g keep head g's running max m_run and rescaled sum l_run; acc
// holds the lane's four dimensions of every head. Every product is an
// explicit, uncontracted operation, so two kernels that run the same steps on
// the same rows produce the same bits.
template <int G, bool kBias, class BiasFn>
__device__ __forceinline__ void flash_step(const float4 (&q4)[G], const float4 (&k4)[4], const float4 (&v4)[4],
                                           int nvalid, int lane, float inv_sqrt_dim, BiasFn bias, float &m_run,
                                           float &l_run, float4 (&acc)[G]) {
    constexpr int GP = 8;     // padded heads: 4 rows x 8 heads = 32 scores, one per lane
    constexpr int kStep = 4;  // rows per step
    const int my_row = lane >> 3, my_head = lane & 7;
    float v[kStep * GP];
#pragma unroll
    for (int i = 0; i < kStep; i++)
#pragma unroll
        for (int g = 0; g < GP; g++) {
            if (g < G) {
                float d = __fmul_rn(q4[g].x, k4[i].x);
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
            v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
        }
    }
    const bool valid = my_row < nvalid && my_head < G;
    float sc;
    if constexpr (kBias) {
        // (score + bias) / sqrt(128): the reference adds the bias before the
        // softmax scales (src/qwen_cache.inc:34, src/qwen_cuda.cu:67).
        sc = valid ? __fmul_rn(__fadd_rn(v[0], bias(my_row)), inv_sqrt_dim) : -INFINITY;
    } else {
        sc = valid ? __fmul_rn(v[0], inv_sqrt_dim) : -INFINITY;
    }
    float mx = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float m_new = fmaxf(m_run, mx);
    const float c = m_run == -INFINITY ? 0.f : expf(__fsub_rn(m_run, m_new));
    const float p = sc == -INFINITY ? 0.f : expf(__fsub_rn(sc, m_new));
    float ps = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 8));
    ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, 16));
    l_run = fmaf(l_run, c, ps);
    m_run = m_new;
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float cg_ = __shfl_sync(0xffffffffu, c, g);
        float4 a = make_float4(__fmul_rn(acc[g].x, cg_), __fmul_rn(acc[g].y, cg_), __fmul_rn(acc[g].z, cg_),
                               __fmul_rn(acc[g].w, cg_));
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
}

// One warp's flash-decoding over rows [r0, r1) of `rows` for the G query
// heads whose 4 dimensions per lane are in q4: four rows per step from r0 on
// (the next step's rows loaded ahead). Returns the warp's state in
// (m[G], l[G], acc[G]) (every lane holds m and l of every head).
template <int G, class Rows>
__device__ __forceinline__ void flash_rows(const Rows &rows, int r0, int r1, const float4 (&q4)[G], int lane,
                                           float inv_sqrt_dim, float (&m)[G], float (&l)[G], float4 (&acc)[G]) {
    constexpr int kStep = 4;
#pragma unroll
    for (int g = 0; g < G; g++) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    float m_run = -INFINITY, l_run = 0.f;
    float4 k4[kStep], v4[kStep], nk4[kStep], nv4[kStep];
    auto load_rows = [&](int t, float4 (&kk)[kStep], float4 (&vv)[kStep]) {
#pragma unroll
        for (int i = 0; i < kStep; i++) {
            if (t + i < r1) {
                rows.load(t + i, lane, kk[i], vv[i]);
            } else {
                kk[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                vv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    };
    if (r0 < r1) load_rows(r0, k4, v4);
    for (int t = r0; t < r1; t += kStep) {
        if (t + kStep < r1) load_rows(t + kStep, nk4, nv4);
        flash_step<G, Rows::kBias>(q4, k4, v4, r1 - t, lane, inv_sqrt_dim, [&](int i) { return rows.bias(t + i); },
                                   m_run, l_run, acc);
#pragma unroll
        for (int i = 0; i < kStep; i++) {
            k4[i] = nk4[i];
            v4[i] = nv4[i];
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = __shfl_sync(0xffffffffu, m_run, g);
        l[g] = __shfl_sync(0xffffffffu, l_run, g);
    }
}

template <int G, class Rows>
__global__ void __launch_bounds__(kDecodeAttnThreads, 2) attn_decode_kernel(
    Rows rows, const float *__restrict__ q, float inv_sqrt_dim, float *__restrict__ part,
    unsigned *__restrict__ counters, float *__restrict__ out, unsigned long long *__restrict__ trace, int defer) {
    static_assert(G <= 8, "query heads per KV head are padded to eight");
    __shared__ float wm[kDecodeAttnWarps][G], wl[kDecodeAttnWarps][G];
    __shared__ __align__(16) float wacc[kDecodeAttnWarps][G][kHeadDim];
    __shared__ __align__(16) float cta_part[kAttnPartialFloats];
    constexpr int kRecvFloats = 2 * kAttnMaxGroup + G * kHeadDim / kCluster;  // 64: what one rank sends another
    __shared__ __align__(16) float recv_s[kCluster][kRecvFloats];
    __shared__ int last_s;
    __shared__ __align__(8) uint64_t kv_bar;
    extern __shared__ __align__(128) unsigned char staged[];  // [K rows][V rows], kStagedRows each (DenseRows)
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int kvh = blockIdx.y, rank = (int)cluster.block_rank(), cid = blockIdx.x / kCluster;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned long long *mark = trace ? trace + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 4 : nullptr;
    if (mark && tid == 0) mark[0] = attn_clock();
    // The token state (position, ring step) is written before a token's first
    // kernel and the cache rows below the newest were written by earlier
    // tokens, so the row split and an L2 prefetch of those rows need not wait
    // for the q/k/v kernel; q and this token's K/V are read after
    // griddepcontrol.wait.
    rows.bind(kvh);
    const int L = rows.length();
    const int clusters = (int)(gridDim.x / kCluster);
    const bool multi = L > kSingleClusterRows && clusters > 1;
    if (!multi && cid > 0) {  // whole clusters leave together
        pdl_trigger();
        if (mark && tid == 0) mark[0] = 0ull;  // no work: not part of the timeline
        return;
    }
    // First phase of a cluster barrier, waited on just before the first
    // remote store: every CTA of the cluster has started by then (the arrive
    // carries no ordering; it only says this CTA is running).
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    const int ctas = multi ? clusters * kCluster : kCluster, cta = multi ? cid * kCluster + rank : rank;
    const int chunk = (L + ctas - 1) / ctas;
    const int t0 = min(L, cta * chunk), t1 = min(L, t0 + chunk);
    const int per_warp = (t1 - t0 + kDecodeAttnWarps - 1) / kDecodeAttnWarps;
    const int r0 = min(t1, t0 + warp * per_warp), r1 = min(t1, r0 + per_warp);
    int stage_from = r0;  // rows below this one are staged in shared memory
    if constexpr (Rows::kStaged) {
        // Stage only into shared memory the launch provided (else load every
        // row from global memory and record the configuration error).
        uint32_t dyn;
        asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
        const bool room = dyn >= kStagedBytes;
        if (!room && tid == 0 && rows.fault) atomicOr(rows.fault, kErrStaging);
        rows.s0 = t0;
        rows.s1 = room ? max(t0, min(min(t1, rows.prefetch_limit()), t0 + kStagedRows)) : t0;
        rows.ks = reinterpret_cast<const float4 *>(staged);
        rows.vs = reinterpret_cast<const float4 *>(staged + kStagedBytes / 2);
        if (tid == 0) {
            mbar_init(&kv_bar, 1);
            mbar_fence_init();
        }
        __syncthreads();
        if (tid == 0) {
            const uint32_t nb = (uint32_t)(rows.s1 - rows.s0) * kHeadDim * sizeof(float);
            if (nb) {
                mbar_expect_tx(&kv_bar, 2 * nb);
                bulk_copy_g2s(staged, rows.kb + (size_t)rows.s0 * (kHeadDim / 4), nb, &kv_bar);
                bulk_copy_g2s(staged + kStagedBytes / 2, rows.vb + (size_t)rows.s0 * (kHeadDim / 4), nb, &kv_bar);
            } else {
                mbar_arrive(&kv_bar);
            }
        }
        stage_from = max(r0, rows.s1);
    }
    {
        constexpr int kRowsPerPass = 32 / Rows::kLines;
        const int limit = min(r1, rows.prefetch_limit());
        for (int t = stage_from + lane / Rows::kLines; t < limit; t += kRowsPerPass)
            rows.prefetch_line(t, lane % Rows::kLines);
    }
    pdl_wait();
    if (mark && tid == 0) mark[1] = attn_clock();
    pdl_trigger();
    // This KV head's G query rows, read once per CTA (every warp needs all of
    // them) and passed on through shared memory: the warps' accumulator
    // buffer, which is not written before cta_merge's first barrier.
    static_assert(G * kHeadDim / 4 <= kDecodeAttnThreads, "one 16-byte piece of q per thread");
    float4 qpiece = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tid < G * kHeadDim / 4) qpiece = __ldcg(reinterpret_cast<const float4 *>(q + (size_t)kvh * G * kHeadDim) + tid);
    rows.current(lane, warp, cta);
    if constexpr (Rows::kStaged) {
        unsigned lost = 0u;
        mbar_wait(&kv_bar, 0, rows.fault ? rows.fault : &lost, kErrFullWait);
    }
    float *q_s = &wacc[0][0][0];
    if (tid < G * kHeadDim / 4) reinterpret_cast<float4 *>(q_s)[tid] = qpiece;
    __syncthreads();

    float4 q4[G], acc[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        q4[g] = reinterpret_cast<const float4 *>(q_s + g * kHeadDim)[lane];
        acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float m[G], l[G];
    flash_rows<G>(rows, r0, r1, q4, lane, inv_sqrt_dim, m, l, acc);
    if (mark && tid == 0) mark[2] = attn_clock();
    // This CTA's slice result into shared memory, then the cluster combine:
    // rank r folds the cluster's partials for outputs [r * kOutPer, ...).
    cta_merge<G>(m, l, acc, wm, wl, wacc, cta_part, nullptr, [] { __syncthreads(); });
    constexpr int kOutPer = G * kHeadDim / kCluster;
    static_assert(G * kHeadDim % kCluster == 0 && kOutPer <= kDecodeAttnThreads, "cluster output split");
    static_assert(kCluster * 16 == kDecodeAttnThreads && kOutPer == 48, "one 16-byte piece per thread");
    // Each CTA sends every rank r what r folds: the maxima and sums (16
    // floats) and its accumulators for outputs [r * kOutPer, ...) (contiguous
    // in the partial), as posted remote stores into r's recv_s row of this
    // CTA; after one cluster barrier every rank folds from its own shared
    // memory and no CTA touches another's again.
    __syncthreads();  // this CTA's partial is complete
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every peer is running
    {
        const int q = tid >> 4, c = tid & 15;
        const float *src = c < 4 ? cta_part + 4 * c : cta_part + 2 * kAttnMaxGroup + q * kOutPer + 4 * (c - 4);
        float *dst = cluster.map_shared_rank(&recv_s[0][0], q) + rank * kRecvFloats + 4 * c;
        *reinterpret_cast<float4 *>(dst) = *reinterpret_cast<const float4 *>(src);
    }
    cluster.sync();
    // Deferred (defer != 0): every used cluster leaves its partial in `part`
    // and the next launch folds them (unused clusters' partials are marked
    // empty); `out` and `counters` are not touched.
    float *cpart = multi || defer ? part + ((size_t)kvh * clusters + cid) * kAttnPartialFloats : nullptr;
    if (tid < kOutPer) {
        const int o = rank * kOutPer + tid, g = o / kHeadDim, d = o % kHeadDim;
        float mr[kCluster], lr[kCluster], ar[kCluster];
#pragma unroll
        for (int r = 0; r < kCluster; r++) {
            mr[r] = recv_s[r][g];
            lr[r] = recv_s[r][kAttnMaxGroup + g];
            ar[r] = recv_s[r][2 * kAttnMaxGroup + tid];
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
        if (!cpart) {
            out[((size_t)kvh * G + g) * kHeadDim + d] = __fdiv_rn(num, den);
        } else {
            cpart[2 * kAttnMaxGroup + g * kHeadDim + d] = num;
            cpart[g] = M;  // every rank touching head g writes the same values
            cpart[kAttnMaxGroup + g] = den;
        }
    }
    if (defer && !multi && rank == 0 && tid < (clusters - 1) * kAttnMaxGroup) {
        const int c = 1 + tid / kAttnMaxGroup, g = tid % kAttnMaxGroup;
        part[((size_t)kvh * clusters + c) * kAttnPartialFloats + g] = -INFINITY;
    }
    if (multi && !defer) {
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
