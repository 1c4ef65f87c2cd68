// Fused batch-1 decode for the Qwen2.5-1.5B decoder on B200 (sm_100a).
//
// Per layer five kernels, per token one readout kernel (reference equations:
// src/qwen.c:248-262,275,289,320,329-330,341,383-387). Every GEMV kernel is a
// persistent grid of one CTA per SM that owns a contiguous share of the rows
// and streams them through a shared-memory ring with bulk copies (stream.cuh);
// the input vector (RMS-normalised where the reference normalises) lives in
// each consumer lane's registers. Kernels are launched with programmatic
// dependent launch and trigger their dependents at once, so the next kernel's
// CTAs become resident beside the running one and their producers fill the
// first stages (up to ~100 KB per SM) before griddepcontrol.wait releases the
// consumers. A whole token is captured once as a CUDA graph and replayed.
#include "common.cuh"
#include "attention.cuh"
#include "attention_decode.cuh"
#include "stream.cuh"
#include "lanes.cuh"
#include "persistent.cuh"
#include "tp.cuh"
#include "kernels.h"
#include "../../include/qwen_b200.h"
#include "../../include/tcm_seeded.h"
#include <type_traits>
#include <mutex>
#include <vector>

namespace tcm {

namespace {

// Optional timeline trace: thread 0 of each CTA stamps the global timer at
// entry (0), when griddepcontrol.wait returned (1), when the input vector is
// ready (2) and when its last group is done (3).
__device__ __forceinline__ void trace_mark(unsigned long long *trace, int event) {
    if (trace && threadIdx.x == 0) trace[(size_t)blockIdx.x * 4 + event] = global_ns();
}

// ---------------------------------------------------------------- stage 1: q/k/v
struct QkvArgs {
    const void *wq, *wk, *wv, *embed;
    const float *bq, *bk, *bv, *norm, *rope_den;
    float *x, *q, *k, *v, *kcache, *vcache;
    DecodeState *st;
    unsigned long long *trace;  // per-CTA timestamps of this launch, or null
    int qheads, kvheads, capacity;
    float eps;
};
// Items are q/k/v rows in RoPE pairs: pair p = (head, d < 64) is rows d and
// d + 64 of that head. Each stage holds R rows = R/2 pairs; the epilogue adds
// the bias, rotates (q and k), stores q / k / v and appends k, v to the cache.
template <typename WT>
__global__ void __launch_bounds__(kStreamThreads, 2) qkv_kernel(QkvArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int R = Geo<WT>::R;
    __shared__ float res[2][R];
    __shared__ float bias_s[2 * kMaxPairsPerCta];
    __shared__ float den_s[kHeadDim / 2];
    __shared__ __align__(16) float nw_s[kHidden], x_s[kHidden];
    __shared__ int fail_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pairs = (a.qheads + 2 * a.kvheads) * 64;
    const int p0 = share_begin(pairs, blockIdx.x, gridDim.x), p1 = share_begin(pairs, blockIdx.x + 1, gridDim.x);
    const int items = 2 * (p1 - p0);
    auto locate = [&](int i, int &kind, int &hl, int &d) -> const WT * {
        const int p = p0 + (i >> 1), head = p >> 6;
        d = (p & 63) + 64 * (i & 1);
        const WT *base;
        if (head < a.qheads) { kind = 0; hl = head; base = (const WT *)a.wq; }
        else if (head < a.qheads + a.kvheads) { kind = 1; hl = head - a.qheads; base = (const WT *)a.wk; }
        else { kind = 2; hl = head - a.qheads - a.kvheads; base = (const WT *)a.wv; }
        return base + (size_t)(hl * kHeadDim + d) * kHidden;
    };
    if (threadIdx.x == 0) fail_s = 0;
    const Ring ring = ring_setup(smem, kStages, kStage<WT>);
    trace_mark(a.trace, 0);
    pdl_trigger();
    if (warp == kConsumerWarps) {
        if (lane == 0)
            ring_produce(ring, items, R, kRow<WT>, [&](int i) { int kd, hl, d; return (const void *)locate(i, kd, hl, d); },
                         &a.st->fault);
        return;
    }
    // Constants first (they do not depend on earlier kernels).
    stage_norm(nw_s, a.norm);
    for (int i = threadIdx.x; i < items; i += kConsumerWarps * 32) {
        int kind, hl, d;
        locate(i, kind, hl, d);
        const float *b = kind == 0 ? a.bq : kind == 1 ? a.bk : a.bv;
        bias_s[i] = b[hl * kHeadDim + d];
    }
    if (threadIdx.x < kHeadDim / 2) den_s[threadIdx.x] = a.rope_den[threadIdx.x];
    pdl_wait();
    trace_mark(a.trace, 1);
    const int pos = a.st->position;
    float xr[kLaneX];
    if (a.embed) {
        load_lane_row<WT>(xr, (const WT *)a.embed + (size_t)a.st->token * kHidden, lane);
        if (blockIdx.x == 0 && warp == 0) store_lane_vec<WT>(a.x, xr, lane);
    } else {
        copy_hidden(x_s, a.x);
    }
    consumers_sync();
    if (!a.embed) load_lane_vec<WT>(xr, x_s, lane);
    rms_lane<WT>(xr, nw_s, a.eps, lane);
    trace_mark(a.trace, 2);
    const int groups = (items + R - 1) / R;
    for (int g = 0; g < groups; g++) {
        const int n = min(R, items - g * R);
        if (ring_acquire(ring, g, &a.st->fault)) {
            const unsigned char *stage = ring.stage(g % kStages);
#pragma unroll
            for (int m = 0; m < R / kConsumerWarps; m++) {
                const int j = warp + kConsumerWarps * m;
                if (j < n) {
                    const float y = row_dot<WT>(stage + (size_t)j * kRow<WT>, xr, lane);
                    if (lane == 0) res[g & 1][j] = y;
                }
            }
        } else {
            fail_s = 1;
        }
        ring_release(ring, g);
        consumers_sync();
        if (fail_s) break;
        if ((int)threadIdx.x < n / 2) {
            const int t = threadIdx.x, i = g * R + 2 * t;
            int kind, hl, d;
            locate(i, kind, hl, d);
            float y0 = __fadd_rn(res[g & 1][2 * t], bias_s[i]), y1 = __fadd_rn(res[g & 1][2 * t + 1], bias_s[i + 1]);
            if (kind < 2) {
                const float angle = __fdiv_rn((float)pos, den_s[d]);
                float sn, cs;
                sincosf(angle, &sn, &cs);
                const float r0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                const float r1 = __fadd_rn(__fmul_rn(y1, cs), __fmul_rn(y0, sn));
                y0 = r0;
                y1 = r1;
            }
            float *dst = kind == 0 ? a.q : kind == 1 ? a.k : a.v;
            dst[hl * kHeadDim + d] = y0;
            dst[hl * kHeadDim + d + 64] = y1;
            float *cache = kind == 1 ? a.kcache : kind == 2 ? a.vcache : nullptr;
            if (cache && pos >= 0 && pos < a.capacity) {
                float *row = cache + ((size_t)hl * a.capacity + pos) * kHeadDim;
                row[d] = y0;
                row[d + 64] = y1;
            }
        }
    }
    trace_mark(a.trace, 3);
}

// ---------------------------------------------------------------- stage 3: O projection + residual
struct ORowsArgs {
    const void *w;
    float *in;           // the attention output (written here when `part` is set)
    const float *part;   // the attention's cluster partials to fold first, or null
    float *x;
    DecodeState *st;
    unsigned long long *trace;  // per-CTA timestamps of this launch, or null
    int group;           // query heads per KV head
};
// The deferred end of attn_decode_kernel: outputs o = threadIdx.x + 256 k
// (head o / 128, dimension o % 128) into v_s, each from the kClustersPerHead
// cluster partials (M, den, num) of its KV head, folded exactly as the
// kernel's own last CTA would fold them; a head with one non-empty partial
// gives num / den directly, as the one-cluster kernel does. M and den of every
// (KV head, cluster) are read once per CTA into ml_s (every thread needs them:
// read per thread, their few lines would take thousands of requests each),
// while each thread's num loads are in flight. Contains two consumers_syncs.
constexpr int kFoldHeads = kHidden / kHeadDim;  // query heads of the fused geometry
__device__ __forceinline__ void fold_attention(float *v_s, float (*ml_s)[kClustersPerHead][2 * kAttnMaxGroup],
                                               const float *__restrict__ part, int group) {
    constexpr int kPer = kHidden / (kConsumerWarps * 32);  // 6 outputs per thread
    constexpr int C = kClustersPerHead;
    const int nml = kFoldHeads / group * C * 2 * kAttnMaxGroup;
    for (int i = threadIdx.x; i < nml; i += kConsumerWarps * 32) {
        const int kc = i / (2 * kAttnMaxGroup), j = i % (2 * kAttnMaxGroup);
        ml_s[kc / C][kc % C][j] = __ldcg(part + (size_t)kc * kAttnPartialFloats + j);
    }
    float ac[kPer][C];
#pragma unroll
    for (int k = 0; k < kPer; k++) {
        const int o = threadIdx.x + kConsumerWarps * 32 * k;
        const int head = o / kHeadDim, kvh = head / group, g = head % group, d = o % kHeadDim;
        const float *hp = part + (size_t)kvh * C * kAttnPartialFloats + 2 * kAttnMaxGroup + g * kHeadDim + d;
#pragma unroll
        for (int c = 0; c < C; c++) ac[k][c] = __ldcg(hp + (size_t)c * kAttnPartialFloats);
    }
    consumers_sync();
#pragma unroll
    for (int k = 0; k < kPer; k++) {
        const int o = threadIdx.x + kConsumerWarps * 32 * k;
        const int head = o / kHeadDim, kvh = head / group, g = head % group;
        float mc[C], lc[C];
#pragma unroll
        for (int c = 0; c < C; c++) {
            mc[c] = ml_s[kvh][c][g];
            lc[c] = ml_s[kvh][c][kAttnMaxGroup + g];
        }
        int valid = 0;
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int c = 0; c < C; c++)
            if (mc[c] != -INFINITY) {
                valid++;
                num = ac[k][c];
                den = lc[c];
            }
        if (valid > 1) {
            float M = -INFINITY;
#pragma unroll
            for (int c = 0; c < C; c++) M = fmaxf(M, mc[c]);
            num = 0.f;
            den = 0.f;
#pragma unroll
            for (int c = 0; c < C; c++) {
                if (mc[c] == -INFINITY) continue;
                const float e = expf(mc[c] - M);
                den = fmaf(e, lc[c], den);
                num = fmaf(e, ac[k][c], num);
            }
        }
        v_s[o] = __fdiv_rn(num, den);
    }
}
template <typename WT>
__global__ void __launch_bounds__(kStreamThreads, 2) oproj_kernel(ORowsArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int R = Geo<WT>::R;
    __shared__ __align__(16) float in_s[kHidden];
    __shared__ float ml_s[kFoldHeads][kClustersPerHead][2 * kAttnMaxGroup];
    __shared__ float x_s[kMaxRowsPerCta];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = share_begin(kHidden, blockIdx.x, gridDim.x), r1 = share_begin(kHidden, blockIdx.x + 1, gridDim.x);
    const int items = r1 - r0;
    const WT *w = (const WT *)a.w;
    const Ring ring = ring_setup(smem, kStages, kStage<WT>);
    trace_mark(a.trace, 0);
    pdl_trigger();
    if (warp == kConsumerWarps) {
        if (lane == 0)
            ring_produce(ring, items, R, kRow<WT>, [&](int i) { return (const void *)(w + (size_t)(r0 + i) * kHidden); },
                         &a.st->fault);
        return;
    }
    pdl_wait();
    trace_mark(a.trace, 1);
    // This CTA's residual rows, read now so that no row's update waits on L2
    // after its dot product (published by the consumers_sync below).
    if ((int)threadIdx.x < items) x_s[threadIdx.x] = a.x[r0 + threadIdx.x];
    if (a.part) fold_attention(in_s, ml_s, a.part, a.group);
    else copy_hidden(in_s, a.in);
    consumers_sync();
    float xr[kLaneX];
    load_lane_vec<WT>(xr, in_s, lane);
    if (a.part && blockIdx.x == 0)  // the attention output, for readers after this launch
        for (int i = threadIdx.x; i < kHidden / 4; i += kConsumerWarps * 32)
            reinterpret_cast<float4 *>(a.in)[i] = reinterpret_cast<const float4 *>(in_s)[i];
    trace_mark(a.trace, 2);
    const int groups = (items + R - 1) / R;
    for (int g = 0; g < groups; g++) {
        if (!ring_acquire(ring, g, &a.st->fault)) break;
        const int n = min(R, items - g * R);
        const unsigned char *stage = ring.stage(g % kStages);
#pragma unroll
        for (int m = 0; m < R / kConsumerWarps; m++) {
            const int j = warp + kConsumerWarps * m;
            if (j < n) {
                const float y = row_dot<WT>(stage + (size_t)j * kRow<WT>, xr, lane);
                if (lane == 0) a.x[r0 + g * R + j] = __fadd_rn(x_s[g * R + j], y);
            }
        }
        ring_release(ring, g);
    }
    trace_mark(a.trace, 3);
}

// ---------------------------------------------------------------- stage 4: gate/up + SwiGLU
struct GateUpArgs {
    const void *wg, *wu;        // this rank's first gate and up rows
    const float *norm, *x;
    float *h;
    DecodeState *st;
    unsigned long long *trace;  // per-CTA timestamps of this launch, or null
    unsigned *sched;            // row-group counter of this launch site
    float eps;
    int inter;                  // intermediate units of this rank (all 8960 on one GPU)
};
// Items alternate gate row j, up row j; the epilogue forms h_j = silu(g) * u
// as g / (1 + exp(-g)) * u (src/qwen_cuda.cu:79).
template <typename WT>
__global__ void __launch_bounds__(kStreamThreads, 2) gateup_kernel(GateUpArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int R = Geo<WT>::R;
    __shared__ float res[2][R];
    __shared__ __align__(16) float nw_s[kHidden], x_s[kHidden];
    __shared__ int fail_s, hdr_s[kStages];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = 2 * a.inter;
    const WT *wg = (const WT *)a.wg, *wu = (const WT *)a.wu;
    if (threadIdx.x == 0) fail_s = 0;
    const Ring ring = ring_setup(smem, kStages, kStage<WT>);
    trace_mark(a.trace, 0);
    pdl_trigger();
    if (warp == kConsumerWarps) {
        if (lane == 0)
            ring_produce_dynamic(ring, items, R, kRow<WT>,
                                 [&](int i) { return (const void *)((i & 1 ? wu : wg) + (size_t)(i >> 1) * kHidden); },
                                 a.sched, hdr_s, &a.st->fault);
        return;
    }
    stage_norm(nw_s, a.norm);
    pdl_wait();
    trace_mark(a.trace, 1);
    float xr[kLaneX];
    copy_hidden(x_s, a.x);
    consumers_sync();
    load_lane_vec<WT>(xr, x_s, lane);
    rms_lane<WT>(xr, nw_s, a.eps, lane);
    trace_mark(a.trace, 2);
    for (int g = 0;; g++) {
        bool failed = false;
        const int grp = ring_next(ring, g, hdr_s, &a.st->fault, &failed);
        const int n = grp >= 0 ? min(R, items - grp * R) : 0;
        if (failed) fail_s = 1;
        if (grp >= 0) {
            const unsigned char *stage = ring.stage(g % kStages);
#pragma unroll
            for (int m = 0; m < R / kConsumerWarps; m++) {
                const int j = warp + kConsumerWarps * m;
                if (j < n) {
                    const float y = row_dot<WT>(stage + (size_t)j * kRow<WT>, xr, lane);
                    if (lane == 0) res[g & 1][j] = y;
                }
            }
            ring_release(ring, g);
        }
        consumers_sync();
        if (fail_s || grp < 0) break;
        if ((int)threadIdx.x < n / 2) {
            const int t = threadIdx.x;
            const float gv = res[g & 1][2 * t], uv = res[g & 1][2 * t + 1];
            a.h[(grp * R) / 2 + t] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.f, expf(-gv))), uv);
        }
    }
    trace_mark(a.trace, 3);
}

// ---------------------------------------------------------------- stage 5: down projection + residual
struct DownArgs {
    const void *w;              // this rank's first column of the down matrix (row stride 8960)
    const float *h;             // this rank's intermediate units
    float *x;
    DecodeState *st;
    unsigned long long *trace;  // per-CTA timestamps of this launch, or null
    TpLink tp;                  // world 1: the sums go straight into the residual
    int layer;
};
// Row geometry of the down projection when a rank reads F = 8960 / SH columns
// of every row: RD rows of F per stage (the stage stays ~35 KB); with fewer
// than eight rows a stage, PIECES warps split each row into contiguous pieces;
// with more, each warp takes RPW whole rows.
template <typename WT, int SH> struct DownGeo {
    static constexpr int E = Geo<WT>::E;
    static constexpr int F = kInter / SH;
    static constexpr int RD = Geo<WT>::RD * SH;
    static constexpr int PIECES = RD >= kConsumerWarps ? 1 : kConsumerWarps / RD;
    static constexpr int RPW = RD >= kConsumerWarps ? RD / kConsumerWarps : 1;
    static constexpr int NVP = F / E / PIECES;  // vectors per piece
    static constexpr int KV = (NVP + 31) / 32;  // per lane
    static constexpr uint32_t kRowBytes = F * sizeof(WT);
    static constexpr uint32_t kStageBytes = RD * kRowBytes;
    static_assert(F % (E * PIECES) == 0 && kRowBytes % 16 == 0, "down row pieces must be whole 16-byte vectors");
    static_assert(PIECES * RD == kConsumerWarps || RPW * kConsumerWarps == RD, "warps must tile a stage");
};
// The pieces of a row are summed in order into the residual row (one GPU), or
// into the rank's partial of that row, which the group then exchanges.
template <typename WT, int SH>
__global__ void __launch_bounds__(kStreamThreads, 2) down_kernel(DownArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    using G = DownGeo<WT, SH>;
    constexpr int RD = G::RD, E = G::E, PIECES = G::PIECES, RPW = G::RPW, NVP = G::NVP, KV = G::KV;
    __shared__ float part_s[2][RD][PIECES];
    __shared__ float x_s[kMaxRowsPerCta];
    __shared__ int fail_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int piece = PIECES > 1 ? warp % PIECES : 0;
    const int r0 = share_begin(kHidden, blockIdx.x, gridDim.x), r1 = share_begin(kHidden, blockIdx.x + 1, gridDim.x);
    const int items = r1 - r0;
    const WT *w = (const WT *)a.w;
    if (threadIdx.x == 0) fail_s = 0;
    const Ring ring = ring_setup(smem, kDownStages, G::kStageBytes);
    trace_mark(a.trace, 0);
    pdl_trigger();
    if (warp == kConsumerWarps) {
        if (lane == 0)
            ring_produce(ring, items, RD, G::kRowBytes, [&](int i) { return (const void *)(w + (size_t)(r0 + i) * kInter); },
                         &a.st->fault);
        return;
    }
    pdl_wait();
    trace_mark(a.trace, 1);
    // This CTA's residual rows, read now (published by the first consumers_sync).
    if ((int)threadIdx.x < items) x_s[threadIdx.x] = a.x[r0 + threadIdx.x];
    float hr[KV * E];
#pragma unroll
    for (int k = 0; k < KV; k++) {
        const int v = piece * NVP + lane + 32 * k;
#pragma unroll
        for (int e = 0; e < E; e += 4) {
            float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
            if (lane + 32 * k < NVP) f = reinterpret_cast<const float4 *>(a.h)[(E * v + e) / 4];
            hr[E * k + e] = f.x;
            hr[E * k + e + 1] = f.y;
            hr[E * k + e + 2] = f.z;
            hr[E * k + e + 3] = f.w;
        }
    }
    trace_mark(a.trace, 2);
    constexpr bool group = SH > 1;  // a rank reads part of each row only inside a group
    const unsigned token = group ? __ldcg(a.tp.epoch) + 1u : 0u;
    const int groups = (items + RD - 1) / RD;
    for (int g = 0; g < groups; g++) {
        const int n = min(RD, items - g * RD);
        if (ring_acquire(ring, g, &a.st->fault)) {
#pragma unroll
            for (int j = 0; j < RPW; j++) {
                const int slot = PIECES > 1 ? warp / PIECES : warp + kConsumerWarps * j;
                if (slot < n) {
                    const uint4 *row = reinterpret_cast<const uint4 *>(ring.stage(g % kDownStages) + (size_t)slot * G::kRowBytes);
                    float acc = 0.f;
#pragma unroll
                    for (int k = 0; k < KV; k++)
                        if (lane + 32 * k < NVP) acc = dot_vec(row[piece * NVP + lane + 32 * k], &hr[E * k], acc, WT());
                    acc = warp_sum(acc);
                    if (lane == 0) part_s[g & 1][slot][piece] = acc;
                }
            }
        } else {
            fail_s = 1;
        }
        ring_release(ring, g);
        consumers_sync();
        if (fail_s) break;
        if ((int)threadIdx.x < n) {
            const int s = threadIdx.x, row = r0 + g * RD + s;
            float sum = part_s[g & 1][s][0];
#pragma unroll
            for (int p = 1; p < PIECES; p++) sum = __fadd_rn(sum, part_s[g & 1][s][p]);
            if (group) {
                const size_t at = ((size_t)a.layer * a.tp.world + a.tp.rank) * kHidden + row;
                for (int p = 0; p < a.tp.world; p++) ll_store(a.tp.part[p] + at, __float_as_uint(sum), token);
            } else {
                a.x[row] = __fadd_rn(x_s[g * RD + s], sum);
            }
        }
    }
    if (group && !fail_s) {
        // This CTA's partial rows are on their way to every rank; add the
        // world's partials of the same rows, in rank order, as they arrive.
        const unsigned long long *mine = a.tp.part[a.tp.rank] + (size_t)a.layer * a.tp.world * kHidden;
        for (int row = r0 + (int)threadIdx.x; row < r1; row += kConsumerWarps * 32) {
            float sum = 0.f;
            bool ok = true;
            for (int p = 0; p < a.tp.world && ok; p++) {
                unsigned bits = 0;
                ok = ll_wait(mine + (size_t)p * kHidden + row, token, &bits, &a.st->fault);
                sum = p ? __fadd_rn(sum, __uint_as_float(bits)) : __uint_as_float(bits);
            }
            if (ok) a.x[row] = __fadd_rn(x_s[row - r0], sum);
        }
    }
    trace_mark(a.trace, 3);
}

// ---------------------------------------------------------------- readout + greedy top-2
struct ReadoutArgs {
    const void *embed;
    const float *norm, *x;
    float *logits;
    float *pv;
    int *pi;
    unsigned *sync;  // [0] block counter, [1] non-finite flag
    DecodeState *st;
    unsigned long long *trace;  // per-CTA timestamps of this launch, or null
    TcmTop2 *log;
    unsigned *sched;            // row-group counter of this launch site
    int vocab;
    float eps;
    TpLink tp;                  // world > 1: this rank's vocabulary rows, logits to every rank, top-2 exchange
};
template <typename WT>
__global__ void __launch_bounds__(kStreamThreads, 2) readout_kernel(ReadoutArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int R = Geo<WT>::R;
    __shared__ float sv[2 * kConsumerWarps];
    __shared__ int si[2 * kConsumerWarps];
    __shared__ __align__(16) float nw_s[kHidden], x_s[kHidden];
    __shared__ int last, hdr_s[kStages];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool group = a.tp.world > 1;
    const int base = group ? a.tp.vocab_begin : 0;
    const int items = group ? a.tp.vocab_end - a.tp.vocab_begin : a.vocab;
    const WT *e = (const WT *)a.embed + (size_t)base * kHidden;
    const Ring ring = ring_setup(smem, kStages, kStage<WT>);
    trace_mark(a.trace, 0);
    pdl_trigger();
    if (warp == kConsumerWarps) {
        if (lane == 0)
            ring_produce_dynamic(ring, items, R, kRow<WT>, [&](int i) { return (const void *)(e + (size_t)i * kHidden); },
                                 a.sched, hdr_s, &a.st->fault);
        return;
    }
    stage_norm(nw_s, a.norm);
    pdl_wait();
    trace_mark(a.trace, 1);
    float xr[kLaneX];
    copy_hidden(x_s, a.x);
    consumers_sync();
    load_lane_vec<WT>(xr, x_s, lane);
    rms_lane<WT>(xr, nw_s, a.eps, lane);
    Top2 t = top2_empty();
    bool bad = false;
    trace_mark(a.trace, 2);
    for (int g = 0;; g++) {
        bool failed = false;
        const int grp = ring_next(ring, g, hdr_s, &a.st->fault, &failed);
        if (grp < 0) break;
        const int n = min(R, items - grp * R);
        const unsigned char *stage = ring.stage(g % kStages);
#pragma unroll
        for (int m = 0; m < R / kConsumerWarps; m++) {
            const int j = warp + kConsumerWarps * m;
            if (j < n) {
                const int row = base + grp * R + j;
                const float y = row_dot<WT>(stage + (size_t)j * kRow<WT>, xr, lane);
                if (!group) {
                    if (lane == 0) a.logits[row] = y;
                } else if (lane < a.tp.world) {
                    a.tp.logits[lane][row] = y;  // every rank's logits buffer (peer stores)
                }
                bad |= !isfinite(y);
                top2_insert(t, y, row);
            }
        }
        ring_release(ring, g);
    }
    trace_mark(a.trace, 3);
    if (group && lane < a.tp.world) __threadfence_system();  // this lane's logits stores reach their rank first
    // Warp results (identical in every lane) -> CTA result -> last CTA merges.
    if (lane == 0) {
        sv[2 * warp] = t.a; sv[2 * warp + 1] = t.b;
        si[2 * warp] = t.ai; si[2 * warp + 1] = t.bi;
        if (bad) atomicOr(&a.sync[1], 1u);
    }
    consumers_sync();
    if (warp == 0) {
        Top2 u = top2_empty();
        if (lane < kConsumerWarps) {
            top2_insert(u, sv[2 * lane], si[2 * lane]);
            top2_insert(u, sv[2 * lane + 1], si[2 * lane + 1]);
        }
        top2_merge_warp(u);
        if (lane == 0) {
            a.pv[2 * blockIdx.x] = u.a; a.pv[2 * blockIdx.x + 1] = u.b;
            a.pi[2 * blockIdx.x] = u.ai; a.pi[2 * blockIdx.x + 1] = u.bi;
            if (group) __threadfence_system();
            else __threadfence();
            last = atomicAdd(&a.sync[0], 1u) == gridDim.x - 1;
        }
    }
    consumers_sync();
    if (!last) return;
    __threadfence();
    Top2 u = top2_empty();
    for (int i = threadIdx.x; i < 2 * (int)gridDim.x; i += kConsumerWarps * 32) top2_insert(u, __ldcg(a.pv + i), __ldcg(a.pi + i));
    top2_merge_warp(u);
    if (lane == 0) {
        sv[2 * warp] = u.a; sv[2 * warp + 1] = u.b;
        si[2 * warp] = u.ai; si[2 * warp + 1] = u.bi;
    }
    consumers_sync();
    if (warp == 0) {
        Top2 z = top2_empty();
        if (lane < kConsumerWarps) {
            top2_insert(z, sv[2 * lane], si[2 * lane]);
            top2_insert(z, sv[2 * lane + 1], si[2 * lane + 1]);
        }
        top2_merge_warp(z);
        if (lane == 0) {
            unsigned flag = atomicExch(&a.sync[1], 0u);
            DecodeState *st = a.st;
            if (group) {
                // Publish this rank's top-2 to every rank, then merge the
                // world's (the order of insertion does not change the result).
                // The fence orders every CTA's logits stores (each CTA fenced
                // before counting itself done) before the published words.
                __threadfence_system();
                const unsigned token = __ldcg(a.tp.epoch) + 1u;
                const unsigned words[5] = {__float_as_uint(z.a), __float_as_uint(z.b), (unsigned)z.ai, (unsigned)z.bi,
                                           flag};
                for (int p = 0; p < a.tp.world; p++)
                    for (int w = 0; w < 5; w++) ll_store(a.tp.top[p] + a.tp.rank * kTpTopWords + w, words[w], token);
                z = top2_empty();
                flag = 0u;
                for (int q = 0; q < a.tp.world; q++) {
                    unsigned v[5];
                    bool ok = true;
                    for (int w = 0; w < 5 && ok; w++)
                        ok = ll_wait(a.tp.top[a.tp.rank] + q * kTpTopWords + w, token, &v[w], &st->fault);
                    if (!ok) break;
                    top2_insert(z, __uint_as_float(v[0]), (int)v[2]);
                    top2_insert(z, __uint_as_float(v[1]), (int)v[3]);
                    flag |= v[4];
                }
                __threadfence_system();  // the peers' logits stores are visible past this kernel's end
                *a.tp.epoch = token;
            }
            TcmTop2 top;
            top.first = z.ai; top.second = z.bi; top.first_value = z.a; top.second_value = z.b;
            st->top = top;
            st->invalid |= (int)flag;
            a.log[st->step % kLogCap] = top;
            st->step += 1;
            st->token = z.ai;
            st->position += 1;
            a.sync[0] = 0u;
        }
    }
}

// ---------------------------------------------------------------- ring token cut
// One CTA per layer moves the 528-byte rows of the write and sample slots
// between the arena and the save area (132 words a row: 4 code segments of 32
// words, then 4 scales); every CTA copies a share of the logits. Mode 0 saves
// both rows, then copies the saved write row into the sample slot (the
// reference's per-layer ring_copy_row, src/bounded_cache.h:38-46, done for all
// layers at the start of the token); mode 1 writes both saved rows back.
constexpr int kRingRowWords = 132;
__device__ __forceinline__ unsigned *ring_word(unsigned char *layer, int rows, int slot, int w) {
    if (w < 128) {
        const int seg = w >> 5, kind = seg >> 1, head = seg & 1;
        return reinterpret_cast<unsigned *>(layer + (size_t)kind * rows * 256 + ((size_t)head * rows + slot) * 128) + (w & 31);
    }
    const int j = w - 128;  // kind * 2 + head
    return reinterpret_cast<unsigned *>(layer + (size_t)rows * 512) + (size_t)j * rows + slot;
}
struct RingCutArgs {
    unsigned char *arena, *save;
    const float *logits;
    float *logits_save;
    const DecodeState *st;  // slots from the token state when set
    int rows, layers, vocab, write_slot, sample_slot, mode;
};
__global__ void __launch_bounds__(256) ring_cut_kernel(RingCutArgs a) {
    pdl_trigger();
    pdl_wait();
    const int ws = a.st ? a.st->ring.write_slot : a.write_slot, ss = a.st ? a.st->ring.sample_slot : a.sample_slot;
    const int l = blockIdx.x, w = threadIdx.x;
    if (l < a.layers && w < kRingRowWords) {
        unsigned char *layer = a.arena + (size_t)l * a.rows * kRingRowBytes;
        unsigned *sw = reinterpret_cast<unsigned *>(a.save + (size_t)l * 2 * kRingRowBytes) + w;
        unsigned *aw = ring_word(layer, a.rows, ws, w);
        if (a.mode == 0) {
            const unsigned old_write = *aw;
            sw[0] = old_write;
            if (ss >= 0) {
                unsigned *as = ring_word(layer, a.rows, ss, w);
                sw[kRingRowWords] = *as;
                *as = old_write;
            }
        } else {
            *aw = sw[0];
            if (ss >= 0) *ring_word(layer, a.rows, ss, w) = sw[kRingRowWords];
        }
    }
    if (a.logits_save) {
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.vocab; i += gridDim.x * blockDim.x)
            a.logits_save[i] = a.logits[i];
    }
}

// ---------------------------------------------------------------- pipeline self-check
// One CTA streams `rows` FP32 rows of 1536 through the same shared-memory ring
// the decode GEMVs use and forms y = W x. With `starve` the producer is told to
// issue nothing, so every consumer warp's first wait runs out at the wait limit,
// records kErrFullWait and returns: no copy is in flight, nothing is left held.
struct SelfCheckArgs {
    const float *w, *x;
    float *y;
    unsigned *fault;
    int rows, starve;
};
__global__ void __launch_bounds__(kStreamThreads, 1) ring_selfcheck_kernel(SelfCheckArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int R = Geo<float>::R;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Ring ring = ring_setup(smem, kStages, kStage<float>);
    if (warp == kConsumerWarps) {
        if (lane == 0)
            ring_produce(ring, a.starve ? 0 : a.rows, R, kRow<float>,
                         [&](int i) { return (const void *)(a.w + (size_t)i * kHidden); }, a.fault);
        return;
    }
    float xr[kLaneX];
    load_lane_vec<float>(xr, a.x, lane);
    const int groups = (a.rows + R - 1) / R;
    for (int g = 0; g < groups; g++) {
        if (!ring_acquire(ring, g, a.fault)) break;
        const int n = min(R, a.rows - g * R);
        const unsigned char *stage = ring.stage(g % kStages);
#pragma unroll
        for (int m = 0; m < R / kConsumerWarps; m++) {
            const int j = warp + kConsumerWarps * m;
            if (j < n) {
                const float y = row_dot<float>(stage + (size_t)j * kRow<float>, xr, lane);
                if (lane == 0) a.y[g * R + j] = y;
            }
        }
        ring_release(ring, g);
    }
}

// Token state from kernel arguments: nothing in host memory is read after the
// launch call returns, so chained enqueues never race a host buffer.
__global__ void set_state_kernel(DecodeState *st, int token, int position) {
    st->token = token;
    st->position = position;
    st->step = 0;
    st->invalid = 0;
    st->fault = 0u;
    st->bar = 0u;
    st->arrive = 0u;
    st->nonfinite = 0u;
}

template <typename T> inline void set_smem(T *kernel, size_t bytes) {
    TCM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

}  // namespace

void set_wait_limit_decode(unsigned long long ns) { set_module_wait_limit(ns); }

__global__ void seeded_fill_kernel(void *dst, int dtype, uint64_t base, size_t n, TcmFill f) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = tcm_seeded_value(base, i, f);
        if (dtype == 2) ((uint16_t *)dst)[i] = tcm_bf16_rne(v);
        else ((float *)dst)[i] = v;
    }
}

}  // namespace tcm

using namespace tcm;

struct QwenB200Decoder {
    QwenB200Shape s;
    int dtype;
    const void *embed;
    const float *norm;
    std::vector<QwenB200Layer> layers;
    float *rope_den;
    size_t weight_bytes;
};

struct QwenB200Runner {
    const QwenB200Decoder *d;
    QwenB200Buffers b;
    std::vector<int> slots;
    DecodeState *st;
    TcmTop2 *log;
    float *attn_part;
    unsigned *attn_counters;
    float *top_pv;
    int *top_pi;
    unsigned *sync;
    DecodeState *host;  // pinned
    TcmTop2 *host_log;  // pinned
    cudaGraphExec_t graph;      // the whole-token graph
    bool graph_ready;
    bool after_host;  // the last stream operation was a host copy: next launch is not programmatic
    unsigned long long *trace;  // timeline buffer (kTraceLaunches x kTraceCtas x 4) or null
    int trace_next;
    int grid, launches;
    unsigned *sched;            // row-group counters, two per launch site (layer * 5 + stage; readout last)
    bool ring_on;               // cache-callback layers are served by `ring`
    QwenB200Ring ring;
    QwenB200RingStep staged;    // written with the next token state
    PersistLayer *pers_layers;  // device copy of the layers for the persistent token kernel
    float *pers_part;           // its attention partials
    bool persistent;            // whole tokens run as one persistent launch (when eligible)
    unsigned lookahead;         // its per-CTA L2 prefetch distance (bytes)
    // Tensor-parallel group (qwen_b200_tp_open / _connect): world 1 when off.
    TpLink tp;
    bool tp_on;                 // connected: launches split the MLP and readout
    unsigned char *tp_area;     // this rank's exchange area (gpu_alloc, exported)
    void *tp_peer_area[kTpMax], *tp_peer_logits[kTpMax];  // opened peer mappings
    int tp_rank, tp_world;
};

int tcm::decoder_view(const QwenB200Decoder *d, QwenB200Shape *shape, const QwenB200Layer **layers, const void **embed,
                 const float **final_norm, const float **rope_den, int *dtype) {
    if (!d) return -1;
    *shape = d->s;
    *layers = d->layers.data();
    *embed = d->embed;
    *final_norm = d->norm;
    *rope_den = d->rope_den;
    *dtype = d->dtype;
    return 0;
}

namespace {

void setup_attention() {
    TCM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<6, DenseRows>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    TCM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<6, DenseRows>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kStagedBytes));
    TCM_CUDA(cudaFuncSetAttribute(attn_decode_kernel<6, ByteRows>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
}
template <typename WT> void setup_kernels_typed() {
    set_smem(qkv_kernel<WT>, ring_smem_bytes(kStages, kStage<WT>));
    set_smem(oproj_kernel<WT>, ring_smem_bytes(kStages, kStage<WT>));
    set_smem(gateup_kernel<WT>, ring_smem_bytes(kStages, kStage<WT>));
    set_smem(down_kernel<WT, 1>, ring_smem_bytes(kDownStages, DownGeo<WT, 1>::kStageBytes));
    set_smem(down_kernel<WT, 2>, ring_smem_bytes(kDownStages, DownGeo<WT, 2>::kStageBytes));
    set_smem(down_kernel<WT, 4>, ring_smem_bytes(kDownStages, DownGeo<WT, 4>::kStageBytes));
    set_smem(down_kernel<WT, 8>, ring_smem_bytes(kDownStages, DownGeo<WT, 8>::kStageBytes));
    set_smem(readout_kernel<WT>, ring_smem_bytes(kStages, kStage<WT>));
    set_smem(ring_selfcheck_kernel, ring_smem_bytes(kStages, kStage<float>));
}
void setup_kernels() {
    static PerDeviceOnce once;
    once.run([] {
        setup_kernels_typed<float>();
        setup_kernels_typed<uint16_t>();
        setup_attention();
    });
}

constexpr int kTraceLaunches = 160, kTraceCtas = 320;
constexpr unsigned kDefaultLookahead = 0u;  // persistent kernel: L2 prefetch distance per CTA (measured: no gain)
// The trace slot of the next launch (launch order within a token), or null.
unsigned long long *trace_slot(QwenB200Runner *r) {
    if (!r->trace) return nullptr;
    return r->trace + (size_t)(r->trace_next++ % kTraceLaunches) * kTraceCtas * 4;
}

bool has_dense(const QwenB200Runner *r, int layer) { return r->slots[layer] >= 0; }
// The counter pair of a launch site. A kernel takes row groups from its pair
// before its dependency wait, so no two launches of one token may share one.
unsigned *sched_slot(const QwenB200Runner *r, int layer, int stage) { return r->sched + 2 * (layer * 5 + stage); }
size_t slot_offset(const QwenB200Runner *r, int layer) {
    const QwenB200Shape &s = r->d->s;
    return (size_t)r->slots[layer] * s.kvheads * r->b.capacity * s.head;
}

// Streamed GEMV kernels launched with two CTAs per SM (each CTA's ring and
// vectors take under half of an SM's shared memory), by kernel and weight
// type: every BF16 kernel, and the FP32 down projection and readout. Two rings
// per SM keep twice the weight bytes in flight; the FP32 q/k/v, O and gate/up
// kernels measured slower that way.
enum GemvKind { kGemvQkv, kGemvOproj, kGemvGateUp, kGemvDown, kGemvReadout };
template <typename WT> constexpr bool gemv_wide(GemvKind k) {
    return std::is_same<WT, uint16_t>::value || k == kGemvDown || k == kGemvReadout;
}
template <typename WT> int gemv_grid(const QwenB200Runner *r, GemvKind k) { return gemv_wide<WT>(k) ? 2 * r->grid : r->grid; }

template <typename WT> void launch_qkv(QwenB200Runner *r, int layer, bool pdl) {
    const QwenB200Decoder *d = r->d;
    const QwenB200Shape &s = d->s;
    const QwenB200Layer &L = d->layers[layer];
    QkvArgs a = {};
    a.wq = L.q; a.wk = L.k; a.wv = L.v;
    a.embed = layer == 0 ? d->embed : nullptr;
    a.bq = L.qb; a.bk = L.kb; a.bv = L.vb; a.norm = L.input_norm; a.rope_den = d->rope_den;
    a.x = r->b.x; a.q = r->b.q; a.k = r->b.k; a.v = r->b.v;
    a.kcache = has_dense(r, layer) ? r->b.keys + slot_offset(r, layer) : nullptr;
    a.vcache = has_dense(r, layer) ? r->b.values + slot_offset(r, layer) : nullptr;
    a.st = r->st;
    a.qheads = s.qheads; a.kvheads = s.kvheads; a.capacity = r->b.capacity; a.eps = s.epsilon;
    a.trace = trace_slot(r);
    launch(qkv_kernel<WT>, dim3(gemv_grid<WT>(r, kGemvQkv)), dim3(kStreamThreads), ring_smem_bytes(kStages, kStage<WT>), stream(), pdl, a);
}
// defer: leave the cluster partials in attn_part for the O projection to fold
// (out is then written by that launch).
template <class Rows>
void launch_attention_rows(QwenB200Runner *r, const Rows &rows, const float *q, float *out, bool pdl, bool defer) {
    const QwenB200Shape &s = r->d->s;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCluster * kClustersPerHead, s.kvheads);
    cfg.blockDim = dim3(kDecodeAttnThreads);
    cfg.dynamicSmemBytes = Rows::kStaged ? kStagedBytes : 0;
    cfg.stream = stream();
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    TCM_CUDA(cudaLaunchKernelEx(&cfg, attn_decode_kernel<6, Rows>, rows, q, 1.0f / sqrtf((float)kHeadDim),
                                r->attn_part, r->attn_counters, out, trace_slot(r),
                                defer ? 1 : 0));
}
void launch_attention(QwenB200Runner *r, int layer, bool pdl, bool defer = false) {
    DenseRows rows = {};
    rows.keys = r->b.keys + slot_offset(r, layer);
    rows.values = r->b.values + slot_offset(r, layer);
    rows.capacity = r->b.capacity;
    rows.position = &r->st->position;
    rows.fault = &r->st->fault;
    launch_attention_rows(r, rows, r->b.q, r->b.attention, pdl, defer);
}
void launch_ring_attention(QwenB200Runner *r, int layer, const float *q, const float *k, const float *v, float *out,
                           bool pdl, bool defer = false) {
    const QwenB200Ring &g = r->ring;
    ByteRows rows = {};
    rows.arena = (const signed char *)g.arena + (size_t)layer * g.rows * kRingRowBytes;
    rows.rows = g.rows;
    rows.anchors = g.anchors;
    rows.reservoir_base = g.anchors + g.recent;
    rows.step = &r->st->ring;
    rows.kcur = k;
    rows.vcur = v;
    rows.invalid = &r->st->invalid;
    launch_attention_rows(r, rows, q, out, pdl, defer);
}
void launch_ring_cut(QwenB200Runner *r, const DecodeState *st, int write_slot, int sample_slot, int mode, bool logits,
                     bool pdl) {
    const QwenB200Ring &g = r->ring;
    RingCutArgs a = {(unsigned char *)g.arena, (unsigned char *)g.save, r->b.logits, logits ? g.logits_save : nullptr,
                     st, g.rows, r->d->s.layers, r->d->s.vocab, write_slot, sample_slot, mode};
    launch(ring_cut_kernel, dim3(r->grid), dim3(256), 0, stream(), pdl, a);
}
// fold: the attention launch before this one deferred its cluster fold.
template <typename WT> void launch_oproj(QwenB200Runner *r, int layer, bool pdl, bool fold = false) {
    const QwenB200Shape &s = r->d->s;
    ORowsArgs o = {r->d->layers[layer].o, r->b.attention, fold ? r->attn_part : nullptr, r->b.x, r->st, trace_slot(r),
                   s.qheads / s.kvheads};
    launch(oproj_kernel<WT>, dim3(gemv_grid<WT>(r, kGemvOproj)), dim3(kStreamThreads), ring_smem_bytes(kStages, kStage<WT>), stream(), pdl, o);
}
// The link the launches of a runner carry (world 1 when no group is connected).
TpLink tp_link(const QwenB200Runner *r) {
    if (r->tp_on) return r->tp;
    TpLink t = {};
    t.world = 1;
    t.inter = kInter;
    t.vocab_end = r->d->s.vocab;
    return t;
}
template <typename WT> void launch_gateup(QwenB200Runner *r, int layer, bool pdl) {
    const QwenB200Layer &L = r->d->layers[layer];
    const TpLink t = tp_link(r);
    const size_t first = (size_t)t.rank * t.inter * kHidden;  // this rank's first unit
    GateUpArgs g = {(const WT *)L.gate + first, (const WT *)L.up + first, L.post_norm, r->b.x, r->b.gate, r->st,
                    trace_slot(r), sched_slot(r, layer, 3), r->d->s.epsilon, t.inter};
    launch(gateup_kernel<WT>, dim3(gemv_grid<WT>(r, kGemvGateUp)), dim3(kStreamThreads), ring_smem_bytes(kStages, kStage<WT>), stream(), pdl, g);
}
template <typename WT, int SH> void launch_down_sh(QwenB200Runner *r, int layer, bool pdl) {
    const TpLink t = tp_link(r);
    DownArgs dn = {(const WT *)r->d->layers[layer].down + (size_t)t.rank * t.inter, r->b.gate, r->b.x, r->st,
                   trace_slot(r), t, layer};
    launch(down_kernel<WT, SH>, dim3(gemv_grid<WT>(r, kGemvDown)), dim3(kStreamThreads),
           ring_smem_bytes(kDownStages, DownGeo<WT, SH>::kStageBytes), stream(), pdl, dn);
}
template <typename WT> void launch_down(QwenB200Runner *r, int layer, bool pdl) {
    switch (r->tp_on ? r->tp.world : 1) {
        case 2: launch_down_sh<WT, 2>(r, layer, pdl); break;
        case 4: launch_down_sh<WT, 4>(r, layer, pdl); break;
        case 8: launch_down_sh<WT, 8>(r, layer, pdl); break;
        default: launch_down_sh<WT, 1>(r, layer, pdl); break;
    }
}
template <typename WT> void launch_mlp(QwenB200Runner *r, int layer, bool pdl, bool fold = false) {
    launch_oproj<WT>(r, layer, pdl, fold);
    launch_gateup<WT>(r, layer, true);
    launch_down<WT>(r, layer, true);
}
template <typename WT> void launch_readout(QwenB200Runner *r, bool pdl) {
    const QwenB200Decoder *d = r->d;
    ReadoutArgs a = {d->embed, d->norm, r->b.x, r->b.logits, r->top_pv, r->top_pi, r->sync, r->st, trace_slot(r),
                     r->log, sched_slot(r, d->s.layers, 0), d->s.vocab, d->s.epsilon, tp_link(r)};
    launch(readout_kernel<WT>, dim3(gemv_grid<WT>(r, kGemvReadout)), dim3(kStreamThreads), ring_smem_bytes(kStages, kStage<WT>), stream(), pdl,
           a);
}

void launch_layer(QwenB200Runner *r, int layer, bool pdl_first) {
    if (r->d->dtype == 2) launch_qkv<uint16_t>(r, layer, pdl_first);
    else launch_qkv<float>(r, layer, pdl_first);
    // The O projection folds the attention's cluster partials (one dependent
    // step less than folding them in the attention's last CTA).
    if (has_dense(r, layer)) launch_attention(r, layer, true, true);
    else launch_ring_attention(r, layer, r->b.q, r->b.k, r->b.v, r->b.attention, true, true);
    if (r->d->dtype == 2) launch_mlp<uint16_t>(r, layer, true, true);
    else launch_mlp<float>(r, layer, true, true);
}
void launch_finish(QwenB200Runner *r, bool pdl) {
    if (r->d->dtype == 2) launch_readout<uint16_t>(r, pdl);
    else launch_readout<float>(r, pdl);
}
void launch_token(QwenB200Runner *r) {
    for (int l = 0; l < r->d->s.layers; l++) launch_layer(r, l, l > 0);
    launch_finish(r, true);
}

bool all_dense(const QwenB200Runner *r) {
    for (int s : r->slots)
        if (s < 0) return false;
    return true;
}
// Every layer has a fused attention: a dense slot, or the attached ring.
bool all_served(const QwenB200Runner *r) { return r->ring_on || all_dense(r); }

// The persistent token kernel serves the runner: every layer has a dense cache
// slot, no ring is attached, the attention split and the barrier timestamps
// fit the grid, and one CTA fits an SM.
int ensure_graph(QwenB200Runner *r);
bool persistent_ok(const QwenB200Runner *r) {
    const QwenB200Shape &s = r->d->s;
    return r->pers_layers && !r->ring_on && !r->tp_on && all_dense(r) && s.kvheads * kPersistAttnCtasPerHead <= r->grid &&
           12 * s.layers + 2 <= kPersistMarks && (size_t)r->grid * kPersistMarks <= (size_t)kTraceLaunches * kTraceCtas * 4 &&
           persistent_blocks_per_sm(r->d->dtype) >= 1;
}
bool use_persistent(const QwenB200Runner *r) { return r->persistent && persistent_ok(r); }
void launch_persistent_token(QwenB200Runner *r) {
    const QwenB200Decoder *d = r->d;
    const QwenB200Shape &s = d->s;
    PersistArgs a = {};
    a.layers = r->pers_layers;
    a.embed = d->embed;
    a.final_norm = d->norm;
    a.rope_den = d->rope_den;
    a.x = r->b.x; a.q = r->b.q; a.k = r->b.k; a.v = r->b.v;
    a.attn = r->b.attention; a.h = r->b.gate; a.logits = r->b.logits;
    a.part = r->pers_part;
    a.pv = r->top_pv;
    a.pi = r->top_pi;
    a.st = r->st;
    a.log = r->log;
    a.trace = r->trace;  // [grid][kPersistMarks] while the persistent kernel serves the runner
    a.nlayers = s.layers; a.qheads = s.qheads; a.kvheads = s.kvheads;
    a.capacity = r->b.capacity; a.vocab = s.vocab;
    a.eps = s.epsilon;
    a.inv_sqrt_dim = 1.0f / sqrtf((float)kHeadDim);
    a.lookahead = r->lookahead;
    launch_persistent(d->dtype, a, r->grid, stream());
    r->after_host = true;
}
// One whole token: the persistent launch, or the token graph.
int run_token(QwenB200Runner *r) {
    if (use_persistent(r)) {
        launch_persistent_token(r);
        return 0;
    }
    if (ensure_graph(r)) return -1;
    TCM_CUDA(cudaGraphLaunch(r->graph, stream()));
    r->after_host = true;
    return 0;
}

void drop_graphs(QwenB200Runner *r) {
    if (r->graph_ready) {
        TCM_CUDA(cudaGraphExecDestroy(r->graph));
        r->graph_ready = false;
    }
}
int ensure_graph(QwenB200Runner *r) {
    if (r->graph_ready) return 0;
    if (!all_served(r)) return -1;
    cudaStream_t s = stream();
    cudaGraph_t g;
    TCM_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    launch_token(r);
    TCM_CUDA(cudaStreamEndCapture(s, &g));
    TCM_CUDA(cudaGraphInstantiate(&r->graph, g, 0));
    TCM_CUDA(cudaGraphDestroy(g));
    r->graph_ready = true;
    return 0;
}

void write_state(QwenB200Runner *r, int token, int position) {
    r->host->token = token;
    r->host->position = position;
    r->host->step = 0;
    r->host->invalid = 0;
    r->host->fault = 0u;
    r->host->bar = 0u;
    r->host->arrive = 0u;
    r->host->nonfinite = 0u;
    r->host->ring = r->staged;
    // With a ring the whole state goes (the step follows the top-2 field).
    const size_t bytes = r->ring_on ? sizeof(DecodeState) : 8 * sizeof(int);
    TCM_CUDA(cudaMemcpyAsync(r->st, r->host, bytes, cudaMemcpyHostToDevice, stream()));
    r->after_host = true;
}
// Opens a token: the state, and with a ring the token cut (row store, sample
// copy, logits) before any layer.
void start_token(QwenB200Runner *r, int token, int position) {
    write_state(r, token, position);
    if (r->ring_on) {
        launch_ring_cut(r, r->st, 0, 0, 0, true, false);
        r->after_host = false;
    }
}
int read_top(QwenB200Runner *r, TcmTop2 *top) {
    TCM_CUDA(cudaMemcpyAsync(r->host, r->st, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream()));
    TCM_CUDA(cudaStreamSynchronize(stream()));
    if (top) *top = r->host->top;
    if (r->host->fault) {
        fprintf(stderr, "B200 decode: a pipeline wait ran out (fault bits 0x%x)\n", r->host->fault);
        return -4;
    }
    if (r->host->invalid & 2) return -5;  // a ring layer encoded a non-finite row: the token aborts first
    return r->host->invalid ? -3 : 0;
}
bool valid_token(const QwenB200Runner *r, int token, int position) {
    const int limit = r->ring_on ? r->ring.positions : r->b.capacity;
    return token >= 0 && token < r->d->s.vocab && position >= 0 && position < limit;
}

cudaEvent_t g_marks[64][16];

}  // namespace

extern "C" {

QwenB200Decoder *qwen_b200_decoder_create(const QwenB200Shape *shape, const float *embedding,
                                          const float *final_norm, const QwenB200Layer *layers, int matrix_dtype) {
    const QwenB200Shape &s = *shape;
    // The fused kernels are built for the Qwen2.5-1.5B geometry: hidden 1536, MLP
    // 8960, head 128, six query heads per KV head. Other shapes use the primitives.
    if (s.head != kHeadDim || s.hidden != kHidden || s.intermediate != kInter || s.kvheads < 1 ||
        s.qheads * s.head != s.hidden || s.qheads != 6 * s.kvheads || s.layers < 1 || s.vocab < 1 ||
        (s.qheads + 2 * s.kvheads) * 64 > kMaxPairsPerCta * 16)
        return nullptr;
    int dtype = matrix_dtype ? matrix_dtype : weight_dtype(embedding);
    if (dtype == 0) dtype = 1;
    if (dtype != 1 && dtype != 2) return nullptr;
    setup_kernels();
    QwenB200Decoder *d = new QwenB200Decoder();
    d->s = s;
    d->dtype = dtype;
    d->embed = embedding;
    d->norm = final_norm;
    d->layers.assign(layers, layers + s.layers);
    float host[kHeadDim / 2];
    for (int i = 0; i < kHeadDim / 2; i++) host[i] = powf(s.theta, 2.0f * i / kHeadDim);
    d->rope_den = (float *)gpu_alloc(sizeof(host));
    gpu_write(d->rope_den, host, sizeof(host));
    const size_t es = dtype == 2 ? 2 : 4, kv = (size_t)s.kvheads * s.head;
    const size_t per_layer = ((size_t)s.hidden * s.hidden * 2 + 2 * kv * s.hidden + 3 * (size_t)s.intermediate * s.hidden) * es +
                             ((size_t)s.hidden * 3 + 2 * kv) * 4;
    d->weight_bytes = per_layer * s.layers + (size_t)s.vocab * s.hidden * es + (size_t)s.hidden * 4;
    return d;
}

void qwen_b200_decoder_free(QwenB200Decoder *d) {
    if (!d) return;
    gpu_free(d->rope_den);
    delete d;
}

size_t qwen_b200_decoder_weight_bytes(const QwenB200Decoder *d) { return d ? d->weight_bytes : 0; }

QwenB200Runner *qwen_b200_runner_create(const QwenB200Decoder *d, const QwenB200Buffers *b) {
    if (!d || !b || b->capacity < 1) return nullptr;
    QwenB200Runner *r = new QwenB200Runner();
    r->d = d;
    r->b = *b;
    r->slots.resize(d->s.layers);
    for (int l = 0; l < d->s.layers; l++) r->slots[l] = b->cache_slots ? b->cache_slots[l] : l;
    r->st = (DecodeState *)gpu_alloc(sizeof(DecodeState));
    gpu_zero(r->st, sizeof(DecodeState));
    r->log = (TcmTop2 *)gpu_alloc(kLogCap * sizeof(TcmTop2));
    r->attn_part = (float *)gpu_alloc((size_t)d->s.kvheads * kClustersPerHead * kAttnPartialFloats * sizeof(float));
    r->attn_counters = (unsigned *)gpu_alloc((size_t)d->s.kvheads * sizeof(unsigned));
    gpu_zero(r->attn_counters, (size_t)d->s.kvheads * sizeof(unsigned));
    r->grid = sm_count();
    if (r->grid * kMaxRowsPerCta < kHidden)  // the O and down kernels stage their residual rows per CTA
        TCM_FATAL("qwen_b200: %d SMs is too few for the fused decoder (needs %d)", r->grid,
                  (kHidden + kMaxRowsPerCta - 1) / kMaxRowsPerCta);
    r->top_pv = (float *)gpu_alloc((size_t)4 * r->grid * sizeof(float));  // two per CTA, up to two CTAs per SM
    r->top_pi = (int *)gpu_alloc((size_t)4 * r->grid * sizeof(int));
    r->sync = (unsigned *)gpu_alloc(2 * sizeof(unsigned));
    gpu_zero(r->sync, 2 * sizeof(unsigned));
    const size_t sched_bytes = (size_t)(d->s.layers * 5 + 1) * 2 * sizeof(unsigned);
    r->sched = (unsigned *)gpu_alloc(sched_bytes);
    gpu_zero(r->sched, sched_bytes);
    TCM_CUDA(cudaMallocHost((void **)&r->host, sizeof(DecodeState)));
    TCM_CUDA(cudaMallocHost((void **)&r->host_log, kLogCap * sizeof(TcmTop2)));
    r->launches = d->s.layers * 5 + 1;
    std::vector<PersistLayer> pl(d->s.layers);
    for (int l = 0; l < d->s.layers; l++) {
        const QwenB200Layer &L = d->layers[l];
        const bool dense = r->slots[l] >= 0;
        pl[l] = PersistLayer{L.q, L.k, L.v, L.o, L.gate, L.up, L.down, L.qb, L.kb, L.vb, L.input_norm, L.post_norm,
                             dense ? b->keys + slot_offset(r, l) : nullptr, dense ? b->values + slot_offset(r, l) : nullptr};
    }
    r->pers_layers = (PersistLayer *)gpu_alloc(pl.size() * sizeof(PersistLayer));
    gpu_write(r->pers_layers, pl.data(), pl.size() * sizeof(PersistLayer));
    r->pers_part = (float *)gpu_alloc((size_t)d->s.kvheads * kPersistAttnCtasPerHead * kAttnPartialFloats * sizeof(float));
    r->persistent = false;  // the token graph measured faster on B200 (persistent kernel: opt-in)
    r->lookahead = kDefaultLookahead;
    return r;
}

void qwen_b200_runner_free(QwenB200Runner *r) {
    if (!r) return;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    qwen_b200_tp_close(r);
    drop_graphs(r);
    gpu_free(r->trace);
    gpu_free(r->st);
    gpu_free(r->log);
    gpu_free(r->attn_part);
    gpu_free(r->attn_counters);
    gpu_free(r->top_pv);
    gpu_free(r->top_pi);
    gpu_free(r->sync);
    gpu_free(r->sched);
    gpu_free(r->pers_layers);
    gpu_free(r->pers_part);
    TCM_CUDA(cudaFreeHost(r->host));
    TCM_CUDA(cudaFreeHost(r->host_log));
    delete r;
}

int qwen_b200_begin(QwenB200Runner *r, int token, int position) {
    if (!r || !valid_token(r, token, position)) return -1;
    start_token(r, token, position);
    return 0;
}

int qwen_b200_layer_qkv(QwenB200Runner *r, int layer) {
    if (!r || layer < 0 || layer >= r->d->s.layers) return -1;
    if (r->d->dtype == 2) launch_qkv<uint16_t>(r, layer, !r->after_host);
    else launch_qkv<float>(r, layer, !r->after_host);
    r->after_host = false;
    return 0;
}
int qwen_b200_layer_attention(QwenB200Runner *r, int layer) {
    if (!r || layer < 0 || layer >= r->d->s.layers || !has_dense(r, layer)) return -1;
    launch_attention(r, layer, !r->after_host);
    r->after_host = false;
    return 0;
}
int qwen_b200_layer_mlp(QwenB200Runner *r, int layer) {
    if (!r || layer < 0 || layer >= r->d->s.layers) return -1;
    if (r->d->dtype == 2) launch_mlp<uint16_t>(r, layer, !r->after_host);
    else launch_mlp<float>(r, layer, !r->after_host);
    r->after_host = false;
    return 0;
}
int qwen_b200_layer(QwenB200Runner *r, int layer) {
    if (!r || layer < 0 || layer >= r->d->s.layers || !has_dense(r, layer)) return -1;
    launch_layer(r, layer, !r->after_host);
    r->after_host = false;
    return 0;
}
int qwen_b200_finish(QwenB200Runner *r, TcmTop2 *top) {
    if (!r) return -1;
    launch_finish(r, !r->after_host);
    r->after_host = true;
    return read_top(r, top);
}

int qwen_b200_token(QwenB200Runner *r, int token, int position, TcmTop2 *top) {
    if (!r || !valid_token(r, token, position) || (!use_persistent(r) && ensure_graph(r))) return -1;
    start_token(r, token, position);
    if (run_token(r)) return -1;
    return read_top(r, top);
}

int qwen_b200_complete(QwenB200Runner *r, TcmTop2 *top) {
    if (!r || run_token(r)) return -1;
    return read_top(r, top);
}

int qwen_b200_can_complete(const QwenB200Runner *r) { return r && all_served(r) ? 1 : 0; }

int qwen_b200_ring_attach(QwenB200Runner *r, const QwenB200Ring *g) {
    if (!r || !g || r->d->s.kvheads != 2 || g->rows < 1 || g->anchors < 0 || g->recent < 1 || g->reservoir < 0 ||
        g->anchors + g->recent + g->reservoir != g->rows || !g->arena || !g->save || !g->logits_save ||
        g->positions < 1 || g->positions > r->d->s.max_position || ((uintptr_t)g->arena & 15))
        return -1;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    drop_graphs(r);
    r->ring = *g;
    r->ring_on = true;
    r->staged = QwenB200RingStep{};
    r->staged.sample_slot = -1;
    r->launches = r->d->s.layers * 5 + 2;  // + the token cut
    return 0;
}

int qwen_b200_ring_stage(QwenB200Runner *r, const QwenB200RingStep *step) {
    if (!r || !r->ring_on || !step) return -1;
    const QwenB200Ring &g = r->ring;
    const QwenB200RingStep &t = *step;
    const bool ok = t.write_slot >= 0 && t.write_slot < g.anchors + g.recent &&
                    (t.sample_slot == -1 || (t.sample_slot >= g.anchors + g.recent && t.sample_slot < g.rows)) &&
                    t.anchors_n >= 0 && t.anchors_n <= g.anchors && t.recent_n >= 0 && t.recent_n <= g.recent &&
                    t.reservoir_n >= 0 && t.reservoir_n <= g.reservoir && t.anchors_n + t.reservoir_n + t.recent_n >= 1;
    if (!ok) return -1;
    r->staged = t;
    return 0;
}

int qwen_b200_ring_attention(QwenB200Runner *r, int layer, const float *q, const float *k, const float *v, float *out) {
    if (!r || !r->ring_on || layer < 0 || layer >= r->d->s.layers || has_dense(r, layer) || !q || !k || !v || !out)
        return -1;
    launch_ring_attention(r, layer, q, k, v, out, !r->after_host);
    r->after_host = false;
    return 0;
}

int qwen_b200_ring_status(QwenB200Runner *r) {
    if (!r) return -1;
    int invalid = 0;
    TCM_CUDA(cudaMemcpyAsync(&r->host->invalid, &r->st->invalid, sizeof(int), cudaMemcpyDeviceToHost, stream()));
    TCM_CUDA(cudaStreamSynchronize(stream()));
    invalid = r->host->invalid;
    r->after_host = true;
    return (invalid & 2) ? -1 : 0;
}

int qwen_b200_enqueue(QwenB200Runner *r, int token, int position, int n) {
    if (!r || r->ring_on || n < 1 || n > kLogCap || !valid_token(r, token, position) || position + n > r->b.capacity ||
        (!use_persistent(r) && ensure_graph(r)))
        return -1;
    set_state_kernel<<<1, 1, 0, stream()>>>(r->st, token, position);
    TCM_CUDA(cudaGetLastError());
    r->after_host = true;
    for (int i = 0; i < n; i++) run_token(r);
    return 0;
}

int qwen_b200_last(QwenB200Runner *r, TcmTop2 *top) { return r ? read_top(r, top) : -1; }

int qwen_b200_generate(QwenB200Runner *r, int token, int position, int n, int *ids, TcmTop2 *tops) {
    if (qwen_b200_enqueue(r, token, position, n)) return -1;
    TCM_CUDA(cudaMemcpyAsync(r->host_log, r->log, (size_t)n * sizeof(TcmTop2), cudaMemcpyDeviceToHost, stream()));
    const int status = read_top(r, nullptr);
    for (int i = 0; i < n; i++) {
        if (ids) ids[i] = r->host_log[i].first;
        if (tops) tops[i] = r->host_log[i];
    }
    return status;
}

int qwen_b200_launches_per_token(const QwenB200Runner *r) { return r ? (use_persistent(r) ? 1 : r->launches) : 0; }

int qwen_b200_persistent_tune(QwenB200Runner *r, int key, int value) {
    if (!r || key != 0 || value < 0 || value > 2048) return -1;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    r->lookahead = (unsigned)value << 10;
    return 0;
}

int qwen_b200_persistent(QwenB200Runner *r, int mode) {
    if (!r || mode < -1 || mode > 1) return -1;
    if (mode >= 0) {
        if (mode == 1 && !persistent_ok(r)) return -1;
        TCM_CUDA(cudaStreamSynchronize(stream()));
        r->persistent = mode == 1;
    }
    return use_persistent(r) ? 1 : 0;
}

int qwen_b200_trace(QwenB200Runner *r, int enable) {
    if (!r) return -1;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    drop_graphs(r);
    if (r->trace) {
        gpu_free(r->trace);
        r->trace = nullptr;
    }
    if (enable) {
        const size_t bytes = (size_t)kTraceLaunches * kTraceCtas * 4 * sizeof(unsigned long long);
        r->trace = (unsigned long long *)gpu_alloc(bytes);
        gpu_zero(r->trace, bytes);
    }
    r->trace_next = 0;
    return 0;
}

int qwen_b200_trace_read(QwenB200Runner *r, unsigned long long *host, size_t count) {
    const size_t total = (size_t)kTraceLaunches * kTraceCtas * 4;
    if (!r || !r->trace || count < total) return -1;
    gpu_read(host, r->trace, total * sizeof(unsigned long long));
    return r->trace_next;
}

float qwen_b200_time_stage(QwenB200Runner *r, int stage, int layer, int position, int reps) {
    if (!r || stage < 0 || stage > 5 || layer < 0 || layer >= r->d->s.layers || reps < 1 ||
        !valid_token(r, 0, position) || (stage == 1 && !has_dense(r, layer) && !r->ring_on) ||
        (r->tp_on && stage >= 4))  // these stages exchange with the group: only whole tokens
        return -1.f;
    const bool bf16 = r->d->dtype == 2;
    auto once = [&](bool pdl) {
        switch (stage) {
            case 0: bf16 ? launch_qkv<uint16_t>(r, layer, pdl) : launch_qkv<float>(r, layer, pdl); break;
            case 1:
                // A ring layer re-encodes the session's current rows into the last token's write slot.
                if (has_dense(r, layer)) launch_attention(r, layer, pdl);
                else launch_ring_attention(r, layer, r->b.q, r->b.k, r->b.v, r->b.attention, pdl);
                break;
            case 2: bf16 ? launch_oproj<uint16_t>(r, layer, pdl) : launch_oproj<float>(r, layer, pdl); break;
            case 3: bf16 ? launch_gateup<uint16_t>(r, layer, pdl) : launch_gateup<float>(r, layer, pdl); break;
            case 4: bf16 ? launch_down<uint16_t>(r, layer, pdl) : launch_down<float>(r, layer, pdl); break;
            default: bf16 ? launch_readout<uint16_t>(r, pdl) : launch_readout<float>(r, pdl); break;
        }
    };
    // The readout advances the device position; each launch restarts it.
    set_state_kernel<<<1, 1, 0, stream()>>>(r->st, 0, position);
    once(false);
    cudaEvent_t a, b;
    TCM_CUDA(cudaEventCreate(&a));
    TCM_CUDA(cudaEventCreate(&b));
    float total = 0.f;
    for (int i = 0; i < reps; i++) {
        set_state_kernel<<<1, 1, 0, stream()>>>(r->st, 0, position);
        TCM_CUDA(cudaEventRecord(a, stream()));
        once(false);
        TCM_CUDA(cudaEventRecord(b, stream()));
        TCM_CUDA(cudaEventSynchronize(b));
        float ms = 0.f;
        TCM_CUDA(cudaEventElapsedTime(&ms, a, b));
        total += ms;
    }
    TCM_CUDA(cudaEventDestroy(a));
    TCM_CUDA(cudaEventDestroy(b));
    r->after_host = true;
    return total / reps;
}

void qwen_b200_ring_rows(void *arena, int rows, int layers, void *save, int write_slot, int sample_slot, int mode) {
    if (!arena || !save || rows < 1 || layers < 1 || layers > 64 || write_slot < 0 || write_slot >= rows ||
        sample_slot < -1 || sample_slot >= rows || (mode != 0 && mode != 1)) {
        fprintf(stderr, "qwen_b200_ring_rows: invalid arguments\n");
        exit(2);
    }
    RingCutArgs a = {(unsigned char *)arena, (unsigned char *)save, nullptr, nullptr, nullptr, rows, layers, 0,
                     write_slot, sample_slot, mode};
    ring_cut_kernel<<<layers, 256, 0, stream()>>>(a);
    TCM_CUDA(cudaGetLastError());
}

// ---------------------------------------------------------------- tensor-parallel group
namespace {
struct TpHandle {
    char magic[8];
    int rank, world, grid, layers, vocab, dtype;
    cudaIpcMemHandle_t area, logits;
};
static_assert(sizeof(TpHandle) <= QWEN_B200_TP_HANDLE_BYTES, "the handle must fit its published size");
constexpr char kTpMagic[8] = "TCMTP01";

typedef int (*AddressRangeFn)(unsigned long long *, size_t *, unsigned long long);
// The base and size of the allocation holding p (driver cuMemGetAddressRange).
bool allocation_of(const void *p, unsigned long long *base, size_t *size) {
    static AddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<AddressRangeFn>(f);
    });
    return fn && fn(base, size, (unsigned long long)(uintptr_t)p) == 0;
}
void tp_unmap(QwenB200Runner *r) {
    for (int p = 0; p < kTpMax; p++) {
        if (r->tp_peer_area[p]) TCM_CUDA(cudaIpcCloseMemHandle(r->tp_peer_area[p]));
        if (r->tp_peer_logits[p]) TCM_CUDA(cudaIpcCloseMemHandle(r->tp_peer_logits[p]));
        r->tp_peer_area[p] = r->tp_peer_logits[p] = nullptr;
    }
}
}  // namespace

int qwen_b200_tp_open(QwenB200Runner *r, int rank, int world, void *handle) {
    if (!r || !handle || (world != 2 && world != 4 && world != 8) || rank < 0 || rank >= world || r->ring_on ||
        !all_dense(r) || r->tp_area || r->d->s.intermediate != kInter || r->d->s.vocab < world)
        return -1;
    // Peers write the logits through an IPC mapping of their allocation, so the
    // buffer must be a whole allocation of its own.
    unsigned long long base = 0;
    size_t size = 0;
    if (!allocation_of(r->b.logits, &base, &size) || base != (unsigned long long)(uintptr_t)r->b.logits ||
        size < (size_t)r->d->s.vocab * sizeof(float)) {
        fprintf(stderr, "qwen_b200_tp_open: the logits buffer must be the start of its own device allocation\n");
        return -1;
    }
    TCM_CUDA(cudaStreamSynchronize(stream()));
    const TpLayout lay = tp_layout(r->d->s.layers, world);
    r->tp_area = (unsigned char *)gpu_alloc(lay.bytes);
    gpu_zero(r->tp_area, lay.bytes);
    TCM_CUDA(cudaStreamSynchronize(stream()));  // zero before any peer can learn the handle
    TpHandle h = {};
    memcpy(h.magic, kTpMagic, sizeof(kTpMagic));
    h.rank = rank;
    h.world = world;
    h.grid = r->grid;
    h.layers = r->d->s.layers;
    h.vocab = r->d->s.vocab;
    h.dtype = r->d->dtype;
    if (cudaIpcGetMemHandle(&h.area, r->tp_area) != cudaSuccess ||
        cudaIpcGetMemHandle(&h.logits, r->b.logits) != cudaSuccess) {
        cudaGetLastError();
        fprintf(stderr, "qwen_b200_tp_open: device memory cannot be exported to peer processes\n");
        gpu_free(r->tp_area);
        r->tp_area = nullptr;
        return -1;
    }
    memset(handle, 0, QWEN_B200_TP_HANDLE_BYTES);
    memcpy(handle, &h, sizeof(h));
    r->tp_rank = rank;
    r->tp_world = world;
    return 0;
}

int qwen_b200_tp_connect(QwenB200Runner *r, const void *handles) {
    if (!r || !handles || !r->tp_area || r->tp_on) return -1;
    const int world = r->tp_world, rank = r->tp_rank;
    TpHandle hs[kTpMax];
    for (int p = 0; p < world; p++) {
        memcpy(&hs[p], (const unsigned char *)handles + (size_t)p * QWEN_B200_TP_HANDLE_BYTES, sizeof(TpHandle));
        const TpHandle &h = hs[p];
        if (memcmp(h.magic, kTpMagic, sizeof(kTpMagic)) || h.rank != p || h.world != world || h.grid != r->grid ||
            h.layers != r->d->s.layers || h.vocab != r->d->s.vocab || h.dtype != r->d->dtype) {
            fprintf(stderr, "qwen_b200_tp_connect: handle %d does not belong to this group\n", p);
            return -1;
        }
    }
    TCM_CUDA(cudaStreamSynchronize(stream()));
    const TpLayout lay = tp_layout(r->d->s.layers, world);
    TpLink t = {};
    for (int p = 0; p < world; p++) {
        unsigned char *area = r->tp_area;
        float *logits = r->b.logits;
        if (p != rank) {
            void *a = nullptr, *l = nullptr;
            if (cudaIpcOpenMemHandle(&a, hs[p].area, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess ||
                (r->tp_peer_area[p] = a, cudaIpcOpenMemHandle(&l, hs[p].logits, cudaIpcMemLazyEnablePeerAccess)) !=
                    cudaSuccess) {
                cudaGetLastError();
                fprintf(stderr, "qwen_b200_tp_connect: cannot map rank %d's memory\n", p);
                tp_unmap(r);
                return -1;
            }
            r->tp_peer_logits[p] = l;
            area = static_cast<unsigned char *>(a);
            logits = static_cast<float *>(l);
        }
        t.part[p] = reinterpret_cast<unsigned long long *>(area + lay.part);
        t.logits[p] = logits;
        t.top[p] = reinterpret_cast<unsigned long long *>(area + lay.top);
    }
    t.epoch = reinterpret_cast<unsigned *>(r->tp_area + lay.epoch);
    t.rank = rank;
    t.world = world;
    t.inter = kInter / world;
    t.vocab_begin = share_begin(r->d->s.vocab, rank, world);
    t.vocab_end = share_begin(r->d->s.vocab, rank + 1, world);
    drop_graphs(r);
    r->tp = t;
    r->tp_on = true;
    return 0;
}

int qwen_b200_tp_close(QwenB200Runner *r) {
    if (!r) return -1;
    if (!r->tp_area) return 0;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    drop_graphs(r);
    tp_unmap(r);
    gpu_free(r->tp_area);
    r->tp_area = nullptr;
    r->tp_on = false;
    r->tp = TpLink{};
    r->tp_rank = 0;
    r->tp_world = 0;
    return 0;
}

int qwen_b200_tp_world(const QwenB200Runner *r) { return r && r->tp_on ? r->tp.world : 1; }

int qwen_b200_wait_limit(unsigned long long ns) {
    if (ns == 0) ns = kWaitLimitNs;
    if (ns < kWaitFloorNs || ns > 60000000000ull) return -1;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    set_module_wait_limit(ns);  // this file's kernels
    set_wait_limit_persistent(ns);
    set_wait_limit_batch(ns);
    return 0;
}

int qwen_b200_pipeline_check(const float *w, int rows, const float *x, float *y, int starve) {
    if (!w || !x || !y || rows < 1 || rows > 4096 || ((uintptr_t)w & 15) || ((uintptr_t)x & 15)) return -1;
    setup_kernels();
    unsigned *fault = (unsigned *)gpu_alloc(sizeof(unsigned));
    gpu_zero(fault, sizeof(unsigned));
    SelfCheckArgs a = {w, x, y, fault, rows, starve ? 1 : 0};
    launch(ring_selfcheck_kernel, dim3(1), dim3(kStreamThreads), ring_smem_bytes(kStages, kStage<float>), stream(), false,
           a);
    unsigned bits = 0;
    gpu_read(&bits, fault, sizeof(bits));
    gpu_free(fault);
    return (int)bits;
}

void qwen_b200_mark(int index) {
    int dev = 0;
    TCM_CUDA(cudaGetDevice(&dev));
    if (index < 0 || index >= 16) return;
    if (!g_marks[dev][index]) TCM_CUDA(cudaEventCreate(&g_marks[dev][index]));
    TCM_CUDA(cudaEventRecord(g_marks[dev][index], stream()));
}
float qwen_b200_elapsed_ms(int from, int to) {
    int dev = 0;
    TCM_CUDA(cudaGetDevice(&dev));
    float ms = 0.f;
    TCM_CUDA(cudaEventSynchronize(g_marks[dev][to]));
    TCM_CUDA(cudaEventElapsedTime(&ms, g_marks[dev][from], g_marks[dev][to]));
    return ms;
}
void qwen_b200_set_device(int device) { TCM_CUDA(cudaSetDevice(device)); }
int qwen_b200_sm_count(void) { return sm_count(); }

void qwen_b200_seeded_fill(void *dst, int dtype, uint64_t seed, uint32_t id, size_t n, float offset, float scale) {
    if (!n) return;
    TcmFill f = {offset, scale};
    seeded_fill_kernel<<<sm_count() * 8, 256, 0, stream()>>>(dst, dtype, tcm_tensor_base(seed, id), n, f);
    TCM_CUDA(cudaGetLastError());
}

}  // extern "C"
