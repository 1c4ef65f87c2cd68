// Whole-token persistent decode for batch 1 on B200 (sm_100a).
//
// One cooperative launch of one CTA per SM runs a whole token: every layer's
// five stages (reference equations src/qwen.c:248-262,275,289,320,329-330,341)
// and the readout with greedy top-2 (src/qwen.c:383-387). A CTA is one
// producer thread and eight consumer warps around a ring of four 48 KB
// shared-memory stages (stream.cuh). The weights do not depend on the token,
// and the cache rows below the current position were written by earlier
// tokens, so the producer streams this CTA's whole share of the token -- its
// q/k/v rows, attention rows, O, gate/up and down rows of every layer, then
// its vocabulary rows -- without waiting for any other CTA: HBM keeps
// streaming while the consumers wait at the grid barriers between stages.
// The consumers take the stages in the same order and run six phases a
// layer, each ended by a grid barrier:
//   Q  RMSNorm (every warp holds the normalised vector in registers) and the
//      q/k/v rows in RoPE pairs: bias, rotation, q/k/v stores and the K/V
//      append at the current position;
//   A  flash-decoding over the cached rows with the split of the cluster
//      attention kernel (16 CTAs a KV head, 64 above 1024 rows; eight warps a
//      CTA; four rows a step), each CTA's partial to global memory;
//   M  the partials folded in the cluster kernel's order (ranks, then
//      clusters) into the attention output;
//   O  O projection + residual;
//   G  RMSNorm, gate/up rows, SwiGLU;
//   D  down projection + residual.
// The per-row dot products, pair epilogues and fold orders are those of the
// per-stage kernels, so a token is bit-identical to the layer-by-layer path.
//
// The grid barrier is a counter in the token state: every CTA adds one per
// barrier and waits until it reaches k x CTAs; the readout's last CTA resets
// it. Every wait is bounded (2 s) and records a fault bit. A CTA whose wait
// gives up sets its abort flag: its producer stops issuing, its consumers run
// the rest of the schedule without waiting or computing (so every named
// barrier still meets), and the other CTAs see the fault bit at their next
// grid barrier and do the same.
#include "common.cuh"
#include "attention.cuh"
#include "attention_decode.cuh"
#include "stream.cuh"
#include "lanes.cuh"
#include "persistent.cuh"
#include "kernels.h"
#include <mutex>

namespace tcm {
namespace {

constexpr int kPStages = 4;
constexpr uint32_t kPStage = 48 * 1024;
static_assert(kStage<float> == kPStage && kStage<uint16_t> == kPStage, "a stage holds one group of 1536-rows");
static_assert(kDownStage<float> <= kPStage && kDownStage<uint16_t> <= kPStage, "a stage holds one group of down rows");
constexpr int kStepRows = 4;                                      // attention rows per warp and step
constexpr uint32_t kKvRow = kHeadDim * sizeof(float);             // one cached K or V row (512 B)
constexpr uint32_t kVOff = kConsumerWarps * kStepRows * kKvRow;   // V rows follow the K rows in a stage
static_assert(2 * kVOff <= kPStage, "an attention stage holds one step of every warp");
constexpr int kGroupQ = 6;  // query heads per KV head
constexpr int kConsumerThreads = kConsumerWarps * 32;
enum : unsigned { kErrGrid = 8u };

// Which share of each stage's work a CTA owns. Shares are rotated by layer and
// phase so the CTAs that take one extra row differ from stage to stage.
struct TokenPlan {
    int grid, cta, pos, rows;  // rows: cache rows attended (position + 1)
    int per_head;              // attention CTAs per KV head: 16, or 64 above 1024 rows
    bool multi;
    __device__ int part(int layer, int phase) const { return (cta + layer * 53 + phase * 17) % grid; }
    __device__ void share(int total, int layer, int phase, int &lo, int &hi) const {
        const int p = part(layer, phase);
        lo = share_begin(total, p, grid);
        hi = share_begin(total, p + 1, grid);
    }
    // This CTA's attention slice of `layer` (the cluster kernel's split):
    // KV head, CTA index within the head, rows [t0, t1) and rows per warp.
    __device__ bool attention(int layer, int kvheads, int &kvh, int &hc, int &t0, int &t1, int &per_warp) const {
        const int a = part(layer, 1);
        if (a >= kvheads * per_head) return false;
        kvh = a / per_head;
        hc = a % per_head;
        const int chunk = (rows + per_head - 1) / per_head;
        t0 = min(rows, hc * chunk);
        t1 = min(rows, t0 + chunk);
        per_warp = (t1 - t0 + kConsumerWarps - 1) / kConsumerWarps;
        return true;
    }
};
__device__ __forceinline__ void warp_rows(int t0, int t1, int per_warp, int w, int &r0, int &r1) {
    r0 = min(t1, t0 + w * per_warp);
    r1 = min(t1, r0 + per_warp);
}

// q/k/v row i of the pairs starting at p0: pair p = (head, d < 64) is rows d
// and d + 64 of that head (items alternate).
template <typename WT>
__device__ __forceinline__ const WT *qkv_row(const PersistArgs &a, const PersistLayer &Ly, int p0, int i, int &kind,
                                             int &hl, int &d) {
    const int p = p0 + (i >> 1), head = p >> 6;
    d = (p & 63) + 64 * (i & 1);
    const WT *base;
    if (head < a.qheads) {
        kind = 0; hl = head; base = (const WT *)Ly.wq;
    } else if (head < a.qheads + a.kvheads) {
        kind = 1; hl = head - a.qheads; base = (const WT *)Ly.wk;
    } else {
        kind = 2; hl = head - a.qheads - a.kvheads; base = (const WT *)Ly.wv;
    }
    return base + (size_t)(hl * kHeadDim + d) * kHidden;
}

__device__ __forceinline__ bool aborted(const volatile int *abort_s) { return *abort_s != 0; }

// Bounded wait that also gives up at once when the CTA aborts.
__device__ __forceinline__ bool wait_phase(uint64_t *bar, uint32_t parity, unsigned *err, unsigned code,
                                           volatile int *abort_s) {
    if (aborted(abort_s)) return false;
    if (mbar_try(bar, parity)) return true;
    const unsigned long long start = global_ns();
    for (;;) {
        if (mbar_try(bar, parity)) return true;
        if (aborted(abort_s)) return false;
        if (wait_expired(global_ns() - start)) {
            atomicOr(err, code);
            *abort_s = 1;
            return false;
        }
    }
}

// ---------------------------------------------------------------- producer
// A position in this CTA's group sequence: group k of phase `phase` of
// `layer` (phases 0..4 = q/k/v, attention, O, gate/up, down; layer == nlayers,
// phase 0 = the readout), with the phase's share and group count. The
// consumers' loops take the same groups in the same order.
struct Walk {
    int layer, phase, k, n;
    int lo, hi;            // the phase's share: pairs, rows, or attention rows [t0, t1)
    int kvh, pw;           // attention: KV head, rows per warp
    bool done;
};
template <typename WT>
__device__ __forceinline__ void walk_enter(Walk &w, const PersistArgs &a, const TokenPlan &plan) {
    constexpr int R = Geo<WT>::R, RD = Geo<WT>::RD, H = R / 2;
    const int pairs = (a.qheads + 2 * a.kvheads) * 64;
    w.k = 0;
    if (w.layer == a.nlayers) {
        plan.share(a.vocab, a.nlayers, 0, w.lo, w.hi);
        w.n = (w.hi - w.lo + R - 1) / R;
        return;
    }
    switch (w.phase) {
        case 0:
            plan.share(pairs, w.layer, 0, w.lo, w.hi);
            w.n = (2 * (w.hi - w.lo) + R - 1) / R;
            break;
        case 1: {
            int hc;
            w.n = plan.attention(w.layer, a.kvheads, w.kvh, hc, w.lo, w.hi, w.pw) ? (w.pw + kStepRows - 1) / kStepRows : 0;
            break;
        }
        case 2:
            plan.share(kHidden, w.layer, 3, w.lo, w.hi);
            w.n = (w.hi - w.lo + R - 1) / R;
            break;
        case 3:
            plan.share(kInter, w.layer, 4, w.lo, w.hi);
            w.n = (w.hi - w.lo + H - 1) / H;
            break;
        default:
            plan.share(kHidden, w.layer, 5, w.lo, w.hi);
            w.n = (w.hi - w.lo + RD - 1) / RD;
            break;
    }
}
// Moves to the next group; false past the last.
template <typename WT>
__device__ __forceinline__ bool walk_next(Walk &w, const PersistArgs &a, const TokenPlan &plan) {
    w.k++;
    while (w.k >= w.n) {
        if (w.layer == a.nlayers) {
            w.done = true;
            return false;
        }
        if (++w.phase == 5) {
            w.phase = 0;
            w.layer++;
        }
        walk_enter<WT>(w, a, plan);
    }
    return true;
}
template <typename WT>
__device__ __forceinline__ void walk_begin(Walk &w, const PersistArgs &a, const TokenPlan &plan) {
    w.layer = 0;
    w.phase = 0;
    w.done = false;
    walk_enter<WT>(w, a, plan);
    if (w.n == 0) {
        w.k = -1;
        walk_next<WT>(w, a, plan);
    }
}

enum GroupOp { kBytes, kCopy, kPrefetch };
// The current group's copies: their total bytes (kBytes), bulk copies into
// `stage` completing on `bar` (kCopy), or L2 prefetches of the same rows
// (kPrefetch). Attention groups cover only rows below the position.
template <typename WT, GroupOp kOp>
__device__ __forceinline__ uint32_t walk_group(const Walk &w, const PersistArgs &a, const TokenPlan &plan,
                                               unsigned char *stage, uint64_t *bar, uint64_t policy) {
    constexpr int R = Geo<WT>::R, RD = Geo<WT>::RD, H = R / 2;
    uint32_t bytes = 0;
    auto move = [&](uint32_t off, const void *src, uint32_t nb) {
        if constexpr (kOp == kCopy) bulk_copy_g2s_hint(stage + off, src, nb, bar, policy);
        if constexpr (kOp == kPrefetch) bulk_prefetch_l2(src, nb);
        bytes += nb;
    };
    if (w.layer == a.nlayers) {
        const int i = w.lo + w.k * R, n = min(R, w.hi - i);
        move(0, (const WT *)a.embed + (size_t)i * kHidden, (uint32_t)n * kRow<WT>);
        return bytes;
    }
    const PersistLayer &Ly = a.layers[w.layer];
    switch (w.phase) {
        case 0: {
            const int items = 2 * (w.hi - w.lo), i0 = w.k * R, n = min(R, items - i0);
            for (int j = 0; j < n; j++) {
                int kind, hl, d;
                move(j * kRow<WT>, qkv_row<WT>(a, Ly, w.lo, i0 + j, kind, hl, d), kRow<WT>);
            }
            break;
        }
        case 1: {
            const float *kb = Ly.kcache + (size_t)w.kvh * a.capacity * kHeadDim;
            const float *vb = Ly.vcache + (size_t)w.kvh * a.capacity * kHeadDim;
            for (int q = 0; q < kConsumerWarps; q++) {
                int r0, r1;
                warp_rows(w.lo, w.hi, w.pw, q, r0, r1);
                const int lo = r0 + kStepRows * w.k, hi = min(min(lo + kStepRows, r1), plan.pos);
                if (hi <= lo) continue;
                const uint32_t off = (uint32_t)(q * kStepRows) * kKvRow, nb = (uint32_t)(hi - lo) * kKvRow;
                move(off, kb + (size_t)lo * kHeadDim, nb);
                move(kVOff + off, vb + (size_t)lo * kHeadDim, nb);
            }
            break;
        }
        case 2: {
            const int i = w.lo + w.k * R, n = min(R, w.hi - i);
            move(0, (const WT *)Ly.wo + (size_t)i * kHidden, (uint32_t)n * kRow<WT>);
            break;
        }
        case 3: {  // H gate rows, then the same H up rows
            const int p = w.lo + w.k * H, n = min(H, w.hi - p);
            move(0, (const WT *)Ly.wg + (size_t)p * kHidden, (uint32_t)n * kRow<WT>);
            move(H * kRow<WT>, (const WT *)Ly.wu + (size_t)p * kHidden, (uint32_t)n * kRow<WT>);
            break;
        }
        default: {
            const int i = w.lo + w.k * RD, n = min(RD, w.hi - i);
            move(0, (const WT *)Ly.wd + (size_t)i * kInter, (uint32_t)n * kDownRow<WT>);
            break;
        }
    }
    return bytes;
}

// The producer: one thread issues every group into the ring, and keeps L2
// prefetches up to `lookahead` bytes ahead of its copies, so HBM keeps
// streaming while the ring is full and the consumers wait at a grid barrier.
// Copies read with an evict-first policy: rows already in shared memory leave
// L2 before the prefetched ones.
template <typename WT>
__device__ __forceinline__ void produce(const PersistArgs &a, const TokenPlan &plan, const Ring &ring,
                                        volatile int *abort_s) {
    unsigned *err = &a.st->fault;
    const uint64_t policy = l2_evict_first_policy();
    const unsigned long long lookahead = a.lookahead;
    Walk w, p;
    walk_begin<WT>(w, a, plan);
    walk_begin<WT>(p, a, plan);
    unsigned long long issued = 0, fetched = 0;
    int gi = 0;
    while (!w.done) {
        while (!p.done && fetched < issued + lookahead) {
            fetched += walk_group<WT, kPrefetch>(p, a, plan, nullptr, nullptr, 0);
            walk_next<WT>(p, a, plan);
        }
        const int s = gi % kPStages;
        if (gi >= kPStages && !wait_phase(&ring.empty[s], ((gi / kPStages) & 1) ^ 1, err, kErrEmptyWait, abort_s)) break;
        if (aborted(abort_s)) break;
        const uint32_t bytes = walk_group<WT, kBytes>(w, a, plan, nullptr, nullptr, 0);
        if (bytes) {
            mbar_expect_tx(&ring.full[s], bytes);
            walk_group<WT, kCopy>(w, a, plan, ring.stage(s), &ring.full[s], policy);
        } else {
            mbar_arrive(&ring.full[s]);
        }
        issued += bytes;
        gi++;
        walk_next<WT>(w, a, plan);
    }
    // Every issued copy lands before the CTA may exit.
    for (int d = gi > kPStages ? gi - kPStages : 0; d < gi; d++)
        if (!mbar_wait(&ring.full[d % kPStages], (d / kPStages) & 1, err, kErrDrain)) break;
}

// ---------------------------------------------------------------- consumers
constexpr int kMaxOut = 16;  // attention outputs one CTA folds in the merge phase
struct ConsumerSmem {
    float *res;      // [2][R]
    float *part_s;   // [2][RD][PIECES]
    float (*wm)[kGroupQ], (*wl)[kGroupQ];
    float (*wacc)[kGroupQ][kHeadDim];  // also the merge phase's staged partials
    float *sv;
    int *si;
    float *nw;       // the next RMSNorm's weights [1536]
    float *bias;     // this CTA's q/k/v biases of the layer [2 * kMaxPairsPerCta]
    float *cs, *sn;  // RoPE cos / sin of the token's position [64]
    float *xo;       // old residual values of this CTA's O or down rows [kMaxOut]
    volatile int *abort_s;
    int *last_s;
};

// Grid-wide barrier k over the consumers of every CTA: a CTA barrier, one
// release-add per CTA, an acquire poll by thread 0. Meanwhile warps 1..7 run
// `pre` (loads of constants the next phase needs; nothing another CTA writes).
template <class Pre>
__device__ __forceinline__ void grid_barrier(DecodeState *st, unsigned target, volatile int *abort_s,
                                             unsigned long long *arrive_mark, unsigned long long *pass_mark, Pre pre) {
    consumers_sync();
    if (threadIdx.x == 0) {
        if (arrive_mark) *arrive_mark = global_ns();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&st->bar) : "memory");
        if (!aborted(abort_s)) {
            const unsigned long long start = global_ns();
            for (;;) {
                unsigned v;
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(&st->bar) : "memory");
                if (v >= target) break;
                if (*(volatile unsigned *)&st->fault) {
                    *abort_s = 1;
                    break;
                }
                if (wait_expired(global_ns() - start)) {
                    atomicOr(&st->fault, kErrGrid);
                    *abort_s = 1;
                    break;
                }
            }
        }
        if (pass_mark) *pass_mark = global_ns();
    } else if (threadIdx.x >= 32) {
        pre((int)threadIdx.x - 32, kConsumerThreads - 32);
    }
    consumers_sync();
}

template <typename WT>
__device__ __forceinline__ void consume(const PersistArgs &a, const TokenPlan &plan, const Ring &ring,
                                        const ConsumerSmem &sm) {
    constexpr int R = Geo<WT>::R, RD = Geo<WT>::RD, E = Geo<WT>::E, H = R / 2;
    constexpr int PIECES = kConsumerWarps / RD;
    constexpr int NVP = kInter / E / PIECES;  // vectors per down-row piece (280)
    constexpr int KV = (NVP + 31) / 32;       // per lane (9)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = warp / PIECES, piece = warp % PIECES;
    volatile int *abort_s = sm.abort_s;
    unsigned *err = &a.st->fault;
    float (*res)[R] = reinterpret_cast<float (*)[R]>(sm.res);
    float (*part_s)[RD][PIECES] = reinterpret_cast<float (*)[RD][PIECES]>(sm.part_s);
    unsigned long long *mark = a.trace ? a.trace + (size_t)blockIdx.x * kPersistMarks : nullptr;
    if (mark && threadIdx.x == 0) mark[0] = global_ns();
    const int token = a.st->token, pos = plan.pos;
    const int pairs = (a.qheads + 2 * a.kvheads) * 64;
    int gi = 0;
    unsigned k = 0;
    // Constants of a phase, loaded by the threads [t, n) in steps of `step`.
    auto stage_vec = [](float *dst, const float *src, int count, int t, int step) {
        for (int i = t; i < count / 4; i += step) reinterpret_cast<float4 *>(dst)[i] = __ldg(reinterpret_cast<const float4 *>(src) + i);
    };
    auto q_consts = [&](int layer, int t, int step) {  // before phase Q of `layer`
        const PersistLayer &Ly = a.layers[layer];
        stage_vec(sm.nw, Ly.in_norm, kHidden, t, step);
        int p0, p1;
        plan.share(pairs, layer, 0, p0, p1);
        for (int i = t; i < 2 * (p1 - p0); i += step) {
            int kind, hl, d;
            qkv_row<WT>(a, Ly, p0, i, kind, hl, d);
            const float *b = kind == 0 ? Ly.bq : kind == 1 ? Ly.bk : Ly.bv;
            sm.bias[i] = __ldg(b + hl * kHeadDim + d);
        }
    };
    auto sync_grid = [&](auto pre) {
        k++;
        grid_barrier(a.st, k * gridDim.x, abort_s, mark ? mark + 2 * k - 1 : nullptr, mark ? mark + 2 * k : nullptr,
                     pre);
    };
    auto no_pre = [](int, int) {};
    auto acquire = [&]() -> bool {
        return wait_phase(&ring.full[gi % kPStages], (gi / kPStages) & 1, err, kErrFullWait, abort_s);
    };
    // The token's RoPE rotation per dimension pair (the per-stage kernel's
    // angle = pos / den, sincosf), and the first layer's constants.
    if (threadIdx.x < kHeadDim / 2) {
        const float angle = __fdiv_rn((float)pos, a.rope_den[threadIdx.x]);
        sincosf(angle, &sm.sn[threadIdx.x], &sm.cs[threadIdx.x]);
    }
    q_consts(0, threadIdx.x, kConsumerThreads);
    consumers_sync();
    float xr[kLaneX];
    for (int layer = 0; layer < a.nlayers; layer++) {
        const PersistLayer &Ly = a.layers[layer];
        {  // ---------------------------------------------------- Q
            int p0, p1;
            plan.share(pairs, layer, 0, p0, p1);
            const int items = 2 * (p1 - p0);
            if (layer == 0) {
                load_lane_row<WT>(xr, (const WT *)a.embed + (size_t)token * kHidden, lane);
                if (blockIdx.x == 0 && warp == 0) store_lane_vec<WT>(a.x, xr, lane);
            } else {
                load_lane_vec<WT, true>(xr, a.x, lane);
            }
            rms_lane<WT>(xr, sm.nw, a.eps, lane);
            for (int i0 = 0; i0 < items; i0 += R, gi++) {
                const int n = min(R, items - i0);
                if (acquire()) {
                    const unsigned char *stage = ring.stage(gi % kPStages);
#pragma unroll
                    for (int m = 0; m < R / kConsumerWarps; m++) {
                        const int j = warp + kConsumerWarps * m;
                        if (j < n) {
                            const float y = row_dot<WT>(stage + (size_t)j * kRow<WT>, xr, lane);
                            if (lane == 0) res[gi & 1][j] = y;
                        }
                    }
                }
                ring_release(ring, gi);
                consumers_sync();
                if (!aborted(abort_s) && (int)threadIdx.x < n / 2) {
                    const int t = threadIdx.x, i = i0 + 2 * t;
                    int kind, hl, d;
                    qkv_row<WT>(a, Ly, p0, i, kind, hl, d);
                    float y0 = __fadd_rn(res[gi & 1][2 * t], sm.bias[i]);
                    float y1 = __fadd_rn(res[gi & 1][2 * t + 1], sm.bias[i + 1]);
                    if (kind < 2) {
                        const float cs = sm.cs[d], sn = sm.sn[d];
                        const float r0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                        const float r1 = __fadd_rn(__fmul_rn(y1, cs), __fmul_rn(y0, sn));
                        y0 = r0;
                        y1 = r1;
                    }
                    float *dst = kind == 0 ? a.q : kind == 1 ? a.k : a.v;
                    dst[hl * kHeadDim + d] = y0;
                    dst[hl * kHeadDim + d + 64] = y1;
                    float *cache = kind == 1 ? Ly.kcache : kind == 2 ? Ly.vcache : nullptr;
                    if (cache && pos >= 0 && pos < a.capacity) {
                        float *row = cache + ((size_t)hl * a.capacity + pos) * kHeadDim;
                        row[d] = y0;
                        row[d + 64] = y1;
                    }
                }
            }
        }
        sync_grid(no_pre);
        {  // ---------------------------------------------------- A
            int kvh, hc, t0, t1, pw;
            if (plan.attention(layer, a.kvheads, kvh, hc, t0, t1, pw)) {
                const float *kb = Ly.kcache + (size_t)kvh * a.capacity * kHeadDim;
                const float *vb = Ly.vcache + (size_t)kvh * a.capacity * kHeadDim;
                float4 q4[kGroupQ], acc[kGroupQ];
                int r0, r1;
                warp_rows(t0, t1, pw, warp, r0, r1);
                // The newest row (appended in phase Q) is read together with q.
                float4 kcur = make_float4(0.f, 0.f, 0.f, 0.f), vcur = kcur;
                if (pos >= r0 && pos < r1) {
                    kcur = __ldcg(reinterpret_cast<const float4 *>(kb + (size_t)pos * kHeadDim) + lane);
                    vcur = __ldcg(reinterpret_cast<const float4 *>(vb + (size_t)pos * kHeadDim) + lane);
                }
#pragma unroll
                for (int g = 0; g < kGroupQ; g++) {
                    q4[g] = __ldcg(reinterpret_cast<const float4 *>(a.q + ((size_t)kvh * kGroupQ + g) * kHeadDim) + lane);
                    acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
                float m_run = -INFINITY, l_run = 0.f;
                const int steps = (pw + kStepRows - 1) / kStepRows;
                for (int s = 0; s < steps; s++, gi++) {
                    const bool ok = acquire();
                    const int t = r0 + kStepRows * s;
                    if (ok && t < r1) {
                        const unsigned char *stage = ring.stage(gi % kPStages);
                        float4 k4[kStepRows], v4[kStepRows];
#pragma unroll
                        for (int i = 0; i < kStepRows; i++) {
                            const int row = t + i;
                            if (row < r1 && row < pos) {
                                const uint32_t off = (uint32_t)(warp * kStepRows + i) * kKvRow;
                                k4[i] = reinterpret_cast<const float4 *>(stage + off)[lane];
                                v4[i] = reinterpret_cast<const float4 *>(stage + kVOff + off)[lane];
                            } else if (row < r1) {  // row == pos
                                k4[i] = kcur;
                                v4[i] = vcur;
                            } else {
                                k4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                                v4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                            }
                        }
                        flash_step<kGroupQ, false>(q4, k4, v4, r1 - t, lane, a.inv_sqrt_dim, [](int) { return 0.f; },
                                                   m_run, l_run, acc);
                    }
                    ring_release(ring, gi);
                }
                float m[kGroupQ], l[kGroupQ];
#pragma unroll
                for (int g = 0; g < kGroupQ; g++) {
                    m[g] = __shfl_sync(0xffffffffu, m_run, g);
                    l[g] = __shfl_sync(0xffffffffu, l_run, g);
                }
                cta_merge<kGroupQ>(m, l, acc, sm.wm, sm.wl, sm.wacc,
                                   a.part + ((size_t)kvh * plan.per_head + hc) * kAttnPartialFloats, nullptr,
                                   [] { consumers_sync(); });
            }
        }
        sync_grid(no_pre);
        {  // ---------------------------------------------------- M
            int o0, o1;
            plan.share(a.kvheads * kGroupQ * kHeadDim, layer, 2, o0, o1);
            const int nout = o1 - o0, C = plan.per_head;
            // Stage every partial value this CTA's outputs fold (parallel L2
            // loads), then fold each output in the cluster kernel's order.
            float *pm = &sm.wacc[0][0][0], *pl = pm + kMaxOut * kPersistAttnCtasPerHead, *pa = pl + kMaxOut * kPersistAttnCtasPerHead;
            {
                // All loads in flight before the first store.
                constexpr int kPer = (kMaxOut * kPersistAttnCtasPerHead + kConsumerThreads - 1) / kConsumerThreads;
                float vm[kPer], vl[kPer], va[kPer];
#pragma unroll
                for (int u = 0; u < kPer; u++) {
                    const int idx = threadIdx.x + u * kConsumerThreads;
                    vm[u] = vl[u] = va[u] = 0.f;
                    if (idx < nout * C) {
                        const int j = idx / C, r = idx - j * C, o = o0 + j;
                        const int kvh = o / (kGroupQ * kHeadDim), g = (o / kHeadDim) % kGroupQ, d = o % kHeadDim;
                        const float *pr = a.part + ((size_t)kvh * C + r) * kAttnPartialFloats;
                        vm[u] = __ldcg(pr + g);
                        vl[u] = __ldcg(pr + kAttnMaxGroup + g);
                        va[u] = __ldcg(pr + 2 * kAttnMaxGroup + g * kHeadDim + d);
                    }
                }
#pragma unroll
                for (int u = 0; u < kPer; u++) {
                    const int idx = threadIdx.x + u * kConsumerThreads;
                    if (idx < nout * C) {
                        pm[idx] = vm[u];
                        pl[idx] = vl[u];
                        pa[idx] = va[u];
                    }
                }
            }
            consumers_sync();
            if ((int)threadIdx.x < nout && !aborted(abort_s)) {
                const int j = threadIdx.x;
                // One cluster's 16 partials folded in rank order (the cluster kernel's DSMEM fold).
                auto fold = [&](int c0, float &M, float &num, float &den) {
                    const float *mr = pm + j * C + c0, *lr = pl + j * C + c0, *ar = pa + j * C + c0;
                    M = -INFINITY;
#pragma unroll
                    for (int r = 0; r < kCluster; r++) M = fmaxf(M, mr[r]);
                    num = 0.f;
                    den = 0.f;
#pragma unroll
                    for (int r = 0; r < kCluster; r++) {
                        if (mr[r] == -INFINITY) continue;
                        const float e = expf(mr[r] - M);
                        den = fmaf(e, lr[r], den);
                        num = fmaf(e, ar[r], num);
                    }
                };
                float out;
                if (!plan.multi) {
                    float M, num, den;
                    fold(0, M, num, den);
                    out = __fdiv_rn(num, den);
                } else {
                    // The clusters' results folded in cluster order (the cluster
                    // kernel's last-CTA merge).
                    float mc[kClustersPerHead], lc[kClustersPerHead], ac[kClustersPerHead];
#pragma unroll
                    for (int c = 0; c < kClustersPerHead; c++) fold(c * kCluster, mc[c], ac[c], lc[c]);
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
                    out = __fdiv_rn(num, den);
                }
                a.attn[o0 + j] = out;
            }
        }
        int r0o, r1o;
        plan.share(kHidden, layer, 3, r0o, r1o);
        sync_grid([&](int t, int step) {  // the O rows' residual values (last written before the previous barrier)
            for (int i = t; i < r1o - r0o; i += step) sm.xo[i] = __ldcg(a.x + r0o + i);
        });
        {  // ---------------------------------------------------- O
            load_lane_vec<WT, true>(xr, a.attn, lane);
            for (int i = r0o; i < r1o; i += R, gi++) {
                const int n = min(R, r1o - i);
                if (acquire()) {
                    const unsigned char *stage = ring.stage(gi % kPStages);
#pragma unroll
                    for (int m = 0; m < R / kConsumerWarps; m++) {
                        const int j = warp + kConsumerWarps * m;
                        if (j < n) {
                            const float y = row_dot<WT>(stage + (size_t)j * kRow<WT>, xr, lane);
                            if (lane == 0) a.x[i + j] = __fadd_rn(sm.xo[i + j - r0o], y);
                        }
                    }
                }
                ring_release(ring, gi);
            }
        }
        sync_grid([&](int t, int step) { stage_vec(sm.nw, Ly.post_norm, kHidden, t, step); });
        {  // ---------------------------------------------------- G
            int q0, q1;
            plan.share(kInter, layer, 4, q0, q1);
            load_lane_vec<WT, true>(xr, a.x, lane);
            rms_lane<WT>(xr, sm.nw, a.eps, lane);
            for (int p = q0; p < q1; p += H, gi++) {
                const int n = min(H, q1 - p);
                if (acquire()) {
                    const unsigned char *stage = ring.stage(gi % kPStages);
#pragma unroll
                    for (int m = 0; m < R / kConsumerWarps; m++) {
                        const int j = warp + kConsumerWarps * m;
                        if (j % H < n) {
                            const float y = row_dot<WT>(stage + (size_t)j * kRow<WT>, xr, lane);
                            if (lane == 0) res[gi & 1][j] = y;
                        }
                    }
                }
                ring_release(ring, gi);
                consumers_sync();
                if (!aborted(abort_s) && (int)threadIdx.x < n) {
                    const int t = threadIdx.x;
                    const float gv = res[gi & 1][t], uv = res[gi & 1][H + t];
                    a.h[p + t] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.f, expf(-gv))), uv);
                }
            }
        }
        int r0d, r1d;
        plan.share(kHidden, layer, 5, r0d, r1d);
        sync_grid([&](int t, int step) {  // the down rows' residual values (written in phase O)
            for (int i = t; i < r1d - r0d; i += step) sm.xo[i] = __ldcg(a.x + r0d + i);
        });
        {  // ---------------------------------------------------- D
            float hr[KV * E];
#pragma unroll
            for (int kk = 0; kk < KV; kk++) {
                const int v = piece * NVP + lane + 32 * kk;
#pragma unroll
                for (int e = 0; e < E; e += 4) {
                    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (lane + 32 * kk < NVP) f = __ldcg(reinterpret_cast<const float4 *>(a.h) + (E * v + e) / 4);
                    hr[E * kk + e] = f.x;
                    hr[E * kk + e + 1] = f.y;
                    hr[E * kk + e + 2] = f.z;
                    hr[E * kk + e + 3] = f.w;
                }
            }
            for (int i = r0d; i < r1d; i += RD, gi++) {
                const int n = min(RD, r1d - i);
                if (acquire() && slot < n) {
                    const uint4 *row =
                        reinterpret_cast<const uint4 *>(ring.stage(gi % kPStages) + (size_t)slot * kDownRow<WT>);
                    float acc = 0.f;
#pragma unroll
                    for (int kk = 0; kk < KV; kk++)
                        if (lane + 32 * kk < NVP) acc = dot_vec(row[piece * NVP + lane + 32 * kk], &hr[E * kk], acc, WT());
                    acc = warp_sum(acc);
                    if (lane == 0) part_s[gi & 1][slot][piece] = acc;
                }
                ring_release(ring, gi);
                consumers_sync();
                if (!aborted(abort_s) && (int)threadIdx.x < n) {
                    const int s = threadIdx.x;
                    float sum = part_s[gi & 1][s][0];
#pragma unroll
                    for (int p = 1; p < PIECES; p++) sum = __fadd_rn(sum, part_s[gi & 1][s][p]);
                    a.x[i + s] = __fadd_rn(sm.xo[i + s - r0d], sum);
                }
            }
        }
        if (layer + 1 < a.nlayers) sync_grid([&](int t, int step) { q_consts(layer + 1, t, step); });
        else sync_grid([&](int t, int step) { stage_vec(sm.nw, a.final_norm, kHidden, t, step); });
    }
    // -------------------------------------------------------- readout + greedy top-2
    int v0, v1;
    plan.share(a.vocab, a.nlayers, 0, v0, v1);
    load_lane_vec<WT, true>(xr, a.x, lane);
    rms_lane<WT>(xr, sm.nw, a.eps, lane);
    Top2 t = top2_empty();
    bool bad = false;
    for (int i = v0; i < v1; i += R, gi++) {
        const int n = min(R, v1 - i);
        if (acquire()) {
            const unsigned char *stage = ring.stage(gi % kPStages);
#pragma unroll
            for (int m = 0; m < R / kConsumerWarps; m++) {
                const int j = warp + kConsumerWarps * m;
                if (j < n) {
                    const int row = i + j;
                    const float y = row_dot<WT>(stage + (size_t)j * kRow<WT>, xr, lane);
                    if (lane == 0) a.logits[row] = y;
                    bad |= !isfinite(y);
                    top2_insert(t, y, row);
                }
            }
        }
        ring_release(ring, gi);
    }
    if (mark && threadIdx.x == 0) mark[2 * k + 1] = global_ns();
    // Warp results (identical in every lane) -> CTA result -> the last CTA merges.
    DecodeState *st = a.st;
    if (lane == 0) {
        sm.sv[2 * warp] = t.a; sm.sv[2 * warp + 1] = t.b;
        sm.si[2 * warp] = t.ai; sm.si[2 * warp + 1] = t.bi;
        if (bad) atomicOr(&st->nonfinite, 1u);
    }
    consumers_sync();
    if (warp == 0) {
        Top2 u = top2_empty();
        if (lane < kConsumerWarps) {
            top2_insert(u, sm.sv[2 * lane], sm.si[2 * lane]);
            top2_insert(u, sm.sv[2 * lane + 1], sm.si[2 * lane + 1]);
        }
        top2_merge_warp(u);
        if (lane == 0) {
            a.pv[2 * blockIdx.x] = u.a; a.pv[2 * blockIdx.x + 1] = u.b;
            a.pi[2 * blockIdx.x] = u.ai; a.pi[2 * blockIdx.x + 1] = u.bi;
            __threadfence();
            *sm.last_s = atomicAdd(&st->arrive, 1u) == gridDim.x - 1;
        }
    }
    consumers_sync();
    if (!*sm.last_s) return;
    __threadfence();
    Top2 u = top2_empty();
    for (int i = threadIdx.x; i < 2 * (int)gridDim.x; i += kConsumerThreads) top2_insert(u, __ldcg(a.pv + i), __ldcg(a.pi + i));
    top2_merge_warp(u);
    if (lane == 0) {
        sm.sv[2 * warp] = u.a; sm.sv[2 * warp + 1] = u.b;
        sm.si[2 * warp] = u.ai; sm.si[2 * warp + 1] = u.bi;
    }
    consumers_sync();
    if (warp == 0) {
        Top2 z = top2_empty();
        if (lane < kConsumerWarps) {
            top2_insert(z, sm.sv[2 * lane], sm.si[2 * lane]);
            top2_insert(z, sm.sv[2 * lane + 1], sm.si[2 * lane + 1]);
        }
        top2_merge_warp(z);
        if (lane == 0) {
            const unsigned flag = atomicExch(&st->nonfinite, 0u);
            TcmTop2 top;
            top.first = z.ai; top.second = z.bi; top.first_value = z.a; top.second_value = z.b;
            st->top = top;
            st->invalid |= (int)flag;
            a.log[st->step % kLogCap] = top;
            st->step += 1;
            st->token = z.ai;
            st->position += 1;
            // Every CTA has passed its last grid barrier (it arrived above).
            st->bar = 0u;
            st->arrive = 0u;
        }
    }
}

template <typename WT>
__global__ void __launch_bounds__(kStreamThreads, 1) token_kernel(PersistArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int R = Geo<WT>::R, RD = Geo<WT>::RD;
    __shared__ float res[2 * R];
    __shared__ float part_s[2 * kConsumerWarps];
    __shared__ float wm[kConsumerWarps][kGroupQ], wl[kConsumerWarps][kGroupQ];
    __shared__ __align__(16) float wacc[kConsumerWarps][kGroupQ][kHeadDim];
    __shared__ __align__(16) float nw[kHidden];
    __shared__ float bias[2 * kMaxPairsPerCta];
    __shared__ float cs[kHeadDim / 2], sn[kHeadDim / 2];
    __shared__ float xo[kMaxOut];
    __shared__ float sv[2 * kConsumerWarps];
    __shared__ int si[2 * kConsumerWarps];
    __shared__ int abort_s, last_s;
    static_assert(2 * RD * (kConsumerWarps / RD) <= 2 * kConsumerWarps, "down partial buffer");
    static_assert(3 * kMaxOut * kPersistAttnCtasPerHead <= kConsumerWarps * kGroupQ * kHeadDim, "merge staging");
    static_assert(kPersistAttnCtasPerHead == kCluster * kClustersPerHead, "attention split");
    if (threadIdx.x == 0) abort_s = 0;
    const Ring ring = ring_setup(smem, kPStages, kPStage);
    TokenPlan plan;
    plan.grid = gridDim.x;
    plan.cta = blockIdx.x;
    plan.pos = a.st->position;
    plan.rows = min(plan.pos + 1, a.capacity);
    plan.multi = plan.rows > kSingleClusterRows;
    plan.per_head = plan.multi ? kCluster * kClustersPerHead : kCluster;
    if (threadIdx.x >= kConsumerThreads) {
        if (threadIdx.x == kConsumerThreads) produce<WT>(a, plan, ring, &abort_s);
        return;
    }
    ConsumerSmem sm = {res, part_s, wm, wl, wacc, sv, si, nw, bias, cs, sn, xo, &abort_s, &last_s};
    consume<WT>(a, plan, ring, sm);
}

size_t token_smem() { return ring_smem_bytes(kPStages, kPStage); }

template <typename WT> int setup_typed() {
    TCM_CUDA(cudaFuncSetAttribute(token_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)token_smem()));
    int n = 0;
    TCM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, token_kernel<WT>, kStreamThreads, token_smem()));
    return n;
}

}  // namespace

void set_wait_limit_persistent(unsigned long long ns) { set_module_wait_limit(ns); }

int persistent_blocks_per_sm(int dtype) {
    static PerDeviceOnce once;
    static int fits[64][2];
    int dev = 0;
    TCM_CUDA(cudaGetDevice(&dev));
    once.run([dev] {
        fits[dev][0] = setup_typed<float>();
        fits[dev][1] = setup_typed<uint16_t>();
    });
    return fits[dev][dtype == 2 ? 1 : 0];
}

void launch_persistent(int dtype, const PersistArgs &a, int grid, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kStreamThreads);
    cfg.dynamicSmemBytes = token_smem();
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (dtype == 2) TCM_CUDA(cudaLaunchKernelEx(&cfg, token_kernel<uint16_t>, a));
    else TCM_CUDA(cudaLaunchKernelEx(&cfg, token_kernel<float>, a));
}

}  // namespace tcm
