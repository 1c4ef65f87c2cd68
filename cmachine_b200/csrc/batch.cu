// Batched decode of independent sessions (sm_100a): one token for each of up
// to 64 sessions per step, sharing one pass over the BF16 weights.
//
// Per layer (reference equations src/qwen.c:248-262,275,289,320,329-330,341,
// applied to every session at its own position):
//   batch_rms_kernel     RMSNorm of each session's x -> BF16 hi/lo rows
//   tc_gemm (EpiQkv)     q/k/v = W x (+ bias, RoPE) on the tensor cores; q to
//                        the batch buffer, k and v appended to each session's
//                        own FP32 cache at its position
//   batch_attn_kernel    split-K flash-decoding over each session's cache
//                        (256 rows a CTA), last CTA per (session, KV head)
//                        folds the slices in order -> BF16 hi/lo rows
//   tc_gemm (EpiResid)   x += O attn
//   batch_rms_kernel     post-attention RMSNorm
//   tc_gemm (EpiSwiglu)  gate/up tiles interleaved 64 + 64 rows, SwiGLU in the
//                        epilogue -> BF16 hi/lo rows of the 8960-wide h
//   tc_gemm (EpiResid)   x += down h
// then the final RMSNorm, the tied-embedding readout on the tensor cores with
// per-tile top-2 (EpiLogits), and batch_top2_kernel (top-2 per session, finite
// check, greedy token feed). A step is captured once into a CUDA graph per
// batch size and replayed; positions, tokens and cache pointers live in a
// device-resident state block.
#include "common.cuh"
#include "attention.cuh"
#include "attention_decode.cuh"
#include "tc_gemm.cuh"
#include "stream.cuh"
#include "kernels.h"
#include "../../include/qwen_b200.h"
#include "../../include/tcm_seeded.h"
#include <cuda.h>
#include <map>
#include <mutex>
#include <vector>

namespace tcm {
namespace {

constexpr int kBN = 64;             // sessions per step (the tensor-core tile's N)
constexpr int kHd = 1536, kFf = 8960;
constexpr int kAttnChunk = 256;     // cache rows per attention CTA
constexpr int kAttnSplitMax = 36;   // up to 9216 cached rows
constexpr int kBatchLogCap = 256;   // steps of top-2 kept for chained decode

// Device-resident batch state: the host writes it before a step; the top-2
// kernel advances token and position for chained greedy steps.
struct BatchState {
    int token[kBN], position[kBN], capacity[kBN];
    float *keys[kBN], *values[kBN], *logits[kBN], *x[kBN];
    int n, step;
    int bad[kBN];       // non-finite logits seen for the session
    unsigned err;       // pipeline wait bits
};

// y = hi + lo + O(2^-17 |y|): both halves round to nearest even.
__device__ __forceinline__ void split_bf16(float y, uint16_t &hi, uint16_t &lo) {
    hi = tcm_bf16_rne(y);
    lo = tcm_bf16_rne(__fsub_rn(y, __uint_as_float((uint32_t)hi << 16)));
}

// ---------------------------------------------------------------- RMSNorm
struct RmsArgs {
    BatchState *st;
    float *x;                 // [kBN][1536] residual stream
    const float *w;           // norm weights (FP32)
    uint16_t *hi, *lo;        // [kBN][1536]
    const uint16_t *embed;    // layer 0: x <- E[token] first
    float eps;
    int copy_x;               // final norm: also copy x to the session's buffer
    const float *part;        // or the residual GEMM's deferred K-split partials: x += their sum first
};
// K splits of a residual GEMM (O, down) whose partials the next RMSNorm sums:
// 12 tiles x 12 splits = 144 CTAs, one wave on 148 SMs.
constexpr int kResidSplits = 12;
constexpr int kRmsThreads = kHd / 4;  // 384: four consecutive elements of x a thread
__global__ void __launch_bounds__(kRmsThreads, 1) batch_rms_kernel(RmsArgs a) {
    __shared__ float red[kRmsThreads / 32];
    const int n = blockIdx.x, tid = threadIdx.x, j0 = 4 * tid;
    float w[4];  // norm weights: constants, read before the dependency wait
#pragma unroll
    for (int c = 0; c < 4; c++) w[c] = a.w[j0 + c];
    pdl_trigger();
    pdl_wait();
    if (n >= a.st->n) return;
    float v[4];
    float *x = a.x + (size_t)n * kHd + j0;
    if (a.embed) {
        const uint2 e = *reinterpret_cast<const uint2 *>(a.embed + (size_t)a.st->token[n] * kHd + j0);  // 4 BF16
        v[0] = __uint_as_float(e.x << 16);
        v[1] = __uint_as_float(e.x & 0xffff0000u);
        v[2] = __uint_as_float(e.y << 16);
        v[3] = __uint_as_float(e.y & 0xffff0000u);
        *reinterpret_cast<float4 *>(x) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        const float4 t = *reinterpret_cast<const float4 *>(x);
        v[0] = t.x;
        v[1] = t.y;
        v[2] = t.z;
        v[3] = t.w;
    }
    if (a.part) {
        // x += the residual GEMM's output, as its K-split partials summed in
        // split order (partial layout [tile][split][session][128]); the 12
        // 16-byte loads are issued before the sums.
        const float *src = a.part + ((size_t)(j0 >> 7) * kResidSplits * kBN + n) * 128 + (j0 & 127);
        float p[kResidSplits][4];
#pragma unroll
        for (int sp = 0; sp < kResidSplits; sp++)  // volatile: kept ahead of every sum below
            asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(p[sp][0]), "=f"(p[sp][1]), "=f"(p[sp][2]), "=f"(p[sp][3])
                         : "l"(src + (size_t)sp * kBN * 128));
#pragma unroll
        for (int c = 0; c < 4; c++) {
            float sum = 0.f;
#pragma unroll
            for (int sp = 0; sp < kResidSplits; sp++)  // volatile: not hoisted between the loads
                asm volatile("add.rn.f32 %0, %0, %1;" : "+f"(sum) : "f"(p[sp][c]));
            v[c] = __fadd_rn(v[c], sum);
        }
        *reinterpret_cast<float4 *>(x) = make_float4(v[0], v[1], v[2], v[3]);
    }
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < 4; c++) ss = fmaf(v[c], v[c], ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int k = 0; k < kRmsThreads / 32; k++) total += red[k];
    const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)kHd), a.eps)));
    uint16_t h[4], l[4];
#pragma unroll
    for (int c = 0; c < 4; c++) split_bf16(__fmul_rn(__fmul_rn(v[c], r), w[c]), h[c], l[c]);
    *reinterpret_cast<uint2 *>(a.hi + (size_t)n * kHd + j0) =
        make_uint2((uint32_t)h[0] | ((uint32_t)h[1] << 16), (uint32_t)h[2] | ((uint32_t)h[3] << 16));
    *reinterpret_cast<uint2 *>(a.lo + (size_t)n * kHd + j0) =
        make_uint2((uint32_t)l[0] | ((uint32_t)l[1] << 16), (uint32_t)l[2] | ((uint32_t)l[3] << 16));
    if (a.copy_x)  // the caller's buffer: no alignment assumed
#pragma unroll
        for (int c = 0; c < 4; c++) a.st->x[n][j0 + c] = v[c];
}

// ---------------------------------------------------------------- GEMM epilogues
// q/k/v: tiles 0..11 are the 12 query heads, 12..13 the K heads, 14..15 the V
// heads; a head is exactly one 128-row tile, so RoPE pairs (d, d + 64) meet in
// the tile. The rotation repeats the single-session kernel's arithmetic.
// Per-session metadata the epilogues read, staged once per CTA.
struct SessionMeta {
    float *keys, *values, *logits;
    int position, capacity;
};
__device__ __forceinline__ void stage_meta(const BatchState *st, unsigned char *scratch, int e) {
    SessionMeta *m = reinterpret_cast<SessionMeta *>(scratch);
    for (int n = e; n < st->n; n += kTcEpiThreads)
        m[n] = SessionMeta{st->keys[n], st->values[n], st->logits[n], st->position[n], st->capacity[n]};
}
static_assert(sizeof(SessionMeta) * kBN <= 2048, "epilogue scratch");

struct EpiQkv {
    BatchState *st;
    const float *bq, *bk, *bv, *rope_den;
    float *q;       // [kBN][1536]
    int layer;
    __device__ TcRows a_rows(int t) const {
        const int m = t < 12 ? 0 : (t < 14 ? 1 : 2), r = (t < 12 ? t : (t < 14 ? t - 12 : t - 14)) * 128;
        return TcRows{m, r, m, r + 64};
    }
    __device__ void init(unsigned char *scratch, int e) const { stage_meta(st, scratch, e); }
    // Row pairs (d, d + 64) for d in [p0, p1), every session; consecutive threads
    // take consecutive d.
    template <int NP>
    __device__ void store(int t, const float (*tile)[NP], int p0, int p1, int e, unsigned char *scratch) const {
        const SessionMeta *meta = reinterpret_cast<const SessionMeta *>(scratch);
        const int kind = t < 12 ? 0 : (t < 14 ? 1 : 2), head = t < 12 ? t : (t < 14 ? t - 12 : t - 14);
        const float *bias = (kind == 0 ? bq : kind == 1 ? bk : bv) + head * 128;
        const int np = p1 - p0, n_active = st->n;
        for (int idx = e; idx < np * n_active; idx += kTcEpiThreads) {
            const int d = p0 + idx % np, n = idx / np;
            float y0 = __fadd_rn(tile[d][n], bias[d]), y1 = __fadd_rn(tile[d + 64][n], bias[d + 64]);
            const SessionMeta &mt = meta[n];
            if (kind < 2) {
                const float angle = __fdiv_rn((float)mt.position, rope_den[d]);
                float sn, cs;
                sincosf(angle, &sn, &cs);
                const float r0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                const float r1 = __fadd_rn(__fmul_rn(y1, cs), __fmul_rn(y0, sn));
                y0 = r0;
                y1 = r1;
            }
            if (kind == 0) {
                q[(size_t)n * kHd + head * 128 + d] = y0;
                q[(size_t)n * kHd + head * 128 + d + 64] = y1;
            } else {
                float *cache = (kind == 1 ? mt.keys : mt.values) + ((size_t)layer * 2 + head) * mt.capacity * 128 +
                               (size_t)mt.position * 128;
                cache[d] = y0;
                cache[d + 64] = y1;
            }
        }
    }
};
// Rows {p, p + 64 : p in [p0, p1)} of an output tile as (row, session) items:
// item i is row rows[i % 2np], session i / 2np.
__device__ __forceinline__ int pair_row(int i, int p0, int np) {
    const int k = i % (2 * np);
    return k < np ? p0 + k : 64 + p0 + (k - np);
}

// x += D (the O and down projections): tile rows are output rows t*128 ...
// The loads of a group of items are issued together, then the sums stored.
struct EpiResid {
    BatchState *st;
    float *x;
    __device__ TcRows a_rows(int t) const { return TcRows{0, t * 128, 0, t * 128 + 64}; }
    __device__ void init(unsigned char *, int) const {}
    template <int NP>
    __device__ void store(int t, const float (*tile)[NP], int p0, int p1, int e, unsigned char *) const {
        const int np = p1 - p0, total = 2 * np * st->n;
        for (int base = 0; base < total; base += kTcEpiThreads * 8) {
            float xv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int i = base + e + kTcEpiThreads * j;
                xv[j] = i < total ? x[(size_t)(i / (2 * np)) * kHd + t * 128 + pair_row(i, p0, np)] : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int i = base + e + kTcEpiThreads * j;
                if (i < total) {
                    const int r = pair_row(i, p0, np), n = i / (2 * np);
                    x[(size_t)n * kHd + t * 128 + r] = __fadd_rn(xv[j], tile[r][n]);
                }
            }
        }
    }
};
// gate rows t*64.. in tile rows 0..63, up rows t*64.. in 64..127; h = silu(g) u
// as g / (1 + exp(-g)) * u (src/qwen_cuda.cu:79), stored as BF16 hi/lo.
struct EpiSwiglu {
    BatchState *st;
    uint16_t *hh, *hl;   // [kBN][8960]
    __device__ TcRows a_rows(int t) const { return TcRows{0, t * 64, 1, t * 64}; }
    __device__ void init(unsigned char *, int) const {}
    template <int NP>
    __device__ void store(int t, const float (*tile)[NP], int p0, int p1, int e, unsigned char *) const {
        const int np = p1 - p0, n_active = st->n;
        for (int idx = e; idx < np * n_active; idx += kTcEpiThreads) {
            const int i = p0 + idx % np, n = idx / np;
            const float g = tile[i][n], u = tile[i + 64][n];
            const float h = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
            uint16_t hi, lo;
            split_bf16(h, hi, lo);
            hh[(size_t)n * kFf + t * 64 + i] = hi;
            hl[(size_t)n * kFf + t * 64 + i] = lo;
        }
    }
};
// Logits to each session's buffer (the top-2 is taken from them afterwards).
struct EpiLogits {
    BatchState *st;
    __device__ TcRows a_rows(int t) const { return TcRows{0, t * 128, 0, t * 128 + 64}; }
    __device__ void init(unsigned char *scratch, int e) const { stage_meta(st, scratch, e); }
    template <int NP>
    __device__ void store(int t, const float (*tile)[NP], int p0, int p1, int e, unsigned char *scratch) const {
        const SessionMeta *meta = reinterpret_cast<const SessionMeta *>(scratch);
        const int np = p1 - p0, total = 2 * np * st->n;
        for (int i = e; i < total; i += kTcEpiThreads) {
            const int r = pair_row(i, p0, np), n = i / (2 * np);
            meta[n].logits[t * 128 + r] = tile[r][n];
        }
    }
};

// y[n][t*128 + r] = D (the plain batched matmul).
struct EpiStore {
    float *y;
    int rows, n;
    __device__ TcRows a_rows(int t) const { return TcRows{0, t * 128, 0, t * 128 + 64}; }
    __device__ void init(unsigned char *, int) const {}
    template <int NP>
    __device__ void store(int t, const float (*tile)[NP], int p0, int p1, int e, unsigned char *) const {
        const int np = p1 - p0, total = 2 * np * n;
        for (int i = e; i < total; i += kTcEpiThreads) {
            const int r = pair_row(i, p0, np), c = i / (2 * np);
            y[(size_t)c * rows + t * 128 + r] = tile[r][c];
        }
    }
};
__global__ void split_rows_kernel(const float *x, uint16_t *hi, uint16_t *lo, size_t count) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        uint16_t h, l;
        split_bf16(x[i], h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

// ---------------------------------------------------------------- attention
// Work items are (session n, KV head h, chunk c of kAttnItemRows cache rows),
// numbered session by session; a persistent grid of one CTA per SM takes items
// blockIdx.x, blockIdx.x + gridDim.x, ... Per CTA one producer thread streams
// each chunk's K and V rows (contiguous in the session's [head][capacity][128]
// slab) into a ring of shared-memory stages with cp.async.bulk, 32 rows of K
// and 32 of V a stage; every consumer warp takes four rows of each stage as
// one flash-decoding step. At the end of an item the eight warps' states merge
// into a partial in global memory; the last CTA of the (session, head) to
// arrive folds the partials in chunk order and writes the output rows as BF16
// hi/lo for the O projection.
constexpr int kAttnRowsPerStage = 32;                  // 8 warps x 4 rows
constexpr int kAttnStageBytes = 2 * kAttnRowsPerStage * kHeadDim * 4;  // K and V: 32 KB
constexpr int kAttnRingStages = 6;
constexpr int kAttnItemRowsMin = 256;   // item sizes are multiples of 32 rows in [256, 2048]
constexpr int kAttnItemMax = (kAttnSplitMax * kAttnChunk) / kAttnItemRowsMin;  // chunks per (session, head)
constexpr size_t kAttnSmem = ring_smem_bytes(kAttnRingStages, kAttnStageBytes);

struct AttnArgs {
    BatchState *st;
    const float *q;        // [kBN][1536]
    int layer;
    float inv_sqrt_dim;
    float *part;           // [kBN][2][kAttnItemMax][kAttnPartialFloats]
    unsigned *counters;    // [kBN][2]
    uint16_t *oh, *ol;     // [kBN][1536]
    unsigned long long *trace;  // per CTA: 0 entry, 1 consumers released, 2 first stage ready, 3 last item done
    unsigned *work;        // [0] next item, [1] CTAs done (reset by the last CTA)
    int item_rows;         // cache rows per work item
};

// One flash-decoding step of a warp over `nrows` (<= 4) rows held in k4/v4 for
// three query heads (q4): the 4 rows x 4 padded heads = 16 partial dots are
// reduced by a reduce-scatter over lane bits 3..0 and one fold over bit 4, so
// lane (row (lane & 15) / 4, head lane & 3) holds a full score; the running
// max and sum of head g live in the lanes with lane & 3 == g. Scores are kept
// in base 2 (scale = log2(e) / sqrt(128)) so the softmax uses exp2; arithmetic
// on pairs of dimensions uses the packed FP32x2 FMA.
__device__ __forceinline__ void flash_step3(const float4 (&q4)[3], const float4 (&k4)[4], const float4 (&v4)[4],
                                            int nrows, int lane, float scale2, float &m_run, float &l_run,
                                            float4 (&acc)[3]) {
    float v[16];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int g = 0; g < 4; g++) {
            if (g < 3) {
                float2 d = __fmul2_rn(make_float2(q4[g].x, q4[g].y), make_float2(k4[i].x, k4[i].y));
                d = __ffma2_rn(make_float2(q4[g].z, q4[g].w), make_float2(k4[i].z, k4[i].w), d);
                v[4 * i + g] = d.x + d.y;
            } else {
                v[4 * i + g] = 0.f;
            }
        }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        const bool upper = (lane & o) != 0;
#pragma unroll
        for (int j = 0; j < o; j++) {
            const float send = upper ? v[j] : v[j + o];
            const float keep = upper ? v[j + o] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    const float dot = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 16);
    const int my_row = (lane & 15) >> 2, my_head = lane & 3;
    const float sc = (my_row < nrows && my_head < 3) ? dot * scale2 : -INFINITY;
    float mx = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    const float m_new = fmaxf(m_run, mx);
    const float c = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
    const float p = sc == -INFINITY ? 0.f : exp2f(sc - m_new);
    float ps = p + __shfl_xor_sync(0xffffffffu, p, 4);
    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
    l_run = fmaf(l_run, c, ps);
    m_run = m_new;
#pragma unroll
    for (int g = 0; g < 3; g++) {
        const float cg_ = __shfl_sync(0xffffffffu, c, g);
        float2 lo = __fmul2_rn(make_float2(acc[g].x, acc[g].y), make_float2(cg_, cg_));
        float2 hi = __fmul2_rn(make_float2(acc[g].z, acc[g].w), make_float2(cg_, cg_));
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float pg = __shfl_sync(0xffffffffu, p, 4 * i + g);
            lo = __ffma2_rn(make_float2(pg, pg), make_float2(v4[i].x, v4[i].y), lo);
            hi = __ffma2_rn(make_float2(pg, pg), make_float2(v4[i].z, v4[i].w), hi);
        }
        acc[g] = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
}

// The first cache row of session n that this step's q/k/v GEMM writes: its
// position, or, when several slots share its cache (a prefill chunk at
// consecutive positions), the smallest of their positions. Copies of rows at or
// above it wait for the GEMM.
__device__ __forceinline__ int first_fresh_row(const BatchState *st, int n_active, int n) {
    int fresh = st->position[n];
    for (int m = 0; m < n_active; m++)
        if (st->keys[m] == st->keys[n]) fresh = min(fresh, st->position[m]);
    return fresh;
}

// 16 consumer warps: warp w takes rows 4 (w / 2) .. + 3 of each 32-row stage for
// query heads 3 (w % 2) .. + 2 of the KV head; one producer warp.
constexpr int kBatchAttnWarps = 16;
constexpr int kBatchAttnThreads = (kBatchAttnWarps + 1) * 32;
__device__ __forceinline__ void attn_consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kBatchAttnWarps * 32) : "memory"); }

__global__ void __launch_bounds__(kBatchAttnThreads, 1) batch_attn_kernel(AttnArgs a) {
    constexpr int G = 6, GH = 3;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int chunk_start[kBN + 1];   // first item of each session (prefix over sessions)
    __shared__ int fresh_s[kBN];           // first cache row of each session this step writes
    __shared__ int stage_item[kAttnRingStages], stage_row[kAttnRingStages];
    __shared__ float wm[kBatchAttnWarps][GH], wl[kBatchAttnWarps][GH];
    __shared__ __align__(16) float wacc[kBatchAttnWarps][GH][kHeadDim];
    __shared__ int last_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Ring ring;
    ring.buf = smem;
    ring.stage_bytes = kAttnStageBytes;
    ring.stages = kAttnRingStages;
    ring.full = reinterpret_cast<uint64_t *>(smem + (size_t)kAttnRingStages * kAttnStageBytes);
    ring.empty = ring.full + kAttnRingStages;
    if (threadIdx.x == 0) {
        for (int st = 0; st < kAttnRingStages; st++) {
            mbar_init(&ring.full[st], 1);
            mbar_init(&ring.empty[st], kBatchAttnWarps);
        }
        mbar_fence_init();
    }
    pdl_trigger();
    if (threadIdx.x == 0 && a.trace) a.trace[(size_t)blockIdx.x * 8 + 0] = global_ns();
    // The state block is written before the step; this token's rows (position)
    // are written by the q/k/v GEMM, so copies that include them wait for it.
    const int n_active = a.st->n;
    if (threadIdx.x == 0) {
        int acc_items = 0;
        for (int n = 0; n < n_active; n++) {
            chunk_start[n] = acc_items;
            acc_items += 2 * ((a.st->position[n] + a.item_rows) / a.item_rows);
        }
        chunk_start[n_active] = acc_items;
    }
    if ((int)threadIdx.x < n_active) fresh_s[threadIdx.x] = first_fresh_row(a.st, n_active, threadIdx.x);
    __syncthreads();
    const int items = chunk_start[n_active];
    auto locate = [&](int item, int &n, int &h, int &c, int &rows0, int &rows1) {
        int lo = 0, hi = n_active - 1;  // last session with chunk_start <= item
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (chunk_start[mid] <= item) lo = mid;
            else hi = mid - 1;
        }
        n = lo;
        const int within = item - chunk_start[n], chunks = (chunk_start[n + 1] - chunk_start[n]) / 2;
        h = within / chunks;
        c = within % chunks;
        const int L = a.st->position[n] + 1;
        rows0 = c * a.item_rows;
        rows1 = min(L, rows0 + a.item_rows);
    };

    if (warp == kBatchAttnWarps) {
        // Producer: items come from a global counter (the first free item goes
        // to the first free CTA), their stages into the ring; each stage carries
        // its item and first row, and a stage with item -1 ends the stream.
        if (lane == 0) {
            bool waited = false, ok = true;
            int g = 0;
            for (;;) {
                const int item = (int)atomicAdd(&a.work[0], 1u);
                const bool done = item >= items;
                int n = 0, h = 0, c = 0, r0 = 0, r1 = 1;
                if (!done) locate(item, n, h, c, r0, r1);
                const int cap = done ? 0 : a.st->capacity[n], last = done ? 0 : fresh_s[n];
                const float *kb = done ? nullptr : a.st->keys[n] + ((size_t)a.layer * 2 + h) * cap * kHeadDim;
                const float *vb = done ? nullptr : a.st->values[n] + ((size_t)a.layer * 2 + h) * cap * kHeadDim;
                for (int t = r0; t < r1; t += kAttnRowsPerStage, g++) {
                    const int s = g % kAttnRingStages, rows = min(kAttnRowsPerStage, r1 - t);
                    if (g >= kAttnRingStages &&
                        !mbar_wait(&ring.empty[s], ((g / kAttnRingStages) & 1) ^ 1, &a.st->err, kErrEmptyWait)) {
                        ok = false;
                        break;
                    }
                    stage_item[s] = done ? -1 : item;
                    stage_row[s] = t;
                    if (done) {
                        mbar_arrive(&ring.full[s]);  // the end marker: no data
                        g++;  // counted, so the drain below sees each stage's latest phase
                        break;
                    }
                    if (!waited && t + rows > last) {  // this stage holds a row the q/k/v GEMM writes
                        pdl_wait();
                        waited = true;
                    }
                    const uint32_t bytes = (uint32_t)rows * kHeadDim * 4;
                    mbar_expect_tx(&ring.full[s], 2 * bytes);
                    bulk_copy_g2s(ring.stage(s), kb + (size_t)t * kHeadDim, bytes, &ring.full[s]);
                    bulk_copy_g2s(ring.stage(s) + kAttnStageBytes / 2, vb + (size_t)t * kHeadDim, bytes, &ring.full[s]);
                }
                if (done || !ok) break;
            }
            for (int d = g > kAttnRingStages ? g - kAttnRingStages : 0; d < g; d++)
                if (!mbar_wait(&ring.full[d % kAttnRingStages], (d / kAttnRingStages) & 1, &a.st->err, kErrDrain)) break;
        }
    } else {
        pdl_wait();
        const int tid = threadIdx.x, quad = warp >> 1, half = warp & 1;
        const float scale2 = a.inv_sqrt_dim * 1.44269504088896340736f;  // log2(e) / sqrt(128): base-2 scores
        if (tid == 0 && a.trace) a.trace[(size_t)blockIdx.x * 8 + 1] = global_ns();
        int g = 0;
        int cur = -1, n = 0, h = 0, c = 0, r0 = 0, r1 = 0;
        float4 q4[GH], acc[GH];
        float m_run = -INFINITY, l_run = 0.f;
        for (;;) {
            if (!mbar_wait(&ring.full[g % kAttnRingStages], (g / kAttnRingStages) & 1, &a.st->err, kErrFullWait)) break;
            const int s = g % kAttnRingStages, item = stage_item[s], t = stage_row[s];
            if (item < 0) break;  // end of the stream (the producer's last stage)
            if (g == 0 && tid == 0 && a.trace) a.trace[(size_t)blockIdx.x * 8 + 2] = global_ns();
            if (item != cur) {
                cur = item;
                locate(item, n, h, c, r0, r1);
#pragma unroll
                for (int gg = 0; gg < GH; gg++) {
                    q4[gg] = reinterpret_cast<const float4 *>(a.q + (size_t)n * kHd + (h * G + GH * half + gg) * kHeadDim)[lane];
                    acc[gg] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
                m_run = -INFINITY;
                l_run = 0.f;
            }
            const int rows = min(kAttnRowsPerStage, r1 - t);
            const float4 *ks = reinterpret_cast<const float4 *>(ring.stage(s));
            const float4 *vs = reinterpret_cast<const float4 *>(ring.stage(s) + kAttnStageBytes / 2);
            const int mine = min(4, rows - 4 * quad);
            float4 k4[4], v4[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const bool in = i < mine;
                k4[i] = in ? ks[(4 * quad + i) * (kHeadDim / 4) + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
                v4[i] = in ? vs[(4 * quad + i) * (kHeadDim / 4) + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&ring.empty[s]);
            g++;
            if (mine > 0) flash_step3(q4, k4, v4, mine, lane, scale2, m_run, l_run, acc);
            if (t + kAttnRowsPerStage < r1) continue;
            // Last stage of the item: merge, per query head, the eight warps that
            // hold it (same half), in warp order, into the chunk's partial.
            attn_consumers_sync();
#pragma unroll
            for (int gg = 0; gg < GH; gg++) {
                reinterpret_cast<float4 *>(wacc[warp][gg])[lane] = acc[gg];
                const float mg = __shfl_sync(0xffffffffu, m_run, gg), lg = __shfl_sync(0xffffffffu, l_run, gg);
                if (lane == 0) {
                    wm[warp][gg] = mg;
                    wl[warp][gg] = lg;
                }
            }
            attn_consumers_sync();
            float *hp = a.part + ((size_t)n * 2 + h) * kAttnItemMax * kAttnPartialFloats;
            float *pc = hp + (size_t)c * kAttnPartialFloats;
            for (int o = tid; o < G * kHeadDim; o += kBatchAttnWarps * 32) {
                const int gq = o / kHeadDim, d = o % kHeadDim, hf = gq / GH, gg = gq % GH;
                float M = -INFINITY;
#pragma unroll
                for (int w = hf; w < kBatchAttnWarps; w += 2) M = fmaxf(M, wm[w][gg]);
                float num = 0.f, den = 0.f;
#pragma unroll
                for (int w = hf; w < kBatchAttnWarps; w += 2) {
                    if (wm[w][gg] == -INFINITY) continue;
                    const float e = exp2f(wm[w][gg] - M);
                    den = fmaf(e, wl[w][gg], den);
                    num = fmaf(e, wacc[w][gg][d], num);
                }
                pc[2 * kAttnMaxGroup + gq * kHeadDim + d] = num;
                if (d == 0) {
                    pc[gq] = M;
                    pc[kAttnMaxGroup + gq] = den;
                }
            }
            __threadfence();
            attn_consumers_sync();
            const int nchunks = (a.st->position[n] + a.item_rows) / a.item_rows;
            unsigned *counter = &a.counters[n * 2 + h];
            if (tid == 0) last_s = atomicAdd(counter, 1u) == (unsigned)(nchunks - 1);
            attn_consumers_sync();
            if (last_s) {
                __threadfence();
                for (int o = tid; o < G * kHeadDim; o += kBatchAttnWarps * 32) {
                    const int gq = o / kHeadDim, d = o % kHeadDim;
                    float M = -INFINITY;
                    for (int cc = 0; cc < nchunks; cc++) M = fmaxf(M, __ldcg(hp + (size_t)cc * kAttnPartialFloats + gq));
                    float num = 0.f, den = 0.f;
                    for (int cc = 0; cc < nchunks; cc++) {
                        const float *pp = hp + (size_t)cc * kAttnPartialFloats;
                        const float mc = __ldcg(pp + gq);
                        if (mc == -INFINITY) continue;
                        const float e = exp2f(mc - M);
                        den = fmaf(e, __ldcg(pp + kAttnMaxGroup + gq), den);
                        num = fmaf(e, __ldcg(pp + 2 * kAttnMaxGroup + gq * kHeadDim + d), num);
                    }
                    uint16_t hi, lo;
                    split_bf16(__fdiv_rn(num, den), hi, lo);
                    a.oh[(size_t)n * kHd + (h * G + gq) * kHeadDim + d] = hi;
                    a.ol[(size_t)n * kHd + (h * G + gq) * kHeadDim + d] = lo;
                }
                if (tid == 0) *counter = 0u;
            }
        }
        if (tid == 0 && a.trace) a.trace[(size_t)blockIdx.x * 8 + 3] = global_ns();
    }
    // The last CTA out resets the work counter for the next launch.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&a.work[1], 1u) == gridDim.x - 1) {
            a.work[0] = 0u;
            a.work[1] = 0u;
        }
    }
}

// ---------------------------------------------------------------- attention on tensor-core fragments
// The same work items, with the arithmetic on the tensor cores (mma.sync
// m16n8k8, TF32 operands, FP32 accumulation) and no sharing between warps:
// each of the CTA's four warps takes whole items from the global counter and
// feeds itself through its own three stages of 8 K rows and 8 V rows (each
// lane moves 16-byte pieces with cp.async; K rows land 576 bytes apart and V
// rows 528, so every fragment load below is free of bank conflicts; a stage's
// barrier completes when all 32 lanes' pieces have landed), issuing the next
// stage's copies as soon as it has read a stage. A warp never waits for
// another.
//
// Per stage and KV head (6 query heads, padded to 8):
//   S = Q K^T: A = [Q_hi; Q_lo] (rows 0-7 the heads' high TF32 parts, rows
//     8-15 the remainders), B = K_hi^T and then K_lo^T, so two products give
//     all four terms of (Q_hi + Q_lo)(K_hi + K_lo); the dimension order inside
//     each k-step of 8 is permuted (lane slot t <-> dimension 4t, slot t + 4
//     <-> 4t + 1 of a 16-dimension block), identically for A and B;
//   online softmax in base 2 on the accumulator layout: lane (g, t) holds
//     head g's scores of rows 2t and 2t + 1 of the 8-row tile; the reference
//     max a head's exponentials use moves only when the tile's max exceeds
//     it by more than kTcLazy (then the accumulators are rescaled), so
//     exponentials stay below 2^kTcLazy and most tiles need no rescale;
//   O += P V: A = [P_hi; P_lo] straight from those registers (row slot t <->
//     row 2t, slot t + 4 <-> 2t + 1), B = V_hi and then V_lo.
// x_hi keeps the TF32 bits of x and x_lo = x - x_hi (exact), so every product
// carries about 21 bits of each operand: FP32-level scores and outputs.
// Each item leaves a partial (max, sum, accumulators) in global memory, and
// batch_attn_merge_kernel folds a (session, head)'s partials in chunk order.
constexpr int kTcWarps = 8;
constexpr int kTcRows = 8;                 // cache rows per stage (one 8-row tile)
constexpr int kTcStages = 3;               // stages per warp
constexpr int kTcKStride = kHeadDim + 16;  // K row stride in floats (576 bytes)
constexpr int kTcVStride = kHeadDim + 4;   // V row stride in floats (528 bytes)
constexpr uint32_t kTcStageBytes = (uint32_t)kTcRows * (kTcKStride + kTcVStride) * 4;
constexpr size_t kTcAttnSmem = (size_t)kTcWarps * kTcStages * kTcStageBytes + (size_t)kTcWarps * kTcStages * 8;
constexpr int kTcItemRowsDefault = 256;
constexpr float kTcLazy = 8.f;             // base-2 headroom of the softmax's reference max
static_assert(kTcAttnSmem <= 227 * 1024, "shared memory");

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 16-byte global -> shared copy (L2 only), and an arrival on `bar` once all of
// this thread's earlier copies have landed (counted in the barrier's arrival
// count, which this does not raise).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ uint32_t tf32_hi(float x) { return __float_as_uint(x) & 0xffffe000u; }
__device__ __forceinline__ uint32_t tf32_lo(float x) { return __float_as_uint(__fsub_rn(x, __uint_as_float(tf32_hi(x)))); }

// O += [P_hi; P_lo] V over one 8-row k-step: v0 and v1 point at this lane's
// rows 2t and 2t + 1 (already offset by 4g dimensions); masked rows read 0.
template <bool kMask>
__device__ __forceinline__ void tc_pv_step(float (&o)[16][4], const uint32_t (&pa)[4], const float *v0, const float *v1,
                                           bool ok0, bool ok1) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
        float4 y = *reinterpret_cast<const float4 *>(v0 + 32 * q), z = *reinterpret_cast<const float4 *>(v1 + 32 * q);
        if constexpr (kMask) {
            if (!ok0) y = make_float4(0.f, 0.f, 0.f, 0.f);
            if (!ok1) z = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float yy[4] = {y.x, y.y, y.z, y.w}, zz[4] = {z.x, z.y, z.z, z.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            mma_tf32(o[4 * q + i], pa, tf32_hi(yy[i]), tf32_hi(zz[i]));
            mma_tf32(o[4 * q + i], pa, tf32_lo(yy[i]), tf32_lo(zz[i]));
        }
    }
}

__global__ void __launch_bounds__(kTcWarps * 32, 1) batch_attn_tc_kernel(AttnArgs a) {
    constexpr int G = 6;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int chunk_start[kBN + 1], fresh_s[kBN], pos_s[kBN];
    __shared__ const float *keys_s[kBN];
    __shared__ int hdr_item[kTcWarps][kTcStages], hdr_row[kTcWarps][kTcStages];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    unsigned char *ring = smem + (size_t)warp * kTcStages * kTcStageBytes;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)kTcWarps * kTcStages * kTcStageBytes) + warp * kTcStages;
    if (lane == 0) {
        for (int st = 0; st < kTcStages; st++) mbar_init(&full[st], 32);  // one arrival per lane
        mbar_fence_init();
    }
    pdl_trigger();
    if (threadIdx.x == 0 && a.trace) a.trace[(size_t)blockIdx.x * 8 + 0] = global_ns();
    // Items are numbered with every (session, head)'s chunks but its last
    // first, session by session (chunk_start: prefix of 2 (chunks - 1)), then
    // the last chunks (n, h) -- the short ones -- so the warps that finish
    // last take the smallest items.
    // The sessions' positions and cache pointers are read once (one load per
    // thread), then the per-session quantities come from shared memory.
    const int n_active = a.st->n;
    if ((int)threadIdx.x < n_active) {
        pos_s[threadIdx.x] = a.st->position[threadIdx.x];
        keys_s[threadIdx.x] = a.st->keys[threadIdx.x];
    }
    __syncthreads();
    if ((int)threadIdx.x < n_active) {
        const int n = threadIdx.x;
        int fresh = pos_s[n];  // first_fresh_row, from the staged copies
        for (int m = 0; m < n_active; m++)
            if (keys_s[m] == keys_s[n]) fresh = min(fresh, pos_s[m]);
        fresh_s[n] = fresh;
    }
    if (threadIdx.x == 0) {
        int acc_items = 0;
        for (int n = 0; n < n_active; n++) {
            chunk_start[n] = acc_items;
            acc_items += 2 * ((pos_s[n] + a.item_rows) / a.item_rows - 1);
        }
        chunk_start[n_active] = acc_items;
    }
    __syncthreads();
    const int full_items = chunk_start[n_active], items = full_items + 2 * n_active;
    auto locate = [&](int item, int &n, int &h, int &c, int &rows0, int &rows1) {
        if (item >= full_items) {
            n = (item - full_items) >> 1;
            h = (item - full_items) & 1;
            c = (pos_s[n] + a.item_rows) / a.item_rows - 1;
        } else {
            int lo = 0, hi = n_active - 1;  // last session with chunk_start <= item
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (chunk_start[mid] <= item) lo = mid;
                else hi = mid - 1;
            }
            n = lo;
            const int within = item - chunk_start[n], chunks = (chunk_start[n + 1] - chunk_start[n]) / 2;
            h = within / chunks;
            c = within % chunks;
        }
        rows0 = c * a.item_rows;
        rows1 = min(pos_s[n] + 1, rows0 + a.item_rows);
    };

    // Producer side (warp-uniform state): the item being copied and its next row.
    int p_item = 0, p_n = 0, p_h = 0, p_c = 0, p_t = 0, p_r1 = 0, produced = 0;
    bool p_end = false, end_issued = false, waited = false;
    auto next_item = [&]() {
        int it = 0;
        if (lane == 0) it = (int)atomicAdd(&a.work[0], 1u);
        it = __shfl_sync(0xffffffffu, it, 0);
        if (it >= items) {
            p_end = true;
            return;
        }
        p_item = it;
        locate(it, p_n, p_h, p_c, p_t, p_r1);
    };
    auto produce = [&]() {
        if (end_issued) return;
        const int s = produced % kTcStages;
        produced++;
        if (p_end) {
            end_issued = true;
            if (lane == 0) hdr_item[warp][s] = -1;
            __syncwarp();
            mbar_arrive(&full[s]);  // the end marker: no data
            return;
        }
        const int rows = min(kTcRows, p_r1 - p_t);
        if (!waited && p_t + rows > fresh_s[p_n]) {  // rows the q/k/v GEMM writes this step
            pdl_wait();
            waited = true;
        }
        if (lane == 0) {
            hdr_item[warp][s] = p_item;
            hdr_row[warp][s] = p_t;
        }
        __syncwarp();
        const size_t base = (((size_t)a.layer * 2 + p_h) * a.st->capacity[p_n] + p_t) * kHeadDim + 4 * lane;
        const float *kg = a.st->keys[p_n] + base, *vg = a.st->values[p_n] + base;
        float *kd = reinterpret_cast<float *>(ring + (size_t)s * kTcStageBytes) + 4 * lane;
        float *vd = kd + kTcRows * kTcKStride;
        for (int r = 0; r < rows; r++) {
            cp_async16(kd + r * kTcKStride, kg + (size_t)r * kHeadDim);
            cp_async16(vd + r * kTcVStride, vg + (size_t)r * kHeadDim);
        }
        cp_async_arrive(&full[s]);
        p_t += rows;
        if (p_t >= p_r1) next_item();
    };
    next_item();
    for (int k = 0; k < kTcStages; k++) produce();
    if (!waited) {  // q is the q/k/v GEMM's output
        pdl_wait();
        waited = true;
    }
    if (threadIdx.x == 0 && a.trace) a.trace[(size_t)blockIdx.x * 8 + 1] = global_ns();

    const float scale2 = a.inv_sqrt_dim * 1.44269504088896340736f;  // log2(e) / sqrt(128): base-2 scores
    uint32_t qa[16][4];
    float o[16][4];
    float m_run = -INFINITY, l_run = 0.f;
    int cur = -1, cn = 0, ch = 0, cc = 0, cr1 = 0;
    auto finish = [&]() {
        float lt = l_run + __shfl_xor_sync(0xffffffffu, l_run, 1);
        lt += __shfl_xor_sync(0xffffffffu, lt, 2);
        float *pc = a.part + (((size_t)cn * 2 + ch) * kAttnItemMax + cc) * kAttnPartialFloats;
        if (g < G) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                float *dst = pc + 2 * kAttnMaxGroup + g * kHeadDim + 32 * q + 8 * t4;
                reinterpret_cast<float4 *>(dst)[0] =
                    make_float4(o[4 * q][0] + o[4 * q][2], o[4 * q + 1][0] + o[4 * q + 1][2],
                                o[4 * q + 2][0] + o[4 * q + 2][2], o[4 * q + 3][0] + o[4 * q + 3][2]);
                reinterpret_cast<float4 *>(dst)[1] =
                    make_float4(o[4 * q][1] + o[4 * q][3], o[4 * q + 1][1] + o[4 * q + 1][3],
                                o[4 * q + 2][1] + o[4 * q + 2][3], o[4 * q + 3][1] + o[4 * q + 3][3]);
            }
            if (t4 == 0) {
                pc[g] = m_run;
                pc[kAttnMaxGroup + g] = lt;
            }
        }
    };
    auto start = [&](int item) {
        int r0;
        locate(item, cn, ch, cc, r0, cr1);
        const float *qb = a.q + (size_t)cn * kHd + (size_t)(ch * G + g) * kHeadDim + 4 * t4;
#pragma unroll
        for (int u = 0; u < 8; u++) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (g < G) v = __ldcg(reinterpret_cast<const float4 *>(qb + 16 * u));
            qa[2 * u][0] = tf32_hi(v.x);
            qa[2 * u][1] = tf32_lo(v.x);
            qa[2 * u][2] = tf32_hi(v.y);
            qa[2 * u][3] = tf32_lo(v.y);
            qa[2 * u + 1][0] = tf32_hi(v.z);
            qa[2 * u + 1][1] = tf32_lo(v.z);
            qa[2 * u + 1][2] = tf32_hi(v.w);
            qa[2 * u + 1][3] = tf32_lo(v.w);
        }
#pragma unroll
        for (int i = 0; i < 16; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
        m_run = -INFINITY;
        l_run = 0.f;
    };
    int k = 0;
    bool failed = false;
    for (;; k++) {
        const int s = k % kTcStages;
        if (!mbar_wait(&full[s], (k / kTcStages) & 1, &a.st->err, kErrFullWait)) {
            failed = true;
            break;
        }
        const int item = hdr_item[warp][s], t0 = hdr_row[warp][s];
        if (item < 0) {  // end of this warp's stream (possibly before any item)
            if (cur >= 0) finish();
            break;
        }
        if (item != cur) {
            if (cur >= 0) finish();
            cur = item;
            start(item);
        }
        if (k == 0 && threadIdx.x == 0 && a.trace) a.trace[(size_t)blockIdx.x * 8 + 2] = global_ns();
        const int nrows = min(kTcRows, cr1 - t0);
        const float *Ks = reinterpret_cast<const float *>(ring + (size_t)s * kTcStageBytes);
        const float *Vs = Ks + kTcRows * kTcKStride;
        // S = [Q_hi; Q_lo] (K_hi + K_lo)^T in four accumulator chains (K_hi or
        // K_lo, even or odd 16-dimension block).
        float sa[2][4], sb[2][4];
#pragma unroll
        for (int c = 0; c < 2; c++)
#pragma unroll
            for (int e = 0; e < 4; e++) sa[c][e] = sb[c][e] = 0.f;
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const float4 kv = *reinterpret_cast<const float4 *>(Ks + g * kTcKStride + 16 * u + 4 * t4);
            mma_tf32(sa[u & 1], qa[2 * u], tf32_hi(kv.x), tf32_hi(kv.y));
            mma_tf32(sb[u & 1], qa[2 * u], tf32_lo(kv.x), tf32_lo(kv.y));
            mma_tf32(sa[u & 1], qa[2 * u + 1], tf32_hi(kv.z), tf32_hi(kv.w));
            mma_tf32(sb[u & 1], qa[2 * u + 1], tf32_lo(kv.z), tf32_lo(kv.w));
        }
        // Scores of head g, rows 2t + e: (Q_hi K) + (Q_lo K).
        float sc[2];
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const float hi = (sa[0][e] + sa[1][e]) + (sb[0][e] + sb[1][e]);
            const float lo = (sa[0][2 + e] + sa[1][2 + e]) + (sb[0][2 + e] + sb[1][2 + e]);
            sc[e] = (2 * t4 + e < nrows && g < G) ? (hi + lo) * scale2 : -INFINITY;
        }
        float mx = fmaxf(sc[0], sc[1]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        if (__any_sync(0xffffffffu, g < G && (m_run == -INFINITY ? mx != -INFINITY : mx > m_run + kTcLazy))) {
            const float m_new = (m_run == -INFINITY || mx > m_run + kTcLazy) ? fmaxf(m_run, mx) : m_run;
            const float corr = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
            l_run *= corr;
#pragma unroll
            for (int i = 0; i < 16; i++)
#pragma unroll
                for (int e = 0; e < 4; e++) o[i][e] *= corr;
            m_run = m_new;
        }
        float p[2];
#pragma unroll
        for (int e = 0; e < 2; e++) p[e] = sc[e] == -INFINITY ? 0.f : exp2f(sc[e] - m_run);
        l_run += p[0] + p[1];
        {
            const uint32_t pa[4] = {tf32_hi(p[0]), tf32_lo(p[0]), tf32_hi(p[1]), tf32_lo(p[1])};
            const float *v0 = Vs + 2 * t4 * kTcVStride + 4 * g, *v1 = v0 + kTcVStride;
            if (nrows < kTcRows)
                tc_pv_step<true>(o, pa, v0, v1, 2 * t4 < nrows, 2 * t4 + 1 < nrows);
            else
                tc_pv_step<false>(o, pa, v0, v1, true, true);
        }
        // This stage's slot is read: the next copies may land in it.
        __syncwarp();
        produce();
    }
    if (failed)  // copies this warp issued must land before it leaves
        for (int j = k + 1; j < produced; j++)
            if (!mbar_wait(&full[j % kTcStages], (j / kTcStages) & 1, &a.st->err, kErrDrain)) break;
    if (threadIdx.x == 0 && a.trace) a.trace[(size_t)blockIdx.x * 8 + 3] = global_ns();
    // The last warp out (every warp has drawn past the last item) resets the
    // work counter for the next launch; no warp waits for the others.
    if (lane == 0) {
        __threadfence();
        if (atomicAdd(&a.work[1], 1u) == gridDim.x * kTcWarps - 1) {
            a.work[0] = 0u;
            a.work[1] = 0u;
        }
    }
}

// Folds the chunk partials of (session blockIdx.x, KV head blockIdx.y) in
// chunk order and writes the heads' output rows as BF16 hi/lo.
struct MergeArgs {
    BatchState *st;
    const float *part;
    uint16_t *oh, *ol;
    int item_rows;
};
__global__ void __launch_bounds__(256) batch_attn_merge_kernel(MergeArgs a) {
    constexpr int G = 6, kPer = G * kHeadDim / 256;  // outputs per thread
    __shared__ float m_s[G][kAttnItemMax], w_s[G][kAttnItemMax], den_s[G];
    pdl_trigger();
    pdl_wait();
    const int n = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    if (n >= a.st->n) return;
    const int nchunks = (a.st->position[n] + a.item_rows) / a.item_rows;
    const float *hp = a.part + ((size_t)n * 2 + h) * kAttnItemMax * kAttnPartialFloats;
    // Every load is issued before any arithmetic: this thread's outputs
    // o = tid + 256 k over all chunks, and per (head, chunk) the chunk's max
    // and sum into shared memory.
    float av[kPer][kAttnItemMax];
#pragma unroll
    for (int k = 0; k < kPer; k++) {
        const int o = tid + 256 * k;
        const float *pa = hp + 2 * kAttnMaxGroup + (o / kHeadDim) * kHeadDim + o % kHeadDim;
#pragma unroll
        for (int c = 0; c < kAttnItemMax; c++) av[k][c] = c < nchunks ? __ldcg(pa + (size_t)c * kAttnPartialFloats) : 0.f;
    }
    for (int i = tid; i < G * nchunks; i += blockDim.x) {
        const int gq = i / nchunks, c = i % nchunks;
        m_s[gq][c] = __ldcg(hp + (size_t)c * kAttnPartialFloats + gq);
        w_s[gq][c] = __ldcg(hp + (size_t)c * kAttnPartialFloats + kAttnMaxGroup + gq);
    }
    __syncthreads();
    // Per head: the weights e_c = 2^(m_c - M) and the denominator, in chunk order.
    if (tid < G) {
        float M = -INFINITY;
        for (int c = 0; c < nchunks; c++) M = fmaxf(M, m_s[tid][c]);
        float den = 0.f;
        for (int c = 0; c < nchunks; c++) {
            const float e = m_s[tid][c] == -INFINITY ? 0.f : exp2f(m_s[tid][c] - M);
            den = m_s[tid][c] == -INFINITY ? den : fmaf(e, w_s[tid][c], den);
            w_s[tid][c] = e;
        }
        den_s[tid] = den;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kPer; k++) {
        const int o = tid + 256 * k, gq = o / kHeadDim, d = o % kHeadDim;
        float num = 0.f;
#pragma unroll
        for (int c = 0; c < kAttnItemMax; c++)
            if (c < nchunks && m_s[gq][c] != -INFINITY) num = fmaf(w_s[gq][c], av[k][c], num);
        uint16_t hi, lo;
        split_bf16(__fdiv_rn(num, den_s[gq]), hi, lo);
        a.oh[(size_t)n * kHd + (h * G + gq) * kHeadDim + d] = hi;
        a.ol[(size_t)n * kHd + (h * G + gq) * kHeadDim + d] = lo;
    }
}

// ---------------------------------------------------------------- top-2 per session
// kTopBlocks blocks per session scan a slice of its logits each (float4 loads,
// finite check) and publish a partial top-2; the last block of the session to
// arrive merges the partials in order, logs the top-2 and feeds top-1 back as
// the session's next token.
constexpr int kTopBlocks = 16;
struct Top2Args {
    BatchState *st;
    Top2 *part;          // [kBN][kTopBlocks]
    unsigned *counters;  // [kBN]
    int vocab;
    TcmTop2 *log;        // [kBatchLogCap][kBN]
};
__global__ void __launch_bounds__(256) batch_top2_kernel(Top2Args a) {
    __shared__ Top2 sh[8];
    __shared__ int last_s;
    pdl_trigger();
    pdl_wait();
    const int n = blockIdx.y, tid = threadIdx.x;
    if (n >= a.st->n) return;
    const int chunk = a.vocab / kTopBlocks, v0 = blockIdx.x * chunk;
    const float4 *lg = reinterpret_cast<const float4 *>(a.st->logits[n] + v0);
    Top2 z = top2_empty();
    bool bad = false;
    for (int i = tid; i < chunk / 4; i += 256) {
        const float4 v = __ldcg(lg + i);
        bad |= !isfinite(v.x) || !isfinite(v.y) || !isfinite(v.z) || !isfinite(v.w);
        const int id = v0 + 4 * i;
        top2_insert(z, v.x, id);
        top2_insert(z, v.y, id + 1);
        top2_insert(z, v.z, id + 2);
        top2_insert(z, v.w, id + 3);
    }
    top2_merge_warp(z);
    if (__syncthreads_or(bad) && tid == 0) a.st->bad[n] = 1;
    if ((tid & 31) == 0) sh[tid >> 5] = z;
    __syncthreads();
    if (tid == 0) {
        Top2 f = sh[0];
        for (int w = 1; w < 8; w++) {
            top2_insert(f, sh[w].a, sh[w].ai);
            top2_insert(f, sh[w].b, sh[w].bi);
        }
        a.part[(size_t)n * kTopBlocks + blockIdx.x] = f;
        __threadfence();
        last_s = atomicAdd(&a.counters[n], 1u) == kTopBlocks - 1;
    }
    __syncthreads();
    if (!last_s || tid != 0) return;
    __threadfence();
    Top2 f = top2_empty();
    for (int b = 0; b < kTopBlocks; b++) {
        const Top2 p = a.part[(size_t)n * kTopBlocks + b];
        top2_insert(f, p.a, p.ai);
        top2_insert(f, p.b, p.bi);
    }
    TcmTop2 top;
    top.first = f.ai; top.second = f.bi; top.first_value = f.a; top.second_value = f.b;
    a.log[(size_t)(a.st->step % kBatchLogCap) * kBN + n] = top;
    a.st->token[n] = f.ai;
    a.st->position[n] += 1;
    a.counters[n] = 0u;
}
__global__ void batch_step_end_kernel(BatchState *st) {
    pdl_wait();
    st->step += 1;
}

// ---------------------------------------------------------------- tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        TCM_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (!p || q != cudaDriverEntryPointSuccess) TCM_FATAL("cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}
// A 2D BF16 map over rows x inner (row-major), 64-element (128-byte) boxes of
// box_rows rows in the 128-byte swizzle.
CUtensorMap bf16_map(const void *base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {inner * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
                                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) TCM_FATAL("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return m;
}

template <class Epi> void gemm_setup() {
    TCM_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<kBN, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)TcGeo<kBN>::kSmem));
    TCM_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<kBN, Epi>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
}

}  // namespace

// The BF16 weights' maps of one layer.
struct LayerMaps {
    CUtensorMap q, k, v, o, gate, up, down;
};

void set_wait_limit_batch(unsigned long long ns) { set_module_wait_limit(ns); }

}  // namespace tcm

using namespace tcm;

struct QwenB200Batch {
    const QwenB200Decoder *d;
    QwenB200Shape s;
    std::vector<LayerMaps> maps;
    CUtensorMap embed, nh_map, nl_map, hh_map, hl_map;
    const std::vector<QwenB200Layer> *layers;
    const void *embed_ptr;
    const float *final_norm, *rope_den;
    BatchState *st;       // device
    BatchState *host;     // pinned mirror
    float *x, *q, *part, *attn_part;
    uint16_t *nh, *nl, *hh, *hl;
    unsigned *counters, *attn_counters, *top_counters, *attn_work;
    Top2 *top_part;
    int cluster_qkv, cluster_o, cluster_down;  // split clusters (0: split K through global memory)
    int attn_item_rows;   // cache rows per attention work item
    int attn_kernel;      // 0: tensor-core fragments + merge kernel; 1: CUDA-core flash-decoding
    int resid_defer;      // 1: the O and down GEMMs leave K-split partials that the next RMSNorm sums
    TcmTop2 *log, *host_log;
    unsigned long long *trace;  // stage timeline (measurement only), or null
    int readout_tiles;
    std::map<int, cudaGraphExec_t> graphs;
    float *prefill_logits, *prefill_x;  // logits and hidden rows of a prefill chunk's non-final tokens (lazy)
};

namespace {

template <class Epi>
void launch_gemm(QwenB200Batch *b, const CUtensorMap &a0, const CUtensorMap &a1, const CUtensorMap &a2,
                 const CUtensorMap &xh, const CUtensorMap &xl, int tiles, int splits, int kblocks, const Epi &epi,
                 bool pdl, int cluster = 1, bool defer = false) {
    TcArgs<kBN, Epi> args;
    args.a[0] = a0;
    args.a[1] = a1;
    args.a[2] = a2;
    args.xh = xh;
    args.xl = xl;
    args.tiles = tiles;
    args.splits = splits;
    args.kblocks = kblocks;
    args.cluster = cluster;
    args.defer = defer ? 1 : 0;
    args.part = b->part;
    args.counters = b->counters;
    args.err = &b->st->err;
    args.trace = b->trace;
    args.epi = epi;
    const int items = tiles * splits;
    if (cluster > 1) {
        // One item per CTA; a cluster of `splits` CTAs per tile.
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(items);
        cfg.blockDim = dim3(kTcThreads);
        cfg.dynamicSmemBytes = TcGeo<kBN>::kSmem;
        cfg.stream = stream();
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = cluster;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 2 : 1;
        TCM_CUDA(cudaLaunchKernelEx(&cfg, tc_gemm_kernel<kBN, Epi>, args));
        return;
    }
    const int grid = items < sm_count() ? items : sm_count();
    launch(tc_gemm_kernel<kBN, Epi>, dim3(grid), dim3(kTcThreads), TcGeo<kBN>::kSmem, stream(), pdl, args);
}

// A K-split GEMM of `tiles` 128-row tiles: split across a cluster when one
// fits (cluster > 0), else 12 splits meeting in global memory; with
// defer_splits > 0, that many splits whose partials the next kernel sums.
template <class Epi>
void launch_split(QwenB200Batch *b, const CUtensorMap &a0, const CUtensorMap &a1, const CUtensorMap &a2,
                  const CUtensorMap &xh, const CUtensorMap &xl, int tiles, int kblocks, const Epi &epi, bool pdl,
                  int cluster, int defer_splits = 0) {
    if (defer_splits > 0) launch_gemm(b, a0, a1, a2, xh, xl, tiles, defer_splits, kblocks, epi, pdl, 1, true);
    else if (cluster > 0) launch_gemm(b, a0, a1, a2, xh, xl, tiles, cluster, kblocks, epi, pdl, cluster);
    else launch_gemm(b, a0, a1, a2, xh, xl, tiles, kblocks < 12 ? kblocks : 12, kblocks, epi, pdl, 1);
}

// How many clusters of `size` GEMM CTAs the GPU can hold at once.
int cluster_capacity(int size) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size * 16);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = TcGeo<kBN>::kSmem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = size;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, tc_gemm_kernel<kBN, EpiResid>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        clusters = 0;
    }
    return clusters;
}
// The largest split cluster (4 <= S <= 16, the fold's slice bound) whose
// `tiles` clusters all fit on the GPU at once; 0 when none does.
int pick_cluster(int tiles, int kblocks) {
    for (int sz = 16; sz >= 4; sz--)
        if (sz <= kblocks && cluster_capacity(sz) >= tiles) return sz;
    return 0;
}

// fold: the residual GEMM before this launch deferred its K-split sum here.
void launch_rms(QwenB200Batch *b, const float *w, bool embed, bool copy_x, bool pdl, bool fold = false) {
    RmsArgs a = {b->st, b->x, w, b->nh, b->nl, embed ? (const uint16_t *)b->embed_ptr : nullptr, b->s.epsilon,
                 copy_x ? 1 : 0, fold ? b->part : nullptr};
    launch(batch_rms_kernel, dim3(kBN), dim3(kRmsThreads), 0, stream(), pdl, a);
}

// The q/k/v projection of `layer` (bias, RoPE and K/V append in its epilogue,
// so its K splits meet in a cluster fold inside the GEMM).
void launch_qkv(QwenB200Batch *b, int layer, bool pdl) {
    const std::vector<QwenB200Layer> &L = *b->layers;
    const LayerMaps &m = b->maps[layer];
    EpiQkv qkv = {b->st, L[layer].qb, L[layer].kb, L[layer].vb, b->rope_den, b->q, layer};
    launch_split(b, m.q, m.k, m.v, b->nh_map, b->nl_map, 16, kHd / kTcKBlock, qkv, pdl, b->cluster_qkv);
}

// The attention of `layer` for n sessions (and its merge, for the tensor-core kernel).
void launch_attention(QwenB200Batch *b, int layer, int n, unsigned long long *trace, bool pdl) {
    AttnArgs at = {b->st, b->q, layer, 1.0f / sqrtf((float)kHeadDim), b->attn_part, b->attn_counters, b->nh, b->nl,
                   trace, b->attn_work + 2 * layer, b->attn_item_rows};
    if (b->attn_kernel == 0) {
        launch(batch_attn_tc_kernel, dim3(sm_count()), dim3(kTcWarps * 32), kTcAttnSmem, stream(), pdl, at);
        MergeArgs ma = {b->st, b->attn_part, b->nh, b->nl, b->attn_item_rows};
        launch(batch_attn_merge_kernel, dim3(n, 2), dim3(256), 0, stream(), true, ma);
    } else {
        launch(batch_attn_kernel, dim3(sm_count()), dim3(kBatchAttnThreads), kAttnSmem, stream(), pdl, at);
    }
}

void launch_step(QwenB200Batch *b, int n) {
    const QwenB200Shape &s = b->s;
    const std::vector<QwenB200Layer> &L = *b->layers;
    launch_rms(b, L[0].input_norm, true, false, false);
    for (int l = 0; l < s.layers; l++) {
        const LayerMaps &m = b->maps[l];
        launch_qkv(b, l, true);
        launch_attention(b, l, n, nullptr, true);
        const bool defer = b->resid_defer != 0;
        EpiResid o = {b->st, b->x};
        launch_split(b, m.o, m.o, m.o, b->nh_map, b->nl_map, 12, kHd / kTcKBlock, o, true, b->cluster_o,
                     defer ? kResidSplits : 0);
        launch_rms(b, L[l].post_norm, false, false, true, defer);
        EpiSwiglu sw = {b->st, b->hh, b->hl};
        launch_gemm(b, m.gate, m.up, m.up, b->nh_map, b->nl_map, kFf / 64, 1, kHd / kTcKBlock, sw, true);
        EpiResid dn = {b->st, b->x};
        launch_split(b, m.down, m.down, m.down, b->hh_map, b->hl_map, 12, kFf / kTcKBlock, dn, true, b->cluster_down,
                     defer ? kResidSplits : 0);
        if (l + 1 < s.layers) launch_rms(b, L[l + 1].input_norm, false, false, true, defer);
    }
    launch_rms(b, b->final_norm, false, true, true, b->resid_defer != 0);
    EpiLogits lg = {b->st};
    launch_gemm(b, b->embed, b->embed, b->embed, b->nh_map, b->nl_map, b->readout_tiles, 1, kHd / kTcKBlock, lg, true);
    Top2Args ta = {b->st, b->top_part, b->top_counters, b->s.vocab, b->log};
    launch(batch_top2_kernel, dim3(kTopBlocks, n), dim3(256), 0, stream(), true, ta);
    launch(batch_step_end_kernel, dim3(1), dim3(1), 0, stream(), true, b->st);
}

cudaGraphExec_t graph_for(QwenB200Batch *b, int n) {
    auto it = b->graphs.find(n);
    if (it != b->graphs.end()) return it->second;
    cudaStream_t s = stream();
    cudaGraph_t g;
    cudaGraphExec_t e;
    TCM_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    launch_step(b, n);
    TCM_CUDA(cudaStreamEndCapture(s, &g));
    TCM_CUDA(cudaGraphInstantiate(&e, g, 0));
    TCM_CUDA(cudaGraphDestroy(g));
    b->graphs[n] = e;
    return e;
}

bool load_sessions(QwenB200Batch *b, int n, const QwenB200BatchSession *ss, const int *tokens, const int *positions) {
    if (n < 1 || n > kBN || !ss || !tokens || !positions) return false;
    BatchState *h = b->host;
    for (int i = 0; i < n; i++) {
        const QwenB200BatchSession &x = ss[i];
        if (!x.keys || !x.values || !x.logits || !x.x || x.capacity < 1 || positions[i] < 0 ||
            positions[i] >= x.capacity || positions[i] >= kAttnSplitMax * kAttnChunk || tokens[i] < 0 ||
            tokens[i] >= b->s.vocab)
            return false;
        h->token[i] = tokens[i];
        h->position[i] = positions[i];
        h->capacity[i] = x.capacity;
        h->keys[i] = x.keys;
        h->values[i] = x.values;
        h->logits[i] = x.logits;
        h->x[i] = x.x;
        h->bad[i] = 0;
    }
    h->n = n;
    h->step = 0;
    h->err = 0u;
    TCM_CUDA(cudaMemcpyAsync(b->st, h, sizeof(BatchState), cudaMemcpyHostToDevice, stream()));
    return true;
}

int read_back(QwenB200Batch *b, int n, int steps, TcmTop2 *tops, bool history = false) {
    TCM_CUDA(cudaMemcpyAsync(b->host, b->st, sizeof(BatchState), cudaMemcpyDeviceToHost, stream()));
    const int last = (steps - 1) % kBatchLogCap;
    if (history)
        TCM_CUDA(cudaMemcpyAsync(b->host_log, b->log, sizeof(TcmTop2) * kBatchLogCap * kBN, cudaMemcpyDeviceToHost,
                                 stream()));
    else
        TCM_CUDA(cudaMemcpyAsync(b->host_log + (size_t)last * kBN, b->log + (size_t)last * kBN,
                                 sizeof(TcmTop2) * kBN, cudaMemcpyDeviceToHost, stream()));
    TCM_CUDA(cudaStreamSynchronize(stream()));
    if (b->host->err) {
        fprintf(stderr, "B200 batch decode: a pipeline wait ran out (bits 0x%x)\n", b->host->err);
        return -4;
    }
    if (tops)
        for (int i = 0; i < n; i++) tops[i] = b->host_log[(size_t)last * kBN + i];
    for (int i = 0; i < n; i++)
        if (b->host->bad[i]) return -3;
    return 0;
}

}  // namespace

extern "C" {

QwenB200Batch *qwen_b200_batch_create(const QwenB200Decoder *d) {
    QwenB200Shape s;
    const QwenB200Layer *layers;
    const void *embed;
    const float *norm, *den;
    int dtype = 0;
    if (!d || decoder_view(d, &s, &layers, &embed, &norm, &den, &dtype) || dtype != 2 || s.hidden != kHd ||
        s.intermediate != kFf || s.qheads != 12 || s.kvheads != 2 || s.head != 128 || s.vocab % 128)
        return nullptr;
    static PerDeviceOnce once;
    once.run([] {
        gemm_setup<EpiQkv>();
        gemm_setup<EpiResid>();
        gemm_setup<EpiSwiglu>();
        gemm_setup<EpiLogits>();
        gemm_setup<EpiStore>();
        TCM_CUDA(cudaFuncSetAttribute(batch_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnSmem));
        TCM_CUDA(cudaFuncSetAttribute(batch_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kTcAttnSmem));
    });
    QwenB200Batch *b = new QwenB200Batch();
    b->d = d;
    b->s = s;
    b->embed_ptr = embed;
    b->final_norm = norm;
    b->rope_den = den;
    auto *lv = new std::vector<QwenB200Layer>(layers, layers + s.layers);
    b->layers = lv;
    for (int l = 0; l < s.layers; l++) {
        const QwenB200Layer &L = layers[l];
        LayerMaps m;
        m.q = bf16_map(L.q, kHd, kHd, 64);
        m.k = bf16_map(L.k, kHd, 256, 64);
        m.v = bf16_map(L.v, kHd, 256, 64);
        m.o = bf16_map(L.o, kHd, kHd, 64);
        m.gate = bf16_map(L.gate, kHd, kFf, 64);
        m.up = bf16_map(L.up, kHd, kFf, 64);
        m.down = bf16_map(L.down, kFf, kHd, 64);
        b->maps.push_back(m);
    }
    b->embed = bf16_map(embed, kHd, (uint64_t)s.vocab, 64);
    b->readout_tiles = s.vocab / 128;
    b->st = (BatchState *)gpu_alloc(sizeof(BatchState));
    gpu_zero(b->st, sizeof(BatchState));
    TCM_CUDA(cudaMallocHost((void **)&b->host, sizeof(BatchState)));
    memset(b->host, 0, sizeof(BatchState));
    b->x = (float *)gpu_alloc((size_t)kBN * kHd * 4);
    b->q = (float *)gpu_alloc((size_t)kBN * kHd * 4);
    b->nh = (uint16_t *)gpu_alloc((size_t)kBN * kHd * 2);
    b->nl = (uint16_t *)gpu_alloc((size_t)kBN * kHd * 2);
    b->hh = (uint16_t *)gpu_alloc((size_t)kBN * kFf * 2);
    b->hl = (uint16_t *)gpu_alloc((size_t)kBN * kFf * 2);
    gpu_zero(b->nh, (size_t)kBN * kHd * 2);
    gpu_zero(b->nl, (size_t)kBN * kHd * 2);
    gpu_zero(b->hh, (size_t)kBN * kFf * 2);
    gpu_zero(b->hl, (size_t)kBN * kFf * 2);
    b->nh_map = bf16_map(b->nh, kHd, kBN, kBN);
    b->nl_map = bf16_map(b->nl, kHd, kBN, kBN);
    b->hh_map = bf16_map(b->hh, kFf, kBN, kBN);
    b->hl_map = bf16_map(b->hl, kFf, kBN, kBN);
    b->part = (float *)gpu_alloc((size_t)16 * 12 * 128 * kBN * 4);
    gpu_zero(b->part, (size_t)16 * 12 * 128 * kBN * 4);  // a stage timed alone may read partials no GEMM wrote
    b->counters = (unsigned *)gpu_alloc(256 * 4);
    gpu_zero(b->counters, 256 * 4);
    b->attn_part = (float *)gpu_alloc((size_t)kBN * 2 * kAttnItemMax * kAttnPartialFloats * 4);
    b->attn_counters = (unsigned *)gpu_alloc((size_t)kBN * 2 * 4);
    gpu_zero(b->attn_counters, (size_t)kBN * 2 * 4);
    b->top_part = (Top2 *)gpu_alloc((size_t)kBN * kTopBlocks * sizeof(Top2));
    b->top_counters = (unsigned *)gpu_alloc(kBN * 4);
    gpu_zero(b->top_counters, kBN * 4);
    // One work counter pair per layer: a launch touches its counters before its
    // dependency wait, so neighbouring layers must not share them.
    b->attn_work = (unsigned *)gpu_alloc((size_t)s.layers * 2 * 4);
    gpu_zero(b->attn_work, (size_t)s.layers * 2 * 4);
    b->attn_item_rows = kTcItemRowsDefault;
    b->attn_kernel = 0;
    b->resid_defer = 1;
    b->cluster_qkv = pick_cluster(16, kHd / kTcKBlock);
    b->cluster_o = pick_cluster(12, kHd / kTcKBlock);
    b->cluster_down = pick_cluster(12, kFf / kTcKBlock);
    b->log = (TcmTop2 *)gpu_alloc(sizeof(TcmTop2) * kBatchLogCap * kBN);
    TCM_CUDA(cudaMallocHost((void **)&b->host_log, sizeof(TcmTop2) * kBatchLogCap * kBN));
    return b;
}

void qwen_b200_batch_free(QwenB200Batch *b) {
    if (!b) return;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    for (auto &g : b->graphs) TCM_CUDA(cudaGraphExecDestroy(g.second));
    void *all[] = {b->st, b->x, b->q, b->nh, b->nl, b->hh, b->hl, b->part, b->counters, b->attn_part,
                   b->attn_counters, b->top_part, b->log, b->top_counters, b->attn_work, b->prefill_logits,
                   b->prefill_x};
    for (void *p : all) gpu_free(p);
    TCM_CUDA(cudaFreeHost(b->host));
    TCM_CUDA(cudaFreeHost(b->host_log));
    delete b->layers;
    delete b;
}

int qwen_b200_batch_max(void) { return kBN; }

int qwen_b200_batch_tune(QwenB200Batch *b, int key, int value) {
    if (!b) return -1;
    if (key == 0 && (value < kAttnItemRowsMin || value > 2048 || value % kAttnRowsPerStage)) return -1;
    if ((key == 1 || key == 2) && value != 0 && value != 1) return -1;
    if (key < 0 || key > 2) return -1;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    for (auto &g : b->graphs) TCM_CUDA(cudaGraphExecDestroy(g.second));
    b->graphs.clear();
    if (key == 0) {  // attention rows per work item
        b->attn_item_rows = value;
    } else if (key == 1) {  // attention kernel, with its own default item size
        b->attn_kernel = value;
        b->attn_item_rows = value == 0 ? kTcItemRowsDefault : 1024;
    } else {  // O and down: K-split sum in the next RMSNorm (1) or in a cluster fold (0)
        b->resid_defer = value;
    }
    return 0;
}

int qwen_b200_batch_cluster_capacity(int size) { return size >= 1 && size <= 16 ? cluster_capacity(size) : -1; }
int qwen_b200_batch_clusters(const QwenB200Batch *b, int *qkv, int *o, int *down) {
    if (!b) return -1;
    *qkv = b->cluster_qkv;
    *o = b->cluster_o;
    *down = b->cluster_down;
    return 0;
}

float qwen_b200_batch_time_stage(QwenB200Batch *b, int n, const QwenB200BatchSession *sessions, const int *tokens,
                                 const int *positions, int stage, int layer, int reps);

int qwen_b200_batch_trace_stage(QwenB200Batch *b, int n, const QwenB200BatchSession *sessions, const int *tokens,
                                const int *positions, int stage, int layer, unsigned long long *host, int ctas) {
    if (!b || !host || ctas < 1 || ctas > 1024) return -1;
    const size_t bytes = (size_t)1024 * 8 * sizeof(unsigned long long);
    b->trace = (unsigned long long *)gpu_alloc(bytes);
    gpu_zero(b->trace, bytes);
    const float ms = qwen_b200_batch_time_stage(b, n, sessions, tokens, positions, stage, layer, 1);
    gpu_read(host, b->trace, (size_t)ctas * 8 * sizeof(unsigned long long));
    gpu_free(b->trace);
    b->trace = nullptr;
    return ms < 0.f ? -1 : 0;
}

float qwen_b200_batch_time_stage(QwenB200Batch *b, int n, const QwenB200BatchSession *sessions, const int *tokens,
                                 const int *positions, int stage, int layer, int reps) {
    if (!b || stage < 0 || stage > 6 || layer < 0 || layer >= b->s.layers || reps < 1 ||
        !load_sessions(b, n, sessions, tokens, positions))
        return -1.f;
    const std::vector<QwenB200Layer> &L = *b->layers;
    const LayerMaps &m = b->maps[layer];
    auto once = [&]() {
        switch (stage) {
            case 0: {
                launch_qkv(b, layer, false);
                break;
            }
            case 1: {
                launch_attention(b, layer, n, b->trace, false);
                break;
            }
            case 2: {
                EpiResid o = {b->st, b->x};
                launch_split(b, m.o, m.o, m.o, b->nh_map, b->nl_map, 12, kHd / kTcKBlock, o, false, b->cluster_o,
                             b->resid_defer ? kResidSplits : 0);
                break;
            }
            case 3: {
                EpiSwiglu sw = {b->st, b->hh, b->hl};
                launch_gemm(b, m.gate, m.up, m.up, b->nh_map, b->nl_map, kFf / 64, 1, kHd / kTcKBlock, sw, false);
                break;
            }
            case 4: {
                EpiResid dn = {b->st, b->x};
                launch_split(b, m.down, m.down, m.down, b->hh_map, b->hl_map, 12, kFf / kTcKBlock, dn, false,
                             b->cluster_down, b->resid_defer ? kResidSplits : 0);
                break;
            }
            case 5: {
                EpiLogits lg = {b->st};
                launch_gemm(b, b->embed, b->embed, b->embed, b->nh_map, b->nl_map, b->readout_tiles, 1,
                            kHd / kTcKBlock, lg, false);
                break;
            }
            default: launch_rms(b, L[layer].post_norm, false, false, false, b->resid_defer != 0); break;
        }
    };
    once();
    cudaEvent_t e0, e1;
    TCM_CUDA(cudaEventCreate(&e0));
    TCM_CUDA(cudaEventCreate(&e1));
    TCM_CUDA(cudaEventRecord(e0, stream()));
    for (int i = 0; i < reps; i++) once();
    TCM_CUDA(cudaEventRecord(e1, stream()));
    TCM_CUDA(cudaEventSynchronize(e1));
    float ms = 0.f;
    TCM_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    TCM_CUDA(cudaEventDestroy(e0));
    TCM_CUDA(cudaEventDestroy(e1));
    return ms / reps;
}

int qwen_b200_batch_matmul(const void *w, int rows, int in, const float *x, int n, float *y, int splits) {
    if (!w || !x || !y || rows < 128 || rows % 128 || in < 64 || in % 64 || n < 1 || n > kBN || splits < 1 ||
        splits > in / 64 || (rows / 128) * splits > 4096)
        return -1;
    static std::once_flag once;
    std::call_once(once, [] { gemm_setup<EpiStore>(); });
    uint16_t *xh = (uint16_t *)gpu_alloc((size_t)kBN * in * 2), *xl = (uint16_t *)gpu_alloc((size_t)kBN * in * 2);
    gpu_zero(xh, (size_t)kBN * in * 2);
    gpu_zero(xl, (size_t)kBN * in * 2);
    split_rows_kernel<<<sm_count(), 256, 0, stream()>>>(x, xh, xl, (size_t)n * in);
    TCM_CUDA(cudaGetLastError());
    const int tiles = rows / 128;
    float *part = (float *)gpu_alloc((size_t)tiles * splits * 128 * kBN * 4);
    unsigned *counters = (unsigned *)gpu_alloc((size_t)tiles * 4), *err = (unsigned *)gpu_alloc(4);
    gpu_zero(counters, (size_t)tiles * 4);
    gpu_zero(err, 4);
    TcArgs<kBN, EpiStore> a;
    a.a[0] = a.a[1] = a.a[2] = bf16_map(w, (uint64_t)in, (uint64_t)rows, 64);
    a.xh = bf16_map(xh, (uint64_t)in, kBN, kBN);
    a.xl = bf16_map(xl, (uint64_t)in, kBN, kBN);
    a.tiles = tiles;
    a.splits = splits;
    a.kblocks = in / 64;
    a.cluster = 1;
    a.defer = 0;
    a.part = part;
    a.counters = counters;
    a.err = err;
    a.trace = nullptr;
    a.epi = EpiStore{y, rows, n};
    const int items = tiles * splits, grid = items < sm_count() ? items : sm_count();
    launch(tc_gemm_kernel<kBN, EpiStore>, dim3(grid), dim3(kTcThreads), TcGeo<kBN>::kSmem, stream(), false, a);
    unsigned bits = 0;
    gpu_read(&bits, err, 4);
    for (void *p : {(void *)xh, (void *)xl, (void *)part, (void *)counters, (void *)err}) gpu_free(p);
    if (bits) {
        fprintf(stderr, "qwen_b200_batch_matmul: a pipeline wait ran out (bits 0x%x)\n", bits);
        return -4;
    }
    return 0;
}
int qwen_b200_batch_launches_per_step(const QwenB200Batch *b) {
    // First RMSNorm; per layer q/k/v, attention (+ its merge), O, RMSNorm,
    // gate/up, down, and the next RMSNorm (the final one after the last
    // layer); vocabulary GEMM, top-2, step end.
    return b ? 1 + b->s.layers * (7 + (b->attn_kernel == 0 ? 1 : 0)) + 3 : 0;
}

int qwen_b200_batch_step(QwenB200Batch *b, int n, const QwenB200BatchSession *sessions, const int *tokens,
                         const int *positions, TcmTop2 *tops) {
    if (!b || !load_sessions(b, n, sessions, tokens, positions)) return -1;
    TCM_CUDA(cudaGraphLaunch(graph_for(b, n), stream()));
    return read_back(b, n, 1, tops);
}

int qwen_b200_batch_prefill(QwenB200Batch *b, const QwenB200BatchSession *session, const int *tokens, int n,
                            int position, TcmTop2 *top) {
    if (!b || !session || !tokens || n < 1 || n > kBN || position < 0 || position + n > session->capacity ||
        position + n > kAttnSplitMax * kAttnChunk)
        return -1;
    if (!b->prefill_logits) {
        b->prefill_logits = (float *)gpu_alloc((size_t)(kBN - 1) * b->s.vocab * sizeof(float));
        b->prefill_x = (float *)gpu_alloc((size_t)(kBN - 1) * kHd * sizeof(float));
    }
    // Slot i is token i at position + i in the session's own cache: the q/k/v
    // epilogue appends every slot's row before the attention kernel reads rows
    // 0..position + i, so the step is causal over the chunk.
    QwenB200BatchSession ss[kBN];
    int pos[kBN];
    TcmTop2 tops[kBN];
    for (int i = 0; i < n; i++) {
        ss[i] = *session;
        if (i < n - 1) {
            ss[i].logits = b->prefill_logits + (size_t)i * b->s.vocab;
            ss[i].x = b->prefill_x + (size_t)i * kHd;
        }
        pos[i] = position + i;
    }
    const int status = qwen_b200_batch_step(b, n, ss, tokens, pos, tops);
    if (status == 0 && top) *top = tops[n - 1];
    return status;
}

int qwen_b200_batch_enqueue(QwenB200Batch *b, int n, const QwenB200BatchSession *sessions, const int *tokens,
                            const int *positions, int steps) {
    if (!b || steps < 1 || steps > kBatchLogCap || !load_sessions(b, n, sessions, tokens, positions)) return -1;
    for (int i = 0; i < n; i++)
        if (positions[i] + steps > sessions[i].capacity || positions[i] + steps > kAttnSplitMax * kAttnChunk) return -1;
    cudaGraphExec_t g = graph_for(b, n);
    for (int i = 0; i < steps; i++) TCM_CUDA(cudaGraphLaunch(g, stream()));
    return 0;
}

int qwen_b200_batch_read(QwenB200Batch *b, int n, int steps, TcmTop2 *tops, TcmTop2 *history) {
    if (!b || n < 1 || n > kBN || steps < 1 || steps > kBatchLogCap) return -1;
    const int status = read_back(b, n, steps, tops, history != nullptr);
    if (history)
        for (int t = 0; t < steps; t++)
            for (int i = 0; i < n; i++) history[(size_t)t * n + i] = b->host_log[(size_t)t * kBN + i];
    return status;
}

}  // extern "C"
