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
constexpr int kAttnSplitMax = 32;   // up to 8192 cached rows
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
};
__global__ void __launch_bounds__(256) batch_rms_kernel(RmsArgs a) {
    __shared__ float red[8];
    pdl_trigger();
    pdl_wait();
    const int n = blockIdx.x, tid = threadIdx.x;
    if (n >= a.st->n) return;
    float v[kHd / 256];
    float *x = a.x + (size_t)n * kHd;
    if (a.embed) {
        const uint16_t *row = a.embed + (size_t)a.st->token[n] * kHd;
#pragma unroll
        for (int i = 0; i < kHd / 256; i++) {
            v[i] = __uint_as_float((uint32_t)row[tid + 256 * i] << 16);
            x[tid + 256 * i] = v[i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < kHd / 256; i++) v[i] = x[tid + 256 * i];
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kHd / 256; i++) ss = fmaf(v[i], v[i], ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++) total += red[w];
    const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)kHd), a.eps)));
#pragma unroll
    for (int i = 0; i < kHd / 256; i++) {
        const int j = tid + 256 * i;
        uint16_t h, l;
        split_bf16(__fmul_rn(__fmul_rn(v[i], r), a.w[j]), h, l);
        a.hi[(size_t)n * kHd + j] = h;
        a.lo[(size_t)n * kHd + j] = l;
        if (a.copy_x) a.st->x[n][j] = v[i];
    }
}

// ---------------------------------------------------------------- GEMM epilogues
// q/k/v: tiles 0..11 are the 12 query heads, 12..13 the K heads, 14..15 the V
// heads; a head is exactly one 128-row tile, so RoPE pairs (d, d + 64) meet in
// the tile. The rotation repeats the single-session kernel's arithmetic.
struct EpiQkv {
    BatchState *st;
    const float *bq, *bk, *bv, *rope_den;
    float *q;       // [kBN][1536]
    int layer;
    __device__ TcRows a_rows(int t) const {
        const int m = t < 12 ? 0 : (t < 14 ? 1 : 2), r = (t < 12 ? t : (t < 14 ? t - 12 : t - 14)) * 128;
        return TcRows{m, r, m, r + 64};
    }
    template <int NP> __device__ void store(int t, const float (*tile)[NP], int e) const {
        const int kind = t < 12 ? 0 : (t < 14 ? 1 : 2), head = t < 12 ? t : (t < 14 ? t - 12 : t - 14);
        const float *bias = (kind == 0 ? bq : kind == 1 ? bk : bv) + head * 128;
        const int n_active = st->n;
        for (int idx = e; idx < 64 * n_active; idx += 128) {
            const int d = idx & 63, n = idx >> 6;
            float y0 = __fadd_rn(tile[d][n], bias[d]), y1 = __fadd_rn(tile[d + 64][n], bias[d + 64]);
            const int pos = st->position[n];
            if (kind < 2) {
                const float angle = __fdiv_rn((float)pos, rope_den[d]);
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
                const int cap = st->capacity[n];
                float *cache = (kind == 1 ? st->keys[n] : st->values[n]) + ((size_t)layer * 2 + head) * cap * 128 +
                               (size_t)pos * 128;
                cache[d] = y0;
                cache[d + 64] = y1;
            }
        }
    }
};
// x += D (the O and down projections): tile rows are output rows t*128 ...
struct EpiResid {
    BatchState *st;
    float *x;
    __device__ TcRows a_rows(int t) const { return TcRows{0, t * 128, 0, t * 128 + 64}; }
    template <int NP> __device__ void store(int t, const float (*tile)[NP], int e) const {
        const int n_active = st->n;
        for (int idx = e; idx < 128 * n_active; idx += 128) {
            const int r = idx & 127, n = idx >> 7;
            float *p = x + (size_t)n * kHd + t * 128 + r;
            *p = __fadd_rn(*p, tile[r][n]);
        }
    }
};
// gate rows t*64.. in tile rows 0..63, up rows t*64.. in 64..127; h = silu(g) u
// as g / (1 + exp(-g)) * u (src/qwen_cuda.cu:79), stored as BF16 hi/lo.
struct EpiSwiglu {
    BatchState *st;
    uint16_t *hh, *hl;   // [kBN][8960]
    __device__ TcRows a_rows(int t) const { return TcRows{0, t * 64, 1, t * 64}; }
    template <int NP> __device__ void store(int t, const float (*tile)[NP], int e) const {
        const int n_active = st->n;
        for (int idx = e; idx < 64 * n_active; idx += 128) {
            const int i = idx & 63, n = idx >> 6;
            const float g = tile[i][n], u = tile[i + 64][n];
            const float h = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
            uint16_t hi, lo;
            split_bf16(h, hi, lo);
            hh[(size_t)n * kFf + t * 64 + i] = hi;
            hl[(size_t)n * kFf + t * 64 + i] = lo;
        }
    }
};
// Logits to each session's buffer, and the tile's top-2 per session.
struct EpiLogits {
    BatchState *st;
    Top2 *part;   // [tiles][kBN]
    __device__ TcRows a_rows(int t) const { return TcRows{0, t * 128, 0, t * 128 + 64}; }
    template <int NP> __device__ void store(int t, const float (*tile)[NP], int e) const {
        const int n_active = st->n;
        for (int idx = e; idx < 128 * n_active; idx += 128) {
            const int r = idx & 127, n = idx >> 7;
            st->logits[n][t * 128 + r] = tile[r][n];
        }
        const int warp = e >> 5, lane = e & 31;
        for (int n = warp; n < n_active; n += 4) {
            Top2 z = top2_empty();
            bool bad = false;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float v = tile[lane + 32 * j][n];
                bad |= !isfinite(v);
                top2_insert(z, v, t * 128 + lane + 32 * j);
            }
            top2_merge_warp(z);
            if (__any_sync(0xffffffffu, bad) && lane == 0) st->bad[n] = 1;
            if (lane == 0) part[(size_t)t * kBN + n] = z;
        }
    }
};

// y[n][t*128 + r] = D (the plain batched matmul).
struct EpiStore {
    float *y;
    int rows, n;
    __device__ TcRows a_rows(int t) const { return TcRows{0, t * 128, 0, t * 128 + 64}; }
    template <int NP> __device__ void store(int t, const float (*tile)[NP], int e) const {
        for (int idx = e; idx < 128 * n; idx += 128) {
            const int r = idx & 127, c = idx >> 7;
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
struct AttnArgs {
    BatchState *st;
    const float *q;        // [kBN][1536]
    int layer;
    float inv_sqrt_dim;
    float *part;           // [kBN][2][kAttnSplitMax][kAttnPartialFloats]
    unsigned *counters;    // [kBN][2]
    uint16_t *oh, *ol;     // [kBN][1536]
};
__global__ void __launch_bounds__(kDecodeAttnThreads, 2) batch_attn_kernel(AttnArgs a) {
    constexpr int G = 6;
    __shared__ float wm[kDecodeAttnWarps][G], wl[kDecodeAttnWarps][G];
    __shared__ __align__(16) float wacc[kDecodeAttnWarps][G][kHeadDim];
    __shared__ int last_s;
    const int s = blockIdx.x, h = blockIdx.y, n = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_trigger();
    // The state block is written before the step: the split needs no wait.
    if (n >= a.st->n) return;
    const int L = a.st->position[n] + 1, splits = (L + kAttnChunk - 1) / kAttnChunk;
    if (s >= splits) return;
    const int cap = a.st->capacity[n];
    DenseRows rows = {};
    rows.keys = a.st->keys[n] + (size_t)a.layer * 2 * cap * kHeadDim;
    rows.values = a.st->values[n] + (size_t)a.layer * 2 * cap * kHeadDim;
    rows.capacity = cap;
    rows.position = &a.st->position[n];
    rows.bind(h);
    const int t0 = s * kAttnChunk, t1 = min(L, t0 + kAttnChunk);
    const int per_warp = kAttnChunk / kDecodeAttnWarps;
    const int r0 = min(t1, t0 + warp * per_warp), r1 = min(t1, r0 + per_warp);
    for (int t = r0 + (lane >> 2); t < min(r1, L - 1); t += 8) rows.prefetch_line(t, lane & 3);
    pdl_wait();
    float4 q4[G], acc[G];
#pragma unroll
    for (int g = 0; g < G; g++) q4[g] = reinterpret_cast<const float4 *>(a.q + (size_t)n * kHd + (h * G + g) * kHeadDim)[lane];
    float m[G], l[G];
    flash_rows<G>(rows, r0, r1, q4, lane, a.inv_sqrt_dim, m, l, acc);
    float *hp = a.part + ((size_t)n * 2 + h) * kAttnSplitMax * kAttnPartialFloats;
    cta_merge<G>(m, l, acc, wm, wl, wacc, hp + (size_t)s * kAttnPartialFloats, nullptr);
    __threadfence();
    __syncthreads();
    unsigned *counter = &a.counters[n * 2 + h];
    if (tid == 0) last_s = atomicAdd(counter, 1u) == (unsigned)(splits - 1);
    __syncthreads();
    if (!last_s) return;
    __threadfence();
    for (int o = tid; o < G * kHeadDim; o += kDecodeAttnThreads) {
        const int g = o / kHeadDim, d = o % kHeadDim;
        float M = -INFINITY;
        for (int c = 0; c < splits; c++) M = fmaxf(M, __ldcg(hp + (size_t)c * kAttnPartialFloats + g));
        float num = 0.f, den = 0.f;
        for (int c = 0; c < splits; c++) {
            const float *pc = hp + (size_t)c * kAttnPartialFloats;
            const float mc = __ldcg(pc + g);
            if (mc == -INFINITY) continue;
            const float e = expf(mc - M);
            den = fmaf(e, __ldcg(pc + kAttnMaxGroup + g), den);
            num = fmaf(e, __ldcg(pc + 2 * kAttnMaxGroup + g * kHeadDim + d), num);
        }
        uint16_t hi, lo;
        split_bf16(__fdiv_rn(num, den), hi, lo);
        a.oh[(size_t)n * kHd + (h * G + g) * kHeadDim + d] = hi;
        a.ol[(size_t)n * kHd + (h * G + g) * kHeadDim + d] = lo;
    }
    if (tid == 0) *counter = 0u;
}

// ---------------------------------------------------------------- top-2 per session
struct Top2Args {
    BatchState *st;
    const Top2 *part;  // [tiles][kBN]
    int tiles;
    TcmTop2 *log;      // [kBatchLogCap][kBN]
};
__global__ void __launch_bounds__(256) batch_top2_kernel(Top2Args a) {
    __shared__ Top2 sh[8];
    pdl_trigger();
    pdl_wait();
    const int n = blockIdx.x, tid = threadIdx.x;
    if (n >= a.st->n) return;
    Top2 z = top2_empty();
    for (int t = tid; t < a.tiles; t += 256) {
        const Top2 p = a.part[(size_t)t * kBN + n];
        top2_insert(z, p.a, p.ai);
        top2_insert(z, p.b, p.bi);
    }
    top2_merge_warp(z);
    if ((tid & 31) == 0) sh[tid >> 5] = z;
    __syncthreads();
    if (tid == 0) {
        Top2 f = sh[0];
        for (int w = 1; w < 8; w++) {
            top2_insert(f, sh[w].a, sh[w].ai);
            top2_insert(f, sh[w].b, sh[w].bi);
        }
        TcmTop2 top;
        top.first = f.ai; top.second = f.bi; top.first_value = f.a; top.second_value = f.b;
        a.log[(size_t)(a.st->step % kBatchLogCap) * kBN + n] = top;
        a.st->token[n] = f.ai;
        a.st->position[n] += 1;
    }
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
}

}  // namespace

// The BF16 weights' maps of one layer.
struct LayerMaps {
    CUtensorMap q, k, v, o, gate, up, down;
};

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
    unsigned *counters, *attn_counters;
    Top2 *top_part;
    TcmTop2 *log, *host_log;
    int readout_tiles;
    std::map<int, cudaGraphExec_t> graphs;
    int launches;
};

namespace {

template <class Epi>
void launch_gemm(QwenB200Batch *b, const CUtensorMap &a0, const CUtensorMap &a1, const CUtensorMap &a2,
                 const CUtensorMap &xh, const CUtensorMap &xl, int tiles, int splits, int kblocks, const Epi &epi,
                 bool pdl) {
    TcArgs<kBN, Epi> args;
    args.a[0] = a0;
    args.a[1] = a1;
    args.a[2] = a2;
    args.xh = xh;
    args.xl = xl;
    args.tiles = tiles;
    args.splits = splits;
    args.kblocks = kblocks;
    args.part = b->part;
    args.counters = b->counters;
    args.err = &b->st->err;
    args.trace = nullptr;
    args.epi = epi;
    const int items = tiles * splits, grid = items < sm_count() ? items : sm_count();
    launch(tc_gemm_kernel<kBN, Epi>, dim3(grid), dim3(kTcThreads), TcGeo<kBN>::kSmem, stream(), pdl, args);
}

void launch_rms(QwenB200Batch *b, const float *w, bool embed, bool copy_x, bool pdl) {
    RmsArgs a = {b->st, b->x, w, b->nh, b->nl, embed ? (const uint16_t *)b->embed_ptr : nullptr, b->s.epsilon,
                 copy_x ? 1 : 0};
    launch(batch_rms_kernel, dim3(kBN), dim3(256), 0, stream(), pdl, a);
}

void launch_step(QwenB200Batch *b, int n) {
    const QwenB200Shape &s = b->s;
    const std::vector<QwenB200Layer> &L = *b->layers;
    launch_rms(b, L[0].input_norm, true, false, false);
    for (int l = 0; l < s.layers; l++) {
        const LayerMaps &m = b->maps[l];
        EpiQkv qkv = {b->st, L[l].qb, L[l].kb, L[l].vb, b->rope_den, b->q, l};
        launch_gemm(b, m.q, m.k, m.v, b->nh_map, b->nl_map, 16, 9, kHd / kTcKBlock, qkv, true);
        AttnArgs at = {b->st, b->q, l, 1.0f / sqrtf((float)kHeadDim), b->attn_part, b->attn_counters, b->nh, b->nl};
        launch(batch_attn_kernel, dim3(kAttnSplitMax, 2, n), dim3(kDecodeAttnThreads), 0, stream(), true, at);
        EpiResid o = {b->st, b->x};
        launch_gemm(b, m.o, m.o, m.o, b->nh_map, b->nl_map, 12, 12, kHd / kTcKBlock, o, true);
        launch_rms(b, L[l].post_norm, false, false, true);
        EpiSwiglu sw = {b->st, b->hh, b->hl};
        launch_gemm(b, m.gate, m.up, m.up, b->nh_map, b->nl_map, kFf / 64, 1, kHd / kTcKBlock, sw, true);
        EpiResid dn = {b->st, b->x};
        launch_gemm(b, m.down, m.down, m.down, b->hh_map, b->hl_map, 12, 12, kFf / kTcKBlock, dn, true);
        if (l + 1 < s.layers) launch_rms(b, L[l + 1].input_norm, false, false, true);
    }
    launch_rms(b, b->final_norm, false, true, true);
    EpiLogits lg = {b->st, b->top_part};
    launch_gemm(b, b->embed, b->embed, b->embed, b->nh_map, b->nl_map, b->readout_tiles, 1, kHd / kTcKBlock, lg, true);
    Top2Args ta = {b->st, b->top_part, b->readout_tiles, b->log};
    launch(batch_top2_kernel, dim3(n), dim3(256), 0, stream(), true, ta);
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

int read_back(QwenB200Batch *b, int n, int steps, TcmTop2 *tops) {
    TCM_CUDA(cudaMemcpyAsync(b->host, b->st, sizeof(BatchState), cudaMemcpyDeviceToHost, stream()));
    TCM_CUDA(cudaMemcpyAsync(b->host_log, b->log, sizeof(TcmTop2) * kBatchLogCap * kBN, cudaMemcpyDeviceToHost,
                             stream()));
    TCM_CUDA(cudaStreamSynchronize(stream()));
    if (b->host->err) {
        fprintf(stderr, "B200 batch decode: a pipeline wait ran out (bits 0x%x)\n", b->host->err);
        return -4;
    }
    if (tops) {
        const int last = (steps - 1) % kBatchLogCap;
        for (int i = 0; i < n; i++) tops[i] = b->host_log[(size_t)last * kBN + i];
    }
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
    static std::once_flag once;
    std::call_once(once, [] {
        gemm_setup<EpiQkv>();
        gemm_setup<EpiResid>();
        gemm_setup<EpiSwiglu>();
        gemm_setup<EpiLogits>();
        gemm_setup<EpiStore>();
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
    b->counters = (unsigned *)gpu_alloc(256 * 4);
    gpu_zero(b->counters, 256 * 4);
    b->attn_part = (float *)gpu_alloc((size_t)kBN * 2 * kAttnSplitMax * kAttnPartialFloats * 4);
    b->attn_counters = (unsigned *)gpu_alloc((size_t)kBN * 2 * 4);
    gpu_zero(b->attn_counters, (size_t)kBN * 2 * 4);
    b->top_part = (Top2 *)gpu_alloc((size_t)b->readout_tiles * kBN * sizeof(Top2));
    b->log = (TcmTop2 *)gpu_alloc(sizeof(TcmTop2) * kBatchLogCap * kBN);
    TCM_CUDA(cudaMallocHost((void **)&b->host_log, sizeof(TcmTop2) * kBatchLogCap * kBN));
    b->launches = 1 + s.layers * 7 + 3;
    return b;
}

void qwen_b200_batch_free(QwenB200Batch *b) {
    if (!b) return;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    for (auto &g : b->graphs) TCM_CUDA(cudaGraphExecDestroy(g.second));
    void *all[] = {b->st, b->x, b->q, b->nh, b->nl, b->hh, b->hl, b->part, b->counters, b->attn_part,
                   b->attn_counters, b->top_part, b->log};
    for (void *p : all) gpu_free(p);
    TCM_CUDA(cudaFreeHost(b->host));
    TCM_CUDA(cudaFreeHost(b->host_log));
    delete b->layers;
    delete b;
}

int qwen_b200_batch_max(void) { return kBN; }

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
int qwen_b200_batch_launches_per_step(const QwenB200Batch *b) { return b ? b->launches : 0; }

int qwen_b200_batch_step(QwenB200Batch *b, int n, const QwenB200BatchSession *sessions, const int *tokens,
                         const int *positions, TcmTop2 *tops) {
    if (!b || !load_sessions(b, n, sessions, tokens, positions)) return -1;
    TCM_CUDA(cudaGraphLaunch(graph_for(b, n), stream()));
    return read_back(b, n, 1, tops);
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
    const int status = read_back(b, n, steps, tops);
    if (history)
        for (int t = 0; t < steps; t++)
            for (int i = 0; i < n; i++) history[(size_t)t * n + i] = b->host_log[(size_t)t * kBN + i];
    return status;
}

}  // extern "C"
