// Fused batch-1 decode for the Qwen2.5 decoder on B200 (sm_100a).
//
// Per layer five kernels, per token one readout kernel; all of them launched
// with programmatic dependent launch so that each kernel's CTAs are resident
// and prefetching their weight rows into L2 while the previous kernel drains,
// and a whole token is captured once as a CUDA graph. Every kernel is a
// warp-per-row GEMV streaming its weights from HBM exactly once (see gemv.cuh)
// with the neighbouring elementwise work fused into its prologue/epilogue.
// Reference equations: src/qwen.c:248-262,275,289,320,329-330,341,383-387.
#include "common.cuh"
#include "gemv.cuh"
#include "attention.cuh"
#include "kernels.h"
#include "../../include/qwen_b200.h"
#include "../../include/tcm_seeded.h"
#include <mutex>
#include <vector>

namespace tcm {

// Device-resident token state: the host writes token/position before a token;
// the readout's last CTA publishes the top-2 and, for chained greedy decode,
// feeds top-1 back as the next token and advances the position.
struct DecodeState {
    int token, position, step, invalid;
    TcmTop2 top;
};
constexpr int kLogCap = 4096;

namespace {

constexpr int kBlock = 256;

// ------------------------------------------------------------------ stage 1
struct QkvArgs {
    const void *wq, *wk, *wv, *embed;
    const float *bq, *bk, *bv, *norm, *rope_den;
    float *x, *q, *k, *v, *kcache, *vcache;
    const DecodeState *st;
    int hidden, qheads, kvheads, capacity;
    float eps;
};

// Task t = (head, d), head over q | k | v heads, d < 64: the warp computes rows
// d and d + 64 of that head, adds the bias, rotates the pair (RoPE, q and k
// only) and stores q, or k/v plus the cache row at the current position.
template <typename WT, int UNROLL>
__global__ void __launch_bounds__(kBlock) qkv_kernel(QkvArgs a) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float red[32];
    const int lane = threadIdx.x & 31;
    const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
    const int tasks = (a.qheads + 2 * a.kvheads) * 64;
    const int nvec = a.hidden / WVec<WT>::kElems;
    auto rows_of = [&](int task, const WT *(&rows)[2], const float *&bias, int &kind, int &hl, int &r0) {
        const int head = task >> 6, d = task & 63;
        const WT *base;
        if (head < a.qheads) { base = (const WT *)a.wq; bias = a.bq; kind = 0; hl = head; }
        else if (head < a.qheads + a.kvheads) { base = (const WT *)a.wk; bias = a.bk; kind = 1; hl = head - a.qheads; }
        else { base = (const WT *)a.wv; bias = a.bv; kind = 2; hl = head - a.qheads - a.kvheads; }
        r0 = hl * kHeadDim + d;
        rows[0] = base + (size_t)r0 * a.hidden;
        rows[1] = base + (size_t)(r0 + 64) * a.hidden;
    };
    if (gwarp < tasks) {
        const WT *rows[2]; const float *bias; int kind, hl, r0;
        rows_of(gwarp, rows, bias, kind, hl, r0);
        prefetch_row_l2(rows[0], (size_t)a.hidden * sizeof(WT), lane);
        prefetch_row_l2(rows[1], (size_t)a.hidden * sizeof(WT), lane);
    }
    pdl_wait();
    pdl_trigger();
    const int pos = a.st->position;
    // Stage the layer input (the token's embedding row for layer 0) and its RMS norm.
    float ss = 0.f;
    if (a.embed) {
        const size_t off = (size_t)a.st->token * a.hidden;
        for (int i = threadIdx.x; i < a.hidden; i += blockDim.x) {
            float v;
            if constexpr (sizeof(WT) == 4) v = ((const float *)a.embed)[off + i];
            else v = __uint_as_float((uint32_t)((const uint16_t *)a.embed)[off + i] << 16);
            xs[i] = v;
            if (blockIdx.x == 0) a.x[i] = v;
            ss = fmaf(v, v, ss);
        }
    } else {
        for (int i = threadIdx.x; i < a.hidden; i += blockDim.x) {
            const float v = a.x[i];
            xs[i] = v;
            ss = fmaf(v, v, ss);
        }
    }
    const float total = block_sum(ss, red);
    const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)a.hidden), a.eps)));
    for (int i = threadIdx.x; i < a.hidden; i += blockDim.x) xs[i] = __fmul_rn(__fmul_rn(xs[i], r), a.norm[i]);
    __syncthreads();
    for (int task = gwarp; task < tasks; task += nwarps) {
        const WT *rows[2]; const float *bias; int kind, hl, r0;
        rows_of(task, rows, bias, kind, hl, r0);
        float acc[2];
        warp_rows_dot<WT, 2, UNROLL>(rows, xs, nvec, lane, acc);
        if (lane == 0) {
            float y0 = __fadd_rn(acc[0], bias[r0]), y1 = __fadd_rn(acc[1], bias[r0 + 64]);
            if (kind < 2) {
                const float angle = __fdiv_rn((float)pos, a.rope_den[task & 63]);
                float sn, cs;
                sincosf(angle, &sn, &cs);
                const float t0 = __fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn));
                const float t1 = __fadd_rn(__fmul_rn(y1, cs), __fmul_rn(y0, sn));
                y0 = t0;
                y1 = t1;
            }
            float *dst = kind == 0 ? a.q : kind == 1 ? a.k : a.v;
            dst[r0] = y0;
            dst[r0 + 64] = y1;
            float *cache = kind == 1 ? a.kcache : kind == 2 ? a.vcache : nullptr;
            if (cache && pos >= 0 && pos < a.capacity) {
                float *row = cache + ((size_t)hl * a.capacity + pos) * kHeadDim;
                row[task & 63] = y0;
                row[(task & 63) + 64] = y1;
            }
        }
    }
}

// ------------------------------------------------------------------ stages 3 and 5
// x[row] += W[row] . in  (O projection over the attention output, and the down
// projection over the SwiGLU output).
struct ResidualArgs {
    const void *w;
    const float *in;
    float *x;
    int in_dim, out_dim;
};
// KSPLIT warps share one row, each streaming a contiguous 1/KSPLIT of it; the
// partial sums meet in shared memory and are added in split order.
template <typename WT, int KSPLIT, int UNROLL>
__global__ void __launch_bounds__(kBlock) residual_gemv_kernel(ResidualArgs a) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float part[kBlock / 32];
    constexpr int kRowsPerCta = (kBlock / 32) / KSPLIT;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int local = warp / KSPLIT, piece = warp % KSPLIT;
    const WT *w = (const WT *)a.w;
    const int nvec = a.in_dim / WVec<WT>::kElems;
    const int per = (nvec + KSPLIT - 1) / KSPLIT;
    const int v0 = min(nvec, piece * per), v1 = min(nvec, v0 + per);
    const size_t piece_bytes = (size_t)(v1 - v0) * 16;
    {
        const int row = blockIdx.x * kRowsPerCta + local;
        if (row < a.out_dim)
            prefetch_row_l2(w + (size_t)row * a.in_dim + (size_t)v0 * WVec<WT>::kElems, piece_bytes, lane);
    }
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < a.in_dim; i += blockDim.x) xs[i] = a.in[i];
    __syncthreads();
    for (int base = blockIdx.x * kRowsPerCta; base < a.out_dim; base += gridDim.x * kRowsPerCta) {
        const int row = base + local;
        float acc[1] = {0.f};
        if (row < a.out_dim) {
            const WT *rows[1] = {w + (size_t)row * a.in_dim + (size_t)v0 * WVec<WT>::kElems};
            warp_rows_partial<WT, 1, UNROLL>(rows, xs + (size_t)v0 * WVec<WT>::kElems, v1 - v0, lane, acc);
            acc[0] = warp_sum(acc[0]);
        }
        if (KSPLIT == 1) {
            if (lane == 0 && row < a.out_dim) a.x[row] = __fadd_rn(a.x[row], acc[0]);
        } else {
            if (lane == 0) part[warp] = acc[0];
            __syncthreads();
            if (piece == 0 && lane == 0 && row < a.out_dim) {
                float sum = part[warp];
#pragma unroll
                for (int k = 1; k < KSPLIT; k++) sum = __fadd_rn(sum, part[warp + k]);
                a.x[row] = __fadd_rn(a.x[row], sum);
            }
            __syncthreads();
        }
    }
}

// ------------------------------------------------------------------ stage 4
struct GateUpArgs {
    const void *wg, *wu;
    const float *norm, *x;
    float *h;
    int hidden, inter;
    float eps;
};
template <typename WT, int UNROLL>
__global__ void __launch_bounds__(kBlock) gateup_kernel(GateUpArgs a) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float red[32];
    const int lane = threadIdx.x & 31;
    const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
    const WT *wg = (const WT *)a.wg, *wu = (const WT *)a.wu;
    if (gwarp < a.inter) {
        prefetch_row_l2(wg + (size_t)gwarp * a.hidden, (size_t)a.hidden * sizeof(WT), lane);
        prefetch_row_l2(wu + (size_t)gwarp * a.hidden, (size_t)a.hidden * sizeof(WT), lane);
    }
    pdl_wait();
    pdl_trigger();
    stage_rms(xs, a.x, a.norm, a.hidden, a.eps, red);
    const int nvec = a.hidden / WVec<WT>::kElems;
    for (int j = gwarp; j < a.inter; j += nwarps) {
        const WT *rows[2] = {wg + (size_t)j * a.hidden, wu + (size_t)j * a.hidden};
        float acc[2];
        warp_rows_dot<WT, 2, UNROLL>(rows, xs, nvec, lane, acc);
        if (lane == 0) a.h[j] = __fmul_rn(__fdiv_rn(acc[0], __fadd_rn(1.f, expf(-acc[0]))), acc[1]);
    }
}

// ------------------------------------------------------------------ readout
struct ReadoutArgs {
    const void *embed;
    const float *norm, *x;
    float *logits;
    float *pv;
    int *pi;
    unsigned *sync;  // [0] block counter, [1] non-finite flag
    DecodeState *st;
    TcmTop2 *log;
    int hidden, vocab;
    float eps;
};
template <typename WT, int UNROLL>
__global__ void __launch_bounds__(kBlock) readout_kernel(ReadoutArgs a) {
    extern __shared__ __align__(16) float xs[];
    __shared__ float red[32];
    __shared__ float sv[2 * 32];
    __shared__ int si[2 * 32];
    __shared__ int last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nwarps = (gridDim.x * blockDim.x) >> 5;
    const WT *e = (const WT *)a.embed;
    if (gwarp < a.vocab) prefetch_row_l2(e + (size_t)gwarp * a.hidden, (size_t)a.hidden * sizeof(WT), lane);
    pdl_wait();
    pdl_trigger();
    stage_rms(xs, a.x, a.norm, a.hidden, a.eps, red);
    const int nvec = a.hidden / WVec<WT>::kElems;
    Top2 t = top2_empty();
    bool bad = false;
    for (int row = gwarp; row < a.vocab; row += nwarps) {
        const WT *rows[1] = {e + (size_t)row * a.hidden};
        float acc[1];
        warp_rows_dot<WT, 1, UNROLL>(rows, xs, nvec, lane, acc);
        if (lane == 0) a.logits[row] = acc[0];
        bad |= !isfinite(acc[0]);
        top2_insert(t, acc[0], row);
    }
    // Warp results (identical in every lane) -> block result.
    if (lane == 0) {
        sv[2 * warp] = t.a; sv[2 * warp + 1] = t.b;
        si[2 * warp] = t.ai; si[2 * warp + 1] = t.bi;
    }
    const int any_bad = __syncthreads_or(bad);
    if (warp == 0) {
        Top2 u = top2_empty();
        if (lane < (int)(blockDim.x >> 5)) {
            top2_insert(u, sv[2 * lane], si[2 * lane]);
            top2_insert(u, sv[2 * lane + 1], si[2 * lane + 1]);
        }
        top2_merge_warp(u);
        if (lane == 0) {
            a.pv[2 * blockIdx.x] = u.a; a.pv[2 * blockIdx.x + 1] = u.b;
            a.pi[2 * blockIdx.x] = u.ai; a.pi[2 * blockIdx.x + 1] = u.bi;
            if (any_bad) atomicOr(&a.sync[1], 1u);
            __threadfence();
            last = atomicAdd(&a.sync[0], 1u) == gridDim.x - 1;
        }
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    Top2 u = top2_empty();
    for (int i = threadIdx.x; i < 2 * (int)gridDim.x; i += blockDim.x) top2_insert(u, __ldcg(a.pv + i), __ldcg(a.pi + i));
    top2_merge_warp(u);
    if (lane == 0) {
        sv[2 * warp] = u.a; sv[2 * warp + 1] = u.b;
        si[2 * warp] = u.ai; si[2 * warp + 1] = u.bi;
    }
    __syncthreads();
    if (warp == 0) {
        Top2 z = top2_empty();
        if (lane < (int)(blockDim.x >> 5)) {
            top2_insert(z, sv[2 * lane], si[2 * lane]);
            top2_insert(z, sv[2 * lane + 1], si[2 * lane + 1]);
        }
        top2_merge_warp(z);
        if (lane == 0) {
            const unsigned flag = atomicExch(&a.sync[1], 0u);
            TcmTop2 top;
            top.first = z.ai; top.second = z.bi; top.first_value = z.a; top.second_value = z.b;
            DecodeState *st = a.st;
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

// Token state from kernel arguments: nothing in host memory is read after the
// launch call returns, so chained enqueues never race a host buffer.
__global__ void set_state_kernel(DecodeState *st, int token, int position) {
    st->token = token;
    st->position = position;
    st->step = 0;
    st->invalid = 0;
}

template <typename T> inline void set_smem(T *kernel, int bytes) {
    TCM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

// GEMV shapes: 16-byte vectors in flight per row per lane (UNROLL) and warps
// per row (KSPLIT). A 1536-wide FP32 row is 12 vectors per lane (one round of
// loads); BF16 is 6. The 8960-wide down rows are split over 4 warps.
template <typename WT> struct Tune;
template <> struct Tune<float> {
    static constexpr int kQkv = 12, kO = 12, kGateUp = 6, kRead = 12, kDownSplit = 4, kDown = 18;
};
template <> struct Tune<uint16_t> {
    static constexpr int kQkv = 6, kO = 6, kGateUp = 6, kRead = 6, kDownSplit = 4, kDown = 9;
};

}  // namespace

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
    cudaGraphExec_t graph;
    bool graph_ready;
    bool after_host;  // the last stream operation was a host copy: next launch is not programmatic
    int grid_gemv, launches;
};

namespace {

template <typename WT> void setup_kernels_typed() {
    set_smem(qkv_kernel<WT, Tune<WT>::kQkv>, 64 * 1024);
    set_smem(residual_gemv_kernel<WT, 1, Tune<WT>::kO>, 96 * 1024);
    set_smem(residual_gemv_kernel<WT, Tune<WT>::kDownSplit, Tune<WT>::kDown>, 96 * 1024);
    set_smem(gateup_kernel<WT, Tune<WT>::kGateUp>, 64 * 1024);
    set_smem(readout_kernel<WT, Tune<WT>::kRead>, 64 * 1024);
}
void setup_kernels() {
    static std::once_flag once;
    std::call_once(once, [] {
        setup_kernels_typed<float>();
        setup_kernels_typed<uint16_t>();
    });
}

bool has_dense(const QwenB200Runner *r, int layer) { return r->slots[layer] >= 0; }
size_t slot_offset(const QwenB200Runner *r, int layer) {
    const QwenB200Shape &s = r->d->s;
    return (size_t)r->slots[layer] * s.kvheads * r->b.capacity * s.head;
}

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
    a.hidden = s.hidden; a.qheads = s.qheads; a.kvheads = s.kvheads; a.capacity = r->b.capacity; a.eps = s.epsilon;
    const int tasks = (s.qheads + 2 * s.kvheads) * 64;
    int grid = (tasks + kBlock / 32 - 1) / (kBlock / 32);
    launch(qkv_kernel<WT, Tune<WT>::kQkv>, dim3(grid), dim3(kBlock), (size_t)s.hidden * 4, stream(), pdl, a);
}
void launch_attention(QwenB200Runner *r, int layer, bool pdl) {
    const QwenB200Shape &s = r->d->s;
    AttnSource src = {};
    src.keys = r->b.keys + slot_offset(r, layer);
    src.values = r->b.values + slot_offset(r, layer);
    attention_split(r->b.q, src, false, r->b.capacity, -1, &r->st->position, s.qheads, s.kvheads, kAttnSplits,
                    r->attn_part, r->attn_counters, r->b.attention, stream(), pdl);
}
template <typename WT> void launch_oproj(QwenB200Runner *r, int layer, bool pdl) {
    const QwenB200Shape &s = r->d->s;
    const QwenB200Layer &L = r->d->layers[layer];
    ResidualArgs o = {L.o, r->b.attention, r->b.x, s.qheads * s.head, s.hidden};
    const int grid = (s.hidden + kBlock / 32 - 1) / (kBlock / 32);
    launch(residual_gemv_kernel<WT, 1, Tune<WT>::kO>, dim3(grid), dim3(kBlock), (size_t)o.in_dim * 4, stream(), pdl, o);
}
template <typename WT> void launch_gateup(QwenB200Runner *r, int layer, bool pdl) {
    const QwenB200Shape &s = r->d->s;
    const QwenB200Layer &L = r->d->layers[layer];
    GateUpArgs g = {L.gate, L.up, L.post_norm, r->b.x, r->b.gate, s.hidden, s.intermediate, s.epsilon};
    int grid = (s.intermediate + kBlock / 32 - 1) / (kBlock / 32);
    if (grid > r->grid_gemv) grid = r->grid_gemv;
    launch(gateup_kernel<WT, Tune<WT>::kGateUp>, dim3(grid), dim3(kBlock), (size_t)s.hidden * 4, stream(), pdl, g);
}
template <typename WT> void launch_down(QwenB200Runner *r, int layer, bool pdl) {
    const QwenB200Shape &s = r->d->s;
    const QwenB200Layer &L = r->d->layers[layer];
    ResidualArgs dn = {L.down, r->b.gate, r->b.x, s.intermediate, s.hidden};
    constexpr int split = Tune<WT>::kDownSplit, rows_per_cta = (kBlock / 32) / split;
    const int grid = (s.hidden + rows_per_cta - 1) / rows_per_cta;
    launch(residual_gemv_kernel<WT, split, Tune<WT>::kDown>, dim3(grid), dim3(kBlock), (size_t)dn.in_dim * 4, stream(),
           pdl, dn);
}
template <typename WT> void launch_mlp(QwenB200Runner *r, int layer, bool pdl) {
    launch_oproj<WT>(r, layer, pdl);
    launch_gateup<WT>(r, layer, true);
    launch_down<WT>(r, layer, true);
}
template <typename WT> void launch_readout(QwenB200Runner *r, bool pdl) {
    const QwenB200Decoder *d = r->d;
    const QwenB200Shape &s = d->s;
    ReadoutArgs a = {d->embed, d->norm, r->b.x, r->b.logits, r->top_pv, r->top_pi, r->sync, r->st, r->log,
                     s.hidden, s.vocab, s.epsilon};
    int grid = (s.vocab + kBlock / 32 - 1) / (kBlock / 32);
    if (grid > r->grid_gemv) grid = r->grid_gemv;
    launch(readout_kernel<WT, Tune<WT>::kRead>, dim3(grid), dim3(kBlock), (size_t)s.hidden * 4, stream(), pdl, a);
}

void launch_layer(QwenB200Runner *r, int layer, bool pdl_first) {
    if (r->d->dtype == 2) launch_qkv<uint16_t>(r, layer, pdl_first);
    else launch_qkv<float>(r, layer, pdl_first);
    launch_attention(r, layer, true);
    if (r->d->dtype == 2) launch_mlp<uint16_t>(r, layer, true);
    else launch_mlp<float>(r, layer, true);
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

int ensure_graph(QwenB200Runner *r) {
    if (r->graph_ready) return 0;
    if (!all_dense(r)) return -1;
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
    TCM_CUDA(cudaMemcpyAsync(r->st, r->host, 4 * sizeof(int), cudaMemcpyHostToDevice, stream()));
    r->after_host = true;
}
int read_top(QwenB200Runner *r, TcmTop2 *top) {
    TCM_CUDA(cudaMemcpyAsync(r->host, r->st, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream()));
    TCM_CUDA(cudaStreamSynchronize(stream()));
    if (top) *top = r->host->top;
    return r->host->invalid ? -3 : 0;
}
bool valid_token(const QwenB200Runner *r, int token, int position) {
    return token >= 0 && token < r->d->s.vocab && position >= 0 && position < r->b.capacity;
}

cudaEvent_t g_marks[64][16];

}  // namespace

extern "C" {

QwenB200Decoder *qwen_b200_decoder_create(const QwenB200Shape *shape, const float *embedding,
                                          const float *final_norm, const QwenB200Layer *layers, int matrix_dtype) {
    const QwenB200Shape &s = *shape;
    if (s.head != kHeadDim || s.kvheads < 1 || s.qheads % s.kvheads || s.qheads / s.kvheads > kAttnMaxGroup ||
        s.hidden % 8 || s.intermediate % 8 || s.layers < 1 || s.vocab < 1 || s.qheads * s.head != s.hidden ||
        s.hidden * 4 > 64 * 1024 || s.intermediate * 4 > 96 * 1024)
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
    const size_t part = (size_t)d->s.kvheads * kAttnSplits * kAttnPartialFloats;
    r->attn_part = (float *)gpu_alloc(part * sizeof(float));
    r->attn_counters = (unsigned *)gpu_alloc((size_t)d->s.kvheads * sizeof(unsigned));
    gpu_zero(r->attn_counters, (size_t)d->s.kvheads * sizeof(unsigned));
    r->grid_gemv = sm_count() * 2;
    r->top_pv = (float *)gpu_alloc((size_t)2 * r->grid_gemv * sizeof(float));
    r->top_pi = (int *)gpu_alloc((size_t)2 * r->grid_gemv * sizeof(int));
    r->sync = (unsigned *)gpu_alloc(2 * sizeof(unsigned));
    gpu_zero(r->sync, 2 * sizeof(unsigned));
    TCM_CUDA(cudaMallocHost((void **)&r->host, sizeof(DecodeState)));
    TCM_CUDA(cudaMallocHost((void **)&r->host_log, kLogCap * sizeof(TcmTop2)));
    r->launches = d->s.layers * 5 + 1;
    return r;
}

void qwen_b200_runner_free(QwenB200Runner *r) {
    if (!r) return;
    TCM_CUDA(cudaStreamSynchronize(stream()));
    if (r->graph_ready) TCM_CUDA(cudaGraphExecDestroy(r->graph));
    gpu_free(r->st);
    gpu_free(r->log);
    gpu_free(r->attn_part);
    gpu_free(r->attn_counters);
    gpu_free(r->top_pv);
    gpu_free(r->top_pi);
    gpu_free(r->sync);
    TCM_CUDA(cudaFreeHost(r->host));
    TCM_CUDA(cudaFreeHost(r->host_log));
    delete r;
}

int qwen_b200_begin(QwenB200Runner *r, int token, int position) {
    if (!r || !valid_token(r, token, position)) return -1;
    write_state(r, token, position);
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
    if (!r || !valid_token(r, token, position) || ensure_graph(r)) return -1;
    write_state(r, token, position);
    TCM_CUDA(cudaGraphLaunch(r->graph, stream()));
    return read_top(r, top);  // leaves after_host set by write_state
}

int qwen_b200_enqueue(QwenB200Runner *r, int token, int position, int n) {
    if (!r || n < 1 || n > kLogCap || !valid_token(r, token, position) || position + n > r->b.capacity ||
        ensure_graph(r))
        return -1;
    set_state_kernel<<<1, 1, 0, stream()>>>(r->st, token, position);
    TCM_CUDA(cudaGetLastError());
    r->after_host = true;
    for (int i = 0; i < n; i++) TCM_CUDA(cudaGraphLaunch(r->graph, stream()));
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

int qwen_b200_launches_per_token(const QwenB200Runner *r) { return r ? r->launches : 0; }

float qwen_b200_time_stage(QwenB200Runner *r, int stage, int layer, int position, int reps) {
    if (!r || stage < 0 || stage > 5 || layer < 0 || layer >= r->d->s.layers || reps < 1 ||
        !valid_token(r, 0, position) || (stage == 1 && !has_dense(r, layer)))
        return -1.f;
    const bool bf16 = r->d->dtype == 2;
    auto once = [&](bool pdl) {
        switch (stage) {
            case 0: bf16 ? launch_qkv<uint16_t>(r, layer, pdl) : launch_qkv<float>(r, layer, pdl); break;
            case 1: launch_attention(r, layer, pdl); break;
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
