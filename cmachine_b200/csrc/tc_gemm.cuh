// Batched weight GEMMs on the 5th-generation tensor cores (sm_100a tcgen05).
//
// D[row][n] = sum_k W[row][k] * X[n][k] for a BF16 weight matrix W (the
// source-BF16 residence, [out][in] row-major) and a batch of FP32 activation
// rows X, n < N sessions. The activations enter as two BF16 halves, hi =
// bf16(x) and lo = bf16(x - hi), and every tile is the sum of two MMAs, W * hi
// + W * lo, accumulated in FP32 in tensor memory: x is carried to about 16
// significant bits, so the product tracks the reference's BF16-weight x FP32
// activation arithmetic to ~1e-5 relative instead of BF16's ~4e-3.
//
// One CTA per SM (persistent over work items), 10 warps:
//   warp 0  producer: one thread issues TMA tile loads (W box 64 x 64 twice per
//           stage for a 128-row tile, X hi and lo boxes 64 x N) into a ring of
//           shared-memory stages in the 128-byte swizzle, each stage completing
//           an mbarrier transaction; the weight loads of the first stages are
//           issued before griddepcontrol.wait (they depend on no kernel);
//   warp 1  MMA: allocates 2N tensor-memory columns (two accumulators), one
//           thread issues tcgen05.mma kind::f16 (M = 128, N, K = 16; four per
//           64-wide k-block and operand half) and tcgen05.commit to release
//           stages and publish accumulators;
//   warps 2-9 epilogue: tcgen05.ld of the accumulator (warp w reads lanes
//           32 * (w % 4) ..., warps 2-5 the first half of the columns and
//           warps 6-9 the second), then either the tile's final values or, with
//           split K, a partial to global memory of which the last CTA to arrive
//           sums the splits in order (deterministic) and finishes the tile, or
//           (defer) a partial that the next kernel sums while it reads the
//           tile's outputs anyway.
//           The epilogue's per-element work (folds, bias, RoPE, SwiGLU, BF16
//           splits) is latency-bound, so two warps per scheduler run it.
// With split K launched as thread-block clusters (one cluster of `splits` CTAs
// per tile, one item per CTA), every CTA leaves its partial tile in shared
// memory, and after a cluster barrier each rank folds its own slice of row
// pairs from all ranks through distributed shared memory, in rank order
// (deterministic), and writes that slice's outputs; a second barrier keeps the
// partials alive until every rank has read them.
// The tile goes to shared memory as [128][N + 1] FP32 and the epilogue functor
// writes the outputs for row pairs (p, p + 64) (bias, RoPE, K/V append,
// residual, SwiGLU, logits ...).
// Every wait is bounded by the global timer and sets a bit in *err.
#pragma once
#include "common.cuh"
#include "stream.cuh"
#include <cuda.h>
#include <cooperative_groups.h>

namespace tcm {

constexpr int kTcEpiThreads = 256;                 // warps 2-9
constexpr int kTcThreads = 64 + kTcEpiThreads;
constexpr int kTcKBlock = 64;  // BF16 elements per k-block (one 128-byte swizzle row)
constexpr uint32_t kTcATile = 128 * 128;  // bytes: 128 rows x 64 BF16

enum : unsigned { kTcErrFull = 16u, kTcErrEmpty = 32u, kTcErrAcc = 64u, kTcErrAccFree = 128u };

template <int N> struct TcGeo {
    static_assert(N % 16 == 0 && N >= 16 && N <= 128, "batch tile N: multiple of 16 up to 128");
    static constexpr uint32_t kBTile = N * 128;                 // bytes: N rows x 64 BF16
    static constexpr uint32_t kStage = kTcATile + 2 * kBTile;   // A, X hi, X lo
    static constexpr int kStages = N <= 64 ? 5 : 4;
    static constexpr int kNP = N + 1;                           // padded tile row (floats)
    static constexpr uint32_t kTileBytes = 128 * kNP * 4;
    static constexpr uint32_t kTmemCols = 2 * N < 32 ? 32 : 2 * N;
    static constexpr uint32_t kScratch = 2048;                  // epilogue metadata (per-session pointers)
    static constexpr size_t kSmem = 1024 + (size_t)kStages * kStage + kTileBytes + kScratch + 256;
    // Instruction descriptor: F32 accumulate, BF16 A and B, both K-major, M = 128.
    static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (8u << 24);
};

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (SBO), base 1024-aligned.
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// 32 lanes x 16 consecutive FP32 columns of tensor memory, one lane per thread.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
// Epilogue warps only (kTcEpiThreads threads, named barrier 2).
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 2, %0;" ::"n"(kTcEpiThreads) : "memory"); }

// The A source of output tile t: rows [r0, r0 + 64) of map m0 and rows
// [r1, r1 + 64) of map m1 form the tile's 128 rows.
struct TcRows {
    int m0, r0, m1, r1;
};

// Optional timeline: per CTA, global-timer stamps (ns) at
//   0 entry after setup, 1 producer released by the dependency wait,
//   2 first stage ready (MMA), 3 last MMA committed, 4 epilogue released,
//   5 first accumulator read, 6 last tile stored, 7 exit.
constexpr int kTcMarks = 8;
__device__ __forceinline__ void tc_mark(unsigned long long *trace, int k) {
    if (trace) trace[(size_t)blockIdx.x * kTcMarks + k] = global_ns();
}

template <int N, class Epi> struct TcArgs {
    CUtensorMap a[3];
    CUtensorMap xh, xl;
    int tiles, splits, kblocks;
    int cluster;          // 1: splits meet in global memory; = splits: in a thread-block cluster
    int defer = 0;        // 1 (with cluster 1): every split leaves its partial in `part` as
                          // [tile][split][session][128] and the next kernel sums them (no fold here)
    float *part;          // split-K partials [tile][split][128][N]
    unsigned *counters;   // per tile, reset by the finishing CTA
    unsigned *err;
    unsigned long long *trace;
    Epi epi;
};

template <int N, class Epi>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ TcArgs<N, Epi> a) {
    using G = TcGeo<N>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float(*tile)[G::kNP] = reinterpret_cast<float(*)[G::kNP]>(smem + (size_t)G::kStages * G::kStage);
    unsigned char *scratch = smem + (size_t)G::kStages * G::kStage + G::kTileBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(scratch + G::kScratch);
    uint64_t *full = bars, *empty = bars + G::kStages, *acc_full = bars + 2 * G::kStages,
             *acc_free = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_free + 2);
    int *flag = reinterpret_cast<int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = a.tiles * a.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_free[b], kTcEpiThreads);
        }
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(G::kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_trigger();
    if (threadIdx.x == 0) tc_mark(a.trace, 0);

    auto krange = [&](int item, int &t, int &k0, int &k1) {
        t = item / a.splits;
        const int s = item % a.splits;
        k0 = (int)((long long)s * a.kblocks / a.splits);
        k1 = (int)((long long)(s + 1) * a.kblocks / a.splits);
    };

    if (warp == 0) {
        if (lane == 0) {
            // Producer. Stage fills g = 0, 1, ... walk (item, k-block) in order.
            int item = blockIdx.x, kb = 0, kend = 0, t = 0;
            TcRows rw{0, 0, 0, 0};
            auto open_item = [&]() {
                int k0;
                krange(item, t, k0, kend);
                kb = k0;
                rw = a.epi.a_rows(t);
            };
            auto step = [&]() {
                if (++kb >= kend) {
                    item += gridDim.x;
                    if (item < items) open_item();
                }
            };
            if (item < items) open_item();
            for (int i = 0; i < 3; i++) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.a[i])) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.xh)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.xl)) : "memory");
            auto load_w = [&](int s) {
                unsigned char *st = smem + (size_t)s * G::kStage;
                mbar_expect_tx(&full[s], G::kStage);
                tma_load_2d(smem_addr(st), &a.a[rw.m0], kb * kTcKBlock, rw.r0, smem_addr(&full[s]));
                tma_load_2d(smem_addr(st + kTcATile / 2), &a.a[rw.m1], kb * kTcKBlock, rw.r1, smem_addr(&full[s]));
            };
            auto load_x = [&](int s, int k) {
                unsigned char *st = smem + (size_t)s * G::kStage;
                tma_load_2d(smem_addr(st + kTcATile), &a.xh, k * kTcKBlock, 0, smem_addr(&full[s]));
                tma_load_2d(smem_addr(st + kTcATile + G::kBTile), &a.xl, k * kTcKBlock, 0, smem_addr(&full[s]));
            };
            // Weights of the first stages before the dependency wait (they are
            // constants); the activations after it.
            int g = 0, pro_kb[G::kStages];
            for (; g < G::kStages && item < items; g++) {
                load_w(g);
                pro_kb[g] = kb;
                step();
            }
            pdl_wait();
            tc_mark(a.trace, 1);
            for (int j = 0; j < g; j++) load_x(j, pro_kb[j]);
            for (; item < items; g++) {
                const int s = g % G::kStages;
                if (!mbar_wait(&empty[s], ((g / G::kStages) & 1) ^ 1, a.err, kTcErrEmpty)) break;
                load_w(s);
                load_x(s, kb);
                step();
            }
            // Drain: every issued stage must land before the CTA may exit.
            for (int d = g > G::kStages ? g - G::kStages : 0; d < g; d++)
                if (!mbar_wait(&full[d % G::kStages], (d / G::kStages) & 1, a.err, kTcErrFull)) break;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int g = 0, local = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x, local++) {
                int t, k0, k1;
                krange(item, t, k0, k1);
                const int buf = local & 1;
                // The epilogue must have drained this accumulator (used two items ago).
                if (local >= 2 && !mbar_wait(&acc_free[buf], ((local >> 1) & 1) ^ 1, a.err, kTcErrAccFree)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * N);
                for (int kb = k0; kb < k1; kb++, g++) {
                    const int s = g % G::kStages;
                    if (!mbar_wait(&full[s], (g / G::kStages) & 1, a.err, kTcErrFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (g == 0) tc_mark(a.trace, 2);
                    const uint32_t base = smem_addr(smem + (size_t)s * G::kStage);
                    const uint64_t ad = tc_desc(base), hd = tc_desc(base + kTcATile),
                                   ld = tc_desc(base + kTcATile + G::kBTile);
#pragma unroll
                    for (int k = 0; k < kTcKBlock / 16; k++) {
                        // +32 bytes per K = 16 step inside the swizzled row: +2 in the address field.
                        tc_mma(d, ad + 2 * k, hd + 2 * k, G::kIdesc, (kb > k0 || k > 0) ? 1u : 0u);
                        tc_mma(d, ad + 2 * k, ld + 2 * k, G::kIdesc, 1u);
                    }
                    tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
                }
                if (!ok) break;
                tc_commit(&acc_full[buf]);
            }
            tc_mark(a.trace, 3);
        }
    } else {
        // Epilogue: kTcEpiThreads threads. Thread e holds row rr of the tile
        // (its tensor-memory lane) and the columns [c0, c0 + H) of its half.
        constexpr int H = N / 2;
        static_assert(H % 16 == 0, "each epilogue half reads whole 16-column loads");
        const int e = (warp - 2) * 32 + lane;
        const int rr = (warp & 3) * 32 + lane;  // warps 2..5 and 6..9 -> lane quarters 2,3,0,1
        const int c0 = ((warp - 2) >> 2) * H;
        pdl_wait();
        if (e == 0) tc_mark(a.trace, 4);
        a.epi.init(scratch, e);
        epi_sync();
        int local = 0;
        for (int item = blockIdx.x; item < items; item += gridDim.x, local++) {
            int t, k0, k1;
            krange(item, t, k0, k1);
            const int buf = local & 1;
            if (!mbar_wait(&acc_full[buf], (local >> 1) & 1, a.err, kTcErrAcc)) break;
            tc_fence_after();
            if (e == 0 && local == 0) tc_mark(a.trace, 5);
            float v[H];
            const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(buf * N + c0);
#pragma unroll
            for (int c = 0; c < H; c += 16) {
                float r[16];
                tc_ld16(taddr + (uint32_t)c, r);
#pragma unroll
                for (int i = 0; i < 16; i++) v[c + i] = r[i];
            }
            tc_fence_before();
            mbar_arrive(&acc_free[buf]);
            if (a.cluster > 1) {
                // Partial to this CTA's shared tile; the cluster folds it below.
                epi_sync();
#pragma unroll
                for (int c = 0; c < H; c++) tile[rr][c0 + c] = v[c];
                continue;
            }
            if (a.defer) {
                // Deferred fold: the partial goes out in the layout its reader
                // wants, each session's 128 rows contiguous (a warp's 32 lanes
                // are 32 consecutive rows, so every store is one 128-byte line).
                float *p = a.part + ((size_t)t * a.splits + item % a.splits) * N * 128 + rr;
#pragma unroll
                for (int c = 0; c < H; c++) p[(size_t)(c0 + c) * 128] = v[c];
                continue;
            }
            bool finish = true;
            if (a.splits > 1) {
                const int split = item % a.splits;
                float4 *p = reinterpret_cast<float4 *>(a.part + (((size_t)t * a.splits + split) * 128 + rr) * N + c0);
#pragma unroll
                for (int c = 0; c < H; c += 4) p[c / 4] = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
                __threadfence();
                epi_sync();
                if (e == 0) *flag = atomicAdd(&a.counters[t], 1u) == (unsigned)(a.splits - 1);
                epi_sync();
                finish = *flag != 0;
                if (finish) {
                    __threadfence();
#pragma unroll
                    for (int c = 0; c < H; c++) v[c] = 0.f;
                    for (int sp = 0; sp < a.splits; sp++) {
                        const float4 *q =
                            reinterpret_cast<const float4 *>(a.part + (((size_t)t * a.splits + sp) * 128 + rr) * N + c0);
#pragma unroll
                        for (int c = 0; c < H; c += 4) {
                            const float4 w = __ldcg(q + c / 4);
                            v[c] += w.x;
                            v[c + 1] += w.y;
                            v[c + 2] += w.z;
                            v[c + 3] += w.w;
                        }
                    }
                    if (e == 0) a.counters[t] = 0u;
                }
            }
            if (finish) {
                epi_sync();  // the previous tile's readers are done with `tile`
#pragma unroll
                for (int c = 0; c < H; c++) tile[rr][c0 + c] = v[c];
                epi_sync();
                a.epi.store(t, tile, 0, 64, e, scratch);
            }
        }
        if (e == 0) tc_mark(a.trace, 6);
    }
    if (a.cluster > 1) {
        // Cluster fold: rank r owns row pairs [r * 64 / S, (r + 1) * 64 / S).
        // After the first barrier every rank's MMAs are done, so its operand
        // ring is idle: each rank writes every row of its partial tile into
        // the ring of the rank that owns the row (posted remote stores,
        // receive layout [source rank][row of the owner's slice][N + 4]).
        // After the second barrier each owner adds its S received slices in
        // rank order, from its own shared memory.
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        constexpr int kRS = N + 4;  // receive row stride (floats; 16-byte rows)
        // S x 2 ceil(64 / S) <= 150 receive rows for every cluster size S <= 16.
        static_assert((size_t)150 * kRS * 4 <= (size_t)G::kStages * G::kStage, "cluster receive buffer");
        const int S = a.cluster, r = (int)cluster.block_rank(), t = blockIdx.x / S;
        const int npmax = (64 + S - 1) / S;
        const int e = (warp - 2) * 32 + lane;  // epilogue thread (warps 2-9)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the ring's async-proxy use is over
        cluster.sync();
        if (warp >= 2) {
            // Thread e sends half ch of tile row e % 128 (row pair pr, upper or lower).
            constexpr int H = N / 2;
            const int row = e & 127, pr = row & 63, half = row >> 6, ch = e >> 7;
            int o = 0;
            while (o + 1 < S && (o + 1) * 64 / S <= pr) o++;
            const int op0 = o * 64 / S, onp = (o + 1) * 64 / S - op0;
            float *dst = cluster.map_shared_rank(reinterpret_cast<float *>(smem), o) +
                         ((size_t)r * 2 * npmax + (pr - op0) + half * onp) * kRS + ch * H;
            const float *src = &tile[row][ch * H];
#pragma unroll
            for (int c = 0; c < H; c += 4)
                *reinterpret_cast<float4 *>(dst + c) = make_float4(src[c], src[c + 1], src[c + 2], src[c + 3]);
        }
        cluster.sync();  // every row has reached its owner
        if (warp >= 2) {
            const int p0 = r * 64 / S, p1 = (r + 1) * 64 / S, np = p1 - p0, count = 2 * np * N;
            const float *recv = reinterpret_cast<const float *>(smem);
            for (int idx = e; idx < count; idx += kTcEpiThreads) {
                const int jr = idx / N, c = idx % N;
                float part[16];  // all of the element's slices requested first
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    part[q] = 0.f;
                    if (q < S)
                        asm volatile("ld.shared.f32 %0, [%1];"
                                     : "=f"(part[q])
                                     : "r"(smem_addr(recv + ((size_t)q * 2 * npmax + jr) * kRS + c)));
                }
                float sum = 0.f;
#pragma unroll
                for (int q = 0; q < 16; q++)
                    if (q < S) sum += part[q];
                tile[jr < np ? p0 + jr : 64 + p0 + (jr - np)][c] = sum;
            }
            epi_sync();
            a.epi.store(t, tile, p0, p1, e, scratch);
            if (e == 0) tc_mark(a.trace, 6);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) tc_mark(a.trace, 7);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::kTmemCols));
    }
}

}  // namespace tcm
