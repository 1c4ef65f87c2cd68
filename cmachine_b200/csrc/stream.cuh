// Weight streaming pipeline for the fused decode kernels (sm_100a).
//
// One producer thread per CTA moves this CTA's weight rows from HBM into a ring
// of shared-memory stages with cp.async.bulk (the TMA engine's untiled bulk
// copy), each stage completing an mbarrier transaction; eight consumer warps
// wait for a stage, do the dot products out of shared memory, and release it.
// The producer never depends on a previous kernel, so it starts filling stages
// before griddepcontrol.wait: while the previous kernel drains, this kernel's
// first stages are already in flight.
//
// Every wait is bounded in time: after the wait limit of polling (global timer;
// kWaitLimitNs unless qwen_b200_wait_limit set another) the waiter records an
// error bit in the caller's error word and returns false; the caller then
// stops, and the producer waits (again bounded) for the copies it issued
// before it exits.
#pragma once
#include "common.cuh"

namespace tcm {

constexpr int kConsumerWarps = 8;
constexpr int kStreamThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s, the default bound of a wait
constexpr unsigned long long kWaitFloorNs = 1000000ull;     // 1 ms: no wait gives up sooner

// The bound of this module's waits. Every .cu file that includes this header
// has its own copy (no device linking); set_module_wait_limit sets it for the
// current device. It is read only once a wait has lasted kWaitFloorNs, so the
// fast path never loads it.
static __device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;
__device__ __forceinline__ bool wait_expired(unsigned long long elapsed) {
    return elapsed > kWaitFloorNs && elapsed > g_wait_limit_ns;
}
static inline void set_module_wait_limit(unsigned long long ns) {
    TCM_CUDA(cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns)));
}

enum : unsigned { kErrFullWait = 1u, kErrEmptyWait = 2u, kErrDrain = 4u };

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait for the phase of `bar` with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned *err, unsigned code) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long start = global_ns();
    for (;;) {
        if (mbar_try(bar, parity)) return true;
        if (wait_expired(global_ns() - start)) {
            atomicOr(err, code);
            return false;
        }
    }
}
// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte
// aligned) completing a transaction on `bar`. No multicast.
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
// The same copy with an L2 cache policy (e.g. evict-first for rows read once).
__device__ __forceinline__ void bulk_copy_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                   uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Asks L2 to fetch `bytes` (multiple of 16, 16-byte aligned) from global memory.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Named barrier among the consumer warps only (the producer warp never joins).
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory"); }

// The ring: STAGES stages of `stage_bytes`, full/empty barrier per stage.
struct Ring {
    unsigned char *buf;
    uint64_t *full, *empty;
    uint32_t stage_bytes;
    int stages;
    __device__ __forceinline__ unsigned char *stage(int s) const { return buf + (size_t)s * stage_bytes; }
};

// Carve a ring from dynamic shared memory (barriers after the stages) and
// initialise it; call from all threads (contains __syncthreads).
__device__ __forceinline__ Ring ring_setup(unsigned char *smem, int stages, uint32_t stage_bytes) {
    Ring r;
    r.buf = smem;
    r.stage_bytes = stage_bytes;
    r.stages = stages;
    r.full = reinterpret_cast<uint64_t *>(smem + (size_t)stages * stage_bytes);
    r.empty = r.full + stages;
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&r.full[s], 1);
            mbar_init(&r.empty[s], kConsumerWarps);
        }
        mbar_fence_init();
    }
    __syncthreads();
    return r;
}
constexpr size_t ring_smem_bytes(int stages, uint32_t stage_bytes) {
    return (size_t)stages * stage_bytes + 2 * stages * sizeof(uint64_t);
}

// Producer loop (one thread): for group g = 0..groups-1, copy items
// [g*R, min(items, (g+1)*R)) into stage g % STAGES, item j of a group at byte
// offset j * item_bytes, source address src(i). Then drain.
template <typename SrcFn>
__device__ __forceinline__ void ring_produce(const Ring &r, int items, int per_stage, uint32_t item_bytes, SrcFn src,
                                             unsigned *err) {
    const int groups = (items + per_stage - 1) / per_stage;
    int issued = 0;
    for (int g = 0; g < groups; g++) {
        const int s = g % r.stages;
        if (g >= r.stages && !mbar_wait(&r.empty[s], ((g / r.stages) & 1) ^ 1, err, kErrEmptyWait)) break;
        const int first = g * per_stage, n = min(per_stage, items - first);
        mbar_expect_tx(&r.full[s], (uint32_t)n * item_bytes);
        for (int j = 0; j < n; j++) bulk_copy_g2s(r.stage(s) + (size_t)j * item_bytes, src(first + j), item_bytes, &r.full[s]);
        issued = g + 1;
    }
    // Every issued copy must land before this thread (and so the CTA) can exit.
    for (int g = issued > r.stages ? issued - r.stages : 0; g < issued; g++)
        if (!mbar_wait(&r.full[g % r.stages], (g / r.stages) & 1, err, kErrDrain)) break;
}

// Dynamic variant: row groups are taken from a global counter (cnt[0]; cnt[1]
// counts finished producers and the last one resets both), so the CTAs that
// stream fastest take more groups and all finish together. Each stage carries
// its group in hdr[stage]; a stage with group -1 (no data) ends the stream.
// The next group's index is fetched while the current stage's wait runs.
template <typename SrcFn>
__device__ __forceinline__ void ring_produce_dynamic(const Ring &r, int items, int per_stage, uint32_t item_bytes,
                                                     SrcFn src, unsigned *cnt, int *hdr, unsigned *err) {
    const int groups = (items + per_stage - 1) / per_stage;
    int g = 0;
    int next = (int)atomicAdd(&cnt[0], 1u);
    for (;; g++) {
        const int grp = next;
        const bool done = grp >= groups;
        if (!done) next = (int)atomicAdd(&cnt[0], 1u);
        const int s = g % r.stages;
        if (g >= r.stages && !mbar_wait(&r.empty[s], ((g / r.stages) & 1) ^ 1, err, kErrEmptyWait)) break;
        hdr[s] = done ? -1 : grp;
        if (done) {
            mbar_arrive(&r.full[s]);  // the end marker: no data
            g++;                      // counted, so the drain sees every stage's latest phase
            break;
        }
        const int first = grp * per_stage, n = min(per_stage, items - first);
        mbar_expect_tx(&r.full[s], (uint32_t)n * item_bytes);
        for (int j = 0; j < n; j++) bulk_copy_g2s(r.stage(s) + (size_t)j * item_bytes, src(first + j), item_bytes, &r.full[s]);
    }
    for (int d = g > r.stages ? g - r.stages : 0; d < g; d++)
        if (!mbar_wait(&r.full[d % r.stages], (d / r.stages) & 1, err, kErrDrain)) break;
    __threadfence();
    if (atomicAdd(&cnt[1], 1u) == gridDim.x - 1) {
        cnt[0] = 0u;
        cnt[1] = 0u;
    }
}
// Consumer side of the dynamic ring: wait for stage g; returns its group, or -1
// at the end of the stream or when the wait ran out (*failed set).
__device__ __forceinline__ int ring_next(const Ring &r, int g, const int *hdr, unsigned *err, bool *failed) {
    if (!mbar_wait(&r.full[g % r.stages], (g / r.stages) & 1, err, kErrFullWait)) {
        *failed = true;
        return -1;
    }
    return hdr[g % r.stages];
}

// Consumer side: wait for group g's stage; release it (one arrive per warp).
__device__ __forceinline__ bool ring_acquire(const Ring &r, int g, unsigned *err) {
    return mbar_wait(&r.full[g % r.stages], (g / r.stages) & 1, err, kErrFullWait);
}
__device__ __forceinline__ void ring_release(const Ring &r, int g) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&r.empty[g % r.stages]);
}

}  // namespace tcm
