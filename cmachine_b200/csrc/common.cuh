// Shared device/host helpers for the B200 (sm_100a) decode library.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <mutex>

// The reference treats every CUDA error as fatal: message on stderr, exit(2)
// (src/qwen_cuda.cu:8). The primitive ABI keeps that contract.
#define TCM_CUDA(call)                                                                      \
    do {                                                                                    \
        cudaError_t e_ = (call);                                                            \
        if (e_ != cudaSuccess) {                                                            \
            fprintf(stderr, "CUDA %s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e_)); \
            exit(2);                                                                        \
        }                                                                                   \
    } while (0)
#define TCM_FATAL(...)                    \
    do {                                  \
        fprintf(stderr, __VA_ARGS__);     \
        fputc('\n', stderr);              \
        exit(2);                          \
    } while (0)

namespace tcm {

// Runs a set-up step once on every device this process uses. Function
// attributes such as the dynamic shared-memory limit belong to the device
// context, so a process that drives several GPUs must set them on each.
struct PerDeviceOnce {
    std::mutex lock;
    bool done[64] = {};
    template <typename Fn> void run(Fn fn) {
        int dev = 0;
        TCM_CUDA(cudaGetDevice(&dev));
        if (dev < 0 || dev >= 64) TCM_FATAL("device index %d out of range", dev);
        std::lock_guard<std::mutex> hold(lock);
        if (!done[dev]) {
            fn();
            done[dev] = true;
        }
    }
};

// The library's stream. It is created with default (blocking) flags, so work
// on it is ordered with the legacy default stream that reference-style callers
// use implicitly; every primitive and fused launch goes here.
cudaStream_t stream();
int sm_count();

constexpr int kWarp = 32;

// ---- Programmatic dependent launch (PDL) -------------------------------------
// A kernel launched with the programmatic-serialization attribute may start
// while its predecessor is still running. It must execute pdl_wait() before it
// reads anything a predecessor wrote or writes anything a predecessor reads.
// Work that depends on no predecessor (weight prefetch) may precede it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Streaming 16-byte load that skips L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Top-2 with the reference's order: larger value first, ties to the lower id
// (src/qwen_cuda.cu:100-101).
struct Top2 {
    float a, b;
    int ai, bi;
};
__device__ __forceinline__ bool better(float v, int id, float w, int wid) { return v > w || (v == w && id < wid); }
__device__ __forceinline__ void top2_insert(Top2 &t, float v, int id) {
    if (id < 0) return;
    if (better(v, id, t.a, t.ai)) {
        t.b = t.a; t.bi = t.ai; t.a = v; t.ai = id;
    } else if (id != t.ai && better(v, id, t.b, t.bi)) {
        t.b = v; t.bi = id;
    }
}
__device__ __forceinline__ Top2 top2_empty() { return Top2{-INFINITY, -INFINITY, 0x7fffffff, 0x7fffffff}; }
__device__ __forceinline__ void top2_merge_warp(Top2 &t) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        float a = __shfl_xor_sync(0xffffffffu, t.a, o), b = __shfl_xor_sync(0xffffffffu, t.b, o);
        int ai = __shfl_xor_sync(0xffffffffu, t.ai, o), bi = __shfl_xor_sync(0xffffffffu, t.bi, o);
        top2_insert(t, a, ai);
        top2_insert(t, b, bi);
    }
}

// Launch helper: optional programmatic-serialization attribute.
template <typename... KArgs, typename... Args>
inline void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                   Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl ? attr : nullptr;
    cfg.numAttrs = pdl ? 1 : 0;
    TCM_CUDA(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

}  // namespace tcm
