// Split-K GQA attention whose scratch lives in a fixed device array.
//
// Who needs it: callers that must not allocate device memory while they run.
// Examples are a host that hands the whole GPU memory to its own pool manager
// and forbids driver allocations after start-up, a latency-critical loop that
// cannot afford the device-wide synchronisation cudaFree implies, and code in
// a context where a lazy allocation could fail late (a nearly full device).
// gpu_attention keeps its split-K partials in memory that its TcmGpu handle
// allocates on first use; gpu_attention_static uses the array below instead
// and never calls cudaMalloc, cudaFree or any allocating routine.
//
// The array is a file-scope __device__ symbol, so every GPU that loads this
// library holds it (kStaticScratchBytes, about 1.2 MB) until the process exits.
// Host code cannot use the symbol's name as a device address; the first call
// on each device asks the runtime for the address (cudaGetSymbolAddress) with
// that device current and keeps it. That first call should therefore happen
// before any stream capture. All calls share the one array and it keeps the
// previous call's contents: the per-head completion counters are cleared by
// each call before its kernel runs, and two calls that overlap on the GPU
// (different streams or processes sharing a context) race on the array.
#include "common.cuh"
#include "attention.cuh"
#include "kernels.h"
#include "../../include/gpu.h"
#include <mutex>

namespace tcm {
namespace {

constexpr int kStaticMaxKvHeads = 4;
constexpr size_t kStaticPartBytes = (size_t)kStaticMaxKvHeads * kAttnSplits * kAttnPartialFloats * sizeof(float);
constexpr size_t kStaticScratchBytes = kStaticPartBytes + 256;  // partials, then the counters

static __device__ __align__(256) unsigned char g_attention_scratch[kStaticScratchBytes];

std::mutex g_setup_lock;
void *g_scratch_address[64];

// Device address of the array for the current device (set up once per device).
unsigned char *scratch_address() {
    int dev = 0;
    TCM_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) TCM_FATAL("gpu_attention_static: device index %d out of range", dev);
    std::lock_guard<std::mutex> hold(g_setup_lock);
    if (!g_scratch_address[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attention_scratch);
        if (e != cudaSuccess || !p)
            TCM_FATAL("gpu_attention_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        g_scratch_address[dev] = p;
    }
    return static_cast<unsigned char *>(g_scratch_address[dev]);
}

}  // namespace
}  // namespace tcm

extern "C" int gpu_attention_static(float *out, const float *q, const float *keys, const float *values, int qheads,
                                    int kvheads, int dim, int capacity, int length) {
    using namespace tcm;
    if (dim != kHeadDim || kvheads < 1 || kvheads > kStaticMaxKvHeads || qheads < kvheads || qheads % kvheads ||
        qheads / kvheads > kAttnMaxGroup || length < 1 || length > capacity) {
        fprintf(stderr,
                "gpu_attention_static: unsupported size (dim %d must be %d; kvheads %d must be 1..%d; "
                "query heads per KV head %d must be <= %d; length %d must be 1..capacity %d)\n",
                dim, kHeadDim, kvheads, kStaticMaxKvHeads, kvheads > 0 ? qheads / kvheads : 0, kAttnMaxGroup, length,
                capacity);
        return -1;
    }
    if (((uintptr_t)keys & 15) || ((uintptr_t)values & 15) || ((uintptr_t)q & 15)) {
        fprintf(stderr, "gpu_attention_static: q, keys and values must be 16-byte aligned\n");
        return -1;
    }
    unsigned char *base = scratch_address();
    float *part = reinterpret_cast<float *>(base);
    unsigned *counters = reinterpret_cast<unsigned *>(base + kStaticPartBytes);
    cudaStream_t s = stream();
    TCM_CUDA(cudaMemsetAsync(counters, 0, (size_t)kvheads * sizeof(unsigned), s));
    AttnSource src = {};
    src.keys = keys;
    src.values = values;
    attention_split(q, src, false, capacity, length, nullptr, qheads, kvheads, kAttnSplits, part, counters, out, s,
                    false);
    return 0;
}
