// Memory registry, copies and the library stream (drop-in for the memory part
// of the reference's src/qwen_cuda.cu:12-24).
//
// The reference keeps a linked list of live cudaMalloc blocks and exits on an
// unknown free (src/qwen_cuda.cu:13-19). Here the registry is a hash map under
// a mutex (the host executor may run sessions on several threads), with the
// same accounting: gpu_live_bytes / gpu_peak_bytes count tracked bytes.
#include "common.cuh"
#include "../../include/gpu.h"
#include <mutex>
#include <unordered_map>

namespace tcm {
namespace {
std::mutex g_lock;
std::unordered_map<void *, size_t> g_blocks;
size_t g_live = 0, g_peak = 0;
cudaStream_t g_stream[64];
bool g_stream_ready[64];
int g_sms[64];
}  // namespace

static int current_device() {
    int d = 0;
    TCM_CUDA(cudaGetDevice(&d));
    if (d < 0 || d >= 64) TCM_FATAL("device index %d out of range", d);
    return d;
}

cudaStream_t stream() {
    int d = current_device();
    if (!g_stream_ready[d]) {
        std::lock_guard<std::mutex> hold(g_lock);
        if (!g_stream_ready[d]) {
            TCM_CUDA(cudaStreamCreateWithFlags(&g_stream[d], cudaStreamDefault));
            TCM_CUDA(cudaDeviceGetAttribute(&g_sms[d], cudaDevAttrMultiProcessorCount, d));
            g_stream_ready[d] = true;
        }
    }
    return g_stream[d];
}

int sm_count() {
    stream();
    return g_sms[current_device()];
}

}  // namespace tcm

extern "C" {

void *gpu_alloc(size_t n) {
    void *p = nullptr;
    TCM_CUDA(cudaMalloc(&p, n ? n : 1));
    std::lock_guard<std::mutex> hold(tcm::g_lock);
    tcm::g_blocks[p] = n;
    tcm::g_live += n;
    if (tcm::g_live > tcm::g_peak) tcm::g_peak = tcm::g_live;
    return p;
}

void gpu_free(void *p) {
    if (!p) return;
    size_t n;
    {
        std::lock_guard<std::mutex> hold(tcm::g_lock);
        auto it = tcm::g_blocks.find(p);
        if (it == tcm::g_blocks.end()) TCM_FATAL("gpu_free: pointer %p was not allocated by gpu_alloc", p);
        n = it->second;
        tcm::g_blocks.erase(it);
        tcm::g_live -= n;
    }
    // cudaFree synchronizes the device, so no queued kernel still uses p.
    TCM_CUDA(cudaFree(p));
}

size_t gpu_live_bytes(void) {
    std::lock_guard<std::mutex> hold(tcm::g_lock);
    return tcm::g_live;
}
size_t gpu_peak_bytes(void) {
    std::lock_guard<std::mutex> hold(tcm::g_lock);
    return tcm::g_peak;
}
size_t gpu_free_bytes(void) {
    size_t f = 0, t = 0;
    TCM_CUDA(cudaMemGetInfo(&f, &t));
    return f;
}

void gpu_zero(void *p, size_t n) {
    if (n) TCM_CUDA(cudaMemsetAsync(p, 0, n, tcm::stream()));
}
void gpu_copy(void *d, const void *s, size_t n) {
    if (n) TCM_CUDA(cudaMemcpyAsync(d, s, n, cudaMemcpyDeviceToDevice, tcm::stream()));
}
void gpu_read(void *d, const void *s, size_t n) {
    cudaStream_t st = tcm::stream();
    if (n) TCM_CUDA(cudaMemcpyAsync(d, s, n, cudaMemcpyDeviceToHost, st));
    TCM_CUDA(cudaStreamSynchronize(st));
}
void gpu_write(void *d, const void *s, size_t n) {
    cudaStream_t st = tcm::stream();
    if (n) TCM_CUDA(cudaMemcpyAsync(d, s, n, cudaMemcpyHostToDevice, st));
    TCM_CUDA(cudaStreamSynchronize(st));
}
void gpu_sync(void) {
    TCM_CUDA(cudaStreamSynchronize(tcm::stream()));
    TCM_CUDA(cudaDeviceSynchronize());
}

}  // extern "C"
