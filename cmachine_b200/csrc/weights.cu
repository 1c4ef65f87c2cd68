// Weight residence profiles (drop-in for src/qwen_weights.inc).
//
// Profile 0 keeps every tensor as FP32 (BF16 sources widened once at load).
// Profile 2 keeps rank-2 matrices as their source BF16 bits; the reference then
// widens 1024-row tiles into a 36.7 MB FP32 scratch tile before each cuBLAS
// GEMV (src/qwen_weights.inc:29-41). Here the GEMV kernels read BF16 straight
// from HBM and widen in registers, so no tile exists: `scratch` and `tiles`
// in gpu_weight_info stay 0, and the reference's tile-derived limits (197
// records, 8960 columns) do not apply. Profile 1 (tiled FP32) therefore has
// the same residence as profile 0; it stays accepted so callers keep working.
#include "common.cuh"
#include "kernels.h"
#include "../../include/gpu.h"
#include "../../include/qwen_b200.h"
#include <mutex>
#include <unordered_map>

namespace tcm {
namespace {
struct Record {
    int in, out, encoded;
    size_t bytes;
};
std::mutex g_lock;
std::unordered_map<const void *, Record> g_records;
int g_mode = 0;
bool g_mode_from_register = false;  // profile 2 entered by registering device matrices
size_t g_matrix_bytes = 0, g_rank1_bytes = 0;
unsigned long long g_matvecs = 0, g_embeddings = 0;

const Record *find(const void *p) {
    auto it = g_records.find(p);
    return it == g_records.end() ? nullptr : &it->second;
}
}  // namespace

int weight_dtype(const void *p) {
    std::lock_guard<std::mutex> hold(g_lock);
    const Record *r = find(p);
    return r ? (r->encoded ? 2 : 1) : 0;
}

__global__ void embedding_widen_kernel(float *out, const uint16_t *src, int width) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < width) out[i] = __uint_as_float((uint32_t)src[i] << 16);
}

}  // namespace tcm

using namespace tcm;

extern "C" {

// src/qwen_weights.inc:9: choose before any matrix is loaded.
void gpu_weight_configure(int mode) {
    std::lock_guard<std::mutex> hold(g_lock);
    if (mode < 0 || mode > 2 || !g_records.empty()) TCM_FATAL("gpu_weight_configure: invalid profile or model loaded");
    g_mode = mode;
}

// src/qwen_weights.inc:10-20.
float *gpu_owned_weight(TcmGpu *, const void *data, uint32_t dtype, size_t count, int rank, int rows, int columns) {
    int mode;
    {
        std::lock_guard<std::mutex> hold(g_lock);
        mode = g_mode;
        if (mode && rank != 2) g_rank1_bytes += count * 4;
    }
    if (!mode || rank != 2) return gpu_weight(data, dtype, count);
    if (rows < 1 || columns < 1 || count != (size_t)rows * columns) TCM_FATAL("gpu_owned_weight: shape mismatch");
    const int encoded = mode == 2;
    float *p;
    if (encoded) {
        if (dtype != 2) TCM_FATAL("exact BF16 matrix source required");
        p = (float *)gpu_alloc(count * 2);
        gpu_write(p, data, count * 2);
    } else {
        p = gpu_weight(data, dtype, count);
    }
    const size_t bytes = count * (encoded ? 2 : 4);
    std::lock_guard<std::mutex> hold(g_lock);
    g_records[p] = Record{columns, rows, encoded, bytes};
    g_matrix_bytes += bytes;
    return p;
}

size_t gpu_owned_weight_bytes(const float *p, size_t count) {
    std::lock_guard<std::mutex> hold(g_lock);
    const Record *r = find(p);
    return r ? r->bytes : count * 4;
}

// src/qwen_weights.inc:23-28.
void gpu_owned_embedding(float *out, const float *embedding, int token, int width) {
    int encoded = 0;
    {
        std::lock_guard<std::mutex> hold(g_lock);
        if (g_mode) {
            const Record *r = find(embedding);
            if (!r || width != r->in || token < 0 || token >= r->out) TCM_FATAL("gpu_owned_embedding: invalid row");
            encoded = r->encoded;
            g_embeddings++;
        }
    }
    if (encoded) {
        const uint16_t *src = reinterpret_cast<const uint16_t *>(embedding) + (size_t)token * width;
        embedding_widen_kernel<<<(width + 255) / 256, 256, 0, stream()>>>(out, src, width);
        TCM_CUDA(cudaGetLastError());
    } else {
        gpu_copy(out, embedding + (size_t)token * width, (size_t)width * 4);
    }
}

// src/qwen_weights.inc:29-41: registered matrices are read in their stored
// type; any other pointer is an ordinary FP32 matrix.
void gpu_matvec(TcmGpu *, const float *w, int in, int out, const float *x, float *y) {
    int dtype = 1;
    {
        std::lock_guard<std::mutex> hold(g_lock);
        g_matvecs++;
        if (g_mode) {
            const Record *r = find(w);
            if (r) {
                if (r->in != in || r->out != out) TCM_FATAL("gpu_matvec: shape differs from the registered matrix");
                dtype = r->encoded ? 2 : 1;
            }
        }
    }
    matvec(w, dtype, in, out, x, y, stream());
}

void qwen_b200_register_matrix(const void *p, int rows, int columns, int encoded) {
    const size_t bytes = (size_t)rows * columns * (encoded ? 2 : 4);
    std::lock_guard<std::mutex> hold(g_lock);
    g_records[p] = Record{columns, rows, encoded ? 1 : 0, bytes};
    g_matrix_bytes += bytes;
    if (encoded && g_mode != 2) {
        g_mode = 2;
        g_mode_from_register = true;
    }
}

int qwen_b200_weight_dtype(const void *p) { return weight_dtype(p) == 2 ? 2 : 1; }

void qwen_b200_unregister_matrix(const void *p) {
    std::lock_guard<std::mutex> hold(g_lock);
    auto it = g_records.find(p);
    if (it == g_records.end()) return;
    g_matrix_bytes -= it->second.bytes;
    g_records.erase(it);
    if (g_records.empty() && g_mode_from_register) {
        g_mode = 0;
        g_mode_from_register = false;
    }
}

void gpu_weight_info(size_t *matrix, size_t *vectors, size_t *scratch, int *count, unsigned long long *matvecs,
                     unsigned long long *tiles, unsigned long long *embeddings) {
    std::lock_guard<std::mutex> hold(g_lock);
    *matrix = g_matrix_bytes;
    *vectors = g_rank1_bytes;
    *scratch = 0;
    *count = (int)g_records.size();
    *matvecs = g_matvecs;
    *tiles = 0;
    *embeddings = g_embeddings;
}

// src/qwen_weights.inc:45: forget the records (their memory is owned and freed
// by the model) and return to profile 0.
void gpu_weight_release(void) {
    std::lock_guard<std::mutex> hold(g_lock);
    g_records.clear();
    g_mode = 0;
    g_mode_from_register = false;
    g_matrix_bytes = g_rank1_bytes = 0;
    g_matvecs = g_embeddings = 0;
}

}  // extern "C"
