// Tensor-parallel batch-1 decode over peer memory (sm_100a, NVLink).
//
// One session's token runs on `world` GPUs at once, one process per GPU. Every
// rank keeps the whole residual stream, the attention and its K/V (replicated:
// they are small), and takes 1/world of the work that dominates a token's
// bytes: the gate/up rows and down columns of every MLP (8960/world of the
// intermediate units) and the rows of the tied-embedding readout
// (vocab/world). Two exchanges per token replace the reference's single-GPU
// data flow (src/qwen.c:320,329-330,341 and 383-387):
//
//   down (per layer): CTA c of every rank owns the same residual rows; it stores
//     its partial sums of those rows into slot [rank] of every rank's exchange
//     area (peer stores over NVLink), raises a flag per peer, waits for the
//     flags of CTA c on every rank, and adds the world partials in rank order to
//     its residual rows. Every rank adds the same numbers in the same order, so
//     the residual stream stays bit-identical on all ranks;
//   readout: each rank computes the logits of its vocabulary rows, stores them
//     into every rank's logits buffer, and its last CTA publishes the rank's
//     top-2 to every rank; each rank merges the world top-2s (larger value,
//     ties to the lower id), so all ranks take the same next token.
//
// Flags carry the token's number (the exchange area's epoch + 1), so they never
// need clearing; a rank cannot reach the same flag of the next token before
// every rank has passed this one. Every wait is bounded (the wait limit) and
// records a fault bit; after a fault the group must be rebuilt. No TMA and no
// multicast: peer memory is written with plain stores and read locally.
#pragma once
#include "common.cuh"
#include "stream.cuh"
#include "../../include/gpu.h"

namespace tcm {

constexpr int kTpMax = 8;

// A rank's published top-2 and whether its logits held a non-finite value.
struct TpTop {
    float a, b;
    int ai, bi;
    unsigned bad, pad[3];
};

// What a launch needs to reach the group. world == 1: no exchange.
struct TpLink {
    float *part[kTpMax];       // rank p's down partials [layers][world][kHidden]
    unsigned *flag[kTpMax];    // rank p's down flags [layers][grid][world]
    float *logits[kTpMax];     // rank p's logits buffer
    TpTop *top[kTpMax];        // rank p's top-2 slots [world]
    unsigned *top_flag[kTpMax];// rank p's top-2 flags [world]
    unsigned *epoch;           // this rank's token counter (tokens finished by the group)
    int rank, world;
    int inter;                 // intermediate units per rank
    int vocab_begin, vocab_end;// this rank's readout rows
};

enum : unsigned { kErrPeerWait = 8u };

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until the flag has reached `want` (token numbers only grow).
// Once a peer wait of the token has run out, later ones give up at once, so a
// lost rank costs one wait limit per token rather than one per exchange.
__device__ __forceinline__ bool wait_flag(const unsigned *p, unsigned want, unsigned *err) {
    if ((int)(ld_acquire_sys(p) - want) >= 0) return true;
    if (*(volatile unsigned *)err & kErrPeerWait) return false;
    const unsigned long long start = global_ns();
    for (;;) {
        if ((int)(ld_acquire_sys(p) - want) >= 0) return true;
        if (wait_expired(global_ns() - start)) {
            atomicOr(err, kErrPeerWait);
            return false;
        }
    }
}

// Byte layout of one rank's exchange area.
struct TpLayout {
    size_t part, flag, top, top_flag, epoch, bytes;
};
inline TpLayout tp_layout(int layers, int world, int grid) {
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    TpLayout t;
    t.part = 0;
    t.flag = up(t.part + (size_t)layers * world * 1536 * sizeof(float));
    t.top = up(t.flag + (size_t)layers * grid * world * sizeof(unsigned));
    t.top_flag = up(t.top + (size_t)world * sizeof(TpTop));
    t.epoch = up(t.top_flag + (size_t)world * sizeof(unsigned));
    t.bytes = up(t.epoch + sizeof(unsigned));
    return t;
}

}  // namespace tcm
