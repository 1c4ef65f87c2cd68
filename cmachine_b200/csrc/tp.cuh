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
//     its partial sum of each of those rows into slot [rank] of every rank's
//     exchange area (peer stores over NVLink), then reads the world's slots of
//     its rows from its own area and adds them in rank order to the residual.
//     Every rank adds the same numbers in the same order, so the residual
//     stream stays bit-identical on all ranks;
//   readout: each rank computes the logits of its vocabulary rows, stores them
//     into every rank's logits buffer, and its last CTA publishes the rank's
//     top-2 to every rank; each rank merges the world top-2s (larger value,
//     ties to the lower id), so all ranks take the same next token.
//
// Every exchanged word travels with the token's number in one 64-bit store
// (value in the low half, token in the high half): a reader that sees the
// token sees the value, with no fence or separate flag on the path. Token
// numbers (the exchange area's epoch + 1) only grow, so slots never need
// clearing, and a rank cannot reach the same slot of the next token before
// every rank has read this one. Every wait is bounded (the wait limit) and
// records a fault bit; after a fault the group must be rebuilt. No TMA and no
// multicast: peer memory is written with plain stores and read locally.
#pragma once
#include "common.cuh"
#include "stream.cuh"
#include "../../include/gpu.h"

namespace tcm {

constexpr int kTpMax = 8;

constexpr int kTpTopWords = 8;  // a rank's published top-2: a, b, ai, bi, non-finite flag (padded)

// What a launch needs to reach the group. world == 1: no exchange.
struct TpLink {
    unsigned long long *part[kTpMax];  // rank p's down slots [layers][world][kHidden] (token << 32 | value)
    float *logits[kTpMax];             // rank p's logits buffer
    unsigned long long *top[kTpMax];   // rank p's top-2 slots [world][kTpTopWords]
    unsigned *epoch;                   // this rank's token counter (tokens finished by the group)
    int rank, world;
    int inter;                         // intermediate units per rank
    int vocab_begin, vocab_end;        // this rank's readout rows
};

enum : unsigned { kErrPeerWait = 8u };

// One exchanged word: the value's bits and the token number, stored and
// loaded as one naturally aligned 64-bit access (single-copy atomic).
__device__ __forceinline__ void ll_store(unsigned long long *slot, unsigned value, unsigned token) {
    const unsigned long long w = ((unsigned long long)token << 32) | value;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(slot), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ll_load(const unsigned long long *slot) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(slot) : "memory");
    return w;
}
// Bounded wait until the slot holds this token's word; its value in *value.
// Once a peer wait of the token has run out, later ones give up at once, so a
// lost rank costs one wait limit per token rather than one per exchange.
__device__ __forceinline__ bool ll_wait(const unsigned long long *slot, unsigned token, unsigned *value, unsigned *err) {
    unsigned long long w = ll_load(slot);
    if ((unsigned)(w >> 32) == token) {
        *value = (unsigned)w;
        return true;
    }
    if (*(volatile unsigned *)err & kErrPeerWait) return false;
    const unsigned long long start = global_ns();
    for (;;) {
        w = ll_load(slot);
        if ((unsigned)(w >> 32) == token) {
            *value = (unsigned)w;
            return true;
        }
        if (wait_expired(global_ns() - start)) {
            atomicOr(err, kErrPeerWait);
            return false;
        }
    }
}

// Byte layout of one rank's exchange area.
struct TpLayout {
    size_t part, top, epoch, bytes;
};
inline TpLayout tp_layout(int layers, int world) {
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    TpLayout t;
    t.part = 0;
    t.top = up(t.part + (size_t)layers * world * 1536 * sizeof(unsigned long long));
    t.epoch = up(t.top + (size_t)world * kTpTopWords * sizeof(unsigned long long));
    t.bytes = up(t.epoch + sizeof(unsigned));
    return t;
}

}  // namespace tcm
