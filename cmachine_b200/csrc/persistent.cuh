// Interface of the persistent whole-token decode kernel (persistent.cu) for
// the batch-1 runner (decode.cu).
#pragma once
#include "lanes.cuh"

namespace tcm {

// One layer's weights and this session's cache slot of that layer
// ([kvheads][capacity][128] FP32 keys and values).
struct PersistLayer {
    const void *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *bq, *bk, *bv, *in_norm, *post_norm;
    float *kcache, *vcache;
};

struct PersistArgs {
    const PersistLayer *layers;  // device array [nlayers]
    const void *embed;
    const float *final_norm, *rope_den;
    float *x, *q, *k, *v, *attn, *h, *logits;
    float *part;                 // attention partials [kvheads][64][kAttnPartialFloats]
    float *pv;                   // per-CTA top-2 values [grid][2]
    int *pi;                     // per-CTA top-2 ids [grid][2]
    DecodeState *st;
    TcmTop2 *log;
    unsigned long long *trace;   // per-CTA barrier timestamps [grid][kPersistMarks], or null
    int nlayers, qheads, kvheads, capacity, vocab;
    float eps, inv_sqrt_dim;
    unsigned lookahead;          // bytes a CTA prefetches into L2 ahead of its copies
};

constexpr int kPersistMarks = 512;          // timestamps per CTA: start, arrival at and passage of each grid barrier, readout done
constexpr int kPersistAttnCtasPerHead = 64;  // attention CTAs of a KV head above 1024 cached rows

// CTAs of the kernel that fit one SM (0: the kernel cannot run on this device).
int persistent_blocks_per_sm(int dtype);
// One token on `stream`: a cooperative launch of `grid` CTAs (one per SM).
void launch_persistent(int dtype, const PersistArgs &a, int grid, cudaStream_t stream);

}  // namespace tcm
