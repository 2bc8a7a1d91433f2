// moe_one.cuh — the one-token layer kernel's host interface (moe_one.cu), used by moe.cu.
#pragma once
#include "common.cuh"

struct cpg_moe_layer;

namespace cpg {

// How the one-token kernel runs a layer (decided once, at layer creation).
struct OnePlan {
    bool ok = false;      // the layer's shape fits the kernel (K <= 8, E <= 256, shared memory)
    int slots = 0;        // 16-row gate/up bands per round held in shared memory
    bool early_down = false;  // the down tiles have their own shared memory area (copied while
                              // gate/up computes); else they reuse the gate/up area
    int grid = 0;         // CTAs: one per SM
    size_t smem = 0;      // dynamic shared memory per CTA
};

int one_plan(const cpg_moe_layer *L, OnePlan *p);
// One token through the layer. ws_hdr: the decode workspace's header (word 0: status); h: its
// (K, F) f32 area; bar: the layer's two barrier counters (zero between launches). Launches on
// one layer must not overlap on the GPU (they share the counters).
int one_launch(const cpg_moe_layer *L, const OnePlan &p, const float *x, const float *attn, float *mlp,
               float *x_out, int *topk, float *wt, float *logits, int *ws_hdr, float *h, unsigned *bar,
               cudaStream_t s);

}  // namespace cpg
