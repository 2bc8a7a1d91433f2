// gemm_tc.cuh — interface of the tcgen05 grouped expert GEMM (gemm_tc.cu).
#pragma once
#include "common.cuh"

namespace cpg {

struct TcArgs {
    const int *n_active;
    const int4 *act;                 // (e, pair offset, tokens, -) per active expert, ascending e
    const void *wmaps;               // (E, 3) CUtensorMap of each expert's gate/up/down Q4_0 rows
    const int *pairs;                // pair -> t*K + j, grouped by expert
    int D, F, K;
    __half *h_out;                   // gate/up output (pairs, F)
    float *y_out;                    // down output (T*K, D)
    int *status;
};

// kind 0: gate/up (h = silu(g)·u) with b = the expert-sorted fp16 token rows (b_rows, D);
// kind 1: down (y per slot) with b = h (b_rows, F). Q4_0 experts; D and F multiples of 256.
int gemm_tc_launch(int kind, const TcArgs &a, const __half *b, int b_rows, int max_tiles, cudaStream_t s);
// Device array of 3E tensor maps over the expert matrices (rows of Q4_0 bytes, boxes of 128 rows ×
// 144 bytes); *d_maps is allocated here and freed by the caller.
int gemm_tc_build_weight_maps(const uint8_t *const *h_ptrs, int E, int D, int F, void **d_maps);

}  // namespace cpg
