// gemm_tc.cuh — interface of the tcgen05 grouped expert GEMM (gemm_tc.cu).
#pragma once
#include "common.cuh"

namespace cpg {

struct TcArgs {
    const int *n_active;
    const int4 *act;                 // (e, pair offset, tokens, -) per active expert, ascending e
    const uint8_t *const *act_ptr;   // (U, 3) gate/up/down pointers
    const int *pairs;                // pair -> t*K + j, grouped by expert
    int D, F, K;
    const __half *bsrc;              // gate/up: xn fp16 (T, D) row-major; down: h fp16 (pairs, F)
    __half *h_out;                   // gate/up output (pairs, F)
    float *y_out;                    // down output (T*K, D)
    int *status;
};

// kind 0: gate/up (h = silu(g)·u), kind 1: down (y per slot). Q4_0 experts.
int gemm_tc_launch(int kind, const TcArgs &a, int max_tiles, cudaStream_t s);

}  // namespace cpg
