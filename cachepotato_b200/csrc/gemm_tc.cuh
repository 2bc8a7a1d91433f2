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
    size_t pass_stride;              // kind 2: floats between the three pass planes of y_out
    int *status;
};

// kind 0: gate/up (h = silu(g)·u) with b = the expert-sorted fp16 token rows (b_rows, D);
// kind 1: down (y per slot) with b = h (b_rows, F). Q4_0 experts; D and F multiples of 256.
int gemm_tc_launch(int kind, const TcArgs &a, const __half *b, int b_rows, int max_tiles, cudaStream_t s);
// Device array of 3E tensor maps over the expert matrices (rows of Q4_0 bytes, boxes of 128 rows ×
// 144 bytes); *d_maps is allocated here and freed by the caller.
int gemm_tc_build_weight_maps(const uint8_t *const *h_ptrs, int E, int D, int F, void **d_maps);

// Dense Q4_0 projections through the same kernel (kind 2: kind 1's layout, one group of all T
// tokens in 128-token tiles, three passes for close to f32 accuracy, W_hi·x_hi, W_hi·x_lo and
// W_lo·x_hi, each pass its own tiles writing its own plane; the planes are then summed).
// gemm_tc_dense_maps: device array of 3n tensor maps, entry 3i+2 over matrix i (rows[i] × k[i],
// rows a multiple of 256, k of 256); *d_maps is allocated here and freed by the caller.
int gemm_tc_dense_maps(const uint8_t *const *w, const int *rows, const int *k, int n, void **d_maps);
// y (T, rows) f32 = W_i · x for the matrix i that tab[0].x names, x16 (T, 2k) fp16 = [x_hi | x_lo]
// with x_hi = fp16(x), x_lo = fp16(x − x_hi); tab = {(i, 0, T, 0), (-1, T, 0, 0)} and
// *n_active = 1 on the device, iota[t] = t for t < T; planes: scratch of 3·T·rows floats.
int gemm_tc_dense(const void *maps, const int4 *tab, const int *n_active, const int *iota, const __half *x16, int T,
                  int rows, int k, float *y, float *planes, int *status, cudaStream_t s);

}  // namespace cpg
