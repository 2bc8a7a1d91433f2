// route_check.cu — routing agreement under ties, on the device: the rule of
// tools/check_qwen3_baseline.py:39-72, which models/qwen3-30b-a3b/MODEL.md section 6 makes the
// definition of "the routing agrees" (router logits are recorded in bf16, so exact ties at the
// K-th place are the norm and "the top K" has several valid answers).
//
// Per token, with p = softmax(logits) (float64 here) and thr = the K-th largest p:
//   the recorded ids, as a set, are a valid top-K when every chosen expert has p >= thr - 1e-12,
//   every expert with p > thr + 1e-12 is chosen, and as many chosen experts lie above
//   thr + 1e-12 as experts do; a valid token is "resolved by a tie" when fewer experts lie above
//   thr + 1e-12 than were chosen. Weights: |sum(w) - 1| and |w - p[ids] / sum(p[ids])|.
// One warp per token; the token's probabilities sit in shared memory.
#include <math.h>
#include <string.h>

#include <climits>

#include "common.cuh"

namespace cpg {

constexpr int RC_WARPS = 8;
constexpr int RC_MAX_E = 256;
constexpr double RC_EPS = 1e-12;

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// cnt: [0] invalid tokens, [1] tokens resolved by a tie, [2] first invalid token (INT_MAX: none);
// err: [0] max |sum(w) - 1|, [1] max weight error, as the bits of non-negative doubles.
__global__ void __launch_bounds__(RC_WARPS * 32) k_route_check(const float *logits, const int *topk, const float *wt,
                                                               int T, int E, int K, int *cnt,
                                                               unsigned long long *err) {
    __shared__ double sp[RC_WARPS][RC_MAX_E];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * RC_WARPS + warp;
    if (t >= T) return;                                    // warp-uniform; no block barrier below
    double *p = sp[warp];
    const float *lg = logits + (size_t)t * E;
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) m = fmaxf(m, lg[e]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    double s = 0.0;
    for (int e = lane; e < E; e += 32) {
        const double v = exp((double)lg[e] - (double)m);
        p[e] = v;
        s += v;
    }
    s = warp_sum_d(s);
    for (int e = lane; e < E; e += 32) p[e] /= s;
    __syncwarp();
    // the K-th largest probability: a value with fewer than K larger and at least K not smaller
    double thr = -1.0;
    for (int e = lane; e < E; e += 32) {
        const double c = p[e];
        int gt = 0, ge = 0;
        for (int f = 0; f < E; ++f) {
            gt += p[f] > c;
            ge += p[f] >= c;
        }
        if (gt < K && ge >= K) thr = c;
    }
    thr = warp_max_d(thr);
    // the recorded ids (lane j < K holds id j) and their distinct members
    const int *ids = topk + (size_t)t * K;
    const int id = lane < K ? ids[lane] : -1;
    const bool all_in = __all_sync(0xffffffffu, lane >= K || (id >= 0 && id < E));
    bool first = lane < K;
    for (int j = 0; j < K; ++j) {
        const int o = __shfl_sync(0xffffffffu, id, j);
        if (j < lane && o == id) first = false;
    }
    const int n_distinct = __popc(__ballot_sync(0xffffffffu, first));
    bool valid = false, tie = false;
    if (all_in) {
        const double pid = lane < K ? p[id] : 0.0;
        const bool chosen_low = first && !(pid >= thr - RC_EPS);
        const int n_above_sel = __popc(__ballot_sync(0xffffffffu, first && pid > thr + RC_EPS));
        int n_above = 0;
        bool unchosen_above = false;
        for (int e = lane; e < E; e += 32) {
            if (p[e] > thr + RC_EPS) {
                ++n_above;
                bool chosen = false;
                for (int j = 0; j < K; ++j) chosen |= ids[j] == e;
                unchosen_above |= !chosen;
            }
        }
        for (int o = 16; o > 0; o >>= 1) n_above += __shfl_xor_sync(0xffffffffu, n_above, o);
        valid = !__any_sync(0xffffffffu, chosen_low) && !__any_sync(0xffffffffu, unchosen_above) &&
                n_above_sel == n_above;
        tie = valid && n_above < n_distinct;
    }
    // weights against softmax + renormalisation over the recorded ids
    const double got = all_in && lane < K ? p[id] : 0.0;
    const double gs = warp_sum_d(got);
    const double w = lane < K ? (double)wt[(size_t)t * K + lane] : 0.0;
    const double werr = warp_max_d(all_in && lane < K ? fabs(got / gs - w) : 0.0);
    const double serr = fabs(warp_sum_d(w) - 1.0);
    if (lane == 0) {
        if (!valid) {
            atomicAdd(&cnt[0], 1);
            atomicMin(&cnt[2], t);
        } else if (tie) {
            atomicAdd(&cnt[1], 1);
        }
        atomicMax(&err[0], (unsigned long long)__double_as_longlong(serr));
        if (all_in) atomicMax(&err[1], (unsigned long long)__double_as_longlong(werr));
    }
}

}  // namespace cpg

using namespace cpg;

extern "C" int cpg_route_check(const float *logits, const int *topk, const float *wt, int T, int E, int K,
                               int *stats, double *errs, void *stream) {
    CPG_REQUIRE(stats && errs && (T == 0 || (logits && topk && wt)), "cpg_route_check: null argument");
    CPG_REQUIRE(T >= 0 && E > 0 && E <= RC_MAX_E && K > 0 && K <= 32 && K <= E,
                "cpg_route_check: T=%d E=%d K=%d (E <= %d, K <= min(32, E))", T, E, K, RC_MAX_E);
    stats[0] = 0;
    stats[1] = 0;
    stats[2] = -1;
    errs[0] = 0.0;
    errs[1] = 0.0;
    if (T == 0) return CPG_OK;
    cudaStream_t s = (cudaStream_t)stream;
    struct Acc { int cnt[4]; unsigned long long err[2]; } h{{0, 0, INT_MAX, 0}, {0ull, 0ull}};
    Acc *d = nullptr;
    CPG_CUDA(cudaMalloc((void **)&d, sizeof(Acc)));
    cudaError_t e = cudaMemcpyAsync(d, &h, sizeof(Acc), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        k_route_check<<<(T + RC_WARPS - 1) / RC_WARPS, RC_WARPS * 32, 0, s>>>(logits, topk, wt, T, E, K, d->cnt, d->err);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h, d, sizeof(Acc), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_fail(e, "cpg_route_check");
    stats[0] = h.cnt[0];
    stats[1] = h.cnt[1];
    stats[2] = h.cnt[2] == INT_MAX ? -1 : h.cnt[2];
    memcpy(&errs[0], &h.err[0], sizeof(double));
    memcpy(&errs[1], &h.err[1], sizeof(double));
    return CPG_OK;
}
