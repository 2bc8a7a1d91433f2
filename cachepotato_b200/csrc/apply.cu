// apply.cu — experts applied to externally routed tokens (prefill, expert-parallel receive side):
// the expert loop of engine/blocks/qwen3_moe.c:199-222 with the routing given by the caller.
//
//   k_apply_prep   validate ids, per-block expert histogram
//   k_apply_group  deterministic token sort: pairs grouped by expert, tokens ascending, plus the
//                  active-expert table the GEMMs schedule from
//   k_apply_gather the token rows in that order as fp16 (the gate/up GEMM's tensor-TMA source)
//   k_gemm_tc<0>   gate/up grouped GEMM on tcgen05, h = silu(g)·u
//   k_gemm_tc<1>   down grouped GEMM on tcgen05, y per (token, slot)
//   k_apply_combine out (+)= sum_j wt_j·y_j over the valid slots, in selection order
// Slots whose expert id is outside [0, n_experts) contribute nothing: an error for
// cpg_moe_apply, empty slots (id -1) by design for cpg_moe_apply_rows (expert-parallel receive).
#include "gemm_tc.cuh"

namespace cpg {

int apply_validate(const cpg_moe_layer *layer, int T, size_t ws_bytes);
// rows_f16: R fp16 rows xstride halves apart; row r's slot ids / weights at + r·istride.
int apply_rows_impl(const cpg_moe_layer *layer, const void *rows_f16, int xstride, int R, const int *slot_expert,
                    const float *slot_wt, int istride, float *out, void *ws, size_t ws_bytes, cudaStream_t s);
int layer_dims(const cpg_moe_layer *L, int *D, int *F, int *E, int *K);
int layer_ptrs(const cpg_moe_layer *L, const uint8_t *const **ptrs, int *enc);
int layer_weight_maps(const cpg_moe_layer *L, const void **maps);

constexpr int AP_BLOCK = 256;            // tokens per grouping block
constexpr int AP_MAX_E = 256;
constexpr int TC_BN_TOK = 256;           // token tile of the tcgen05 GEMM

struct ApplyWs {
    size_t status, n_active, act, act_ptr, blk_cnt, pairs, xs, h, y, total;
};

static size_t al(size_t v) { return (v + 255) / 256 * 256; }

static ApplyWs apply_layout(int D, int F, int E, int K, int T) {
    ApplyWs w{};
    size_t o = 0;
    const int nblk = (T + AP_BLOCK - 1) / AP_BLOCK;
    w.status = o; o = al(o + 16 * sizeof(int));
    w.n_active = o; o = al(o + sizeof(int));
    w.act = o; o = al(o + sizeof(int4) * (E + 1));
    w.act_ptr = o; o = al(o + sizeof(void *) * 3 * E);
    w.blk_cnt = o; o = al(o + sizeof(int) * (size_t)nblk * E);
    w.pairs = o; o = al(o + sizeof(int) * (size_t)T * K);
    w.xs = o; o = al(o + sizeof(__half) * (size_t)T * K * D);
    w.h = o; o = al(o + sizeof(__half) * (size_t)T * K * F);
    w.y = o; o = al(o + sizeof(float) * (size_t)T * K * D);
    w.total = o;
    return w;
}

// per-block expert counts, id validation (negative ids are empty slots when empty_ok). The
// status words are cleared on the stream before this launch, so a bad id any block records stays.
__global__ void __launch_bounds__(AP_BLOCK) k_apply_prep(int T, int E, int K, const int *__restrict__ idx, int istride,
                                                          int *__restrict__ blk_cnt, int *status, int empty_ok) {
    __shared__ int s_cnt[AP_MAX_E];
    const int b = blockIdx.x, t0 = b * AP_BLOCK;
    for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
    __syncthreads();
    const int nt = min(AP_BLOCK, T - t0);
    for (int i = threadIdx.x; i < nt * K; i += blockDim.x) {
        const int e = idx[(size_t)(t0 + i / K) * istride + i % K];
        if (e >= 0 && e < E) atomicAdd(&s_cnt[e], 1);
        else if (!(empty_ok && e < 0)) atomicExch(status, ST_BAD_ITEM);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) blk_cnt[(size_t)b * E + e] = s_cnt[e];
}

// Deterministic counting sort of the (token, slot) pairs by expert. Block b places its pairs at
// off[e] + (pairs of e in blocks < b) + (pairs of e from earlier tokens of block b).
__global__ void __launch_bounds__(AP_BLOCK) k_apply_group(int T, int E, int K, const int *__restrict__ idx, int istride,
                                                           const int *__restrict__ blk_cnt, int nblk,
                                                           const uint8_t *const *ptrs, int *pairs, int4 *act,
                                                           const uint8_t **act_ptr, int *n_active) {
    __shared__ int s_base[AP_MAX_E], s_tot[AP_MAX_E], s_off[AP_MAX_E];
    __shared__ uint32_t s_mask[AP_MAX_E];
    const int b = blockIdx.x, t0 = b * AP_BLOCK, tid = threadIdx.x;
    for (int e = tid; e < E; e += blockDim.x) {
        int before = 0, tot = 0;
        for (int c = 0; c < nblk; ++c) {
            const int v = blk_cnt[(size_t)c * E + e];
            before += c < b ? v : 0;
            tot += v;
        }
        s_base[e] = before;
        s_tot[e] = tot;
    }
    __syncthreads();
    if (tid == 0) {
        int o = 0;
        for (int e = 0; e < E; ++e) { s_off[e] = o; o += s_tot[e]; }
    }
    __syncthreads();
    if (b == 0 && tid == 0) {               // active-expert table (ascending expert id)
        int u = 0;
        for (int e = 0; e < E; ++e) {
            if (s_tot[e] > 0) {
                act[u] = make_int4(e, s_off[e], s_tot[e], 0);
                act_ptr[3 * u + 0] = ptrs[3 * e + 0];
                act_ptr[3 * u + 1] = ptrs[3 * e + 1];
                act_ptr[3 * u + 2] = ptrs[3 * e + 2];
                ++u;
            }
        }
        act[u] = make_int4(-1, s_off[E - 1] + s_tot[E - 1], 0, 0);
        *n_active = u;
    }
    const int nt = min(AP_BLOCK, T - t0);
    for (int c0 = 0; c0 < nt; c0 += 32) {
        for (int e = tid; e < E; e += blockDim.x) s_mask[e] = 0;
        __syncthreads();
        for (int i = tid; i < 32 * K; i += blockDim.x) {
            const int tl = i / K, t = t0 + c0 + tl;
            if (c0 + tl < nt) {
                const int e = idx[(size_t)t * istride + i % K];
                if (e >= 0 && e < E) atomicOr(&s_mask[e], 1u << tl);
            }
        }
        __syncthreads();
        for (int i = tid; i < 32 * K; i += blockDim.x) {
            const int tl = i / K, j = i % K, t = t0 + c0 + tl;
            if (c0 + tl < nt) {
                const int slot = t * K + j;
                const int e = idx[(size_t)t * istride + j];
                if (e >= 0 && e < E) {
                    const int r = s_base[e] + __popc(s_mask[e] & ((1u << tl) - 1u));
                    pairs[s_off[e] + r] = slot;
                }
            }
        }
        __syncthreads();
        for (int e = tid; e < E; e += blockDim.x) s_base[e] += __popc(s_mask[e]);
        __syncthreads();
    }
}

// xs[p] = fp16(xn[token of pair p]) for the valid pairs (one warp per row, 8 values per lane
// step); from fp16 rows xh (xstride halves apart) instead when xn is null
__global__ void __launch_bounds__(256) k_apply_gather(const float *__restrict__ xn, const __half *__restrict__ xh,
                                                       int D, int xstride, int K, const int *__restrict__ pairs,
                                                       const int4 *__restrict__ act, const int *__restrict__ n_active,
                                                       __half *__restrict__ xs, int max_pairs) {
    const int n_valid = act[*n_active].y;
    const int lane = threadIdx.x & 31;
    for (int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < n_valid && p < max_pairs;
         p += (gridDim.x * blockDim.x) >> 5) {
        const size_t row = (size_t)(pairs[p] / K) * D;
        uint4 *dst = reinterpret_cast<uint4 *>(xs + (size_t)p * D);
        if (!xn) {
            const uint4 *src16 = reinterpret_cast<const uint4 *>(xh + (size_t)(pairs[p] / K) * xstride);
            for (int i = lane; i < D / 8; i += 32) dst[i] = src16[i];
            continue;
        }
        const float4 *src = reinterpret_cast<const float4 *>(xn + row);
        for (int i = lane; i < D / 8; i += 32) {
            const float4 a = src[2 * i], b = src[2 * i + 1];
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
            dst[i] = make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                                *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
        }
    }
}

// out[t] (+)= sum_j wt[t,j]·y[t*K+j] over slots with a valid id, in selection order with one
// rounding per product and per sum (qwen3_moe.c:221); accumulate = 0 starts from zero.
__global__ void __launch_bounds__(256) k_apply_combine(int T, int D, int K, int E, const int *__restrict__ idx,
                                                        const float *__restrict__ wt, int istride,
                                                        const float *__restrict__ y, float *out, int accumulate) {
    const int n4 = T * D / 4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const int t = (i * 4) / D, k = i * 4 - t * D;
        float4 acc = accumulate ? reinterpret_cast<const float4 *>(out)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < K; ++j) {
            const int e = __ldg(idx + (size_t)t * istride + j);
            if (e < 0 || e >= E) continue;
            const float w = __ldg(wt + (size_t)t * istride + j);
            const float4 v = __ldg(reinterpret_cast<const float4 *>(y + ((size_t)t * K + j) * D + k));
            acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
        }
        reinterpret_cast<float4 *>(out)[i] = acc;
    }
}

}  // namespace cpg

using namespace cpg;

extern "C" size_t cpg_moe_apply_workspace_bytes(const cpg_moe_layer *layer, int max_T) {
    int D, F, E, K;
    if (!layer || max_T <= 0 || layer_dims(layer, &D, &F, &E, &K) != CPG_OK) return 0;
    return apply_layout(D, F, E, K, max_T).total;
}

// Everything apply_impl rejects before it launches anything, and the layer's tensor maps built:
// the expert-parallel path calls this before its first collective, so a bad argument can never
// leave the peers waiting in a collective this rank does not join.
int cpg::apply_validate(const cpg_moe_layer *layer, int T, size_t ws_bytes) {
    CPG_REQUIRE(layer, "cpg_moe_apply: null layer");
    CPG_REQUIRE(T > 0, "cpg_moe_apply: T=%d", T);
    int D, F, E, K, enc;
    const uint8_t *const *ptrs;
    int rc = layer_dims(layer, &D, &F, &E, &K);
    if (rc == CPG_OK) rc = layer_ptrs(layer, &ptrs, &enc);
    if (rc) return rc;
    CPG_REQUIRE(enc == CPG_ENC_Q4, "cpg_moe_apply: the tcgen05 grouped GEMM takes Q4_0 experts");
    CPG_REQUIRE(E <= AP_MAX_E, "cpg_moe_apply: n_experts=%d > %d", E, AP_MAX_E);
    CPG_REQUIRE(F % 256 == 0 && D % 256 == 0, "cpg_moe_apply: d_exp %% 256 and d_model %% 256 must be 0");
    const ApplyWs W = apply_layout(D, F, E, K, T);
    CPG_REQUIRE(ws_bytes >= W.total, "cpg_moe_apply: workspace %zu < %zu bytes for T=%d", ws_bytes, W.total, T);
    const void *maps = nullptr;
    return layer_weight_maps(layer, &maps);
}

// Input rows: xn (f32, D apart) or xh (fp16, xstride halves apart); row t's K slot ids and
// weights at topk_idx / wt + t·istride. empty_ok: negative ids are empty slots, not errors.
// accumulate: mlp += the block output, else mlp = it. ev: null, or 5 events recorded around the
// sort, gate/up, down and combine phases.
static int apply_impl(const cpg_moe_layer *layer, const float *xn, const __half *xh, int xstride, int T,
                      const int *topk_idx, const float *wt, int istride, float *mlp, int accumulate, int empty_ok,
                      void *ws, size_t ws_bytes, cudaStream_t s, cudaEvent_t *ev) {
    CPG_REQUIRE(layer && (xn || xh) && topk_idx && wt && mlp && ws, "cpg_moe_apply: null argument");
    int rc = apply_validate(layer, T, ws_bytes);
    if (rc) return rc;
    int D, F, E, K, enc;
    const uint8_t *const *ptrs;
    layer_dims(layer, &D, &F, &E, &K);
    layer_ptrs(layer, &ptrs, &enc);
    const ApplyWs W = apply_layout(D, F, E, K, T);
    CPG_REQUIRE((((uintptr_t)xn | (uintptr_t)xh | (uintptr_t)mlp | (uintptr_t)ws) & 15) == 0,
                "cpg_moe_apply: 16-byte alignment");
    uint8_t *w = (uint8_t *)ws;
    int *status = (int *)(w + W.status);
    const int nblk = (T + AP_BLOCK - 1) / AP_BLOCK;
    if (ev) CPG_CUDA(cudaEventRecord(ev[0], s));
    CPG_CUDA(cudaMemsetAsync(status, 0, 16 * sizeof(int), s));
    k_apply_prep<<<nblk, AP_BLOCK, 0, s>>>(T, E, K, topk_idx, istride, (int *)(w + W.blk_cnt), status, empty_ok);
    CPG_CUDA(cudaGetLastError());
    k_apply_group<<<nblk, AP_BLOCK, 0, s>>>(T, E, K, topk_idx, istride, (const int *)(w + W.blk_cnt), nblk, ptrs,
                                            (int *)(w + W.pairs), (int4 *)(w + W.act), (const uint8_t **)(w + W.act_ptr),
                                            (int *)(w + W.n_active));
    CPG_CUDA(cudaGetLastError());
    {
        const int P = T * K;
        int ggrid = (P + 7) / 8;
        if (ggrid > sm_count() * 8) ggrid = sm_count() * 8;
        k_apply_gather<<<ggrid, 256, 0, s>>>(xn, xh, D, xstride, K, (const int *)(w + W.pairs), (const int4 *)(w + W.act),
                                             (const int *)(w + W.n_active), (__half *)(w + W.xs), P);
        CPG_CUDA(cudaGetLastError());
    }
    TcArgs a{};
    a.n_active = (const int *)(w + W.n_active);
    a.act = (const int4 *)(w + W.act);
    rc = layer_weight_maps(layer, &a.wmaps);
    if (rc) return rc;
    a.pairs = (const int *)(w + W.pairs);
    a.D = D; a.F = F; a.K = K;
    a.status = status;
    const int max_tok_tiles = (T * K + TC_BN_TOK - 1) / TC_BN_TOK + (E < T * K ? E : T * K);
    a.h_out = (__half *)(w + W.h);
    a.y_out = (float *)(w + W.y);
    if (ev) CPG_CUDA(cudaEventRecord(ev[1], s));
    rc = gemm_tc_launch(0, a, (const __half *)(w + W.xs), T * K, max_tok_tiles * (F / 128), s);
    if (rc) return rc;
    if (ev) CPG_CUDA(cudaEventRecord(ev[2], s));
    rc = gemm_tc_launch(1, a, (const __half *)(w + W.h), T * K, max_tok_tiles * (D / 256), s);
    if (rc) return rc;
    if (ev) CPG_CUDA(cudaEventRecord(ev[3], s));
    const int n4 = T * D / 4;
    int cgrid = (n4 + 255) / 256;
    if (cgrid > sm_count() * 8) cgrid = sm_count() * 8;
    k_apply_combine<<<cgrid, 256, 0, s>>>(T, D, K, E, topk_idx, wt, istride, (const float *)(w + W.y), mlp, accumulate);
    CPG_CUDA(cudaGetLastError());
    if (ev) CPG_CUDA(cudaEventRecord(ev[4], s));
    return CPG_OK;
}

extern "C" int cpg_moe_apply(const cpg_moe_layer *layer, const float *xn, int T, const int *topk_idx,
                             const float *wt, float *mlp, void *ws, size_t ws_bytes, void *stream) {
    int D = 0, F, E, K = 0;
    if (layer) layer_dims(layer, &D, &F, &E, &K);
    return apply_impl(layer, xn, nullptr, D, T, topk_idx, wt, K, mlp, 1, 0, ws, ws_bytes, (cudaStream_t)stream,
                      nullptr);
}

int cpg::apply_rows_impl(const cpg_moe_layer *layer, const void *rows_f16, int xstride, int R, const int *slot_expert,
                         const float *slot_wt, int istride, float *out, void *ws, size_t ws_bytes, cudaStream_t s) {
    CPG_REQUIRE(rows_f16, "cpg_moe_apply_rows: null rows");
    return apply_impl(layer, nullptr, (const __half *)rows_f16, xstride, R, slot_expert, slot_wt, istride, out, 0, 1,
                      ws, ws_bytes, s, nullptr);
}

extern "C" int cpg_moe_apply_rows(const cpg_moe_layer *layer, const void *rows_f16, int R, const int *slot_expert,
                                  const float *slot_wt, float *out, void *ws, size_t ws_bytes, void *stream) {
    CPG_REQUIRE(rows_f16, "cpg_moe_apply_rows: null rows");
    int D = 0, F, E, K = 0;
    if (layer) layer_dims(layer, &D, &F, &E, &K);
    return apply_impl(layer, nullptr, (const __half *)rows_f16, D, R, slot_expert, slot_wt, K, out, 0, 1, ws, ws_bytes,
                      (cudaStream_t)stream, nullptr);
}

extern "C" int cpg_moe_apply_profile(const cpg_moe_layer *layer, const float *xn, int T, const int *topk_idx,
                                     const float *wt, float *mlp, void *ws, size_t ws_bytes, void *stream,
                                     float *phase_ms) {
    CPG_REQUIRE(phase_ms, "cpg_moe_apply_profile: null phase_ms");
    cudaEvent_t ev[5] = {};
    for (int i = 0; i < 5; ++i) {
        const cudaError_t ce = cudaEventCreate(&ev[i]);
        if (ce != cudaSuccess) {
            for (int j = 0; j < i; ++j) cudaEventDestroy(ev[j]);
            return cuda_fail(ce, "cpg_moe_apply_profile: event");
        }
    }
    int D = 0, F, E, K = 0;
    if (layer) layer_dims(layer, &D, &F, &E, &K);
    int rc = apply_impl(layer, xn, nullptr, D, T, topk_idx, wt, K, mlp, 1, 0, ws, ws_bytes, (cudaStream_t)stream, ev);
    if (rc == CPG_OK) {
        const cudaError_t ce = cudaEventSynchronize(ev[4]);
        if (ce != cudaSuccess) rc = cuda_fail(ce, "cpg_moe_apply_profile: synchronize");
        for (int i = 0; rc == CPG_OK && i < 4; ++i) {
            const cudaError_t e2 = cudaEventElapsedTime(&phase_ms[i], ev[i], ev[i + 1]);
            if (e2 != cudaSuccess) rc = cuda_fail(e2, "cpg_moe_apply_profile: elapsed time");
        }
    }
    for (int i = 0; i < 5; ++i) cudaEventDestroy(ev[i]);
    return rc;
}

extern "C" int cpg_moe_apply_check(const void *ws, void *stream) {
    CPG_REQUIRE(ws, "cpg_moe_apply_check: null workspace");
    int st = 0;
    CPG_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    CPG_CUDA(cudaMemcpy(&st, ws, sizeof(int), cudaMemcpyDeviceToHost));
    if (st == ST_BAD_ITEM) {
        set_error("cpg_moe_apply: expert id outside [0, n_experts) (those slots contributed zero)");
        return CPG_EINVAL;
    }
    if (st != ST_OK) {
        set_error("device-side wait timed out (status %d)", st);
        return CPG_ETIMEOUT;
    }
    return CPG_OK;
}
