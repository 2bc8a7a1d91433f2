// moe.cu — the Qwen3-MoE block (engine/blocks/qwen3_moe.c:169-223) on B200.
//
// Three or four launches per layer, all enqueued on one stream and free of host syncs:
//   k_router   RMSNorm(x + attn), f32 router GEMV, softmax over experts, strict-'>' top-k,
//              renormalisation (qwen3_moe.c:178-197). The CTAs of one token tile form a thread-
//              block cluster (each holds a slice of the experts); after a cluster barrier, CTA r
//              routes token r of the tile.
//   k_experts<GATEUP>  per (expert, 64 features, chunk of up to 12 tokens): gate and up GEMMs
//              on interleaved gate/up tiles, h = silu(g)·u (qwen3_moe.c:217-219). Each CTA first groups the (token, slot)
//              pairs by expert in its own shared memory (CTA 0 publishes the table for the
//              later kernels); batches over EX_GROUP_MAX pairs are grouped by k_group instead.
//   k_experts<DOWN>    per (expert, 128-row tile, token chunk): y = Wd·h (qwen3_moe.c:220)
//   k_experts<BOTH>    the two above in one launch when the gate/up items outnumber the SMs
//              (every batch of two or more tokens): gate/up items first, then down items, each
//              down item waiting (bounded) for its token chunk's h
//   k_combine  mlp += sum_j wt_j·y_j in selection order (qwen3_moe.c:221) and the residual
//              x + (attn + mlp) of run_layers (engine/api/cachepotato.c:157-159)
//
// Expert kernels: two producer warps fill an mbarrier ring of stages. One thread deals the work
// items and streams the weight rows from the layer's decode tile copy (k_tile_experts) by one
// bulk copy per stage (one 256-value K slice of the item's rows, no multicast); the
// other warp copies the same K slice of the item's token rows by 16-byte cp.async. Eight
// consumer warps decode Q4_0 / Q8_0 groups in registers (exact integers in fp16) and feed
// mma.m16n8k16 with fp32 accumulators; the group scale is applied in fp32 after each group's
// MMAs. Weights are read exactly once per layer.
//
// Activations keep f32 accuracy on fp16 tensor cores: every f32 operand value v (xn, h) is
// stored as two fp16 halves, hi = fp16(v) and lo = fp16(v - hi), so hi + lo carries about 22
// significant bits. The halves are neighbouring N columns of the MMA (token j of an item ->
// columns 2j and 2j+1), so a column pair's two partial sums land in one thread's accumulator
// pair and add up in fp32 after the K loop; the Q4/Q8 integers are exact in fp16. One 8-column
// MMA tile therefore carries four tokens, and an item of at most four tokens (a one-token decode
// step, most experts of a 64-token batch) issues no more MMAs than a single fp16 operand would.
#include <math.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "expert_tile.cuh"
#include "layout.cuh"
#include "moe_one.cuh"

namespace cpg {

// ------------------------------------------------------------------ constants and layouts
constexpr int R_TB = 8;          // router: tokens per CTA (one warp per token); 1-2 for tiny batches
constexpr int R_THREADS = 256;
constexpr int MAX_E = 256;
constexpr int MAX_K = 32;

constexpr int KIND_GATEUP = 0;
constexpr int KIND_DOWN = 1;
constexpr int KIND_BOTH = 2;     // gate/up then down items in one launch
constexpr int EX_NW = 8;         // consumer warps per CTA
constexpr int EX_NP = 2;         // producer warps: weight tiles, token rows (one issuing warp's
                                 // copies are served one after another on B200)
constexpr int EX_NCH = 3;        // 8-column MMA tiles per item (four tokens each: hi and lo columns);
                                 // 12 tokens per item measured ahead of 8 and 16 (two 35 KB or
                                 // three 26 KB stages per CTA against three 31 KB ones)
constexpr int EX_NCHUNK = 4 * EX_NCH;   // tokens per item (an expert with more is split)
constexpr int EX_GROUP_MAX = 1024;       // pairs the gate/up kernel groups itself (T ≤ 128)
constexpr int R_CLUSTER_MAX = 16;        // router CTAs per token tile (one cluster)

// workspace words
enum { WS_STATUS = 0, WS_ITEMS_GATEUP = 2, WS_ITEMS_DOWN = 3, WS_HDR_INTS = 16 };

struct WsLayout {
    size_t zero_row, n_active, act, pairs, topk, wt, logits, xn, h, y, dep, total;
};

// Token chunks of a batch: at most one partial chunk per active expert plus the full ones.
static int max_token_chunks(int E, int K, int T) {
    const int max_active = T * K < E ? T * K : E;
    return max_active + T * K / EX_NCHUNK;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static WsLayout ws_layout(int D, int F, int E, int K, int T) {
    WsLayout L{};
    size_t o = WS_HDR_INTS * sizeof(int);
    o = align_up(o, 256);
    L.zero_row = o; o += sizeof(__half) * (size_t)(D > F ? D : F);   // operand for padded tokens
    o = align_up(o, 256);
    L.n_active = o; o += sizeof(int);
    o = align_up(o, 256);
    L.act = o; o = align_up(o + sizeof(int4) * (size_t)(E + 1), 256);
    L.pairs = o; o = align_up(o + sizeof(int) * (size_t)T * K, 256);
    L.topk = o; o = align_up(o + sizeof(int) * (size_t)T * K, 256);
    L.wt = o; o = align_up(o + sizeof(float) * (size_t)T * K, 256);
    L.logits = o; o = align_up(o + sizeof(float) * (size_t)T * E, 256);
    L.xn = o; o = align_up(o + sizeof(__half) * 2 * (size_t)T * D, 256);       // per token: hi | lo
    L.h = o; o = align_up(o + sizeof(__half) * 2 * (size_t)T * K * F, 256);    // per pair: hi | lo
    L.y = o; o = align_up(o + sizeof(float) * (size_t)T * K * D, 256);
    L.dep = o; o = align_up(o + sizeof(int) * (size_t)max_token_chunks(E, K, T), 256);
    L.total = o;
    return L;
}

__constant__ Perm64 c_perm[2] = {kPermQ4, kPermQ8};
__device__ __forceinline__ const Perm64 &perm_of(int enc) { return c_perm[enc == CPG_ENC_Q4 ? 0 : 1]; }

// ------------------------------------------------------------------ router
struct RouterArgs {
    const float *x, *attn, *ln2, *wgate;
    int T, D, E, K;
    float eps;
    int xn_enc;                  // permutation of the xn copy the gate/up kernel reads
    int F;
    int eb;                      // experts per CTA
    float *logits;
    int *topk;
    float *wt;
    __half *xn_perm;
    int *status;                 // workspace header (status word, counters)
    __half *zero_row;
    int *n_active, *pairs;
    int4 *act;                   // active experts ascending: (e, pair offset, tokens, token chunks before)
    int *dep;                    // per token chunk counters of the one-launch expert kernel
    int n_dep;
};

// group (token, slot) pairs by expert, tokens ascending inside an expert; one CTA
__device__ __forceinline__ int warp_incl_scan(int v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Group (token, slot) pairs by expert, tokens ascending inside an expert, and publish the
// active-expert table the expert kernels schedule from. One CTA; top-k ids staged in shared
// memory (they fit for decode batches; larger batches read them from global memory).
__device__ void group_pairs(const RouterArgs &a) {
    __shared__ int s_cnt[MAX_E], s_off[MAX_E], s_base[MAX_E], s_uidx[MAX_E], s_chp[MAX_E];
    __shared__ uint32_t s_mask[MAX_E];
    __shared__ int s_tk[8 * 8 * MAX_K];
    __shared__ int s_tot[3];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int TK = a.T * a.K;
    const bool staged = TK <= 8 * 8 * MAX_K;
    for (int e = tid; e < a.E; e += blockDim.x) { s_cnt[e] = 0; s_base[e] = 0; }
    if (staged)
        for (int i = tid; i < TK; i += blockDim.x) s_tk[i] = __ldcg(a.topk + i);
    __syncthreads();
    const int *tk = staged ? s_tk : a.topk;
    for (int i = tid; i < TK; i += blockDim.x) atomicAdd(&s_cnt[staged ? tk[i] : __ldcg(a.topk + i)], 1);
    __syncthreads();
    if (warp == 0) {                     // exclusive scans over experts, 32 at a time
        int o = 0, u = 0, chp = 0;
        for (int e0 = 0; e0 < a.E; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < a.E ? s_cnt[e] : 0;
            const int ch = (c + EX_NCHUNK - 1) / EX_NCHUNK, act = c > 0;
            const int ic = warp_incl_scan(c), ich = warp_incl_scan(ch), ia = warp_incl_scan(act);
            if (e < a.E) {
                s_off[e] = o + ic - c;
                s_chp[e] = chp + ich - ch;
                s_uidx[e] = act ? u + ia - 1 : -1;
            }
            o += __shfl_sync(0xffffffffu, ic, 31);
            chp += __shfl_sync(0xffffffffu, ich, 31);
            u += __shfl_sync(0xffffffffu, ia, 31);
        }
        if (lane == 0) {
            a.act[u] = make_int4(-1, o, 0, chp);
            *a.n_active = u;
        }
    }
    __syncthreads();
    for (int e = tid; e < a.E; e += blockDim.x) {
        const int u = s_uidx[e];
        if (u >= 0) a.act[u] = make_int4(e, s_off[e], s_cnt[e], s_chp[e]);
    }
    (void)s_tot;
    for (int c0 = 0; c0 < a.T; c0 += 32) {
        for (int e = tid; e < a.E; e += blockDim.x) s_mask[e] = 0;
        __syncthreads();
        for (int i = tid; i < 32 * a.K; i += blockDim.x) {
            const int tl = i / a.K, t = c0 + tl;
            if (t < a.T) {
                const int idx = t * a.K + i % a.K;
                atomicOr(&s_mask[staged ? tk[idx] : __ldcg(a.topk + idx)], 1u << tl);
            }
        }
        __syncthreads();
        for (int i = tid; i < 32 * a.K; i += blockDim.x) {
            const int tl = i / a.K, j = i % a.K, t = c0 + tl;
            if (t < a.T) {
                const int idx = t * a.K + j;
                const int e = staged ? tk[idx] : __ldcg(a.topk + idx);
                const int r = s_base[e] + __popc(s_mask[e] & ((1u << tl) - 1u));
                a.pairs[s_off[e] + r] = idx;
            }
        }
        __syncthreads();
        for (int e = tid; e < a.E; e += blockDim.x) s_base[e] += __popc(s_mask[e]);
        __syncthreads();
    }
}

// The grouping of group_pairs inside one CTA, into shared memory: s_act[0..U) = (expert, first
// pair, pairs, token chunks before), s_act[U] = (-1, T·K, 0, all chunks); s_pairs = the pair
// indices t·K + j, experts ascending, tokens ascending within an expert (the same order).
// scratch: (4·E + E·ceil(T/32) + T·K + 1) ints of shared memory. Every thread calls it; it
// returns U after a barrier.
__device__ int group_cta(const int *topk, int T, int K, int E, int4 *s_act, int *s_pairs, int *scratch) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int TK = T * K, W = (T + 31) >> 5;
    int *s_cnt = scratch, *s_off = s_cnt + E, *s_chp = s_off + E, *s_uidx = s_chp + E;
    uint32_t *s_mask = reinterpret_cast<uint32_t *>(s_uidx + E);     // (E, W): tokens of expert e
    int *s_tk = reinterpret_cast<int *>(s_mask + E * W);
    int *s_u = s_tk + TK;
    for (int e = tid; e < E; e += blockDim.x) s_cnt[e] = 0;
    for (int i = tid; i < E * W; i += blockDim.x) s_mask[i] = 0u;
    for (int i = tid; i < TK; i += blockDim.x) s_tk[i] = __ldcg(topk + i);
    __syncthreads();
    for (int i = tid; i < TK; i += blockDim.x) {      // a token's experts are distinct
        const int e = s_tk[i], t = i / K;
        atomicAdd(&s_cnt[e], 1);
        atomicOr(&s_mask[e * W + (t >> 5)], 1u << (t & 31));
    }
    __syncthreads();
    if (warp == 0) {                                  // exclusive scans over experts, 32 at a time
        int o = 0, u = 0, chp = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < E ? s_cnt[e] : 0;
            const int ch = (c + EX_NCHUNK - 1) / EX_NCHUNK, act = c > 0;
            const int ic = warp_incl_scan(c), ich = warp_incl_scan(ch), ia = warp_incl_scan(act);
            if (e < E) {
                s_off[e] = o + ic - c;
                s_chp[e] = chp + ich - ch;
                s_uidx[e] = act ? u + ia - 1 : -1;
            }
            o += __shfl_sync(0xffffffffu, ic, 31);
            chp += __shfl_sync(0xffffffffu, ich, 31);
            u += __shfl_sync(0xffffffffu, ia, 31);
        }
        if (lane == 0) {
            s_act[u] = make_int4(-1, o, 0, chp);
            *s_u = u;
        }
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
        const int u = s_uidx[e];
        if (u >= 0) s_act[u] = make_int4(e, s_off[e], s_cnt[e], s_chp[e]);
    }
    for (int i = tid; i < TK; i += blockDim.x) {      // rank = tokens before t that chose e
        const int e = s_tk[i], t = i / K;
        const uint32_t *m = s_mask + e * W;
        int r = __popc(m[t >> 5] & ((1u << (t & 31)) - 1u));
        for (int w = 0; w < (t >> 5); ++w) r += __popc(m[w]);
        s_pairs[s_off[e] + r] = i;
    }
    __syncthreads();
    return *s_u;
}

// Sum of each of the N values over the warp's 32 lanes: for N = 32 or 64 by halving exchanges
// (N - 2 or N - 1 shuffles; lane L ends with the sums of values (N/32)·L + j in v[j]), else one
// warp sum per value (every lane ends with all N sums).
template <int N>
__device__ __forceinline__ void warp_sums(float (&v)[N]) {
    const int lane = threadIdx.x & 31;
    if constexpr (N == 32 || N == 64) {
#pragma unroll
        for (int o = 16, n = N / 2; o >= 1; o >>= 1, n >>= 1) {
            const bool up = lane & o;                   // keep the upper half of the current range
#pragma unroll
            for (int i = 0; i < n; ++i) {
                const float send = up ? v[i] : v[n + i];
                const float keep = up ? v[n + i] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = warp_sum(v[i]);
    }
}

// TB tokens per CTA: 8, or the batch itself for one or two tokens (a tile of 8 costs a lone token
// the larger staging and the unrolled token loops). Dynamic shared memory: the tile's (TB, D)
// rows and the gain (D), copied in at kernel entry (it does not depend on the previous kernel).
// The router rows are read from L2 (prefetched at entry): staged in shared memory they make the
// CTA too large to share an SM with the previous kernel's CTAs, and the clusters start late.
template <int TB>
__global__ void __launch_bounds__(R_THREADS, 2) k_router(RouterArgs a) {
    extern __shared__ __align__(16) float xs[];           // (TB, D): hh, then xn; then the gain
    __shared__ uint8_t s_p2e[64];
    __shared__ float s_red[R_THREADS / 32][TB];
    __shared__ float s_inv[TB];
    __shared__ float s_part[R_THREADS / 32][TB * 4];
    __shared__ float s_lg[TB][MAX_E];                     // logits of the tokens this CTA routes
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.y * TB, nt = min(TB, a.T - t0);
    if (tid < 64) s_p2e[tid] = perm_of(a.xn_enc).pos_to_elem[tid];
    const int e0 = blockIdx.x * a.eb;
    const int ne = max(0, min(a.eb, a.E - e0));
    const int D = a.D, D4 = D / 4;
    float *gsm = xs + TB * D;
    // the GEMV's router rows (below): a warp's K chunks of four experts at a time. When they fit
    // one set of registers (d_model <= 2048) the first group is loaded here, before the wait on
    // the previous kernel, and each next group while the current one is reduced.
    constexpr int RC = 2;
    const bool one_pass = D / 128 <= RC * (R_THREADS / 32);
    const float *wrow = a.wgate + (size_t)e0 * D;
    float4 w[RC][4];
    auto load_w = [&](int eg, int c0) {
#pragma unroll
        for (int r = 0; r < RC; ++r) {
            const int c = c0 + r * (R_THREADS / 32);
#pragma unroll
            for (int el = 0; el < 4; ++el)
                w[r][el] = c < D / 128 && eg + el < ne
                               ? __ldg(reinterpret_cast<const float4 *>(wrow + (size_t)(eg + el) * D) + c * 32 + lane)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    if (one_pass) load_w(0, warp);
    {   // the gain into shared memory, the remaining router rows into L2
        for (int i = tid; i < D4; i += R_THREADS)
            cp_async16(reinterpret_cast<float4 *>(gsm) + i, reinterpret_cast<const float4 *>(a.ln2) + i);
        const char *wb = reinterpret_cast<const char *>(wrow);
        const size_t wbytes = (size_t)ne * D * sizeof(float);
        for (size_t o = (size_t)tid * 128; o < wbytes; o += (size_t)R_THREADS * 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(wb + o));
    }
    pdl_wait();                                           // x comes from the previous kernel
    pdl_launch_dependents();
    if (blockIdx.x == 0 && blockIdx.y == 0) {
        // per-forward state: status word and counters, the padding operand row
        if (tid < WS_HDR_INTS) a.status[tid] = 0;
        for (int i = tid; i < a.n_dep; i += R_THREADS) a.dep[i] = 0;
        for (int i = tid; i < (D > a.F ? D : a.F) / 2; i += R_THREADS)
            reinterpret_cast<uint32_t *>(a.zero_row)[i] = 0u;
    }

    // hh = x + attn (qwen3_moe.c:178), then rmsnorm (kernels.c:408-413): inv = 1 / sqrt(sum(x^2)/n
    // + eps); xn = x * inv * g. When a token row is exactly two float4 per thread (d_model 2048
    // with 256 threads) the tile stays in registers from the loads to the normalised store: thread
    // i holds float4 columns i and i + 256 of every token, its sums of squares per token are
    // reduced over the warp and then over the warps in order. Otherwise the same steps run through
    // shared memory. The loads are all in flight before any is used (the kernel is latency-bound).
    if (TB == R_TB && D4 == 2 * R_THREADS) {
        const float4 *x4 = reinterpret_cast<const float4 *>(a.x + (size_t)t0 * D);
        const float4 *a4 = a.attn ? reinterpret_cast<const float4 *>(a.attn + (size_t)t0 * D) : nullptr;
        float4 v[TB][2];
#pragma unroll
        for (int t = 0; t < TB; ++t)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                v[t][h] = t < nt ? __ldg(x4 + t * D4 + h * R_THREADS + tid) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (a4) {
#pragma unroll
            for (int t = 0; t < TB; ++t)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    if (t < nt) {
                        const float4 b = __ldg(a4 + t * D4 + h * R_THREADS + tid);
                        v[t][h].x += b.x; v[t][h].y += b.y; v[t][h].z += b.z; v[t][h].w += b.w;
                    }
                }
        }
        float ss[TB];
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            float q = 0.0f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                q = fmaf(v[t][h].x, v[t][h].x, q);
                q = fmaf(v[t][h].y, v[t][h].y, q);
                q = fmaf(v[t][h].z, v[t][h].z, q);
                q = fmaf(v[t][h].w, v[t][h].w, q);
            }
            ss[t] = warp_sum(q);
        }
        if (lane == 0)
#pragma unroll
            for (int t = 0; t < TB; ++t) s_red[warp][t] = ss[t];
        cp_async_wait_all();                              // this thread's gain copies
        __syncthreads();
        if (tid < nt) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < R_THREADS / 32; ++w) tot += s_red[w][tid];
            s_inv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(tot, (float)D) + a.eps));
        }
        __syncthreads();
        const float4 *g4 = reinterpret_cast<const float4 *>(gsm);
        const float4 g0 = g4[tid], g1 = g4[R_THREADS + tid];
        float4 *s4 = reinterpret_cast<float4 *>(xs);
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            if (t < nt) {
                const float inv = s_inv[t];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float4 gv = h ? g1 : g0;
                    float4 o;
                    o.x = __fmul_rn(__fmul_rn(v[t][h].x, inv), gv.x);
                    o.y = __fmul_rn(__fmul_rn(v[t][h].y, inv), gv.y);
                    o.z = __fmul_rn(__fmul_rn(v[t][h].z, inv), gv.z);
                    o.w = __fmul_rn(__fmul_rn(v[t][h].w, inv), gv.w);
                    s4[t * D4 + h * R_THREADS + tid] = o;
                }
            }
        }
    } else {
        {
            const float4 *x4 = reinterpret_cast<const float4 *>(a.x + (size_t)t0 * D);
            const float4 *a4 = a.attn ? reinterpret_cast<const float4 *>(a.attn + (size_t)t0 * D) : nullptr;
            float4 *s4 = reinterpret_cast<float4 *>(xs);
            const int n4 = nt * D4;
            for (int i0 = tid; i0 < n4; i0 += 16 * R_THREADS) {
                float4 v[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const int i = i0 + u * R_THREADS;
                    if (i < n4) v[u] = __ldg(x4 + i);
                }
                if (a4) {
#pragma unroll
                    for (int u = 0; u < 16; ++u) {
                        const int i = i0 + u * R_THREADS;
                        if (i < n4) {
                            const float4 b = __ldg(a4 + i);
                            v[u].x += b.x; v[u].y += b.y; v[u].z += b.z; v[u].w += b.w;
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const int i = i0 + u * R_THREADS;
                    if (i < n4) s4[i] = v[u];
                }
            }
        }
        __syncthreads();
        const float4 *s4 = reinterpret_cast<const float4 *>(xs);
        float ss[TB];
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            ss[t] = 0.0f;
            if (t < nt)
                for (int c = tid; c < D4; c += R_THREADS) {
                    const float4 v = s4[t * D4 + c];
                    ss[t] = fmaf(v.x, v.x, ss[t]);
                    ss[t] = fmaf(v.y, v.y, ss[t]);
                    ss[t] = fmaf(v.z, v.z, ss[t]);
                    ss[t] = fmaf(v.w, v.w, ss[t]);
                }
        }
#pragma unroll
        for (int t = 0; t < TB; ++t) ss[t] = warp_sum(ss[t]);
        if (lane == 0)
#pragma unroll
            for (int t = 0; t < TB; ++t) s_red[warp][t] = ss[t];
        cp_async_wait_all();                              // this thread's gain copies
        __syncthreads();
        if (tid < nt) {
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < R_THREADS / 32; ++w) tot += s_red[w][tid];
            s_inv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(tot, (float)D) + a.eps));
        }
        __syncthreads();
        const float4 *g4 = reinterpret_cast<const float4 *>(gsm);
        float4 *r4 = reinterpret_cast<float4 *>(xs);
        for (int i = tid; i < nt * D4; i += R_THREADS) {
            const int t = i / D4;
            const float inv = s_inv[t];
            const float4 gv = g4[i - t * D4];
            float4 v = r4[i];
            v.x = __fmul_rn(__fmul_rn(v.x, inv), gv.x);
            v.y = __fmul_rn(__fmul_rn(v.y, inv), gv.y);
            v.z = __fmul_rn(__fmul_rn(v.z, inv), gv.z);
            v.w = __fmul_rn(__fmul_rn(v.w, inv), gv.w);
            r4[i] = v;
        }
    }
    __syncthreads();
    // xn for the expert kernels as fp16 hi | lo halves (row of 2·D), in their K order: CTA x of
    // the cluster writes token x of the tile, eight values (two 16-byte stores) per thread
    for (int t = blockIdx.x; t < nt; t += gridDim.x) {
        const float *row = xs + t * D;
        __half *dst = a.xn_perm + (size_t)(t0 + t) * 2 * D;
        for (int p0 = tid * 8; p0 < D; p0 += R_THREADS * 8) {
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int q0 = p0 + 2 * k, q1 = q0 + 1;
                split_half2(row[(q0 & ~63) + s_p2e[q0 & 63]], row[(q1 & ~63) + s_p2e[q1 & 63]], hi[k], lo[k]);
            }
            *reinterpret_cast<uint4 *>(dst + p0) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4 *>(dst + D + p0) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
    }
    // logits = Wgate·xn (matmul_wx, kernels.c:84-95), four experts of the CTA at a time: warp w
    // takes the 128-value K chunks w, w + 8, ... of every (token, expert) pair (lane l: values
    // 4l..4l+3 of the chunk; the router rows' loads of a group are all in flight before its
    // FMAs), then the lanes' and the warps' partial sums are added (warps in order). Each logit
    // goes to the logits output and into the shared memory of the cluster CTA that routes its
    // token (rank t mod cluster size).
    const int rank = cluster_ctarank(), csz = cluster_nctarank();
    const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
    for (int eg = 0; eg < ne; eg += 4) {
        float acc[TB * 4];
#pragma unroll
        for (int i = 0; i < TB * 4; ++i) acc[i] = 0.0f;
        for (int c0 = warp; c0 < D / 128; c0 += RC * (R_THREADS / 32)) {
            if (!one_pass) load_w(eg, c0);
#pragma unroll
            for (int r = 0; r < RC; ++r) {
                const int c = c0 + r * (R_THREADS / 32);
                if (c >= D / 128) break;
#pragma unroll
                for (int t = 0; t < TB; ++t) {
                    if (t < nt) {
                        const float4 xv = xs4[t * D4 + c * 32 + lane];
#pragma unroll
                        for (int el = 0; el < 4; ++el) {
                            float v = acc[t * 4 + el];
                            v = fmaf(w[r][el].x, xv.x, v);
                            v = fmaf(w[r][el].y, xv.y, v);
                            v = fmaf(w[r][el].z, xv.z, v);
                            v = fmaf(w[r][el].w, xv.w, v);
                            acc[t * 4 + el] = v;
                        }
                    }
                }
            }
        }
        if (one_pass && eg + 4 < ne) load_w(eg + 4, warp);     // in flight during the reduction
        warp_sums<TB * 4>(acc);
        if constexpr (TB * 4 == 32) {
            s_part[warp][lane] = acc[0];
        } else {
            if (lane == 0)
#pragma unroll
                for (int i = 0; i < TB * 4; ++i) s_part[warp][i] = acc[i];
        }
        __syncthreads();
        if (tid < TB * 4) {
            const int t = tid >> 2, el = tid & 3;
            if (t < nt && eg + el < ne) {
                float v = 0.0f;
#pragma unroll
                for (int w2 = 0; w2 < R_THREADS / 32; ++w2) v += s_part[w2][tid];
                const int e = e0 + eg + el;
                a.logits[(size_t)(t0 + t) * a.E + e] = v;
                const uint32_t dst = smem_u32(&s_lg[t / csz][e]);
                uint32_t remote;
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(dst), "r"(t % csz));
                asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
            }
        }
        __syncthreads();
    }
    // every logit of the tile is in its routing CTA's shared memory once the cluster (all CTAs of
    // this token tile) has passed the barrier (release/acquire at cluster scope); CTA r then
    // routes tokens r, r + cluster size, ... of the tile, each with the whole CTA
    cluster_sync();
    __shared__ __align__(16) float s_p[MAX_E + MAX_K];
    __shared__ int s_e[MAX_K];
    __shared__ float s_w[MAX_K];
    for (int r = rank, j = 0; r < nt; r += csz, ++j) {
        const int t = t0 + r;
        select_topk<MAX_E, MAX_K, true>(s_lg[j], a.E, a.K, s_e, s_w, s_p);
        if (tid < a.K) {
            a.topk[(size_t)t * a.K + tid] = s_e[tid];
            a.wt[(size_t)t * a.K + tid] = s_w[tid];
        }
        __syncthreads();
    }
}

// Batches of more than EX_GROUP_MAX pairs: one CTA groups the (token, slot) pairs by expert
// into the workspace (smaller batches are grouped by the gate/up kernel itself).
constexpr int RT_THREADS = 512;
__global__ void __launch_bounds__(RT_THREADS) k_group(RouterArgs a) {
    pdl_wait();                                           // top-k from k_router
    pdl_launch_dependents();
    group_pairs(a);
}

// ------------------------------------------------------------------ experts
struct ExpertArgs {
    int D, F, K;
    const int *n_active, *pairs;
    const int4 *act;             // active-expert table (see RouterArgs)
    // GATEUP with topk set: group topk (T, K) over E experts in each CTA, CTA 0 writing the
    // table to the three pointers below for the later kernels; otherwise read it from above
    const int *topk;
    int T, E;
    int *g_n_active, *g_pairs;
    int4 *g_act;
    const __half *bsrc;          // GATEUP: xn_perm (T, D); DOWN: h_perm (pairs, F)
    __half *h_out;               // GATEUP output (pairs, F), permuted for Wd
    float *y_out;                // DOWN output (T*K, D), row = t*K + j
    int h_enc;                   // encoding of Wd (permutation of h_out)
    const __half *zero_row;      // operand row for padded token columns (zeroed with the header)
    int *status;
    int *item_ctr;               // dynamic work counter (zeroed with the header)
    int *dep;                    // KIND_BOTH: per token chunk, gate/up warps whose h is stored (zeroed by the router)
    int stages;
    const uint8_t *tiles;        // the layer's expert matrices in the decode tile layout, (E, 3)
};

// An item is one row block of one active expert for one chunk of its tokens; it streams through
// the stage ring in K slices of 256 values (eight groups per row: 144 B of Q4_0, 272 B of Q8_0).
// GATEUP: features [64m, 64m + 64) of gate and up, 8 interleaved tiles; warp w holds tile w
// (gate rows 8w..8w+7 over the same up rows), so each thread ends with the gate and the up sum of
// its feature and forms h itself.
// DOWN: 128 rows of Wd, warp w holds tile w. Every warp keeps its rows over the whole K.
template <int ENC, int KIND>
struct ExCfg {
    static constexpr int GB = ENC == CPG_ENC_Q4 ? 18 : 34;
    static constexpr int SLB = 8 * GB;                        // bytes of one row's K slice
    static constexpr int MATS = KIND == KIND_GATEUP ? 2 : 1;
    static constexpr int RB = KIND == KIND_GATEUP ? 64 : 128; // rows per matrix per item
    static constexpr int WBYTES = MATS * RB * SLB;             // weight tiles of a stage
    // one token's row slice in shared memory: hi half (512 B), 16 B gap, lo half, 16 B gap. The
    // gap puts a row's hi and lo reads on different banks (lanes 2i and 2i+1 of a quarter warp
    // read the two halves of one token).
    static constexpr int LOFF = EX_KSL * 2 + 16;
    static constexpr int BROW = 2 * LOFF;
    static constexpr int STAGE = WBYTES + EX_NCHUNK * BROW;    // + the chunk's token rows
    static constexpr int WPAIR = GB / 2;                       // 32-bit words per group pair
};

struct StageMeta { int item, m, off, cnt, s, kind, chunk, pad; };   // off/cnt: the item's token chunk; s: K slice;
                                                                      // chunk: its index over all experts

// Item -> (active expert u, row tile m, token chunk c). Items run expert-major, then row tile,
// then chunk, so the chunks of one weight tile are fetched back to back (the later fetches hit
// L2). items_before(u) = tiles * chunks_before(u), from the router's table in shared memory.
__device__ __forceinline__ void decode_item(const int4 *act, int U, int tiles, int item, int &u, int &m, int &c) {
    int lo = 0, hi = U;                       // last u with items_before(u) <= item
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (tiles * act[mid].w <= item) lo = mid; else hi = mid;
    }
    u = lo;
    const int nch = act[u + 1].w - act[u].w;
    const int local = item - tiles * act[u].w;
    m = local / nch;
    c = local - m * nch;
}


// One K slice of a tile against NTL token tiles: the eight groups one at a time (two k16 MMAs
// into a fresh sum per token tile, then the group's fp32 scale), so that only one group's
// fragments (8 registers) and one token tile's operand are live. Holding a whole group pair's
// fragments and the next pair's operands in registers instead spilled at the kernel's 96
// registers and measured 4 % slower (k_experts<Q4, BOTH>, 64 tokens).
template <int ENC, int NTL, int TSTRIDE>
__device__ __forceinline__ void slice_mma(const uint8_t *tp, int lane, const uint8_t *bs, float (&acc)[EX_NCH][4]) {
    using X = ExTile<ENC>;
    const uint2 *sc = reinterpret_cast<const uint2 *>(tp + X::DB + (lane >> 2) * 32);   // scales, 2 pairs a load
#pragma unroll
    for (int P = 0; P < 4; ++P) {
        const uint2 sg = sc[(P >> 1)], s8 = sc[2 + (P >> 1)];
        const uint32_t dg = P & 1 ? sg.y : sg.x, d8 = P & 1 ? s8.y : s8.x;
        const float2 fg = __half22float2(*reinterpret_cast<const __half2 *>(&dg));
        const float2 f8 = __half22float2(*reinterpret_cast<const __half2 *>(&d8));
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {                     // group 2P + hf
            uint32_t fh[2][4];
            group_frags<ENC>(tp, P, hf, lane, fh);
            const float d0 = hf ? fg.y : fg.x, d1 = hf ? f8.y : f8.x;   // rows g / g + 8
#pragma unroll
            for (int nt = 0; nt < NTL; ++nt) {
                const uint4 bq = *reinterpret_cast<const uint4 *>(bs + nt * TSTRIDE + P * 128 + hf * 16);
                const float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                float sj[4];
                mma_16816(sj, fh[0], bq.x, bq.y, z);
                mma_16816(sj, fh[1], bq.z, bq.w, sj);
                fma2_f32(acc[nt][0], acc[nt][1], d0, sj[0], sj[1]);
                fma2_f32(acc[nt][2], acc[nt][3], d1, sj[2], sj[3]);
            }
        }
    }
}

// Builds the decode tiles of every expert of a layer from the raw Q4_0/Q8_0 rows: per expert
// (3·MB bytes) the interleaved gate/up matrix (2·d_exp rows, tile rt = gate rows [8rt, 8rt + 8)
// over the same up rows) and then the down matrix; one thread per (expert, tile, lane). mats:
// device table (E·3) of matrix pointers, [3e + kind].
template <int ENC>
__global__ void k_tile_experts(const uint8_t *const *mats, uint8_t *out, int E, int D, int F) {
    using X = ExTile<ENC>;
    const size_t MB = (size_t)F * D / 32 * X::GB;             // bytes per matrix, every kind
    const int ntile = (F / 16) * (D / EX_KSL);                 // tiles per matrix, every kind
    const long n = (long)E * 3 * ntile * 32;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const long q = i >> 5;
        const int e = (int)(q / (3 * ntile)), r = (int)(q - (long)e * 3 * ntile);
        uint8_t *dst = out + (size_t)e * 3 * MB + (size_t)r * X::TB;
        if (r < 2 * ntile) {                                   // gate/up: D/256 slices of 2F/16 tiles
            const int RT = F / 8, s = r / RT, rt = r - s * RT;
            const size_t rowb = (size_t)D / 32 * X::GB, off = (size_t)rt * 8 * rowb + (size_t)s * 8 * X::GB;
            tile_build_lane<ENC>(mats[3 * e] + off, mats[3 * e + 1] + off, rowb, dst, lane);
        } else {                                               // down: F/256 slices of D/16 tiles
            const int RT = D / 16, s = (r - 2 * ntile) / RT, rt = (r - 2 * ntile) - s * RT;
            const size_t rowb = (size_t)F / 32 * X::GB;
            const uint8_t *src = mats[3 * e + 2] + (size_t)rt * 16 * rowb + (size_t)s * 8 * X::GB;
            tile_build_lane<ENC>(src, src + 8 * rowb, rowb, dst, lane);
        }
    }
}

// Bounded wait until *p >= need (gpu-scope acquire). Returns false after kWaitLimitNs.
__device__ __forceinline__ bool wait_count_geq(const int *p, int need) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= need) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        __nanosleep(64);
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (v >= need) return true;
        if ((i & 63u) == 0 && global_ns() - t0 > kWaitLimitNs) return false;
    }
}

// KIND_GATEUP, KIND_DOWN: one matrix kind per launch. KIND_BOTH: one launch for the whole
// block: the gate/up items first, then the down items, from one work counter. A down item needs
// the h rows of its token chunk, which the chunk's F/64 gate/up items store: each consumer warp
// of those bumps the chunk's counter (release) after its stores, and the down item's token-row
// warp waits for F/64 × 8 (acquire, bounded) before copying the rows. Items are claimed in order, so a down
// item only ever waits for gate/up items that running CTAs have already claimed: no CTA needs
// another to become resident, and the down items fill the SMs the gate/up tail leaves idle.
template <int ENC, int KIND>
__global__ void __launch_bounds__((EX_NP + EX_NW) * 32, 2) k_experts(ExpertArgs a) {
    using C = ExCfg<ENC, KIND>;
    using X = ExTile<ENC>;
    constexpr bool HAS_GU = KIND != KIND_DOWN, HAS_DN = KIND != KIND_GATEUP;
    // Dynamic shared memory starts after the static arrays, 16-byte aligned only; the stages
    // (bulk copy destinations) are placed on 128 bytes (the launch adds the slack).
    // Layout: stages | barriers | stage metadata.
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t *const smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    __shared__ Perm64 s_perm;
    __shared__ int s_abort;
    __shared__ int4 s_act[MAX_E + 1];
    __shared__ int s_pairs[HAS_GU ? EX_GROUP_MAX : 1];
    const int S = a.stages;
    const int tiles_gu = a.F / 64, tiles_dn = a.D / 128;     // row blocks per matrix and chunk
    const int ns_gu = a.D / EX_KSL, ns_dn = a.F / EX_KSL;     // K slices per item
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S * C::STAGE);   // STAGE: a multiple of 16
    uint64_t *empty = full + S;
    uint64_t *mready = empty + S;                              // stage metadata written
    StageMeta *meta = reinterpret_cast<StageMeta *>(mready + S);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t MB = (size_t)a.D * a.F / 32 * X::GB;          // bytes per expert matrix

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1 + 32);           // weight producer + the 32 token-row lanes
            mbar_init(&empty[s], EX_NW);
            mbar_init(&mready[s], 1);
        }
        fence_mbar_init();
        s_abort = 0;
    }
    if (threadIdx.x < 64) {
        const Perm64 &pm = perm_of(a.h_enc);
        s_perm.pos_to_elem[threadIdx.x] = pm.pos_to_elem[threadIdx.x];
        s_perm.elem_to_pos[threadIdx.x] = pm.elem_to_pos[threadIdx.x];
    }
    pdl_wait();                                  // top-k from k_router / table and h from gate-up
    pdl_launch_dependents();
    const bool self_group = HAS_GU && a.topk != nullptr;
    int U;
    if (self_group) {
        // the stage ring is not in use yet: it holds the grouping scratch
        U = group_cta(a.topk, a.T, a.K, a.E, s_act, s_pairs, reinterpret_cast<int *>(smem));
        if (blockIdx.x == 0) {                   // the table for the down and combine kernels
            for (int u = threadIdx.x; u <= U; u += blockDim.x) a.g_act[u] = s_act[u];
            for (int i = threadIdx.x; i < a.T * a.K; i += blockDim.x) a.g_pairs[i] = s_pairs[i];
            if (threadIdx.x == 0) *a.g_n_active = U;
        }
    } else {
        U = *a.n_active;
        for (int u = threadIdx.x; u <= U; u += blockDim.x) s_act[u] = a.act[u];
        __syncthreads();
    }
    const int chunks = s_act[U].w;
    const int total_gu = HAS_GU ? tiles_gu * chunks : 0;
    const int total = total_gu + (HAS_DN ? tiles_dn * chunks : 0);
    const int *pairs = self_group ? s_pairs : a.pairs;

    if (warp == 1) {
        // ---------------- token-row producer: the whole warp, the chunk's rows of each K slice by
        // 16-byte asynchronous copies (lane l copies bytes [16l, 16l + 16) of every row's slice;
        // the copies of one warp instruction read 512 contiguous bytes). A bulk copy per row would
        // queue up to 16 copies per stage behind one issuing thread. Each lane's copies count as
        // one arrival on the stage's full barrier once they have landed.
        int trow[EX_NCHUNK];                                    // source row of each token column
        const __half *src = a.bsrc;
        int cur = -1, rlen = 0;
        for (int it = 0;; ++it) {
            const int st = it % S;
            if (!mbar_wait(&mready[st], (uint32_t)(it / S) & 1u)) {
                if (lane == 0) atomicCAS(a.status + WS_STATUS, ST_OK, ST_TIMEOUT_FULL);
                break;
            }
            const StageMeta md = meta[st];
            if (md.item < 0) {                                 // sentinel
                mbar_arrive(&full[st]);
                break;
            }
            if (md.item != cur) {                              // the chunk's token rows (fp16, permuted K)
                cur = md.item;
                const bool gu = md.kind == KIND_GATEUP;
                if (KIND == KIND_BOTH && !gu) {                // h of this chunk stored by its gate/up items
                    if (!wait_count_geq(a.dep + md.chunk, tiles_gu * EX_NW) && lane == 0)
                        atomicCAS(a.status + WS_STATUS, ST_OK, ST_TIMEOUT_FULL);
                    __threadfence();
                }
                src = KIND == KIND_BOTH && !gu ? a.h_out : a.bsrc;
                rlen = gu ? a.D : a.F;                         // a source row is hi | lo, rlen each
#pragma unroll
                for (int j = 0; j < EX_NCHUNK; ++j) {
                    const int p = md.off + min(j, md.cnt - 1);
                    trow[j] = gu ? pairs[p] / a.K : p;
                }
            }
            uint8_t *dst = smem + (size_t)st * C::STAGE + C::WBYTES + lane * 16;
            const __half *sl = src + (size_t)md.s * EX_KSL + lane * 8;
#pragma unroll
            for (int j = 0; j < EX_NCHUNK; ++j) {              // columns past cnt keep stale rows: their
                if (j < md.cnt) {                              // results are never stored
                    const __half *r = sl + (size_t)trow[j] * 2 * rlen;
                    cp_async16(dst + j * C::BROW, r);
                    cp_async16(dst + j * C::BROW + C::LOFF, r + rlen);
                }
            }
            cp_async_mbar_arrive(&full[st]);
        }
        cp_async_wait_all();                                   // nothing in flight when the warp leaves
        return;
    }
    if (warp == 0) {
        // ---------------- weight producer: one thread, one bulk copy per matrix and K slice;
        // it deals the items and publishes each stage's metadata to the token-row producer
        if (lane != 0) return;
        int it = 0;
        bool ok = true, done = false;
        while (!done) {
            const int item = atomicAdd(a.item_ctr, 1);
            const bool gu = HAS_GU && item < total_gu;
            const int kind = gu ? KIND_GATEUP : KIND_DOWN;
            const int li = gu ? item : item - total_gu;
            const int ns = gu ? ns_gu : ns_dn;
            int u = 0, m = 0, c = 0;
            if (item < total) decode_item(s_act, U, gu ? tiles_gu : tiles_dn, li, u, m, c);
            const int4 ex = s_act[u];
            const int c0 = c * EX_NCHUNK;
            const int cnt = item < total ? min(EX_NCHUNK, ex.z - c0) : 0;
            for (int sl = 0; sl < (item < total ? ns : 1); ++sl, ++it) {
                const int st = it % S;
                if (it >= S && !mbar_wait(&empty[st], (uint32_t)(it / S - 1) & 1u)) {
                    atomicCAS(a.status + WS_STATUS, ST_OK, ST_TIMEOUT_EMPTY);
                    ok = false;
                    break;
                }
                if (item >= total) {                           // sentinel: no more items
                    meta[st].item = -1;
                    mbar_arrive(&mready[st]);
                    mbar_arrive(&full[st]);
                    done = true;
                    ++it;
                    break;
                }
                meta[st] = StageMeta{item, m, ex.y + c0, cnt, sl, kind, ex.w + c, 0};
                mbar_arrive(&mready[st]);                      // release: the metadata is visible
                mbar_arrive_expect_tx(&full[st], (uint32_t)C::WBYTES);
                uint8_t *dst = smem + (size_t)st * C::STAGE;
                // the item's row tiles of K slice sl: contiguous in the tile layout
                const uint8_t *te = a.tiles + (size_t)(3 * ex.x) * MB;
                if (gu) {                                      // 8 interleaved gate/up tiles
                    const size_t toff = ((size_t)sl * (a.F / 8) + (size_t)m * 8) * X::TB;
                    bulk_g2s(dst, te + toff, 8 * X::TB, &full[st]);
                } else {
                    const size_t toff = ((size_t)sl * (a.D / 16) + (size_t)m * 8) * X::TB;
                    bulk_g2s(dst, te + 2 * MB + toff, 8 * X::TB, &full[st]);
                }
            }
            if (!ok) break;
        }
        // keep the CTA alive until every issued copy has landed (bounded)
        for (int k = 1; k <= S && it - k >= 0; ++k) {
            const int j = it - k;
            mbar_wait(&full[j % S], (uint32_t)(j / S) & 1u);
        }
        return;
    }

    // ---------------- consumers: gate/up items: warp cw owns 16 rows of matrix cw & 1 (tile
    // cw >> 1 of the item's 64); down items: 16 rows (tile cw of the item's 128); over the whole K
    const int cw = warp - EX_NP;
    const int g = lane >> 2, t = lane & 3;
    // MMA column 8·nt + c holds token 4·nt + c/2 of the item, its hi half for even c, lo for
    // odd c. This lane feeds column g of every tile and receives columns 2t, 2t+1: accumulator
    // acc[nt][0] + acc[nt][1] is token 4·nt + t at row g, acc[nt][2] + acc[nt][3] at row g + 8.
    float acc[EX_NCH][4];
    int ntl = 1;                                           // 8-column tiles in use: ceil(cnt / 4)
    for (int it = 0;; ++it) {
        const int st = it % S;
        if (!mbar_wait(&full[st], (uint32_t)(it / S) & 1u)) {
            if (lane == 0) atomicCAS(a.status + WS_STATUS, ST_OK, ST_TIMEOUT_FULL);
            break;
        }
        const StageMeta md = meta[st];
        if (md.item < 0) break;
        const bool gu = HAS_GU && (!HAS_DN || md.kind == KIND_GATEUP);
        if (md.s == 0) {                                   // a new item
            ntl = (md.cnt + 3) >> 2;
#pragma unroll
            for (int nt = 0; nt < EX_NCH; ++nt)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[nt][c] = 0.0f;
        }
        constexpr int TS = 4 * C::BROW;                    // bytes from one 8-column tile's rows to the next
        const uint8_t *bs = smem + (size_t)st * C::STAGE + C::WBYTES + (g >> 1) * C::BROW + (g & 1) * C::LOFF + t * 32;
        const uint8_t *tp = smem + (size_t)st * C::STAGE + (size_t)cw * X::TB;
        switch (ntl) {
            case 1: slice_mma<ENC, 1, TS>(tp, lane, bs, acc); break;
            case 2: slice_mma<ENC, 2, TS>(tp, lane, bs, acc); break;
            default: slice_mma<ENC, 3, TS>(tp, lane, bs, acc); break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);           // this warp is done with the stage
        if (md.s != (gu ? ns_gu : ns_dn) - 1) continue;
        // ---------------- epilogue of the item: hi and lo partial sums added in fp32
        if (gu) {
            // row g: gate, row g + 8: up, of feature fr
            const int fr = md.m * 64 + cw * 8 + g;
            const int pos = (fr & ~63) + s_perm.elem_to_pos[fr & 63];
#pragma unroll
            for (int nt = 0; nt < EX_NCH; ++nt) {
                const int col = nt * 4 + t;                                                   // token of the item
                if (nt >= ntl || col >= md.cnt) continue;
                const float gv = acc[nt][0] + acc[nt][1], uv = acc[nt][2] + acc[nt][3];
                const float h = gv / (1.0f + expf(-gv)) * uv;                                 // kernels.c:416, qwen3_moe.c:219
                __half *hr = a.h_out + (size_t)(md.off + col) * 2 * a.F;                      // hi | lo
                split_half(h, hr[pos], hr[a.F + pos]);
            }
            if (KIND == KIND_BOTH) {
                __syncwarp();
                if (lane == 0) {
                    __threadfence();                       // the warp's h stores before the count
                    atomicAdd(a.dep + md.chunk, 1);
                }
            }
        } else {
            const int row = md.m * 128 + cw * 16 + g;                                         // rows row, row + 8
#pragma unroll
            for (int nt = 0; nt < EX_NCH; ++nt) {
                const int col = nt * 4 + t;
                if (nt >= ntl || col >= md.cnt) continue;
                float *yr = a.y_out + (size_t)pairs[md.off + col] * a.D;
                yr[row] = acc[nt][0] + acc[nt][1];
                yr[row + 8] = acc[nt][2] + acc[nt][3];
            }
        }
    }
}

// ------------------------------------------------------------------ combine
__global__ void k_combine(const float *__restrict__ x, const float *__restrict__ attn, int T, int D, int K,
                          const float *__restrict__ wt, const float *__restrict__ y, float *mlp, float *x_out) {
    pdl_wait();                                  // y from the down-projection kernel
    pdl_launch_dependents();
    const int n4 = T * D / 4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const int t = (i * 4) / D, k = i * 4 - t * D;
        float4 acc = mlp ? reinterpret_cast<const float4 *>(mlp)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float *wt_t = wt + t * K;
        const float *y_t = y + (size_t)t * K * D + k;
        for (int j0 = 0; j0 < K; j0 += 8) {      // qwen3_moe.c:221: selection order, no fusion
            float4 v[8];
            float w[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (j0 + j < K) {
                    v[j] = __ldg(reinterpret_cast<const float4 *>(y_t + (size_t)(j0 + j) * D));
                    w[j] = __ldg(wt_t + j0 + j);
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (j0 + j < K) {
                    acc.x = __fadd_rn(acc.x, __fmul_rn(w[j], v[j].x));
                    acc.y = __fadd_rn(acc.y, __fmul_rn(w[j], v[j].y));
                    acc.z = __fadd_rn(acc.z, __fmul_rn(w[j], v[j].z));
                    acc.w = __fadd_rn(acc.w, __fmul_rn(w[j], v[j].w));
                }
            }
        }
        if (mlp) reinterpret_cast<float4 *>(mlp)[i] = acc;
        if (x_out) {
            const float4 xv = reinterpret_cast<const float4 *>(x)[i];
            float4 av = attn ? reinterpret_cast<const float4 *>(attn)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            reinterpret_cast<float4 *>(x_out)[i] =
                make_float4(xv.x + (av.x + acc.x), xv.y + (av.y + acc.y), xv.z + (av.z + acc.z), xv.w + (av.w + acc.w));
        }
    }
}

// ------------------------------------------------------------------ host side
struct KernelPlan {
    int stages = 0, ctas = 0;
    size_t smem = 0;
};


}  // namespace cpg

struct cpg_moe_layer {
    int D, F, E, K;
    float eps;
    int enc;                       // expert encoding (Q4 or Q8)
    const float *ln2;
    const float *wgate;
    const uint8_t **d_ptrs;        // device (E, 3)
    std::vector<const uint8_t *> h_ptrs;   // host copy of the same table
    void *d_wmaps = nullptr;       // device (E, 3) TMA tensor maps of the expert matrices, built
                                   // on the first tcgen05 call (cpg_moe_apply)
    uint8_t *d_tiles = nullptr;    // device copy of the expert matrices in the decode tile layout
                                   // (k_tile_experts), built here
    std::mutex wmaps_mu;
    cpg::KernelPlan gateup, down, both;      // two CTAs per SM (Q4_0), ~100 KB of stages each
    cpg::KernelPlan gateup_deep, down_deep;  // one CTA per SM with all the shared memory in stages:
                                             // for launches with at most one item per SM
    cpg::OnePlan one;                        // the one-token layer kernel (moe_one.cu), if it fits
    unsigned *d_one_bar = nullptr;           // its grid-barrier counters (zeroed at creation)
};

namespace cpg {

template <int ENC, int KIND>
static int plan_kernel(KernelPlan &p, bool deep) {
    using C = ExCfg<ENC, KIND>;
    auto *k = k_experts<ENC, KIND>;
    const size_t fixed = 8 * (sizeof(StageMeta) + 24) + 256;
    cudaFuncAttributes fa;
    CPG_CUDA(cudaFuncGetAttributes(&fa, k));
    const size_t limit = (size_t)smem_optin() - fa.sharedSizeBytes;
    // two CTAs per SM (latency hiding comes from warps); stages fill about 100 KB per CTA (three
    // 31 KB Q4_0 stages; Q8_0's 48 KB stages leave room for one CTA per SM). Deep: one CTA per
    // SM, as many stages as fit (up to 8 = every K slice of a gate/up item in flight)
    int S = (int)(((deep ? limit : 100 * 1024) - fixed) / C::STAGE);
    if (S < 2) S = 2;
    if (S > 8) S = 8;
    while (S > 1 && fixed + (size_t)S * C::STAGE > limit) --S;
    CPG_REQUIRE(fixed + (size_t)S * C::STAGE <= limit, "expert kernel: a %d-byte stage does not fit in shared memory",
                C::STAGE);
    p.stages = S;
    p.smem = (size_t)S * C::STAGE + S * sizeof(StageMeta) + 3 * S * sizeof(uint64_t) +
             128;                                           // alignment slack
    int rc = allow_max_smem((const void *)k);
    if (rc) return rc;
    int per_sm = 0;
    CPG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, (EX_NP + EX_NW) * 32, p.smem));
    CPG_REQUIRE(per_sm >= 1, "expert kernel: no CTA fits on an SM");
    p.ctas = per_sm * sm_count();
    return CPG_OK;
}

static int launch_experts(const cpg_moe_layer *L, int KIND, const ExpertArgs &a, int max_items, cudaStream_t s) {
    // few items (one token: 8 experts): one CTA per SM with the whole item's slices in flight
    const bool deep = KIND != KIND_BOTH && max_items <= sm_count();
    const KernelPlan &p = KIND == KIND_BOTH ? L->both
                          : KIND == KIND_GATEUP ? (deep ? L->gateup_deep : L->gateup) : (deep ? L->down_deep : L->down);
    const int grid = max_items < p.ctas ? (max_items > 0 ? max_items : 1) : p.ctas;
    ExpertArgs b = a;
    b.stages = p.stages;
    b.tiles = L->d_tiles;
    const dim3 block((EX_NP + EX_NW) * 32);
    auto *k = L->enc == CPG_ENC_Q4
                  ? (KIND == KIND_BOTH ? k_experts<CPG_ENC_Q4, KIND_BOTH>
                     : KIND == KIND_GATEUP ? k_experts<CPG_ENC_Q4, KIND_GATEUP> : k_experts<CPG_ENC_Q4, KIND_DOWN>)
                  : (KIND == KIND_BOTH ? k_experts<CPG_ENC_Q8, KIND_BOTH>
                     : KIND == KIND_GATEUP ? k_experts<CPG_ENC_Q8, KIND_GATEUP> : k_experts<CPG_ENC_Q8, KIND_DOWN>);
    CPG_CUDA(launch_pdl(k, dim3(grid), block, p.smem, s, b));
    return CPG_OK;
}

}  // namespace cpg

namespace cpg {
int layer_dims(const cpg_moe_layer *L, int *D, int *F, int *E, int *K) {
    CPG_REQUIRE(L, "null layer");
    *D = L->D; *F = L->F; *E = L->E; *K = L->K;
    return CPG_OK;
}
int layer_ptrs(const cpg_moe_layer *L, const uint8_t *const **ptrs, int *enc) {
    CPG_REQUIRE(L, "null layer");
    *ptrs = L->d_ptrs;
    *enc = L->enc;
    return CPG_OK;
}
int layer_one_info(const cpg_moe_layer *L, int *D, int *F, int *E, int *K, int *enc, const float **ln2,
                   const float **wgate, const uint8_t **tiles, float *eps) {
    CPG_REQUIRE(L, "null layer");
    *D = L->D; *F = L->F; *E = L->E; *K = L->K; *enc = L->enc;
    *ln2 = L->ln2; *wgate = L->wgate; *tiles = L->d_tiles; *eps = L->eps;
    return CPG_OK;
}
int gemm_tc_build_weight_maps(const uint8_t *const *h_ptrs, int E, int D, int F, void **d_maps);
int layer_weight_maps(const cpg_moe_layer *Lc, const void **maps) {
    CPG_REQUIRE(Lc, "null layer");
    cpg_moe_layer *L = const_cast<cpg_moe_layer *>(Lc);
    std::lock_guard<std::mutex> g(L->wmaps_mu);
    if (!L->d_wmaps) {
        const int rc = gemm_tc_build_weight_maps(L->h_ptrs.data(), L->E, L->D, L->F, &L->d_wmaps);
        if (rc) return rc;
    }
    *maps = L->d_wmaps;
    return CPG_OK;
}
}  // namespace cpg

using namespace cpg;

namespace cpg {
int router_cluster(int E, int *eb);

// The decode kernels' copy of the layer's expert matrices (k_tile_experts), made from the
// matrices as they are now: the caller's weights must hold their final values.
static int build_tiles(cpg_moe_layer *L) {
    const size_t gb = L->enc == CPG_ENC_Q4 ? 18 : 34;
    const size_t bytes = (size_t)3 * L->E * L->F * L->D / 32 * gb;
    CPG_CUDA(cudaDeviceSynchronize());              // the weights' writers, on any stream
    CPG_CUDA(cudaMalloc((void **)&L->d_tiles, bytes));
    const long threads = (long)L->E * 3 * (L->F / 16) * (L->D / EX_KSL) * 32;
    const int grid = (int)std::min<long>((threads + 255) / 256, (long)sm_count() * 8);
    if (L->enc == CPG_ENC_Q4)
        k_tile_experts<CPG_ENC_Q4><<<grid, 256>>>(L->d_ptrs, L->d_tiles, L->E, L->D, L->F);
    else
        k_tile_experts<CPG_ENC_Q8><<<grid, 256>>>(L->d_ptrs, L->d_tiles, L->E, L->D, L->F);
    CPG_CUDA(cudaGetLastError());
    CPG_CUDA(cudaDeviceSynchronize());
    return CPG_OK;
}
int router_cluster_check(int E, int rsmem, int *n_active = nullptr);
}  // namespace cpg

extern "C" int cpg_moe_layer_create(const cpg_moe_desc *d, cpg_moe_layer **out) {
    CPG_REQUIRE(d && out, "cpg_moe_layer_create: null argument");
    *out = nullptr;
    CPG_REQUIRE(d->d_model > 0 && d->d_model % 256 == 0, "d_model=%d must be a positive multiple of 256", d->d_model);
    CPG_REQUIRE(d->d_exp > 0 && d->d_exp % 256 == 0, "d_exp=%d must be a positive multiple of 256", d->d_exp);
    CPG_REQUIRE(d->n_experts > 0 && d->n_experts <= MAX_E, "n_experts=%d outside [1, %d]", d->n_experts, MAX_E);
    CPG_REQUIRE(d->topk > 0 && d->topk <= MAX_K && d->topk <= d->n_experts, "topk=%d outside [1, min(%d, n_experts)]", d->topk, MAX_K);
    CPG_REQUIRE(d->ln2 && d->wgate.p && d->experts, "cpg_moe_layer_create: null tensor");
    CPG_REQUIRE(d->wgate.enc == CPG_ENC_F32, "router weights must be f32 (the reference keeps Wgate f32)");
    CPG_REQUIRE(((uintptr_t)d->wgate.p & 15) == 0, "router weights must be 16-byte aligned");
    CPG_REQUIRE(((uintptr_t)d->ln2 & 15) == 0, "ln2 must be 16-byte aligned");
    const int enc = d->experts[0].enc;
    CPG_REQUIRE(enc == CPG_ENC_Q4 || enc == CPG_ENC_Q8, "expert encoding %d is not Q4_0/Q8_0", enc);
    const int E = d->n_experts;
    const uint8_t **h = (const uint8_t **)malloc(sizeof(void *) * 3 * E);
    CPG_REQUIRE(h != nullptr, "host allocation failed");
    for (int i = 0; i < 3 * E; ++i) {
        if (!d->experts[i].p || d->experts[i].enc != enc || ((uintptr_t)d->experts[i].p & 15)) {
            free(h);
            CPG_REQUIRE(false, "expert tensor %d (expert %d kind %d): null, unaligned or encoding != %d", i, i / 3, i % 3, enc);
        }
        h[i] = (const uint8_t *)d->experts[i].p;
    }
    cpg_moe_layer *L = new cpg_moe_layer();
    L->D = d->d_model; L->F = d->d_exp; L->E = E; L->K = d->topk; L->eps = d->rms_eps;
    L->enc = enc; L->ln2 = d->ln2; L->wgate = (const float *)d->wgate.p;
    L->h_ptrs.assign(h, h + 3 * E);
    cudaError_t ce = cudaMalloc((void **)&L->d_ptrs, sizeof(void *) * 3 * E);
    if (ce == cudaSuccess) ce = cudaMemcpy(L->d_ptrs, h, sizeof(void *) * 3 * E, cudaMemcpyHostToDevice);
    free(h);
    if (ce != cudaSuccess) {
        cudaFree(L->d_ptrs);
        delete L;
        return cuda_fail(ce, "cpg_moe_layer_create: expert table upload");
    }
    int rc;
    if (enc == CPG_ENC_Q4) {
        rc = plan_kernel<CPG_ENC_Q4, KIND_GATEUP>(L->gateup, false);
        if (rc == CPG_OK) rc = plan_kernel<CPG_ENC_Q4, KIND_BOTH>(L->both, false);
        if (rc == CPG_OK) rc = plan_kernel<CPG_ENC_Q4, KIND_DOWN>(L->down, false);
        if (rc == CPG_OK) rc = plan_kernel<CPG_ENC_Q4, KIND_GATEUP>(L->gateup_deep, true);
        if (rc == CPG_OK) rc = plan_kernel<CPG_ENC_Q4, KIND_DOWN>(L->down_deep, true);
    } else {
        rc = plan_kernel<CPG_ENC_Q8, KIND_GATEUP>(L->gateup, false);
        if (rc == CPG_OK) rc = plan_kernel<CPG_ENC_Q8, KIND_BOTH>(L->both, false);
        if (rc == CPG_OK) rc = plan_kernel<CPG_ENC_Q8, KIND_DOWN>(L->down, false);
        if (rc == CPG_OK) rc = plan_kernel<CPG_ENC_Q8, KIND_GATEUP>(L->gateup_deep, true);
        if (rc == CPG_OK) rc = plan_kernel<CPG_ENC_Q8, KIND_DOWN>(L->down_deep, true);
    }
    if (rc == CPG_OK) rc = build_tiles(L);
    if (rc == CPG_OK) rc = one_plan(L, &L->one);
    if (rc == CPG_OK && L->one.ok) {
        cudaError_t ce = cudaMalloc((void **)&L->d_one_bar, 2 * sizeof(unsigned));
        if (ce == cudaSuccess) ce = cudaMemset(L->d_one_bar, 0, 2 * sizeof(unsigned));
        if (ce != cudaSuccess) rc = cuda_fail(ce, "cpg_moe_layer_create: barrier counters");
    }
    if (rc == CPG_OK) {
        // the token tile's rows, plus the CTA's router rows when they fit beside them (static
        // shared memory of the kernel: about 12 KB)
        const int rsmem = (R_TB + 1) * L->D * (int)sizeof(float);        // the tile's rows and the gain
        if (rsmem > smem_optin() - 16 * 1024) {
            set_error("d_model=%d too large for the router kernel", L->D);
            rc = CPG_EINVAL;
        } else {
            rc = allow_max_smem((const void *)k_router<1>);
            if (rc == CPG_OK) rc = allow_max_smem((const void *)k_router<2>);
            if (rc == CPG_OK) rc = allow_max_smem((const void *)k_router<R_TB>);
            if (rc == CPG_OK) rc = router_cluster_check(E, rsmem);
        }
    }
    if (rc != CPG_OK) {
        cudaFree(L->d_ptrs);
        if (L->d_tiles) cudaFree(L->d_tiles);
        if (L->d_one_bar) cudaFree(L->d_one_bar);
        delete L;
        return rc;
    }
    *out = L;
    return CPG_OK;
}

namespace cpg {
// CTAs per router cluster for E experts (experts per CTA: at least one per warp).
int router_cluster(int E, int *eb) {
    const int min_eb = (E + R_CLUSTER_MAX - 1) / R_CLUSTER_MAX;
    *eb = min_eb > R_THREADS / 32 ? min_eb : R_THREADS / 32;
    return (E + *eb - 1) / *eb;
}

// The router's clusters must fit on this device (checked once per layer).
int router_cluster_check(int E, int rsmem, int *n_active) {
    int eb = 0;
    const int csz = router_cluster(E, &eb);
    CPG_CUDA(cudaFuncSetAttribute(k_router<1>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    CPG_CUDA(cudaFuncSetAttribute(k_router<2>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    CPG_CUDA(cudaFuncSetAttribute(k_router<R_TB>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(csz, 1);
    cfg.blockDim = dim3(R_THREADS);
    cfg.dynamicSmemBytes = (size_t)rsmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)csz;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    CPG_CUDA(cudaOccupancyMaxActiveClusters(&n, k_router<R_TB>, &cfg));
    if (n_active) *n_active = n;
    CPG_REQUIRE(n >= 1, "router kernel: a cluster of %d CTAs does not fit on this device", csz);
    return CPG_OK;
}
}  // namespace cpg

extern "C" void cpg_moe_layer_destroy(cpg_moe_layer *L) {
    if (!L) return;
    cudaFree(L->d_ptrs);
    if (L->d_tiles) cudaFree(L->d_tiles);
    if (L->d_wmaps) cudaFree(L->d_wmaps);
    if (L->d_one_bar) cudaFree(L->d_one_bar);
    delete L;
}

extern "C" size_t cpg_moe_workspace_bytes(const cpg_moe_layer *L, int max_T) {
    if (!L || max_T <= 0) return 0;
    return ws_layout(L->D, L->F, L->E, L->K, max_T).total;
}

namespace cpg {
// ev (optional, 5 events): recorded before the router, gate/up, down and combine launches and
// after the combine, so a caller can time each phase on the stream it runs on.
int moe_forward_impl(const cpg_moe_layer *L, const float *x, const float *attn, int T, float *mlp,
                     float *x_out, int *topk_idx, float *wt, float *router, void *ws, size_t ws_bytes,
                     cudaStream_t s, cudaEvent_t *ev);
}

extern "C" int cpg_moe_forward(const cpg_moe_layer *L, const float *x, const float *attn, int T,
                               float *mlp, float *x_out, int *topk_idx, float *wt, float *router,
                               void *ws, size_t ws_bytes, void *stream) {
    return moe_forward_impl(L, x, attn, T, mlp, x_out, topk_idx, wt, router, ws, ws_bytes,
                            (cudaStream_t)stream, nullptr);
}

int cpg::moe_forward_impl(const cpg_moe_layer *L, const float *x, const float *attn, int T, float *mlp,
                          float *x_out, int *topk_idx, float *wt, float *router, void *ws, size_t ws_bytes,
                          cudaStream_t s, cudaEvent_t *ev) {
    CPG_REQUIRE(L && x && ws, "cpg_moe_forward: null argument");
    CPG_REQUIRE(T > 0, "cpg_moe_forward: T=%d", T);
    const WsLayout W = ws_layout(L->D, L->F, L->E, L->K, T);
    CPG_REQUIRE(ws_bytes >= W.total, "cpg_moe_forward: workspace %zu < %zu bytes for T=%d", ws_bytes, W.total, T);
    CPG_REQUIRE((((uintptr_t)x | (uintptr_t)attn | (uintptr_t)mlp | (uintptr_t)x_out | (uintptr_t)ws) & 15) == 0,
                "cpg_moe_forward: buffers must be 16-byte aligned");
    uint8_t *w = (uint8_t *)ws;
    int *hdr = (int *)w;
    if (ev) CPG_CUDA(cudaEventRecordWithFlags(ev[0], s, cudaEventRecordExternal));
    if (T == 1 && L->one.ok) {
        // one token: the whole block in one cooperative launch (moe_one.cu); its time is the
        // router phase of the phase events
        const int rc = one_launch(L, L->one, x, attn, mlp, x_out, topk_idx ? topk_idx : (int *)(w + W.topk),
                                  wt ? wt : (float *)(w + W.wt), router ? router : (float *)(w + W.logits), hdr,
                                  (float *)(w + W.h), L->d_one_bar, s);
        if (rc) return rc;
        if (ev)
            for (int i = 1; i < 5; ++i) CPG_CUDA(cudaEventRecordWithFlags(ev[i], s, cudaEventRecordExternal));
        return CPG_OK;
    }

    RouterArgs ra{};
    ra.x = x; ra.attn = attn; ra.ln2 = L->ln2; ra.wgate = L->wgate;
    ra.T = T; ra.D = L->D; ra.F = L->F; ra.E = L->E; ra.K = L->K; ra.eps = L->eps; ra.xn_enc = L->enc;
    ra.logits = router ? router : (float *)(w + W.logits);
    ra.topk = topk_idx ? topk_idx : (int *)(w + W.topk);
    ra.wt = wt ? wt : (float *)(w + W.wt);
    ra.xn_perm = (__half *)(w + W.xn);
    ra.status = hdr;
    ra.zero_row = (__half *)(w + W.zero_row);
    ra.n_active = (int *)(w + W.n_active);
    ra.act = (int4 *)(w + W.act);
    ra.pairs = (int *)(w + W.pairs);
    ra.dep = (int *)(w + W.dep);
    ra.n_dep = max_token_chunks(L->E, L->K, T);
    // one cluster of at most R_CLUSTER_MAX CTAs per token tile, one expert row per warp when
    // E ≤ 8 · R_CLUSTER_MAX (16 CTAs, 128 per 64 tokens for Qwen3-30B-A3B)
    const int csz = router_cluster(L->E, &ra.eb);
    const int tb = T <= 2 ? T : R_TB;
    const dim3 rgrid(csz, (T + tb - 1) / tb);
    auto *rk = tb == 1 ? k_router<1> : tb == 2 ? k_router<2> : k_router<R_TB>;
    const size_t rsm = (size_t)(tb + 1) * L->D * sizeof(float);
    CPG_CUDA(launch_pdl_cluster(rk, rgrid, dim3(R_THREADS), rsm, s, csz, ra));
    // the gate/up kernel groups small batches itself; its scratch (group_cta) must fit in two
    // stages of the smallest stage ring (Q4 gate/up: 2 × 26,880 bytes)
    const size_t group_scratch = sizeof(int) * (4 * (size_t)L->E + (size_t)L->E * ((T + 31) / 32) + (size_t)T * L->K + 1);
    const bool self_group = T * L->K <= EX_GROUP_MAX && group_scratch <= 40960;
    if (!self_group) CPG_CUDA(launch_pdl(k_group, dim3(1), dim3(RT_THREADS), 0, s, ra));

    ExpertArgs ea{};
    ea.D = L->D; ea.F = L->F; ea.K = L->K;
    ea.n_active = ra.n_active; ea.act = ra.act;
    ea.zero_row = ra.zero_row;
    ea.pairs = ra.pairs; ea.h_enc = L->enc; ea.status = hdr;
    const int max_chunks = ra.n_dep;
    const int gu_items = max_chunks * (L->F / 64), dn_items = max_chunks * (L->D / 128);

    ea.bsrc = ra.xn_perm;
    ea.h_out = (__half *)(w + W.h);
    ea.y_out = (float *)(w + W.y);
    ea.dep = ra.dep;
    ea.item_ctr = hdr + WS_ITEMS_GATEUP;
    if (self_group) {
        ea.topk = ra.topk; ea.T = T; ea.E = L->E;
        ea.g_n_active = ra.n_active; ea.g_act = ra.act; ea.g_pairs = ra.pairs;
    }
    if (ev) CPG_CUDA(cudaEventRecordWithFlags(ev[1], s, cudaEventRecordExternal));
    int rc;
    if (gu_items > sm_count()) {
        // more items than SMs: gate/up and down in one launch (the down items fill the gate/up tail)
        rc = launch_experts(L, KIND_BOTH, ea, gu_items + dn_items, s);
        if (rc) return rc;
        if (ev) CPG_CUDA(cudaEventRecordWithFlags(ev[2], s, cudaEventRecordExternal));
    } else {
        // a few items (one token: 8 experts): each kind on one CTA per SM with all its K slices
        // in flight
        rc = launch_experts(L, KIND_GATEUP, ea, gu_items, s);
        if (rc) return rc;
        ea.bsrc = (const __half *)(w + W.h);
        ea.item_ctr = hdr + WS_ITEMS_DOWN;
        ea.topk = nullptr;
        if (ev) CPG_CUDA(cudaEventRecordWithFlags(ev[2], s, cudaEventRecordExternal));
        rc = launch_experts(L, KIND_DOWN, ea, dn_items, s);
        if (rc) return rc;
    }

    const int n4 = T * L->D / 4;
    int cgrid = (n4 + 255) / 256;
    if (cgrid > sm_count() * 8) cgrid = sm_count() * 8;
    if (ev) CPG_CUDA(cudaEventRecordWithFlags(ev[3], s, cudaEventRecordExternal));
    CPG_CUDA(launch_pdl(k_combine, dim3(cgrid), dim3(256), 0, s, x, attn, T, L->D, L->K, (const float *)ra.wt,
                        (const float *)(w + W.y), mlp, x_out));
    if (ev) CPG_CUDA(cudaEventRecordWithFlags(ev[4], s, cudaEventRecordExternal));
    return CPG_OK;
}

extern "C" int cpg_moe_check(const void *ws, void *stream) {
    CPG_REQUIRE(ws, "cpg_moe_check: null workspace");
    int st = 0;
    CPG_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    CPG_CUDA(cudaMemcpy(&st, ws, sizeof(int), cudaMemcpyDeviceToHost));
    if (st != ST_OK) {
        set_error("device-side wait timed out (status %d)", st);
        return CPG_ETIMEOUT;
    }
    return CPG_OK;
}
