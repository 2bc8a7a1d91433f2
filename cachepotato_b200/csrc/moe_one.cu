// moe_one.cu — the Qwen3-MoE block for ONE token (a decode step of batch 1) in one launch.
//
// The block of engine/blocks/qwen3_moe.c:169-223 plus the residual of run_layers
// (engine/api/cachepotato.c:157-159) for T = 1 is a chain of small dependent steps: the router
// needs all of xn, top-k needs all 128 logits, each down row needs all 768 h values of every
// selected expert. As separate launches each step costs a launch and a pipeline fill, and the
// router alone ran on 16 SMs. Here one cooperative launch (one CTA per SM, co-residency
// guaranteed by the runtime) runs the whole block with two grid-wide barriers:
//
//   phase R   every CTA: hh = x + attn, RMSNorm (ln2) -> xn, kept in shared memory; CTA c < E
//             writes logit c = Wgate[c]·xn (f32)                                   -> barrier 1
//   phase S   every CTA (one warp): softmax, strict-'>' top-k, renormalisation (qwen3_moe.c:
//             181-197) from the E logits; CTA 0 writes topk / wt. Each CTA then starts the bulk
//             copies of its gate/up units and an L2 prefetch of the down tiles it will need
//   phase G   unit = (selected expert j, 16-row band b of the expert's F rows): gate and up
//             bands over the whole K, one K slice per warp, partial sums added across warps in
//             warp order, h = silu(g)·u (qwen3_moe.c:217-219) to the workspace  -> barrier 2
//   phase D   CTA c owns output rows [16c, 16c + 16): Wd of every selected expert on those rows
//             (one expert per warp), then mlp += wt_j·y_j in selection order (qwen3_moe.c:221)
//             and x_out = x + (attn + mlp)
//
// Weights come from the layer's decode tile copy (k_tile_experts) by 16-byte cp.async from every
// thread and are decoded in registers into mma.m16n8k16 exactly as in the batched expert
// kernels; the token's f32 activations are fp16 hi + lo halves in MMA columns 0 and 1. The grid
// barriers' waits are bounded by %globaltimer and record a status code; their counters return to
// zero at the end of every launch (the last CTA to finish resets them, also after a wait that
// gave up), so they live with the layer and are zeroed once, when it is created.
#include <math.h>

#include "common.cuh"
#include "expert_tile.cuh"
#include "layout.cuh"
#include "moe_one.cuh"

namespace cpg {

constexpr int O_THREADS = 256;
constexpr int O_NW = O_THREADS / 32;
constexpr int O_MAXK = 8;           // selected experts per token (one warp each in phase D)
constexpr int O_MAXE = 256;

__constant__ Perm64 c_perm_one[2] = {kPermQ4, kPermQ8};

struct OneArgs {
    const float *x, *attn, *ln2, *wgate;
    const uint8_t *tiles;           // decode tile copy of the layer, (E, 3) matrices of MB bytes
    int D, F, E, K, enc;
    float eps;
    int slots;                      // 16-row gate/up bands per round (shared memory)
    int early_down;                 // the down tiles have their own shared memory area
    float *logits;                  // (E)
    int *topk;                      // (K)
    float *wt;                      // (K)
    float *mlp, *x_out;             // (D), either may be null
    float *h;                       // workspace (K, F) f32
    int *status;                    // workspace word 0 (cleared by CTA 0 at the start)
    unsigned *bar;                  // the layer's counters: [0] barrier arrivals, [1] finished CTAs
};

// Bounded grid barrier: arrive, then wait until `target` arrivals (all CTAs of the launch, which
// is cooperative: every CTA is resident). Memory written before it is visible after it.
__device__ __forceinline__ void grid_sync(unsigned *ctr, unsigned target, int *status) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(ctr, 1u);
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
        if (v < target) {
            const uint64_t t0 = global_ns();
            for (uint32_t i = 1;; ++i) {
                __nanosleep(32);
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
                if (v >= target) break;
                if ((i & 63u) == 0 && global_ns() - t0 > kWaitLimitNs) {
                    atomicCAS(status, ST_OK, ST_TIMEOUT_FULL);
                    break;
                }
            }
        }
        __threadfence();
    }
    __syncthreads();
}

// One 16-row tile of one K slice against the token's operand columns: acc[0] + acc[1] is row g,
// acc[2] + acc[3] row g + 8 (lanes with t == 0; other lanes hold unused columns). b points at
// this lane's 32 bytes of the slice's pair 0 (hi or lo half by column).
template <int ENC>
__device__ __forceinline__ void tile_one(const uint8_t *tp, const uint8_t *b, int lane, float (&acc)[4]) {
    using X = ExTile<ENC>;
    const uint2 *sc = reinterpret_cast<const uint2 *>(tp + X::DB + (lane >> 2) * 32);
#pragma unroll
    for (int P = 0; P < 4; ++P) {
        uint32_t fr[4][4];
        tile_frags<ENC>(tp, P, lane, fr);
        const uint4 b0 = *reinterpret_cast<const uint4 *>(b + P * 128);
        const uint4 b1 = *reinterpret_cast<const uint4 *>(b + P * 128 + 16);
        const uint2 sg = sc[P >> 1], s8 = sc[2 + (P >> 1)];
        const uint32_t dg = P & 1 ? sg.y : sg.x, d8 = P & 1 ? s8.y : s8.x;
        const float2 fg = __half22float2(*reinterpret_cast<const __half2 *>(&dg));
        const float2 f8 = __half22float2(*reinterpret_cast<const __half2 *>(&d8));
        const float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        float sj[4], sj1[4];
        mma_16816(sj, fr[0], b0.x, b0.y, z);
        mma_16816(sj, fr[1], b0.z, b0.w, sj);
        mma_16816(sj1, fr[2], b1.x, b1.y, z);
        mma_16816(sj1, fr[3], b1.z, b1.w, sj1);
        fma2_f32(acc[0], acc[1], fg.x, sj[0], sj[1]);
        fma2_f32(acc[0], acc[1], fg.y, sj1[0], sj1[1]);
        fma2_f32(acc[2], acc[3], f8.x, sj[2], sj[3]);
        fma2_f32(acc[2], acc[3], f8.y, sj1[2], sj1[3]);
    }
}

// Vector loads a thread keeps in flight: D <= O_XV * 4 * O_THREADS values in phase R,
// K * F <= O_HV * 4 * O_THREADS in phase D (every load of a phase is issued before any is used).
constexpr int O_XV = 4;
constexpr int O_HV = 12;

template <int ENC>
__global__ void __launch_bounds__(O_THREADS, 1) k_moe_one(OneArgs a) {
    using X = ExTile<ENC>;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t *const smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    __shared__ uint64_t s_bar[2];                       // [0] gate/up rounds, [1] down tiles
    __shared__ int s_sel_e[O_MAXK];
    __shared__ float s_sel_w[O_MAXK];
    __shared__ float s_red[O_NW];
    __shared__ Perm64 s_perm;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int D = a.D, F = a.F, E = a.E, K = a.K, G = gridDim.x, c = blockIdx.x;
    const int nsd = D / EX_KSL, nsf = F / EX_KSL;                   // K slices of gate/up, of down
    const int NB = a.slots;                                         // 16-row bands per round
    const size_t MB = (size_t)D * F / 32 * X::GB;                   // bytes per expert matrix
    // shared memory: xs f32 (D) | xb fp16 hi (D) | xb fp16 lo (D) | red (NW, 2, 32, 4) f32 |
    // region: phase G (nsd, 2·NB) interleaved gate/up tiles (a 16-row band b of both matrices =
    // tiles 2b, 2b + 1); phase D (K, nsf) tiles, then h as hi | lo per expert
    float *xs = reinterpret_cast<float *>(smem);
    __half *xb = reinterpret_cast<__half *>(xs + D);
    float *red = reinterpret_cast<float *>(xb + 2 * D);
    uint8_t *region = reinterpret_cast<uint8_t *>(red + O_NW * 2 * 32 * 4);

    // the router row this CTA scores, in flight while the rest of phase R runs
    const int D4 = D / 4;
    float4 wv[O_XV];
    if (c < E) {
        const float4 *w4 = reinterpret_cast<const float4 *>(a.wgate + (size_t)c * D);
#pragma unroll
        for (int k = 0; k < O_XV; ++k)
            if (tid + k * O_THREADS < D4) wv[k] = __ldg(w4 + tid + k * O_THREADS);
    }
    if (tid == 0) {
        mbar_init(&s_bar[0], 1);
        mbar_init(&s_bar[1], 1);
        fence_mbar_init();
    }
    if (tid < 64) {
        const Perm64 &pm = c_perm_one[ENC == CPG_ENC_Q4 ? 0 : 1];
        s_perm.pos_to_elem[tid] = pm.pos_to_elem[tid];
        s_perm.elem_to_pos[tid] = pm.elem_to_pos[tid];
    }

    if (c == 0 && tid == 0) *a.status = ST_OK;                      // this launch's status word
    // ---------------- phase R: hh = x + attn, xn = RMSNorm(hh) (kernels.c:408-413), logits
    {
        const float4 *x4 = reinterpret_cast<const float4 *>(a.x);
        const float4 *a4 = reinterpret_cast<const float4 *>(a.attn);
        const float4 *g4 = reinterpret_cast<const float4 *>(a.ln2);
        float4 hv[O_XV], gv[O_XV];
#pragma unroll
        for (int k = 0; k < O_XV; ++k) {
            const int i = tid + k * O_THREADS;
            if (i < D4) {
                hv[k] = __ldg(x4 + i);
                gv[k] = __ldg(g4 + i);
            }
        }
        if (a.attn) {
#pragma unroll
            for (int k = 0; k < O_XV; ++k) {
                const int i = tid + k * O_THREADS;
                if (i < D4) {
                    const float4 b = __ldg(a4 + i);
                    hv[k].x += b.x; hv[k].y += b.y; hv[k].z += b.z; hv[k].w += b.w;
                }
            }
        }
        float ss = 0.0f;
#pragma unroll
        for (int k = 0; k < O_XV; ++k)
            if (tid + k * O_THREADS < D4) {
                ss = fmaf(hv[k].x, hv[k].x, ss);
                ss = fmaf(hv[k].y, hv[k].y, ss);
                ss = fmaf(hv[k].z, hv[k].z, ss);
                ss = fmaf(hv[k].w, hv[k].w, ss);
            }
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < O_NW; ++w) tot += s_red[w];
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(tot, (float)D) + a.eps));
        float lg = 0.0f;
#pragma unroll
        for (int k = 0; k < O_XV; ++k) {
            const int i = tid + k * O_THREADS;
            if (i < D4) {
                float4 v = hv[k];
                v.x = __fmul_rn(__fmul_rn(v.x, inv), gv[k].x);
                v.y = __fmul_rn(__fmul_rn(v.y, inv), gv[k].y);
                v.z = __fmul_rn(__fmul_rn(v.z, inv), gv[k].z);
                v.w = __fmul_rn(__fmul_rn(v.w, inv), gv[k].w);
                reinterpret_cast<float4 *>(xs)[i] = v;
                if (c < E) {                                         // logit c = Wgate[c]·xn
                    lg = fmaf(wv[k].x, v.x, lg);
                    lg = fmaf(wv[k].y, v.y, lg);
                    lg = fmaf(wv[k].z, v.z, lg);
                    lg = fmaf(wv[k].w, v.w, lg);
                }
            }
        }
        __syncthreads();                                             // s_red reused below
        lg = warp_sum(lg);
        if (lane == 0) s_red[warp] = lg;
        __syncthreads();
        if (tid == 0 && c < E) {
            float v = 0.0f;
            for (int w = 0; w < O_NW; ++w) v += s_red[w];
            a.logits[c] = v;
        }
    }
    for (int e = c + G; e < E; e += G) {                             // more experts than CTAs
        const float4 *w4 = reinterpret_cast<const float4 *>(a.wgate + (size_t)e * D);
        float acc = 0.0f;
        for (int i = tid; i < D4; i += O_THREADS) {
            const float4 w = __ldg(w4 + i), v = reinterpret_cast<const float4 *>(xs)[i];
            acc = fmaf(w.x, v.x, acc);
            acc = fmaf(w.y, v.y, acc);
            acc = fmaf(w.z, v.z, acc);
            acc = fmaf(w.w, v.w, acc);
        }
        acc = warp_sum(acc);
        __syncthreads();
        if (lane == 0) s_red[warp] = acc;
        __syncthreads();
        if (tid == 0) {
            float v = 0.0f;
            for (int w = 0; w < O_NW; ++w) v += s_red[w];
            a.logits[e] = v;
        }
    }
    // the operand copy for the gate/up MMAs: hi | lo halves in the expert kernels' K order
    for (int p = tid; p < D; p += O_THREADS) {
        const float v = xs[(p & ~63) + s_perm.pos_to_elem[p & 63]];
        split_half(v, xb[p], xb[D + p]);
    }
    grid_sync(a.bar, (unsigned)G, a.status);

    // ---------------- phase S: routing; this CTA's gate/up bands are a consecutive range
    {
        __shared__ __align__(16) float s_p[O_MAXE + O_MAXK];   // probabilities, then the selected ones
        select_topk<O_MAXE, O_MAXK>(a.logits, E, K, s_sel_e, s_sel_w, s_p);
    }
    if (c == 0 && tid < K) {
        a.topk[tid] = s_sel_e[tid];
        a.wt[tid] = s_sel_w[tid];
    }
    const int bands = F / 16, n_units = K * bands;
    const int n0 = (int)((long)c * n_units / G), n1 = (int)((long)(c + 1) * n_units / G);
    // one round: bands [r0, r1) of the range; per (expert chunk, K slice) one bulk copy of the
    // chunk's consecutive interleaved tiles (contiguous in the tile layout). The bulk operations of
    // one warp are served one after another, so they are dealt round robin over all warps.
    auto issue_round = [&](int r0, int r1) {
        if (tid == 0) mbar_arrive_expect_tx(&s_bar[0], (uint32_t)(r1 - r0) * 2u * nsd * X::TB);
        __syncthreads();
        int q = 0;
        for (int n = r0; n < r1;) {
            const int j = n / bands, b = n - j * bands, cnt = min(r1 - n, bands - b);
            const uint8_t *te = a.tiles + (size_t)(3 * s_sel_e[j]) * MB;
            for (int s = 0; s < nsd; ++s, ++q)
                if (lane == 0 && q % O_NW == warp)
                    bulk_g2s(region + ((size_t)s * 2 * NB + 2 * (n - r0)) * X::TB,
                             te + ((size_t)s * 2 * bands + 2 * b) * X::TB, (uint32_t)cnt * 2 * X::TB, &s_bar[0]);
            n += cnt;
        }
    };
    // the down tiles of this CTA's (first) output band: copied now into their own area when it
    // fits (they land while gate/up computes), else prefetched into L2 and copied in phase D
    const uint32_t dbytes = (uint32_t)(K * nsf) * X::TB;
    uint8_t *dtiles = a.early_down ? region + (size_t)NB * 2 * nsd * X::TB : region;
    auto issue_down = [&](int bd, bool to_smem) {
        if (to_smem && tid == 0) mbar_arrive_expect_tx(&s_bar[1], dbytes);
        __syncthreads();
        if (lane == 0)
            for (int q = warp; q < K * nsf; q += O_NW) {
                const int j = q / nsf, s = q - j * nsf;
                const uint8_t *src = a.tiles + (size_t)(3 * s_sel_e[j] + 2) * MB + ((size_t)s * (D / 16) + bd) * X::TB;
                if (to_smem) bulk_g2s(dtiles + (size_t)q * X::TB, src, X::TB, &s_bar[1]);
                else asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"((uint32_t)X::TB) : "memory");
            }
    };
    if (n0 < n1) issue_round(n0, min(n1, n0 + NB));
    if (c < D / 16) issue_down(c, a.early_down != 0);

    // ---------------- phase G: h = silu(Wg·xn) · (Wu·xn) for this CTA's 16-row bands
    for (int r0 = n0; r0 < n1; r0 += NB) {
        const int r1 = min(n1, r0 + NB);
        if (!mbar_wait(&s_bar[0], (uint32_t)((r0 - n0) / NB) & 1u) && tid == 0)
            atomicCAS(a.status, ST_OK, ST_TIMEOUT_FULL);
        for (int n = r0; n < r1; ++n) {
            const int j = n / bands, b = n - j * bands, k = n - r0;
            float ag[4] = {0.0f, 0.0f, 0.0f, 0.0f}, au[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const int g = lane >> 2, t = lane & 3;
            for (int s = warp; s < nsd; s += O_NW) {
                const uint8_t *bp = reinterpret_cast<const uint8_t *>(xb + (g == 1 ? D : 0) + s * EX_KSL) + t * 32;
                tile_one<ENC>(region + ((size_t)s * 2 * NB + 2 * k) * X::TB, bp, lane, ag);       // features 16b..+7
                tile_one<ENC>(region + ((size_t)s * 2 * NB + 2 * k + 1) * X::TB, bp, lane, au);   // 16b+8..+15
            }
            float4 *r4 = reinterpret_cast<float4 *>(red);
            r4[(warp * 2 + 0) * 32 + lane] = make_float4(ag[0], ag[1], ag[2], ag[3]);
            r4[(warp * 2 + 1) * 32 + lane] = make_float4(au[0], au[1], au[2], au[3]);
            __syncthreads();
            if (tid < 16) {                                          // feature 16b + tid: MMA row rg of
                const int rg = tid & 7, hi8 = tid >> 3;              // tile 2k + hi8 (gate), rg + 8 (up)
                float gs = 0.0f, us = 0.0f;
                for (int w = 0; w < O_NW; ++w) {
                    const float4 v = r4[(w * 2 + hi8) * 32 + rg * 4];
                    gs += v.x + v.y;
                    us += v.z + v.w;
                }
                const float silu = gs / (1.0f + expf(-gs));          // kernels.c:416
                a.h[(size_t)j * F + b * 16 + tid] = silu * us;      // qwen3_moe.c:219
            }
            __syncthreads();
        }
        if (r1 < n1) issue_round(r1, min(n1, r1 + NB));              // the region is free again
    }
    grid_sync(a.bar, 2u * G, a.status);

    // ---------------- phase D: y_j = Wd_j·h_j on this CTA's 16-row bands, then the combine
    __half *hb = reinterpret_cast<__half *>(dtiles + dbytes);       // (K, 2, F) after the tiles
    for (int bd = c, it = 0; bd < D / 16; bd += G, ++it) {
        if (!(a.early_down && it == 0)) issue_down(bd, true);
        if (bd == c) {
            // h of every selected expert as hi | lo fp16 in Wd's K order (all loads in flight)
            const int KF4 = K * F / 4;
            float4 hv[O_HV];
#pragma unroll
            for (int k = 0; k < O_HV; ++k)
                if (tid + k * O_THREADS < KF4) hv[k] = __ldcg(reinterpret_cast<const float4 *>(a.h) + tid + k * O_THREADS);
#pragma unroll
            for (int k = 0; k < O_HV; ++k) {
                const int i = tid + k * O_THREADS;
                if (i < KF4) {
                    const int q = i * 4, j = q / F, e0 = q - j * F;     // four values e0..e0+3 of expert j
                    __half *hj = hb + (size_t)j * 2 * F + (e0 & ~63);
                    const float v4[4] = {hv[k].x, hv[k].y, hv[k].z, hv[k].w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int pos = s_perm.elem_to_pos[(e0 + u) & 63];
                        split_half(v4[u], hj[pos], hj[F + pos]);
                    }
                }
            }
        }
        float xr = 0.0f, ar = 0.0f, mr = 0.0f;                       // the combine's operands, early
        if (tid < 16) {
            const int row = bd * 16 + tid;
            xr = a.x[row];
            if (a.attn) ar = a.attn[row];
            if (a.mlp) mr = a.mlp[row];
        }
        __syncthreads();
        if (!mbar_wait(&s_bar[1], (uint32_t)it & 1u) && tid == 0) atomicCAS(a.status, ST_OK, ST_TIMEOUT_FULL);
        const int g = lane >> 2, t = lane & 3;
        float4 *r4 = reinterpret_cast<float4 *>(red);
        for (int j = warp; j < K; j += O_NW) {
            float ay[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int s = 0; s < nsf; ++s) {
                const uint8_t *bp = reinterpret_cast<const uint8_t *>(hb + (size_t)j * 2 * F + (g == 1 ? F : 0) + s * EX_KSL) + t * 32;
                tile_one<ENC>(dtiles + (size_t)(j * nsf + s) * X::TB, bp, lane, ay);
            }
            r4[j * 32 + lane] = make_float4(ay[0], ay[1], ay[2], ay[3]);
        }
        __syncthreads();
        if (tid < 16) {                                              // row 16·bd + tid
            const int rg = tid & 7, hi8 = tid >> 3, row = bd * 16 + tid;
            float acc = mr;
            for (int j = 0; j < K; ++j) {                            // selection order, qwen3_moe.c:221
                const float4 v = r4[j * 32 + rg * 4];
                acc = __fadd_rn(acc, __fmul_rn(s_sel_w[j], hi8 ? v.z + v.w : v.x + v.y));
            }
            if (a.mlp) a.mlp[row] = acc;
            if (a.x_out) a.x_out[row] = xr + (ar + acc);
        }
        __syncthreads();
    }

    // ---------------- the last CTA to finish returns the barrier counters to zero
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(a.bar + 1, 1u) == (unsigned)G - 1) {
            a.bar[0] = 0u;
            a.bar[1] = 0u;
            __threadfence();
        }
    }
}

}  // namespace cpg

namespace cpg {

int layer_one_info(const cpg_moe_layer *L, int *D, int *F, int *E, int *K, int *enc, const float **ln2,
                   const float **wgate, const uint8_t **tiles, float *eps);

// Whether (and how) the one-token kernel runs this layer: K <= 8, E <= 256, D <= 4096 and
// K·F <= 12288 (the vector loads a thread keeps in flight), and shared memory for at least one
// gate/up band per round and for the down phase's tiles and h; one CTA per SM resident.
int one_plan(const cpg_moe_layer *L, OnePlan *p) {
    int D, F, E, K, enc;
    const float *ln2, *wg;
    const uint8_t *tiles;
    float eps;
    int rc = layer_one_info(L, &D, &F, &E, &K, &enc, &ln2, &wg, &tiles, &eps);
    if (rc) return rc;
    p->ok = false;
    if (K > O_MAXK || E > O_MAXE || D % 256 || F % 256 || D > O_XV * 4 * O_THREADS ||
        (long)K * F > (long)O_HV * 4 * O_THREADS)
        return CPG_OK;
    const size_t TB = (size_t)16 * 8 * (enc == CPG_ENC_Q4 ? 18 : 34);
    const size_t band = 2 * (size_t)(D / 256) * TB;                 // one 16-row band of gate and up
    const size_t fixed = (size_t)D * 4 + (size_t)D * 4 + O_NW * 2 * 32 * 16 + 128;
    const size_t down = (size_t)K * (F / 256) * TB + (size_t)K * 2 * F * 2;
    const long limit = smem_optin() - 2048;                          // static shared memory and slack
    const int G = sm_count();
    const int per_cta = (K * (F / 16) + G - 1) / G;                  // bands a CTA owns
    int NB = (int)((limit - (long)fixed) / (long)band);
    if (NB > per_cta) NB = per_cta;
    if (NB < 1) return CPG_OK;
    size_t region = (size_t)NB * band + down;                       // the down tiles in their own area
    p->early_down = fixed + region <= (size_t)limit;
    if (!p->early_down) region = (size_t)NB * band > down ? (size_t)NB * band : down;   // reused
    if (fixed + region > (size_t)limit) return CPG_OK;
    p->slots = NB;
    p->smem = fixed + region;
    auto *k = enc == CPG_ENC_Q4 ? k_moe_one<CPG_ENC_Q4> : k_moe_one<CPG_ENC_Q8>;
    rc = allow_max_smem((const void *)k);
    if (rc) return rc;
    int per_sm = 0;
    CPG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, O_THREADS, p->smem));
    if (per_sm < 1) return CPG_OK;
    p->grid = G;
    p->ok = true;
    return CPG_OK;
}

int one_launch(const cpg_moe_layer *L, const OnePlan &p, const float *x, const float *attn, float *mlp,
               float *x_out, int *topk, float *wt, float *logits, int *ws_hdr, float *h, unsigned *bar,
               cudaStream_t s) {
    OneArgs a{};
    const uint8_t *tiles;
    int rc = layer_one_info(L, &a.D, &a.F, &a.E, &a.K, &a.enc, &a.ln2, &a.wgate, &tiles, &a.eps);
    if (rc) return rc;
    a.tiles = tiles;
    a.x = x; a.attn = attn; a.mlp = mlp; a.x_out = x_out;
    a.topk = topk; a.wt = wt; a.logits = logits; a.h = h;
    a.status = ws_hdr;
    a.bar = bar;
    a.slots = p.slots;
    a.early_down = p.early_down ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(O_THREADS);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;                     // every CTA resident: the grid barriers end
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    auto *k = a.enc == CPG_ENC_Q4 ? k_moe_one<CPG_ENC_Q4> : k_moe_one<CPG_ENC_Q8>;
    CPG_CUDA(cudaLaunchKernelEx(&cfg, k, a));
    return CPG_OK;
}

}  // namespace cpg
