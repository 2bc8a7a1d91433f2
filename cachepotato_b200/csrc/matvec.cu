// matvec.cu — out[t] = W·x[t] for f32 / Q8_0 / Q4_0 row-major W, fp32 arithmetic throughout.
//
// The kernel-level entry points of the reference (matmul_wx, matmul_wx_q8, matmul_wx_q4 in
// engine/kernels/kernels.c:84-95, 368-396, 514-540): each weight is decoded to (float)q * d
// exactly and multiply-added in fp32, so results agree with the reference within its own
// kernel-gate tolerance (rel 1e-5, tools/verify_q8_kernels.py). One warp per output row;
// lanes take 64-value group pairs (36 B for Q4, 68 B for Q8, 4-byte aligned), x is staged in
// shared memory, up to 8 vectors share each weight load.
#include <algorithm>

#include "common.cuh"

namespace cpg {

constexpr int MV_WARPS = 8;
constexpr int MV_TOK = 8;          // vectors per pass (accumulators per lane)

__device__ __forceinline__ int sext4(uint32_t v) { return (int)(v << 28) >> 28; }

template <int ENC>
__device__ __forceinline__ void row_partial(const uint8_t *__restrict__ row, int n_in,
                                            const float *__restrict__ xs, int ntok, float acc[MV_TOK],
                                            bool aligned4) {
    const int lane = threadIdx.x & 31;
    if (ENC == CPG_ENC_F32) {
        const float *w = reinterpret_cast<const float *>(row);
        for (int k = lane * 4; k < n_in; k += 128) {
            const float4 wv = *reinterpret_cast<const float4 *>(w + k);
#pragma unroll
            for (int t = 0; t < MV_TOK; ++t) {
                if (t < ntok) {
                    const float4 xv = *reinterpret_cast<const float4 *>(xs + t * n_in + k);
                    acc[t] = fmaf(wv.x, xv.x, acc[t]);
                    acc[t] = fmaf(wv.y, xv.y, acc[t]);
                    acc[t] = fmaf(wv.z, xv.z, acc[t]);
                    acc[t] = fmaf(wv.w, xv.w, acc[t]);
                }
            }
        }
        return;
    }
    constexpr int GB = ENC == CPG_ENC_Q4 ? 18 : 34;
    const int ng = n_in / 32;
    if (aligned4 && (ng % 2) == 0) {
        constexpr int NW = GB / 2;                      // words per group pair: 9 or 17
        const int np = ng / 2;                          // x staged as xs[t][k][p] (k < 64)
        for (int p = lane; p < np; p += 32) {
            const uint32_t *wp = reinterpret_cast<const uint32_t *>(row + (size_t)p * 2 * GB);
            uint32_t w[NW];
#pragma unroll
            for (int i = 0; i < NW; ++i) w[i] = __ldg(wp + i);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int b0 = half * GB;               // byte offset of this group in the span
                const uint32_t sb = (w[b0 / 4] >> ((b0 % 4) * 8)) & 0xFFFFu;
                const float d = f16_bits_to_f32(sb);
                const float *xp = xs + (half * 32) * np + p;   // element (half*32 + k) at xp[k*np]
                if (ENC == CPG_ENC_Q4) {
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int bo = b0 + 2 + k;
                        const uint32_t byte = (w[bo / 4] >> ((bo % 4) * 8)) & 0xFFu;
                        const float lo = __fmul_rn((float)sext4(byte), d);
                        const float hi = __fmul_rn((float)sext4(byte >> 4), d);
#pragma unroll
                        for (int t = 0; t < MV_TOK; ++t) {
                            if (t < ntok) {
                                acc[t] = fmaf(lo, xp[t * n_in + k * np], acc[t]);
                                acc[t] = fmaf(hi, xp[t * n_in + (k + 16) * np], acc[t]);
                            }
                        }
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 32; ++k) {
                        const int bo = b0 + 2 + k;
                        const int q = (int)(int8_t)((w[bo / 4] >> ((bo % 4) * 8)) & 0xFFu);
                        const float v = __fmul_rn((float)q, d);
#pragma unroll
                        for (int t = 0; t < MV_TOK; ++t)
                            if (t < ntok) acc[t] = fmaf(v, xp[t * n_in + k * np], acc[t]);
                    }
                }
            }
        }
    } else {
        // any alignment: one group per lane, byte loads; x staged as xs[t][k][g] (k < 32)
        for (int g = lane; g < ng; g += 32) {
            const uint8_t *blk = row + (size_t)g * GB;
            const float d = f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
            const float *xp = xs + g;
            if (ENC == CPG_ENC_Q4) {
                for (int k = 0; k < 16; ++k) {
                    const uint32_t byte = blk[2 + k];
                    const float lo = __fmul_rn((float)sext4(byte), d);
                    const float hi = __fmul_rn((float)sext4(byte >> 4), d);
#pragma unroll
                    for (int t = 0; t < MV_TOK; ++t) {
                        if (t < ntok) {
                            acc[t] = fmaf(lo, xp[t * n_in + k * ng], acc[t]);
                            acc[t] = fmaf(hi, xp[t * n_in + (k + 16) * ng], acc[t]);
                        }
                    }
                }
            } else {
                for (int k = 0; k < 32; ++k) {
                    const float v = __fmul_rn((float)(int8_t)blk[2 + k], d);
#pragma unroll
                    for (int t = 0; t < MV_TOK; ++t)
                        if (t < ntok) acc[t] = fmaf(v, xp[t * n_in + k * ng], acc[t]);
                }
            }
        }
    }
}

// ---------------------------------------------------------------- streaming GEMV (T ≤ 4)
// For decode-sized T the weight rows are the only traffic: 16 consecutive rows at a time arrive
// in shared memory by one 1D bulk copy (a 4-deep ring filled by one producer thread), and each
// lane decodes whole 64-value group pairs from there (word stride 9 or 17, odd: no bank
// conflicts), with the same exact (float)q·d and fp32 FMA as the row-per-warp kernel above.
constexpr int GV_ROWS = 16;
// Sixteen consumer warps, one row each per stage: with eight (two rows each) the Q8 lm_head's
// consumers issued ~0.33 instructions per scheduler cycle; sixteen took whole-model decode from
// 345 to 351 tok/s (at <= 96 registers a CTA fills an SM's register file: one CTA per SM).
constexpr int GV_CONS = 16;
constexpr int GV_MAXT = 4;

template <int ENC, int NT>
__device__ __forceinline__ void gemv_pair(const uint32_t *__restrict__ wp, const float *__restrict__ xp, int np,
                                          int n_in, float (&acc)[NT]) {
    constexpr int GB = ENC == CPG_ENC_Q4 ? 18 : 34;
    constexpr int NW = GB / 2;
    // independent partial sums per vector (one vector: four FMA chains of 16 instead of one of
    // 64), added in a fixed order at the end
    constexpr int NA = NT == 1 ? 4 : NT == 2 ? 2 : 1;
    uint32_t w[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = wp[i];
    float part[NT][NA];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int j = 0; j < NA; ++j) part[t][j] = 0.0f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int b0 = half * GB;
        const float d = f16_bits_to_f32((w[b0 / 4] >> ((b0 % 4) * 8)) & 0xFFFFu);
        const float *xh = xp + (half * 32) * np;
        if (ENC == CPG_ENC_Q4) {
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int bo = b0 + 2 + k;
                const uint32_t byte = (w[bo / 4] >> ((bo % 4) * 8)) & 0xFFu;
                const float lo = __fmul_rn((float)sext4(byte), d);
                const float hi = __fmul_rn((float)sext4(byte >> 4), d);
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    part[t][(2 * k) % NA] = fmaf(lo, xh[t * n_in + k * np], part[t][(2 * k) % NA]);
                    part[t][(2 * k + 1) % NA] = fmaf(hi, xh[t * n_in + (k + 16) * np], part[t][(2 * k + 1) % NA]);
                }
            }
        } else {
#pragma unroll
            for (int k = 0; k < 32; ++k) {
                const int bo = b0 + 2 + k;
                const float v = __fmul_rn((float)(int)(int8_t)((w[bo / 4] >> ((bo % 4) * 8)) & 0xFFu), d);
#pragma unroll
                for (int t = 0; t < NT; ++t) part[t][k % NA] = fmaf(v, xh[t * n_in + k * np], part[t][k % NA]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        if constexpr (NA == 4) acc[t] += (part[t][0] + part[t][1]) + (part[t][2] + part[t][3]);
        else if constexpr (NA == 2) acc[t] += part[t][0] + part[t][1];
        else acc[t] += part[t][0];
    }
}

// Up to three matrices of the same width and encoding read the same vectors (the attention
// projections Wq, Wk, Wv); their 16-row tiles are numbered one after the other. With `norm`
// set, x is first RMS-normalised per vector with that gain (kernels.c:408-413: inv = 1/sqrt(Σx²/n
// + eps), xn = (x·inv)·g), so the layer's first RMSNorm needs no launch of its own.
struct GemvSeg {
    const uint8_t *w;
    float *out;
    int n_out;
};
struct GemvArgs {
    GemvSeg seg[3];
    int nseg;
    const float *x;
    const float *norm;
    float eps;
    int n_in;
    long rowbytes;
    int stages;
};

template <int ENC, int NT>
__global__ void __launch_bounds__((GV_CONS + 1) * 32) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(16) uint8_t gsm[];
    const int n_in = a.n_in;
    float *xs = reinterpret_cast<float *>(gsm);                           // (NT, n_in) pair-permuted
    uint8_t *ring = gsm + (size_t)NT * n_in * sizeof(float);
    __shared__ uint64_t full[8], empty[8];
    __shared__ float s_red[GV_CONS + 1][NT];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int np = n_in / 64;
    int t0[4] = {0, 0, 0, 0};
    for (int i = 0; i < a.nseg; ++i) t0[i + 1] = t0[i] + (a.seg[i].n_out + GV_ROWS - 1) / GV_ROWS;
    const int ntiles = t0[a.nseg];
    const size_t stage_bytes = (size_t)GV_ROWS * a.rowbytes;
    const int stages = a.stages;
    if (threadIdx.x == 0) {
        for (int i = 0; i < stages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], GV_CONS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    if (warp == GV_CONS) {
        // weights do not depend on the previous kernel: the ring fills while it finishes
        if (lane != 0) return;
        int it = 0;
        for (int tl = blockIdx.x; tl < ntiles; tl += gridDim.x, ++it) {
            const int st = it % stages;
            if (it >= stages && !mbar_wait(&empty[st], (uint32_t)(it / stages - 1) & 1u)) break;
            int sg = 0;
            while (tl >= t0[sg + 1]) ++sg;
            const int r0 = (tl - t0[sg]) * GV_ROWS, nr = min(GV_ROWS, a.seg[sg].n_out - r0);
            mbar_arrive_expect_tx(&full[st], (uint32_t)(nr * a.rowbytes));
            bulk_g2s(ring + st * stage_bytes, a.seg[sg].w + (size_t)r0 * a.rowbytes, (uint32_t)(nr * a.rowbytes), &full[st]);
        }
        for (int q = it > stages ? it - stages : 0; q < it; ++q) mbar_wait(&full[q % stages], (uint32_t)(q / stages) & 1u);
        return;
    }
    pdl_wait();                                        // x comes from the previous kernel
    float inv[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) inv[t] = 1.0f;
    if (a.norm) {
        float ss[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) ss[t] = 0.0f;
        for (int i = threadIdx.x; i < n_in; i += GV_CONS * 32) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const float v = a.x[(size_t)t * n_in + i];
                ss[t] = fmaf(v, v, ss[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss[t] += __shfl_xor_sync(0xffffffffu, ss[t], o);
            if (lane == 0) s_red[warp][t] = ss[t];
        }
        named_bar_sync(1, GV_CONS * 32);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float tot = 0.0f;
            for (int w = 0; w < GV_CONS; ++w) tot += s_red[w][t];
            inv[t] = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(tot, (float)n_in) + a.eps));
        }
    }
    for (int i = threadIdx.x; i < NT * n_in; i += GV_CONS * 32) {
        const int t = i / n_in, e = i - t * n_in;
        float v = a.x[i];
        if (a.norm) v = __fmul_rn(__fmul_rn(v, inv[t]), a.norm[e]);
        xs[t * n_in + (e % 64) * np + e / 64] = v;
    }
    named_bar_sync(1, GV_CONS * 32);
    int it = 0;
    for (int tl = blockIdx.x; tl < ntiles; tl += gridDim.x, ++it) {
        const int st = it % stages;
        if (!mbar_wait(&full[st], (uint32_t)(it / stages) & 1u)) break;
        int sg = 0;
        while (tl >= t0[sg + 1]) ++sg;
        const int r0 = (tl - t0[sg]) * GV_ROWS, n_out = a.seg[sg].n_out, nr = min(GV_ROWS, n_out - r0);
#pragma unroll
        for (int rr = 0; rr < GV_ROWS / GV_CONS; ++rr) {
            const int r = warp * (GV_ROWS / GV_CONS) + rr;
            if (r >= nr) break;
            const uint32_t *row = reinterpret_cast<const uint32_t *>(ring + st * stage_bytes + (size_t)r * a.rowbytes);
            float acc[NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
            for (int p = lane; p < np; p += 32) gemv_pair<ENC, NT>(row + p * (ENC == CPG_ENC_Q4 ? 9 : 17), xs + p, np, n_in, acc);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
            }
            if (lane == 0) {
#pragma unroll
                for (int t = 0; t < NT; ++t) a.seg[sg].out[(size_t)t * n_out + r0 + r] = acc[t];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
}

template <int ENC, int NT>
static int gemv_launch(const GemvArgs &ga, cudaStream_t s) {
    auto *k = k_gemv<ENC, NT>;
    const size_t xbytes = (size_t)NT * ga.n_in * sizeof(float);
    const size_t stage = (size_t)GV_ROWS * ga.rowbytes;
    const int avail = smem_optin() - 4096;
    int stages = (int)((avail - (long)xbytes) / (long)stage);
    if (stages > 4) stages = 4;
    if (stages < 2) return 1;                                 // too wide: the row kernel takes it
    GemvArgs a = ga;
    a.stages = stages;
    const size_t smem = xbytes + stages * stage;
    CPG_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int ntiles = 0;
    for (int i = 0; i < a.nseg; ++i) ntiles += (a.seg[i].n_out + GV_ROWS - 1) / GV_ROWS;
    // as many CTAs as fit (two per SM for the attention projections' 18 KB tiles): more tiles in
    // flight and fewer tiles per CTA, which is what bounds a small matrix
    int per_sm = 1;
    CPG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, (GV_CONS + 1) * 32, smem));
    if (per_sm < 1) per_sm = 1;
    const int grid = ntiles < per_sm * sm_count() ? ntiles : per_sm * sm_count();
    CPG_CUDA(launch_pdl(k, dim3(grid), dim3((GV_CONS + 1) * 32), smem, s, a));
    return CPG_OK;
}

// Streaming GEMV over up to three matrices of one width (nseg ≤ 3), optional RMSNorm of x first.
// Returns 1 when the shape does not suit the streaming kernel (the caller falls back).
int gemv_multi(const GemvSeg *segs, int nseg, const float *x, int T, const float *norm, float eps, int n_in, int enc,
               cudaStream_t s) {
    const long rb = row_bytes(enc, n_in);
    if (enc == CPG_ENC_F32 || T < 1 || T > GV_MAXT || nseg < 1 || nseg > 3 || n_in % 64 || rb % 16 || ((uintptr_t)x & 15))
        return 1;
    GemvArgs a{};
    for (int i = 0; i < nseg; ++i) {
        if ((uintptr_t)segs[i].w & 15) return 1;
        a.seg[i] = segs[i];
    }
    a.nseg = nseg; a.x = x; a.norm = norm; a.eps = eps; a.n_in = n_in; a.rowbytes = rb;
    if (enc == CPG_ENC_Q4)
        return T == 1 ? gemv_launch<CPG_ENC_Q4, 1>(a, s) : T == 2 ? gemv_launch<CPG_ENC_Q4, 2>(a, s)
             : T == 3 ? gemv_launch<CPG_ENC_Q4, 3>(a, s) : gemv_launch<CPG_ENC_Q4, 4>(a, s);
    return T == 1 ? gemv_launch<CPG_ENC_Q8, 1>(a, s) : T == 2 ? gemv_launch<CPG_ENC_Q8, 2>(a, s)
         : T == 3 ? gemv_launch<CPG_ENC_Q8, 3>(a, s) : gemv_launch<CPG_ENC_Q8, 4>(a, s);
}

template <int ENC>
__global__ void __launch_bounds__(MV_WARPS * 32)
k_matvec(float *__restrict__ out, const float *__restrict__ x, const uint8_t *__restrict__ w,
         int n_in, int n_out, int T, int tok_per_cta, long rowbytes) {
    extern __shared__ float xs[];                       // (tok_per_cta, n_in), lane-friendly order
    const int t0 = blockIdx.y * tok_per_cta;
    const int nt = min(tok_per_cta, T - t0);
    const bool aligned4 = (((uintptr_t)w | (uintptr_t)rowbytes) & 3) == 0;
    // element e of a vector goes to: f32 -> e; Q pairs -> (e%64)*np + e/64; Q groups -> (e%32)*ng + e/32
    const int ng = n_in / 32;
    const bool pairs = ENC != CPG_ENC_F32 && aligned4 && (ng % 2) == 0;
    for (int i = threadIdx.x; i < nt * n_in; i += blockDim.x) {
        const int t = i / n_in, e = i - t * n_in;
        int o = e;
        if (ENC != CPG_ENC_F32) o = pairs ? (e % 64) * (ng / 2) + e / 64 : (e % 32) * ng + e / 32;
        xs[t * n_in + o] = x[(size_t)(t0 + t) * n_in + e];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = blockIdx.x * MV_WARPS + warp; r < n_out; r += gridDim.x * MV_WARPS) {
        const uint8_t *row = w + (size_t)r * rowbytes;
        for (int tc = 0; tc < nt; tc += MV_TOK) {
            float acc[MV_TOK];
#pragma unroll
            for (int t = 0; t < MV_TOK; ++t) acc[t] = 0.0f;
            row_partial<ENC>(row, n_in, xs + tc * n_in, min(MV_TOK, nt - tc), acc, aligned4);
#pragma unroll
            for (int t = 0; t < MV_TOK; ++t) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
            }
            if (lane == 0) {
#pragma unroll
                for (int t = 0; t < MV_TOK; ++t)
                    if (tc + t < nt) out[(size_t)(t0 + tc + t) * n_out + r] = acc[t];
            }
        }
    }
}

// f32 W·x of any shape and alignment (matmul_wx takes any n_in, kernels.c:84-95): one warp per
// (token, output row), lane-strided scalar loads, fp32 FMA, a warp reduction.
__global__ void __launch_bounds__(256) k_matvec_f32_any(float *__restrict__ out, const float *__restrict__ x,
                                                        const float *__restrict__ w, int n_in, int n_out, int T) {
    const int lane = threadIdx.x & 31;
    const long nw = (long)gridDim.x * (blockDim.x >> 5);
    for (long i = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < (long)T * n_out; i += nw) {
        const int t = (int)(i / n_out), r = (int)(i - (long)t * n_out);
        const float *row = w + (size_t)r * n_in, *xt = x + (size_t)t * n_in;
        float acc = 0.0f;
        for (int k = lane; k < n_in; k += 32) acc = fmaf(__ldg(row + k), __ldg(xt + k), acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) out[(size_t)t * n_out + r] = acc;
    }
}

int matvec_launch(float *out, const float *x, cpg_tensor w, int n_in, int n_out, int T,
                  cudaStream_t s) {
    CPG_REQUIRE(out && x && w.p, "cpg_matvec: null pointer");
    CPG_REQUIRE(n_in > 0 && n_out > 0 && T > 0, "cpg_matvec: empty shape (%d, %d, T=%d)", n_in, n_out, T);
    CPG_REQUIRE(w.enc == CPG_ENC_F32 || w.enc == CPG_ENC_Q4 || w.enc == CPG_ENC_Q8,
                "cpg_matvec: unknown encoding %d", w.enc);
    CPG_REQUIRE(w.enc == CPG_ENC_F32 || n_in % 32 == 0, "cpg_matvec: n_in=%d not a multiple of 32", n_in);
    if (w.enc == CPG_ENC_F32 && (n_in % 4 != 0 || ((uintptr_t)w.p & 15) != 0)) {
        long warps = (long)T * n_out;
        int grid = (int)std::min<long>((warps + 7) / 8, (long)sm_count() * 16);
        k_matvec_f32_any<<<grid, 256, 0, s>>>(out, x, (const float *)w.p, n_in, n_out, T);
        CPG_CUDA(cudaGetLastError());
        return CPG_OK;
    }
    const long rb = row_bytes(w.enc, n_in);
    // decode-sized batches of quantised rows: the streaming kernel
    {
        const GemvSeg seg{(const uint8_t *)w.p, out, n_out};
        const int r = gemv_multi(&seg, 1, x, T, nullptr, 0.0f, n_in, w.enc, s);
        if (r != 1) return r;
    }
    // tokens per CTA: as many as fit 96 KB of staged x
    int tpc = (int)((96 * 1024) / ((long)n_in * 4));
    CPG_REQUIRE(tpc >= 1, "cpg_matvec: n_in=%d too large to stage", n_in);
    if (tpc > T) tpc = T;
    const size_t smem = (size_t)tpc * n_in * sizeof(float);
    const int ty = (T + tpc - 1) / tpc;
    int gx = (n_out + MV_WARPS - 1) / MV_WARPS;
    const int cap = sm_count() * 8;
    if (gx > cap) gx = cap;
    dim3 grid(gx, ty);
    auto *kq4 = k_matvec<CPG_ENC_Q4>;
    auto *kq8 = k_matvec<CPG_ENC_Q8>;
    auto *kf = k_matvec<CPG_ENC_F32>;
    auto *k = w.enc == CPG_ENC_Q4 ? kq4 : w.enc == CPG_ENC_Q8 ? kq8 : kf;
    const int rc = allow_max_smem((const void *)k);
    if (rc) return rc;
    k<<<grid, MV_WARPS * 32, smem, s>>>(out, x, (const uint8_t *)w.p, n_in, n_out, T, tpc, rb);
    CPG_CUDA(cudaGetLastError());
    return CPG_OK;
}

}  // namespace cpg

extern "C" int cpg_matvec(float *out, const float *x, cpg_tensor w, int n_in, int n_out, int T,
                          void *stream) {
    return cpg::matvec_launch(out, x, w, n_in, n_out, T, (cudaStream_t)stream);
}
