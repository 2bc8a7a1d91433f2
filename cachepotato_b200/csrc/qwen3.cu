// qwen3.cu — the whole Qwen3-MoE model on the device (the whole-model benchmark): the attention half of
// qwen3_layer_kv (engine/blocks/qwen3_moe.c:110-167), the MoE half through cpg_moe_forward, and the
// model loop of cp_chat (engine/api/cachepotato.c:108-166, 315-378): embed_rows, run_layers,
// apply_head, greedy argmax.
//
// Per layer, for T new tokens at positions pos0..pos0+T-1:
//   k_rmsnorm       xn = RMSNorm(x, ln1)                                   kernels.c:408-413
//   cpg_matvec ×3   q = Wq·xn, k = Wk·xn, v = Wv·xn (k, v straight into the f32 KV cache)
//                   (T ≤ 4: one streaming GEMV launch with the RMSNorm fused; a prompt of
//                   QW_DENSE_MIN_T tokens or more with Q4_0 projections: the tcgen05 GEMM of
//                   gemm_tc.cu, operands split into two fp16 terms each, three passes, which
//                   keeps the result within f32 rounding of the GEMV's)
//   k_qk_norm_rope  per-head RMSNorm of q and k (head_rmsnorm, qwen3_moe.c:44-49), then RoPE at
//                   each token's position (rope_apply_from, kernels.c:425-447); a one-token step
//                   does this inside the attention kernel
//   attention       causal GQA: s = q·k / sqrt(hd), softmax, Σ s·v (qwen3_moe.c:135-155):
//                   k_attention_split (decode-sized T: position ranges per head, merged),
//                   k_attention_prompt (prompts: 32 queries per block), k_attention (fallback)
//   cpg_matvec      attn = Wo·ao
//   cpg_moe_forward RMSNorm(x + attn, ln2) → router → experts → x += attn + mlp (fused residual)
// Head: RMSNorm of the last position with final_norm, lm_head GEMV, k_argmax (first maximum wins).
// Head dimension 128 (one warp per head, four values per lane).
#include <math.h>

#include <algorithm>

#include <vector>

#include "common.cuh"
#include "expert_tile.cuh"
#include "gemm_tc.cuh"

namespace cpg {

constexpr int QW_HD = 128;
constexpr int QW_DENSE_MIN_T = 32;     // prompt length from which projections run on tcgen05

__device__ __forceinline__ float block_sum(float v, float *s_red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) s_red[warp] = v;
    __syncthreads();
    float r = 0.0f;
    for (int i = 0; i < nw; ++i) r += s_red[i];
    __syncthreads();
    return r;
}

// embed_rows (cachepotato.c:108-133): row ids[t] of the Q8_0/Q4_0 table, q·d exact in fp32.
__global__ void __launch_bounds__(256) k_embed(const uint8_t *__restrict__ tab, int enc, const int *__restrict__ ids,
                                                int D, float *__restrict__ x) {
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    const int gb = enc == CPG_ENC_Q4 ? 18 : 34;
    const uint8_t *row = tab + (size_t)ids[t] * (size_t)(D / 32) * gb;
    for (int g = threadIdx.x; g < D / 32; g += blockDim.x) {
        const uint8_t *blk = row + (size_t)g * gb;
        const float d = f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
        float *o = x + (size_t)t * D + g * 32;
        if (enc == CPG_ENC_Q8) {
            for (int i = 0; i < 32; ++i) o[i] = __fmul_rn((float)(int8_t)blk[2 + i], d);
        } else {
            for (int k = 0; k < 16; ++k) {
                const int b = blk[2 + k];
                const int lo = (b & 0x0F) > 7 ? (b & 0x0F) - 16 : (b & 0x0F);
                const int hi = (b >> 4) > 7 ? (b >> 4) - 16 : (b >> 4);
                o[k] = __fmul_rn((float)lo, d);
                o[k + 16] = __fmul_rn((float)hi, d);
            }
        }
    }
}

// rmsnorm (kernels.c:408-413): inv = 1/sqrt(Σx²/n + eps), out = (x·inv)·g; one block per row.
__global__ void __launch_bounds__(256) k_rmsnorm(const float *__restrict__ x, const float *__restrict__ g, int D,
                                                  float eps, float *__restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float s_red[8];
    const float *xr = x + (size_t)blockIdx.x * D;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < D; k += blockDim.x) ss = fmaf(xr[k], xr[k], ss);
    ss = block_sum(ss, s_red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(ss, (float)D) + eps));
    float *o = out + (size_t)blockIdx.x * D;
    for (int k = threadIdx.x; k < D; k += blockDim.x) o[k] = __fmul_rn(__fmul_rn(xr[k], inv), g[k]);
}

// hi = fp16(v), lo = fp16(v − hi): v to about 22 bits in two fp16 terms.
__device__ __forceinline__ void split_f16(float v, __half &hi, __half &lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

// k_rmsnorm as the operand of the tensor-core projections: row t of out (2·D halves) holds
// [hi(xn_t) | lo(xn_t)].
__global__ void __launch_bounds__(256) k_rmsnorm_f16(const float *__restrict__ x, const float *__restrict__ g, int D,
                                                      float eps, __half *__restrict__ out) {
    __shared__ float s_red[8];
    const float *xr = x + (size_t)blockIdx.x * D;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < D; k += blockDim.x) ss = fmaf(xr[k], xr[k], ss);
    ss = block_sum(ss, s_red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(ss, (float)D) + eps));
    __half *o = out + (size_t)blockIdx.x * 2 * D;
    for (int k = threadIdx.x; k < D; k += blockDim.x)
        split_f16(__fmul_rn(__fmul_rn(xr[k], inv), g[k]), o[k], o[D + k]);
}

// (T, n) f32 rows -> (T, 2n) [hi | lo] fp16 rows.
__global__ void k_split_f16(const float *__restrict__ x, int T, int n, __half *__restrict__ out) {
    const size_t total = (size_t)T * n;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t t = i / n, c = i - t * n;
        split_f16(x[i], out[t * 2 * n + c], out[t * 2 * n + n + c]);
    }
}

// The single-group tables of the dense projections: group p (0..3 = q, k, v, o) holds all T
// tokens in order.
__global__ void k_dense_tab(int4 *tab, int *n_active, int T) {
    const int p = threadIdx.x;
    if (p < 4) {
        tab[2 * p] = make_int4(p, 0, T, 0);
        tab[2 * p + 1] = make_int4(-1, T, 0, 0);
    }
    if (p == 0) *n_active = 1;
}

__global__ void k_iota(int *v, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) v[i] = i;
}

// One warp: head RMSNorm with gain g (head_rmsnorm, qwen3_moe.c:44-49), then RoPE at `pos`
// (rope_apply_from, kernels.c:425-447), of the 128 values at src into dst (may alias). Lane l
// holds elements l, l+32 (first half) and l+64, l+96 (their rotation partners). Products and
// sums are rounded one at a time, as the reference's ISO C.
__device__ __forceinline__ void head_norm_rope(const float *src, const float *__restrict__ g, float pos, float theta,
                                               float eps, float *dst) {
    const int lane = threadIdx.x & 31;
    float e[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = src[lane + 32 * i];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) ss = fmaf(e[i], e[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(ss, (float)QW_HD) + eps));
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = __fmul_rn(__fmul_rn(e[i], inv), g[lane + 32 * i]);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int fi = lane + 32 * i;                               // frequency index in [0, 64)
        const float invf = powf(theta, __fdiv_rn(-2.0f * (float)fi, (float)QW_HD));
        const float ang = __fmul_rn(pos, invf);
        const float c = cosf(ang), s = sinf(ang);
        const float a = e[i], b = e[i + 2];
        e[i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
        e[i + 2] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = e[i];
}

// One warp per (token, head) of q (heads 0..H-1) and k (heads H..H+KV-1): head_norm_rope at
// position pos0 + t (pos0 read from the device, so a captured step serves every position). q is
// updated in place; k and v go from their staging rows (T, KV·hd) into the cache at pos0 + t.
__global__ void __launch_bounds__(256) k_qk_norm_rope(float *__restrict__ q, const float *__restrict__ kst,
                                                       const float *__restrict__ vst, float *__restrict__ kc,
                                                       float *__restrict__ vc, int T, const int *__restrict__ d_pos,
                                                       int H, int KV, const float *__restrict__ qn,
                                                       const float *__restrict__ kn, float theta, float eps) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nh = H + KV;
    if (w >= T * nh) return;
    const int pos0 = *d_pos;
    const int t = w / nh, h = w - t * nh;
    const bool isq = h < H;
    const size_t krow = ((size_t)t * KV + (h - H)) * QW_HD, kdst = ((size_t)(pos0 + t) * KV + (h - H)) * QW_HD;
    const float *src = isq ? q + ((size_t)t * H + h) * QW_HD : kst + krow;
    float *v = isq ? q + ((size_t)t * H + h) * QW_HD : kc + kdst;
    const float *g = isq ? qn : kn;
    if (!isq) {
#pragma unroll
        for (int i = 0; i < 4; ++i) vc[kdst + lane + 32 * i] = vst[krow + lane + 32 * i];
    }
    head_norm_rope(src, g, (float)(pos0 + t), theta, eps, v);
}

// Causal GQA attention (qwen3_moe.c:135-155), one block of 256 threads per (query token i,
// head h) over the n = pos0 + i + 1 cached positions:
//   scores   one thread per position: s = Σ_e q[e]·k[e] in element order with one rounding per
//            product and per sum (the reference's loop, ISO C without contraction), then / √hd
//   softmax  max, expf(s - max), sum, divide (block reductions: the sum's order differs)
//   output   warp w takes positions [w·n/8, (w+1)·n/8), lane l elements 4l..4l+3 (float4 rows),
//            the eight partial sums added in warp order
constexpr int AT_THREADS = 256;
constexpr int AT_WARPS = AT_THREADS / 32;
__global__ void __launch_bounds__(AT_THREADS) k_attention(const float *__restrict__ q, const float *__restrict__ kc,
                                                           const float *__restrict__ vc, const int *__restrict__ d_pos,
                                                           int H, int KV, float *__restrict__ ao) {
    pdl_wait();
    pdl_launch_dependents();
    const int pos0 = *d_pos;
    extern __shared__ float sc[];                        // (n) scores
    __shared__ float s_red[AT_WARPS];
    __shared__ __align__(16) float s_q[QW_HD];
    __shared__ __align__(16) float s_out[AT_WARPS][QW_HD];
    const int h = blockIdx.x, i = blockIdx.y;
    const int kh = h / (H / KV);
    const int n = pos0 + i + 1;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x < QW_HD) s_q[threadIdx.x] = q[((size_t)i * H + h) * QW_HD + threadIdx.x];
    __syncthreads();
    const float scale = __fsqrt_rn((float)QW_HD);
    const size_t ks = (size_t)KV * QW_HD;
    for (int j = threadIdx.x; j < n; j += AT_THREADS) {
        const float4 *kj = reinterpret_cast<const float4 *>(kc + (size_t)j * ks + (size_t)kh * QW_HD);
        const float4 *q4 = reinterpret_cast<const float4 *>(s_q);
        float s = 0.0f;
#pragma unroll 8
        for (int e = 0; e < QW_HD / 4; ++e) {
            const float4 kv = __ldg(kj + e), qv = q4[e];
            s = __fadd_rn(s, __fmul_rn(qv.x, kv.x));
            s = __fadd_rn(s, __fmul_rn(qv.y, kv.y));
            s = __fadd_rn(s, __fmul_rn(qv.z, kv.z));
            s = __fadd_rn(s, __fmul_rn(qv.w, kv.w));
        }
        sc[j] = __fdiv_rn(s, scale);
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < n; j += AT_THREADS) mx = fmaxf(mx, sc[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = s_red[0];
#pragma unroll
    for (int w = 1; w < AT_WARPS; ++w) mx = fmaxf(mx, s_red[w]);
    __syncthreads();
    float sum = 0.0f;
    for (int j = threadIdx.x; j < n; j += AT_THREADS) {
        const float ex = expf(__fsub_rn(sc[j], mx));
        sc[j] = ex;
        sum += ex;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) s_red[warp] = sum;
    __syncthreads();
    sum = 0.0f;
#pragma unroll
    for (int w = 0; w < AT_WARPS; ++w) sum += s_red[w];
    for (int j = threadIdx.x; j < n; j += AT_THREADS) sc[j] = __fdiv_rn(sc[j], sum);
    __syncthreads();
    const int per = (n + AT_WARPS - 1) / AT_WARPS;
    const int j0 = warp * per, j1 = min(n, j0 + per);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float *vb = vc + (size_t)kh * QW_HD + lane * 4;
    int j = j0;
    for (; j + 4 <= j1; j += 4) {                        // four rows in flight
        float4 vv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) vv[u] = __ldg(reinterpret_cast<const float4 *>(vb + (size_t)(j + u) * ks));
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float p = sc[j + u];
            acc.x = __fadd_rn(acc.x, __fmul_rn(p, vv[u].x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(p, vv[u].y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(p, vv[u].z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(p, vv[u].w));
        }
    }
    for (; j < j1; ++j) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(vb + (size_t)j * ks));
        const float p = sc[j];
        acc.x = __fadd_rn(acc.x, __fmul_rn(p, v.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(p, v.y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(p, v.z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(p, v.w));
    }
    *reinterpret_cast<float4 *>(&s_out[warp][lane * 4]) = acc;
    __syncthreads();
    if (threadIdx.x < QW_HD) {
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < AT_WARPS; ++w) o = __fadd_rn(o, s_out[w][threadIdx.x]);
        ao[((size_t)i * H + h) * QW_HD + threadIdx.x] = o;
    }
}

// The same attention for a prompt (T ≥ QW_DENSE_MIN_T new tokens): one block per (head h,
// AP_QT consecutive queries), so each key and value row read from the cache serves AP_QT queries.
//   scores   key tiles of AP_KT rows in shared memory; a thread holds 4 queries × 2 keys, each
//            score a sequential f32 sum over the 128 elements (fused multiply-adds), then / √hd
//   softmax  one warp per query row: max, expf(s - max), sum, divide (rows past the causal end
//            are zero)
//   output   value tiles in shared memory; warp w holds queries 4w..4w+3, lane l elements
//            4l..4l+3, summed over positions in order
// Shared memory: the (AP_QT, n_cap) score rows, one key/value tile, the query rows.
constexpr int AP_QT = 32, AP_KT = 64, AP_KS = QW_HD + 4;        // row stride: conflict-free float4
__global__ void __launch_bounds__(256) k_attention_prompt(const float *__restrict__ q, const float *__restrict__ kc,
                                                          const float *__restrict__ vc, const int *__restrict__ d_pos,
                                                          int T, int H, int KV, int n_cap, float *__restrict__ ao) {
    extern __shared__ __align__(16) float smp[];
    const int ss = (n_cap + 3) & ~3;                          // score row stride (16-byte rows)
    float *sS = smp;                                          // (AP_QT, ss)
    float *sK = sS + (size_t)AP_QT * ss;                      // (AP_KT, AP_KS) keys, then values
    float *sQ = sK + AP_KT * AP_KS;                           // (AP_QT, hd)
    const int h = blockIdx.x, q0 = blockIdx.y * AP_QT;
    const int kh = h / (H / KV);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int pos0 = *d_pos;
    const int nq = min(AP_QT, T - q0);
    const int nmax = min(n_cap, pos0 + q0 + nq);              // keys the last query of the tile sees
    const size_t ks = (size_t)KV * QW_HD;
    for (int i = tid; i < AP_QT * QW_HD / 4; i += 256) {
        const int qi = i / (QW_HD / 4), d4 = i % (QW_HD / 4);
        const float4 v = qi < nq ? *reinterpret_cast<const float4 *>(q + ((size_t)(q0 + qi) * H + h) * QW_HD + 4 * d4)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4 *>(sQ + qi * QW_HD + 4 * d4) = v;
    }
    const float scale = __fsqrt_rn((float)QW_HD);
    const int qg = warp, kg = lane;                           // queries 4qg..4qg+3, keys kg, kg+32
    for (int kt0 = 0; kt0 < nmax; kt0 += AP_KT) {
        __syncthreads();
        for (int i = tid; i < AP_KT * QW_HD / 4; i += 256) {
            const int r = i / (QW_HD / 4), d4 = i % (QW_HD / 4);
            const float4 v = kt0 + r < nmax ? *reinterpret_cast<const float4 *>(kc + (size_t)(kt0 + r) * ks + (size_t)kh * QW_HD + 4 * d4)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4 *>(sK + r * AP_KS + 4 * d4) = v;
        }
        __syncthreads();
        float acc[4][2] = {};
#pragma unroll 4
        for (int d4 = 0; d4 < QW_HD / 4; ++d4) {
            float4 qv[4], kv[2];
#pragma unroll
            for (int a = 0; a < 4; ++a) qv[a] = *reinterpret_cast<const float4 *>(sQ + (4 * qg + a) * QW_HD + 4 * d4);
#pragma unroll
            for (int b = 0; b < 2; ++b) kv[b] = *reinterpret_cast<const float4 *>(sK + (kg + 32 * b) * AP_KS + 4 * d4);
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    float t = acc[a][b];
                    t = fmaf(qv[a].x, kv[b].x, t);
                    t = fmaf(qv[a].y, kv[b].y, t);
                    t = fmaf(qv[a].z, kv[b].z, t);
                    t = fmaf(qv[a].w, kv[b].w, t);
                    acc[a][b] = t;
                }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const int j = kt0 + kg + 32 * b;
                if (j < nmax) sS[(size_t)(4 * qg + a) * ss + j] = __fdiv_rn(acc[a][b], scale);
            }
    }
    __syncthreads();
    for (int qi = warp; qi < AP_QT; qi += 8) {                // softmax per row, zeros past the end
        float *row = sS + (size_t)qi * ss;
        const int n = qi < nq ? min(nmax, pos0 + q0 + qi + 1) : 0;
        float mx = -INFINITY;
        for (int j = lane; j < n; j += 32) mx = fmaxf(mx, row[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.0f;
        for (int j = lane; j < n; j += 32) {
            const float ex = expf(__fsub_rn(row[j], mx));
            row[j] = ex;
            sum += ex;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        for (int j = lane; j < nmax; j += 32) row[j] = j < n ? __fdiv_rn(row[j], sum) : 0.0f;
    }
    float4 out[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) out[a] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int vt0 = 0; vt0 < nmax; vt0 += AP_KT) {
        __syncthreads();
        for (int i = tid; i < AP_KT * QW_HD / 4; i += 256) {
            const int r = i / (QW_HD / 4), d4 = i % (QW_HD / 4);
            const float4 v = vt0 + r < nmax ? *reinterpret_cast<const float4 *>(vc + (size_t)(vt0 + r) * ks + (size_t)kh * QW_HD + 4 * d4)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4 *>(sK + r * AP_KS + 4 * d4) = v;
        }
        __syncthreads();
        const int jn = min(AP_KT, nmax - vt0);
        for (int j = 0; j < jn; ++j) {
            const float4 v = *reinterpret_cast<const float4 *>(sK + j * AP_KS + 4 * lane);
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const float p = sS[(size_t)(4 * warp + a) * ss + vt0 + j];
                out[a].x = fmaf(p, v.x, out[a].x);
                out[a].y = fmaf(p, v.y, out[a].y);
                out[a].z = fmaf(p, v.z, out[a].z);
                out[a].w = fmaf(p, v.w, out[a].w);
            }
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int qi = 4 * warp + a;
        if (qi < nq) *reinterpret_cast<float4 *>(ao + ((size_t)(q0 + qi) * H + h) * QW_HD + 4 * lane) = out[a];
    }
}

// Decode-sized T: the positions of each (query, head) are split into gridDim.y ≤ AS_SPLIT ranges,
// one block each, so that a step's attention spreads over enough blocks whatever the context
// (as_splits: 16 for one query, one range once the T·H pairs alone fill the GPU):
//   block    scores of its range (warp per position, lane l elements 4l..4l+3, shuffle sum),
//            local max m and sum l of expf(s - m), o = Σ expf(s - m)·v (positions in order per
//            warp, warps added in order); (m, l, o) to part
//   last     the block that finishes last for (query, head) (a counter per pair, reset by that
//            block) merges the ranges: M = max m, out = Σ o·e^(m-M) / Σ l·e^(m-M)
// The range length follows the device position, so a captured step serves every position.
// With `nr` set (each query a new token: a decode step), the head norm and RoPE of
// k_qk_norm_rope happen here: every block normalises its q row, the block whose range holds the
// new position normalises the new key itself (and takes the new value from the staging row), and
// of the heads sharing a KV head the first writes both into the cache for the later steps.
// With `seq.tok_pos` set (a step of several sequences), query i is the new token of its own
// sequence: position tok_pos[i], cache rows at kc/vc + tok_slot[i]·slot_elems; otherwise the T
// queries are consecutive tokens of one sequence at positions *d_pos + i.
struct AttnNorm {
    const float *kst, *vst, *qn, *kn;
    float theta, eps;
    int on;
};
struct AttnSeqs {
    const int *tok_slot, *tok_pos;
    size_t slot_elems;
};
constexpr int AS_SPLIT = 16, AS_THREADS = 256;
constexpr int AS_B = 4;                                           // positions per warp with loads in flight
// At most 64 registers (four blocks per SM): a decode step's 512 blocks stay one wave.
__global__ void __launch_bounds__(AS_THREADS, 4) k_attention_split(const float *__restrict__ q, float *__restrict__ kc,
                                                                float *__restrict__ vc, const int *__restrict__ d_pos,
                                                                int H, int KV, float *__restrict__ part, int *__restrict__ cnt,
                                                                float *__restrict__ ao, const AttnNorm nr, const AttnSeqs seq) {
    pdl_wait();
    pdl_launch_dependents();
    extern __shared__ float s_sc[];                               // the range's scores
    __shared__ float s_red[AS_THREADS / 32];
    __shared__ __align__(16) float s_o[AS_THREADS / 32][QW_HD];
    __shared__ __align__(16) float s_qk[3][QW_HD];               // normalised q, new k, new v
    __shared__ int s_last;
    const int h = blockIdx.x, b = blockIdx.y, i = blockIdx.z;
    const int kh = h / (H / KV);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int pnew;                                                     // this query's position
    if (seq.tok_pos) {
        pnew = seq.tok_pos[i];
        const size_t off = (size_t)seq.tok_slot[i] * seq.slot_elems;
        kc += off;
        vc += off;
    } else {
        pnew = *d_pos + i;
    }
    const int n = pnew + 1;
    const int ns = gridDim.y;
    const int chunk = (n + ns - 1) / ns;
    const int j0 = b * chunk, len = max(0, min(n, j0 + chunk) - j0);
    const size_t ks = (size_t)KV * QW_HD;
    const bool holds_new = nr.on && pnew >= j0 && pnew < j0 + len;   // this range ends at the new key
    if (nr.on) {
        const size_t krow = ((size_t)i * KV + kh) * QW_HD;
        if (warp == 0) head_norm_rope(q + ((size_t)i * H + h) * QW_HD, nr.qn, (float)pnew, nr.theta, nr.eps, s_qk[0]);
        if (holds_new && warp == 1) head_norm_rope(nr.kst + krow, nr.kn, (float)pnew, nr.theta, nr.eps, s_qk[1]);
        if (holds_new && warp == 2)
            for (int e = lane; e < QW_HD; e += 32) s_qk[2][e] = nr.vst[krow + e];
        __syncthreads();
        if (holds_new && h % (H / KV) == 0 && tid < 2 * QW_HD) {  // the cache row for later steps
            float *dst = (tid < QW_HD ? kc : vc) + (size_t)pnew * ks + (size_t)kh * QW_HD;
            dst[tid % QW_HD] = s_qk[1 + tid / QW_HD][tid % QW_HD];
        }
    }
    const float4 qv = nr.on ? *reinterpret_cast<const float4 *>(&s_qk[0][4 * lane])
                            : *reinterpret_cast<const float4 *>(q + ((size_t)i * H + h) * QW_HD + 4 * lane);
    const float scale = __fsqrt_rn((float)QW_HD);
    const float *kb = kc + (size_t)kh * QW_HD + 4 * lane, *vb = vc + (size_t)kh * QW_HD + 4 * lane;
    constexpr int NW = AS_THREADS / 32;
    // a warp's positions warp, warp + NW, ...: AS_B key rows requested before any is used
    for (int j = warp; j < len; j += NW * AS_B) {
        float4 kv[AS_B];
#pragma unroll
        for (int u = 0; u < AS_B; ++u) {
            const int jj = j + NW * u;
            kv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (jj < len)
                kv[u] = holds_new && j0 + jj == pnew ? *reinterpret_cast<const float4 *>(&s_qk[1][4 * lane])
                                                     : *reinterpret_cast<const float4 *>(kb + (size_t)(j0 + jj) * ks);
        }
#pragma unroll
        for (int u = 0; u < AS_B; ++u) {
            const int jj = j + NW * u;
            float sv = fmaf(qv.x, kv[u].x, fmaf(qv.y, kv[u].y, fmaf(qv.z, kv[u].z, __fmul_rn(qv.w, kv[u].w))));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sv += __shfl_xor_sync(0xffffffffu, sv, o);
            if (lane == 0 && jj < len) s_sc[jj] = __fdiv_rn(sv, scale);
        }
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int jj = tid; jj < len; jj += AS_THREADS) mx = fmaxf(mx, s_sc[jj]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = s_red[0];
#pragma unroll
    for (int w = 1; w < AS_THREADS / 32; ++w) mx = fmaxf(mx, s_red[w]);
    __syncthreads();
    float sum = 0.0f;
    for (int jj = tid; jj < len; jj += AS_THREADS) {
        const float ex = expf(__fsub_rn(s_sc[jj], mx));
        s_sc[jj] = ex;
        sum += ex;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) s_red[warp] = sum;
    __syncthreads();
    sum = 0.0f;
#pragma unroll
    for (int w = 0; w < AS_THREADS / 32; ++w) sum += s_red[w];
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = warp; j < len; j += NW * AS_B) {                // value rows in flight the same way,
        float4 vv[AS_B];                                          // added in position order
#pragma unroll
        for (int u = 0; u < AS_B; ++u) {
            const int jj = j + NW * u;
            vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (jj < len)
                vv[u] = holds_new && j0 + jj == pnew ? *reinterpret_cast<const float4 *>(&s_qk[2][4 * lane])
                                                     : *reinterpret_cast<const float4 *>(vb + (size_t)(j0 + jj) * ks);
        }
#pragma unroll
        for (int u = 0; u < AS_B; ++u) {
            const int jj = j + NW * u;
            if (jj >= len) break;
            const float p = s_sc[jj];
            acc.x = fmaf(p, vv[u].x, acc.x);
            acc.y = fmaf(p, vv[u].y, acc.y);
            acc.z = fmaf(p, vv[u].z, acc.z);
            acc.w = fmaf(p, vv[u].w, acc.w);
        }
    }
    *reinterpret_cast<float4 *>(&s_o[warp][4 * lane]) = acc;
    __syncthreads();
    float *pp = part + (((size_t)i * H + h) * ns + b) * (QW_HD + 2);
    if (tid < QW_HD) {
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < AS_THREADS / 32; ++w) o += s_o[w][tid];
        pp[2 + tid] = o;
    }
    if (tid == 0) {
        pp[0] = mx;
        pp[1] = sum;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&cnt[i * H + h], 1) == ns - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid < QW_HD) {
        const float *p0 = part + ((size_t)i * H + h) * ns * (QW_HD + 2);
        float M = -INFINITY;
        for (int r = 0; r < ns; ++r) {
            const float l = __ldcg(p0 + r * (QW_HD + 2) + 1);
            if (l > 0.0f) M = fmaxf(M, __ldcg(p0 + r * (QW_HD + 2)));
        }
        float L = 0.0f, o = 0.0f;
        for (int r = 0; r < ns; ++r) {
            const float l = __ldcg(p0 + r * (QW_HD + 2) + 1);
            if (l > 0.0f) {
                const float e = expf(__fsub_rn(__ldcg(p0 + r * (QW_HD + 2)), M));
                L = fmaf(l, e, L);
                o = fmaf(__ldcg(p0 + r * (QW_HD + 2) + 2 + tid), e, o);
            }
        }
        ao[((size_t)i * H + h) * QW_HD + tid] = __fdiv_rn(o, L);
    }
    if (tid == 0) cnt[i * H + h] = 0;                             // ready for the next launch
}

// A step of several sequences, one block per (KV head, token): the H/KV query heads sharing the
// KV head are the block's warps, so each cached key and value row is read once for all of them
// (qwen3_moe.c:135-155 per head). The head norm and RoPE of q and of the new key happen here (as
// in k_attention_split with `nr`), and the new key and value go into the token's slot at its
// position. Positions are taken in chunks of AG_CHUNK rows staged in shared memory (rows padded
// to AG_RS floats, so lane j reads row j without bank conflicts); per warp:
//   scores   lane j: s_j = Σ_e q[e]·k_j[e] (fused multiply-adds in element order) / √hd
//   softmax  online over the chunks: running max m, sum l and output o rescaled by e^(m - m')
//            when a chunk raises the max
//   output   lane l holds elements 4l..4l+3: o += e^(s_j - m)·v_j, positions in order; o / l
constexpr int AG_CHUNK = 64, AG_RS = QW_HD + 4;
static size_t attention_group_smem() { return (size_t)2 * AG_CHUNK * AG_RS * sizeof(float); }
__global__ void __launch_bounds__(256) k_attention_group(const float *__restrict__ q, float *__restrict__ kc,
                                                         float *__restrict__ vc, int H, int KV, const AttnNorm nr,
                                                         const AttnSeqs seq, float *__restrict__ ao) {
    pdl_wait();
    pdl_launch_dependents();
    extern __shared__ __align__(16) float ag[];
    float *sK = ag, *sV = ag + AG_CHUNK * AG_RS;
    __shared__ __align__(16) float s_q[8][QW_HD];
    __shared__ __align__(16) float s_new[2][QW_HD];
    const int kh = blockIdx.x, i = blockIdx.y, G = H / KV;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int h = kh * G + w;
    const int pos = seq.tok_pos[i], n = pos + 1;
    const size_t off = (size_t)seq.tok_slot[i] * seq.slot_elems, ks = (size_t)KV * QW_HD;
    kc += off;
    vc += off;
    const size_t krow = ((size_t)i * KV + kh) * QW_HD;
    if (w < G) head_norm_rope(q + ((size_t)i * H + h) * QW_HD, nr.qn, (float)pos, nr.theta, nr.eps, s_q[w]);
    if (w == 0) head_norm_rope(nr.kst + krow, nr.kn, (float)pos, nr.theta, nr.eps, s_new[0]);
    if (w == 1)
        for (int e = lane; e < QW_HD; e += 32) s_new[1][e] = nr.vst[krow + e];
    __syncthreads();
    for (int e = tid; e < 2 * QW_HD; e += blockDim.x)            // the cache rows for later steps
        ((e < QW_HD ? kc : vc) + (size_t)pos * ks + (size_t)kh * QW_HD)[e % QW_HD] = s_new[e / QW_HD][e % QW_HD];
    const float scale = __fsqrt_rn((float)QW_HD);
    float m = -INFINITY, l = 0.0f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < n; c0 += AG_CHUNK) {
        const int cn = min(AG_CHUNK, n - c0);
        __syncthreads();                                          // the previous chunk is consumed
        for (int idx = tid; idx < cn * (QW_HD / 4); idx += blockDim.x) {
            const int r = idx / (QW_HD / 4), c4 = idx % (QW_HD / 4), j = c0 + r;
            float4 kv, vv;
            if (j == pos) {
                kv = *reinterpret_cast<const float4 *>(&s_new[0][4 * c4]);
                vv = *reinterpret_cast<const float4 *>(&s_new[1][4 * c4]);
            } else {
                kv = __ldg(reinterpret_cast<const float4 *>(kc + (size_t)j * ks + (size_t)kh * QW_HD) + c4);
                vv = __ldg(reinterpret_cast<const float4 *>(vc + (size_t)j * ks + (size_t)kh * QW_HD) + c4);
            }
            *reinterpret_cast<float4 *>(sK + r * AG_RS + 4 * c4) = kv;
            *reinterpret_cast<float4 *>(sV + r * AG_RS + 4 * c4) = vv;
        }
        __syncthreads();
        if (w >= G) continue;
        float sc[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int r = lane + 32 * u;
            if (r < cn) {
                const float4 *kr = reinterpret_cast<const float4 *>(sK + r * AG_RS);
                const float4 *qr = reinterpret_cast<const float4 *>(s_q[w]);
                float acc = 0.0f;
#pragma unroll 8
                for (int c = 0; c < QW_HD / 4; ++c) {
                    const float4 kv = kr[c], qv = qr[c];
                    acc = fmaf(qv.x, kv.x, acc);
                    acc = fmaf(qv.y, kv.y, acc);
                    acc = fmaf(qv.z, kv.z, acc);
                    acc = fmaf(qv.w, kv.w, acc);
                }
                sc[u] = __fdiv_rn(acc, scale);
            } else {
                sc[u] = -INFINITY;
            }
        }
        const float mn = fmaxf(m, warp_max(fmaxf(sc[0], sc[1])));
        const float rs = expf(__fsub_rn(m, mn));                  // 0 on the first chunk
        const float p0 = expf(__fsub_rn(sc[0], mn)), p1 = expf(__fsub_rn(sc[1], mn));
        l = fmaf(l, rs, warp_sum(p0 + p1));
        o.x *= rs; o.y *= rs; o.z *= rs; o.w *= rs;
        for (int r = 0; r < cn; ++r) {
            const float p = __shfl_sync(0xffffffffu, r < 32 ? p0 : p1, r & 31);
            const float4 v = *reinterpret_cast<const float4 *>(sV + r * AG_RS + 4 * lane);
            o.x = fmaf(p, v.x, o.x);
            o.y = fmaf(p, v.y, o.y);
            o.z = fmaf(p, v.z, o.z);
            o.w = fmaf(p, v.w, o.w);
        }
        m = mn;
    }
    if (w < G)
        *reinterpret_cast<float4 *>(ao + ((size_t)i * H + h) * QW_HD + 4 * lane) =
            make_float4(__fdiv_rn(o.x, l), __fdiv_rn(o.y, l), __fdiv_rn(o.z, l), __fdiv_rn(o.w, l));
}

// Ranges per (query, head) for T queries of H heads: enough blocks for four waves of 148 SMs.
static int as_splits(int T, int H) {
    const int pairs = T * H, want = 4 * 148;
    return pairs >= want ? 1 : std::min(AS_SPLIT, (want + pairs - 1) / pairs);
}

static size_t attention_prompt_smem(int n_cap) {
    return sizeof(float) * ((size_t)AP_QT * ((n_cap + 3) & ~3) + AP_KT * AP_KS + AP_QT * QW_HD);
}

// argmax with the first maximum winning (cachepotato.c:353-356), NaN-free logits: each block
// takes one contiguous chunk (partial results), then one block combines them; ties go to the
// smaller index at every level.
constexpr int AM_BLOCKS = 148;
__device__ __forceinline__ void argmax_block(float best, int bi, float *out_v, int *out_i) {
    __shared__ float s_v[32];
    __shared__ int s_i[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    if (lane == 0) { s_v[warp] = best; s_i[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (s_v[w] > best || (s_v[w] == best && s_i[w] < bi)) { best = s_v[w]; bi = s_i[w]; }
        *out_v = best;
        *out_i = bi;
    }
}

// Row r = blockIdx.y of (rows, n) logits; its partials at part + r·gridDim.x.
__global__ void __launch_bounds__(512) k_argmax_part(const float *__restrict__ v, int n, float *part_v, int *part_i) {
    pdl_wait();
    pdl_launch_dependents();
    v += (size_t)blockIdx.y * n;
    part_v += (size_t)blockIdx.y * gridDim.x;
    part_i += (size_t)blockIdx.y * gridDim.x;
    const int chunk = (n + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = lo + threadIdx.x; j < hi; j += blockDim.x) {
        const float x = v[j];
        if (x > best) { best = x; bi = j; }                 // j ascends: ties keep the first
    }
    argmax_block(best, bi, part_v + blockIdx.x, part_i + blockIdx.x);
}

// Row r = blockIdx.x: its nparts partials, the id to out[r].
__global__ void __launch_bounds__(256) k_argmax_final(const float *__restrict__ part_v, const int *__restrict__ part_i,
                                                       int nparts, int *out) {
    pdl_wait();
    pdl_launch_dependents();
    part_v += (size_t)blockIdx.x * nparts;
    part_i += (size_t)blockIdx.x * nparts;
    out += blockIdx.x;
    __shared__ float s_best;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = threadIdx.x; j < nparts; j += blockDim.x) {
        const float x = part_v[j];
        const int i = part_i[j];
        if (x > best || (x == best && i < bi)) { best = x; bi = i; }
    }
    argmax_block(best, bi, &s_best, out);
}

// After a step: the argmax becomes the next step's input id, the position advances, and the id
// is recorded at out[*d_pos - base] when out is given.
__global__ void k_advance(const int *__restrict__ next, int *__restrict__ ids, int *__restrict__ d_pos, int T,
                          int *__restrict__ out, int base) {
    pdl_wait();
    pdl_launch_dependents();
    const int id = *next;
    const int p = *d_pos + T;
    *d_pos = p;
    ids[0] = id;
    if (out) out[p - base] = id;
}

// A step of several sequences: token t is the new token of slot tok_slot[t], at that slot's
// position.
__global__ void k_batch_begin(const int *__restrict__ tok_slot, const int *__restrict__ slot_pos,
                              int *__restrict__ tok_pos, int n) {
    pdl_wait();
    pdl_launch_dependents();
    for (int t = threadIdx.x; t < n; t += blockDim.x) tok_pos[t] = slot_pos[tok_slot[t]];
}

// After such a step: every slot of the step advances by one position, its argmax becomes its
// next input id and is recorded at out[step·n + t], step = *d_step, which then advances.
__global__ void k_batch_advance(const int *__restrict__ next, int *__restrict__ ids, const int *__restrict__ tok_slot,
                                int *__restrict__ slot_pos, int n, int *__restrict__ out, int *__restrict__ d_step) {
    pdl_wait();
    pdl_launch_dependents();
    const int step = *d_step;
    __syncthreads();
    for (int t = threadIdx.x; t < n; t += blockDim.x) {
        const int id = next[t];
        slot_pos[tok_slot[t]] += 1;
        ids[t] = id;
        out[(size_t)step * n + t] = id;
    }
    if (threadIdx.x == 0) *d_step = step + 1;
}

int matvec_launch(float *out, const float *x, cpg_tensor w, int n_in, int n_out, int T, cudaStream_t s);
struct GemvSeg {
    const uint8_t *w;
    float *out;
    int n_out;
};
int gemv_multi(const GemvSeg *segs, int nseg, const float *x, int T, const float *norm, float eps, int n_in, int enc,
               cudaStream_t s);
int layer_dims(const cpg_moe_layer *L, int *D, int *F, int *E, int *K);
bool dense_ok(int enc, int rows, int k);
size_t dense_act_bytes(int T, int K);
int dense_build(const void *w, int enc, int rows, int k, uint8_t **tiles, cudaStream_t s);
int dense_prep(const float *x, int T, int K, const float *gain, float eps, int enc, uint8_t *xh, cudaStream_t s);
int dense_run(const uint8_t *const *tiles, const int *rows, float *const *outs, int nseg, int enc, int K,
              const uint8_t *xh, int T, float *planes, size_t planes_floats, int *counters, int n_counters,
              int *status, cudaStream_t s);
constexpr int QW_DENSE_DEC_MIN_T = 5, QW_DENSE_DEC_MAX_T = 64;   // steps of several sequences on dense.cu

// Decode tile copies of the attention projections and the lm_head (dense.cu) with their operand
// and split-K buffers, built by the first batch of at least QW_DENSE_DEC_MIN_T slots and kept
// with the model: steps of QW_DENSE_DEC_MIN_T .. QW_DENSE_DEC_MAX_T sequences run their
// projections and head on the tensor cores. One sequence keeps the streaming GEMV, which is
// faster at one token (measured: 2.95 against 3.92 ms per token for the whole model).
struct QwDense {
    std::vector<uint8_t *> attn;                   // 4 per layer: Wq, Wk, Wv, Wo
    uint8_t *head = nullptr;
    uint8_t *xh = nullptr;
    float *planes = nullptr;
    size_t planes_floats = 0;
    int *counters = nullptr;                       // split K, one per band
    int *status = nullptr;
};
constexpr int QW_DENSE_COUNTERS = 1024;

}  // namespace cpg

struct cpg_qwen3 {
    int D, H, KV, V, L, max_ctx;
    float theta, eps;
    cpg_tensor embed, lm_head;
    const float *final_norm;
    std::vector<cpg_qwen3_attn> attn;
    std::vector<const cpg_moe_layer *> moe;
    float *x = nullptr, *xn = nullptr, *q = nullptr, *ao = nullptr, *at = nullptr, *kv = nullptr, *logits = nullptr;
    float *kst = nullptr, *vst = nullptr;          // (max_ctx, KV·hd) k and v before the cache
    float *am_v = nullptr;                         // argmax partials
    int *am_i = nullptr;
    int *d_ids = nullptr, *d_next = nullptr, *h_next = nullptr, *d_pos = nullptr, *d_out = nullptr;
    cudaGraphExec_t step_graph = nullptr;          // one decode step, T = 1, any position
    // prompts on the tensor cores (Q4_0 projections): per layer 12 tensor maps (entry 3p+2 over
    // Wq, Wk, Wv, Wo), the four single-group tables, t -> t, the fp16 operand rows, a status word
    void *dmaps = nullptr;
    int4 *dtab = nullptr;
    int *dn_active = nullptr, *iota = nullptr, *d_status = nullptr;
    __half *x16 = nullptr;
    float *planes = nullptr;                       // the projection GEMM's three pass planes
    float *as_part = nullptr;                      // split attention: (T < QW_DENSE_MIN_T, H, AS_SPLIT, 2 + hd)
    int *as_cnt = nullptr;                         // and a counter per (query, head), zero between launches
    size_t ap_smem = 0;                            // shared memory k_attention_prompt may use
    cpg::QwDense dn;                               // dense.cu tiles and buffers (empty: not built)
    void *ws = nullptr;
    size_t ws_bytes = 0;
    int pos = 0;
    cudaStream_t s = nullptr;
};

using namespace cpg;

static void free_dense(QwDense &dn) {
    for (uint8_t *p : dn.attn) cudaFree(p);
    cudaFree(dn.head); cudaFree(dn.xh); cudaFree(dn.planes); cudaFree(dn.status); cudaFree(dn.counters);
    dn = QwDense{};
}

static void qwen3_free(cpg_qwen3 *m) {
    cudaFree(m->x); cudaFree(m->xn); cudaFree(m->q); cudaFree(m->ao); cudaFree(m->at); cudaFree(m->kv);
    cudaFree(m->logits); cudaFree(m->d_ids); cudaFree(m->d_next); cudaFree(m->ws);
    cudaFree(m->kst); cudaFree(m->vst); cudaFree(m->d_pos); cudaFree(m->d_out);
    cudaFree(m->am_v); cudaFree(m->am_i);
    cudaFree(m->dmaps); cudaFree(m->dtab); cudaFree(m->dn_active); cudaFree(m->iota); cudaFree(m->d_status);
    cudaFree(m->x16); cudaFree(m->planes); cudaFree(m->as_part); cudaFree(m->as_cnt);
    free_dense(m->dn);
    if (m->step_graph) cudaGraphExecDestroy(m->step_graph);
    if (m->h_next) cudaFreeHost(m->h_next);
    if (m->s) cudaStreamDestroy(m->s);
    delete m;
}

// The dense.cu copies of every projection and of the lm_head, when every matrix is Q4_0 / Q8_0 of
// a usable shape (otherwise the streaming GEMV and the row kernel serve them). All or nothing.
static int build_dense(cpg_qwen3 *m) {
    const int QD = m->H * QW_HD, KDi = m->KV * QW_HD, D = m->D;
    bool ok = true;
    for (int l = 0; l < m->L && ok; ++l) {
        const cpg_qwen3_attn &A = m->attn[l];
        ok = A.wk.enc == A.wq.enc && A.wv.enc == A.wq.enc && dense_ok(A.wq.enc, QD, D) && dense_ok(A.wk.enc, KDi, D) &&
             dense_ok(A.wo.enc, D, QD);
    }
    if (!ok) return CPG_OK;
    QwDense &dn = m->dn;
    int rc = CPG_OK;
    for (int l = 0; l < m->L && !rc; ++l) {
        const cpg_qwen3_attn &A = m->attn[l];
        const cpg_tensor w[4] = {A.wq, A.wk, A.wv, A.wo};
        const int rows[4] = {QD, KDi, KDi, D}, ks[4] = {D, D, D, QD};
        for (int i = 0; i < 4 && !rc; ++i) {
            uint8_t *t = nullptr;
            rc = dense_build(w[i].p, w[i].enc, rows[i], ks[i], &t, m->s);
            if (!rc) dn.attn.push_back(t);
        }
    }
    if (!rc && dense_ok(m->lm_head.enc, m->V, D)) rc = dense_build(m->lm_head.p, m->lm_head.enc, m->V, D, &dn.head, m->s);
    if (rc) {
        cudaStreamSynchronize(m->s);
        free_dense(dn);
        return rc;
    }
    const int kmax = QD > D ? QD : D;
    dn.planes_floats = (size_t)16 * QW_DENSE_DEC_MAX_T * (QD + 2 * KDi > D ? QD + 2 * KDi : D);
    cudaError_t ce = cudaMalloc(&dn.xh, dense_act_bytes(QW_DENSE_DEC_MAX_T, kmax));
    if (ce == cudaSuccess) ce = cudaMalloc(&dn.planes, dn.planes_floats * sizeof(float));
    if (ce == cudaSuccess) ce = cudaMalloc(&dn.status, sizeof(int));
    if (ce == cudaSuccess) ce = cudaMemsetAsync(dn.status, 0, sizeof(int), m->s);
    if (ce == cudaSuccess) ce = cudaMalloc(&dn.counters, QW_DENSE_COUNTERS * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMemsetAsync(dn.counters, 0, QW_DENSE_COUNTERS * sizeof(int), m->s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(m->s);
    if (ce == cudaSuccess) return CPG_OK;
    free_dense(dn);
    return cuda_fail(ce, "cpg_qwen3_batch_create: dense projections");
}

extern "C" int cpg_qwen3_create(const cpg_qwen3_desc *d, cpg_qwen3 **out) {
    CPG_REQUIRE(d && out, "cpg_qwen3_create: null argument");
    *out = nullptr;
    CPG_REQUIRE(d->head_dim == QW_HD, "cpg_qwen3_create: head_dim %d (this build: %d)", d->head_dim, QW_HD);
    CPG_REQUIRE(d->n_heads > 0 && d->n_kv > 0 && d->n_heads % d->n_kv == 0, "cpg_qwen3_create: heads %d / kv %d",
                d->n_heads, d->n_kv);
    CPG_REQUIRE(d->d_model > 0 && d->d_model % 32 == 0 && d->vocab > 0 && d->n_layers > 0 && d->max_ctx > 0,
                "cpg_qwen3_create: bad dimensions");
    CPG_REQUIRE(d->embed.p && d->lm_head.p && d->final_norm && d->attn && d->moe, "cpg_qwen3_create: null tensor");
    CPG_REQUIRE(d->embed.enc == CPG_ENC_Q8 || d->embed.enc == CPG_ENC_Q4, "cpg_qwen3_create: embed must be Q8_0/Q4_0");
    for (int l = 0; l < d->n_layers; ++l) {
        int D, F, E, K;
        CPG_REQUIRE(d->moe[l] && layer_dims(d->moe[l], &D, &F, &E, &K) == CPG_OK && D == d->d_model,
                    "cpg_qwen3_create: layer %d: MoE half missing or d_model mismatch", l);
        const cpg_qwen3_attn &A = d->attn[l];
        CPG_REQUIRE(A.ln1 && A.q_norm && A.k_norm && A.wq.p && A.wk.p && A.wv.p && A.wo.p,
                    "cpg_qwen3_create: layer %d: null attention tensor", l);
    }
    cpg_qwen3 *m = new cpg_qwen3();
    m->D = d->d_model; m->H = d->n_heads; m->KV = d->n_kv; m->V = d->vocab; m->L = d->n_layers;
    m->max_ctx = d->max_ctx; m->theta = d->rope_theta; m->eps = d->rms_eps;
    m->embed = d->embed; m->lm_head = d->lm_head; m->final_norm = d->final_norm;
    m->attn.assign(d->attn, d->attn + d->n_layers);
    m->moe.assign(d->moe, d->moe + d->n_layers);
    const size_t C = (size_t)d->max_ctx, D = d->d_model, QD = (size_t)d->n_heads * QW_HD, KD = (size_t)d->n_kv * QW_HD;
    m->ws_bytes = cpg_moe_workspace_bytes(d->moe[0], d->max_ctx);
    cudaError_t ce = cudaStreamCreateWithFlags(&m->s, cudaStreamNonBlocking);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->x, C * D * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->xn, C * D * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->at, C * D * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->q, C * QD * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->ao, C * QD * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->kv, (size_t)d->n_layers * 2 * C * KD * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->logits, (size_t)d->vocab * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->d_ids, C * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->d_next, 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->kst, C * KD * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->vst, C * KD * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->d_pos, 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->am_v, AM_BLOCKS * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->am_i, AM_BLOCKS * 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->d_out, (C + 1) * 4);
    if (ce == cudaSuccess) ce = cudaMallocHost(&m->h_next, 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->ws, m->ws_bytes);
    if (ce == cudaSuccess)
        ce = cudaMalloc(&m->as_part, (size_t)QW_DENSE_MIN_T * d->n_heads * AS_SPLIT * (QW_HD + 2) * sizeof(float));
    if (ce == cudaSuccess) ce = cudaMalloc(&m->as_cnt, (size_t)QW_DENSE_MIN_T * d->n_heads * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMemset(m->as_cnt, 0, (size_t)QW_DENSE_MIN_T * d->n_heads * sizeof(int));
    if (ce != cudaSuccess) {
        qwen3_free(m);
        return cuda_fail(ce, "cpg_qwen3_create: allocation");
    }
    const size_t asmem = C * sizeof(float);            // attention scores of every position
    if (asmem > 32 * 1024) {                           // beyond the default with the static arrays
        if (asmem > 200 * 1024) {
            qwen3_free(m);
            CPG_REQUIRE(false, "cpg_qwen3_create: max_ctx %d too long for the attention kernel", d->max_ctx);
        }
        ce = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)asmem);
        if (ce == cudaSuccess)       // one range per (query, head): the scores of every position
            ce = cudaFuncSetAttribute(k_attention_split, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)asmem);
        if (ce != cudaSuccess) {
            qwen3_free(m);
            return cuda_fail(ce, "cpg_qwen3_create: attention shared memory");
        }
    }
    // tensor-core projections for prompts, when every projection is Q4_0 of a usable shape
    bool dense = D % 256 == 0 && QD % 256 == 0 && KD % 256 == 0;
    for (int l = 0; l < d->n_layers && dense; ++l) {
        const cpg_qwen3_attn &A = d->attn[l];
        dense = A.wq.enc == CPG_ENC_Q4 && A.wk.enc == CPG_ENC_Q4 && A.wv.enc == CPG_ENC_Q4 && A.wo.enc == CPG_ENC_Q4;
    }
    if (dense) {
        std::vector<const uint8_t *> w;
        std::vector<int> rows, k;
        for (int l = 0; l < d->n_layers; ++l) {
            const cpg_qwen3_attn &A = d->attn[l];
            const uint8_t *p[4] = {(const uint8_t *)A.wq.p, (const uint8_t *)A.wk.p, (const uint8_t *)A.wv.p,
                                   (const uint8_t *)A.wo.p};
            const int r[4] = {(int)QD, (int)KD, (int)KD, (int)D}, kk[4] = {(int)D, (int)D, (int)D, (int)QD};
            for (int i = 0; i < 4; ++i) {
                w.push_back(p[i]); rows.push_back(r[i]); k.push_back(kk[i]);
            }
        }
        int rc = gemm_tc_dense_maps(w.data(), rows.data(), k.data(), (int)w.size(), &m->dmaps);
        if (rc) {
            qwen3_free(m);
            return rc;
        }
        ce = cudaMalloc(&m->dtab, 8 * sizeof(int4));
        if (ce == cudaSuccess) ce = cudaMalloc(&m->dn_active, sizeof(int));
        if (ce == cudaSuccess) ce = cudaMalloc(&m->iota, C * sizeof(int));
        if (ce == cudaSuccess) ce = cudaMalloc(&m->d_status, sizeof(int));
        if (ce == cudaSuccess) ce = cudaMalloc(&m->x16, C * 2 * (QD > D ? QD : D) * sizeof(__half));
        if (ce == cudaSuccess) ce = cudaMalloc(&m->planes, C * 3 * (QD > D ? QD : D) * sizeof(float));
        if (ce == cudaSuccess) ce = cudaMemsetAsync(m->d_status, 0, sizeof(int), m->s);
        if (ce == cudaSuccess) {
            k_iota<<<(int)((C + 255) / 256), 256, 0, m->s>>>(m->iota, (int)C);
            ce = cudaGetLastError();
        }
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(m->s);
        if (ce != cudaSuccess) {
            qwen3_free(m);
            return cuda_fail(ce, "cpg_qwen3_create: dense projection tables");
        }
    }
    // prompt attention: the score rows of the whole context when they fit in shared memory
    const size_t ap = attention_prompt_smem(d->max_ctx);
    if (ap <= (size_t)smem_optin()) {
        ce = cudaFuncSetAttribute(k_attention_prompt, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ap);
        if (ce != cudaSuccess) {
            qwen3_free(m);
            return cuda_fail(ce, "cpg_qwen3_create: prompt attention shared memory");
        }
        m->ap_smem = ap;
    }
    *out = m;
    return CPG_OK;
}

extern "C" void cpg_qwen3_destroy(cpg_qwen3 *m) {
    if (m) qwen3_free(m);
}

// Where the T tokens of one enqueue belong. The KV cache holds S slots of C positions per layer:
// layer l's keys of slot j at kv + ((2l)·S + j)·C·KD, its values at kv + ((2l + 1)·S + j)·C·KD
// (S = 1: the model's own sequence). Either the T tokens are consecutive tokens of slot `slot`
// from the device position *d_pos (a prompt, or the model's own decode step), or (slot < 0)
// token t is the new token of slot tok_slot[t] at position tok_pos[t] (a step of several
// sequences). The head runs on the last row (one sequence) or on every row (several), into
// logits (rows, V) and the argmax into d_next[row].
struct QwSeq {
    float *kv;
    int S, C;
    const int *d_pos;
    int slot;
    const int *tok_slot, *tok_pos;
    int n_cap;                      // one sequence: its length after these T tokens
    float *as_part;
    int *as_cnt;
    float *logits, *am_v;
    int *am_i, *d_next;
    const QwDense *dn;              // several sequences: the dense.cu path, or null
};

// Enqueue T tokens (ids in m->d_ids[0..T)) through embed, the layers and the head. Nothing here
// reads a position on the host, so a decode step is captured once and replayed at every position.
static int qwen3_enqueue(cpg_qwen3 *m, const QwSeq &sq, int T, cudaStream_t s) {
    const int D = m->D, H = m->H, KV = m->KV, QD = H * QW_HD, KD = KV * QW_HD;
    const size_t C = (size_t)sq.C, S = (size_t)sq.S;
    const bool multi = sq.slot < 0;
    CPG_CUDA(launch_pdl(k_embed, dim3(T), dim3(256), 0, s, (const uint8_t *)m->embed.p, m->embed.enc,
                        (const int *)m->d_ids, D, m->x));
    const bool dense = m->dmaps && T >= QW_DENSE_MIN_T;
    if (dense) {
        k_dense_tab<<<1, 32, 0, s>>>(m->dtab, m->dn_active, T);
        CPG_CUDA(cudaGetLastError());
    }
    const AttnSeqs aseq{multi ? sq.tok_slot : nullptr, multi ? sq.tok_pos : nullptr, C * KD};
    for (int l = 0; l < m->L; ++l) {
        const cpg_qwen3_attn &A = m->attn[l];
        float *kc = sq.kv + (size_t)(2 * l) * S * C * KD, *vc = kc + S * C * KD;
        if (!multi) {
            kc += (size_t)sq.slot * C * KD;
            vc += (size_t)sq.slot * C * KD;
        }
        const void *maps = dense ? (const void *)((const uint8_t *)m->dmaps + (size_t)l * 12 * 128) : nullptr;
        // RMSNorm(x, ln1) and q, k, v: prompts on the tensor cores; decode-sized T in one
        // streaming launch; otherwise separately
        const int enc = A.wq.enc;
        int rc = 1;
        const bool ddec = sq.dn && T >= QW_DENSE_DEC_MIN_T && T <= QW_DENSE_DEC_MAX_T;
        if (ddec) {
            const uint8_t *tl[3] = {sq.dn->attn[4 * l], sq.dn->attn[4 * l + 1], sq.dn->attn[4 * l + 2]};
            const int rows[3] = {QD, KD, KD};
            float *const outs[3] = {m->q, m->kst, m->vst};
            rc = dense_prep(m->x, T, D, A.ln1, m->eps, enc, sq.dn->xh, s);
            if (!rc) rc = dense_run(tl, rows, outs, 3, enc, D, sq.dn->xh, T, sq.dn->planes, sq.dn->planes_floats,
                                    sq.dn->counters, QW_DENSE_COUNTERS, sq.dn->status, s);
            if (rc) return rc;
        } else if (dense) {
            k_rmsnorm_f16<<<T, 256, 0, s>>>(m->x, A.ln1, D, m->eps, m->x16);
            CPG_CUDA(cudaGetLastError());
            rc = gemm_tc_dense(maps, m->dtab + 0, m->dn_active, m->iota, m->x16, T, QD, D, m->q, m->planes, m->d_status, s);
            if (!rc) rc = gemm_tc_dense(maps, m->dtab + 2, m->dn_active, m->iota, m->x16, T, KD, D, m->kst, m->planes, m->d_status, s);
            if (!rc) rc = gemm_tc_dense(maps, m->dtab + 4, m->dn_active, m->iota, m->x16, T, KD, D, m->vst, m->planes, m->d_status, s);
            if (rc) return rc;
        } else if (A.wk.enc == enc && A.wv.enc == enc) {
            const GemvSeg seg[3] = {{(const uint8_t *)A.wq.p, m->q, QD}, {(const uint8_t *)A.wk.p, m->kst, KD},
                                    {(const uint8_t *)A.wv.p, m->vst, KD}};
            rc = gemv_multi(seg, 3, m->x, T, A.ln1, m->eps, D, enc, s);
        }
        if (rc == 1) {
            k_rmsnorm<<<T, 256, 0, s>>>(m->x, A.ln1, D, m->eps, m->xn);
            CPG_CUDA(cudaGetLastError());
            rc = matvec_launch(m->q, m->xn, A.wq, D, QD, T, s);
            if (!rc) rc = matvec_launch(m->kst, m->xn, A.wk, D, KD, T, s);
            if (!rc) rc = matvec_launch(m->vst, m->xn, A.wv, D, KD, T, s);
        }
        if (rc) return rc;
        const int warps = T * (H + KV);
        AttnNorm nr{};                               // new tokens, one per sequence: fused into the attention
        if (T == 1 || multi) nr = AttnNorm{m->kst, m->vst, A.q_norm, A.k_norm, m->theta, m->eps, 1};
        else
            CPG_CUDA(launch_pdl(k_qk_norm_rope, dim3((warps + 7) / 8), dim3(256), 0, s, m->q, (const float *)m->kst,
                                (const float *)m->vst, kc, vc, T, sq.d_pos, H, KV, A.q_norm, A.k_norm,
                                m->theta, m->eps));
        const int n_cap = sq.n_cap;                                  // prompt: positions known here
        if (!multi && T >= QW_DENSE_MIN_T && attention_prompt_smem(n_cap) <= m->ap_smem) {
            k_attention_prompt<<<dim3(H, (T + AP_QT - 1) / AP_QT), 256, attention_prompt_smem(n_cap), s>>>(
                (const float *)m->q, (const float *)kc, (const float *)vc, sq.d_pos, T, H, KV, n_cap, m->ao);
            CPG_CUDA(cudaGetLastError());
        } else if (multi && T * KV >= 148 && H / KV <= 8) {
            CPG_CUDA(launch_pdl(k_attention_group, dim3(KV, T), dim3(32 * (H / KV)), attention_group_smem(), s,
                                (const float *)m->q, kc, vc, H, KV, nr, aseq, m->ao));
        } else if (multi || T < QW_DENSE_MIN_T) {
            const int ns = as_splits(T, H);
            const size_t ssmem = (size_t)((sq.C + ns - 1) / ns) * sizeof(float);
            CPG_CUDA(launch_pdl(k_attention_split, dim3(H, ns, T), dim3(AS_THREADS), ssmem, s, (const float *)m->q,
                                kc, vc, sq.d_pos, H, KV, sq.as_part, sq.as_cnt, m->ao, nr, aseq));
        } else {
            const size_t asmem = (size_t)sq.C * sizeof(float);          // scores of every cached position
            CPG_CUDA(launch_pdl(k_attention, dim3(H, T), dim3(AT_THREADS), asmem, s, (const float *)m->q,
                                (const float *)kc, (const float *)vc, sq.d_pos, H, KV, m->ao));
        }
        if (ddec) {
            const uint8_t *tl[1] = {sq.dn->attn[4 * l + 3]};
            const int rows[1] = {D};
            float *const outs[1] = {m->at};
            rc = dense_prep(m->ao, T, QD, nullptr, 0.0f, A.wo.enc, sq.dn->xh, s);
            if (!rc) rc = dense_run(tl, rows, outs, 1, A.wo.enc, QD, sq.dn->xh, T, sq.dn->planes, sq.dn->planes_floats,
                                    sq.dn->counters, QW_DENSE_COUNTERS, sq.dn->status, s);
        } else if (dense) {
            const size_t n = (size_t)T * QD;
            k_split_f16<<<(int)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184), 256, 0, s>>>(m->ao, T, QD, m->x16);
            CPG_CUDA(cudaGetLastError());
            rc = gemm_tc_dense(maps, m->dtab + 6, m->dn_active, m->iota, m->x16, T, D, QD, m->at, m->planes, m->d_status, s);
        } else {
            rc = matvec_launch(m->at, m->ao, A.wo, QD, D, T, s);
        }
        if (rc) return rc;
        rc = cpg_moe_forward(m->moe[l], m->x, m->at, T, nullptr, m->x, nullptr, nullptr, nullptr, m->ws, m->ws_bytes, s);
        if (rc) return rc;
    }
    // head: RMSNorm with final_norm fused into the lm_head GEMV, of the last position (one
    // sequence) or of every row (one new token per sequence)
    const int hr = multi ? T : 1;
    const float *xl = m->x + (size_t)(T - hr) * D;
    const GemvSeg hseg{(const uint8_t *)m->lm_head.p, sq.logits, m->V};
    int rc = 1;
    if (multi && sq.dn && sq.dn->head && hr >= QW_DENSE_DEC_MIN_T && hr <= QW_DENSE_DEC_MAX_T) {
        const uint8_t *tl[1] = {sq.dn->head};
        const int rows[1] = {m->V};
        float *const outs[1] = {sq.logits};
        rc = dense_prep(xl, hr, D, m->final_norm, m->eps, m->lm_head.enc, sq.dn->xh, s);
        if (!rc) rc = dense_run(tl, rows, outs, 1, m->lm_head.enc, D, sq.dn->xh, hr, sq.dn->planes,
                                sq.dn->planes_floats, sq.dn->counters, QW_DENSE_COUNTERS, sq.dn->status, s);
        if (rc) return rc;
    } else if (m->lm_head.enc != CPG_ENC_F32) {
        rc = gemv_multi(&hseg, 1, xl, hr, m->final_norm, m->eps, D, m->lm_head.enc, s);
    }
    if (rc == 1) {
        k_rmsnorm<<<hr, 256, 0, s>>>(xl, m->final_norm, D, m->eps, m->xn);
        CPG_CUDA(cudaGetLastError());
        rc = matvec_launch(sq.logits, m->xn, m->lm_head, D, m->V, hr, s);
    }
    if (rc) return rc;
    const int parts = std::min(AM_BLOCKS, std::max(4, (2 * AM_BLOCKS + hr - 1) / hr));   // chunks per row
    CPG_CUDA(launch_pdl(k_argmax_part, dim3(parts, hr), dim3(512), 0, s, (const float *)sq.logits, m->V, sq.am_v,
                        sq.am_i));
    CPG_CUDA(launch_pdl(k_argmax_final, dim3(hr), dim3(256), 0, s, (const float *)sq.am_v, (const int *)sq.am_i,
                        parts, sq.d_next));
    return CPG_OK;
}

// The model's own sequence: slot 0 of its own cache.
static QwSeq own_seq(cpg_qwen3 *m, int T) {
    return QwSeq{m->kv, 1, m->max_ctx, m->d_pos, 0, nullptr, nullptr, m->pos + T, m->as_part, m->as_cnt,
                 m->logits, m->am_v, m->am_i, m->d_next, nullptr};
}

// One token at the current device position: the captured step graph (built on first use).
static int qwen3_step_device(cpg_qwen3 *m, int *out, int base) {
    CPG_REQUIRE(m->pos + 1 <= m->max_ctx, "cpg_qwen3: position %d reached max_ctx %d", m->pos, m->max_ctx);
    if (!m->step_graph) {
        cudaGraph_t g = nullptr;
        CPG_CUDA(cudaStreamBeginCapture(m->s, cudaStreamCaptureModeThreadLocal));
        int rc = qwen3_enqueue(m, own_seq(m, 1), 1, m->s);
        const cudaError_t ce = cudaStreamEndCapture(m->s, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (ce != cudaSuccess) return cuda_fail(ce, "cpg_qwen3: step capture");
        const cudaError_t ie = cudaGraphInstantiate(&m->step_graph, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) return cuda_fail(ie, "cpg_qwen3: step instantiate");
    }
    CPG_CUDA(cudaGraphLaunch(m->step_graph, m->s));
    k_advance<<<1, 1, 0, m->s>>>(m->d_next, m->d_ids, m->d_pos, 1, out, base);
    CPG_CUDA(cudaGetLastError());
    m->pos += 1;
    return CPG_OK;
}

static int qwen3_read_next(cpg_qwen3 *m, int *next_id) {
    CPG_CUDA(cudaMemcpyAsync(m->h_next, m->d_next, 4, cudaMemcpyDeviceToHost, m->s));
    CPG_CUDA(cudaStreamSynchronize(m->s));
    if (next_id) *next_id = *m->h_next;
    return CPG_OK;
}

// The projection GEMM's bounded waits (prompts and steps of QW_DENSE_MIN_T tokens or more).
static int qwen3_status(cpg_qwen3 *m, const char *fn) {
    const int *words[2] = {m->d_status, m->dn.status};
    for (const int *w : words) {
        if (!w) continue;
        int st = 0;
        CPG_CUDA(cudaMemcpy(&st, w, sizeof(int), cudaMemcpyDeviceToHost));
        if (st != ST_OK) {
            set_error("%s: a bounded wait in a projection kernel timed out (status %d)", fn, st);
            return CPG_ETIMEOUT;
        }
    }
    return CPG_OK;
}

extern "C" int cpg_qwen3_prefill(cpg_qwen3 *m, const int *ids, int T, int *next_id) {
    CPG_REQUIRE(m && ids && T > 0, "cpg_qwen3_prefill: bad argument");
    CPG_REQUIRE(T <= m->max_ctx, "cpg_qwen3_prefill: %d tokens > max_ctx %d", T, m->max_ctx);
    for (int t = 0; t < T; ++t) CPG_REQUIRE(ids[t] >= 0 && ids[t] < m->V, "cpg_qwen3_prefill: id %d out of range", ids[t]);
    m->pos = 0;
    CPG_CUDA(cudaMemsetAsync(m->d_pos, 0, 4, m->s));
    CPG_CUDA(cudaMemcpyAsync(m->d_ids, ids, sizeof(int) * (size_t)T, cudaMemcpyHostToDevice, m->s));
    const int rc = qwen3_enqueue(m, own_seq(m, T), T, m->s);
    if (rc) return rc;
    int rc2 = 0;
    k_advance<<<1, 1, 0, m->s>>>(m->d_next, m->d_ids, m->d_pos, T, nullptr, 0);
    CPG_CUDA(cudaGetLastError());
    m->pos = T;
    rc2 = qwen3_read_next(m, next_id);
    return rc2 ? rc2 : qwen3_status(m, "cpg_qwen3_prefill");
}

extern "C" int cpg_qwen3_append(cpg_qwen3 *m, const int *ids, int T, int *next_id) {
    CPG_REQUIRE(m && ids && T > 0, "cpg_qwen3_append: bad argument");
    CPG_REQUIRE(m->pos + T <= m->max_ctx, "cpg_qwen3_append: %d + %d tokens > max_ctx %d", m->pos, T, m->max_ctx);
    for (int t = 0; t < T; ++t) CPG_REQUIRE(ids[t] >= 0 && ids[t] < m->V, "cpg_qwen3_append: id %d out of range", ids[t]);
    CPG_CUDA(cudaMemcpyAsync(m->d_ids, ids, sizeof(int) * (size_t)T, cudaMemcpyHostToDevice, m->s));
    const int rc = qwen3_enqueue(m, own_seq(m, T), T, m->s);
    if (rc) return rc;
    k_advance<<<1, 1, 0, m->s>>>(m->d_next, m->d_ids, m->d_pos, T, nullptr, 0);
    CPG_CUDA(cudaGetLastError());
    m->pos += T;
    const int rc2 = qwen3_read_next(m, next_id);
    return rc2 ? rc2 : qwen3_status(m, "cpg_qwen3_append");
}

extern "C" int cpg_qwen3_rewind(cpg_qwen3 *m, int pos) {
    CPG_REQUIRE(m && pos >= 0 && pos <= m->pos, "cpg_qwen3_rewind: position %d (current %d)", pos, m ? m->pos : -1);
    m->pos = pos;
    int *h = m->h_next;                                  // pinned staging word
    *h = pos;
    CPG_CUDA(cudaMemcpyAsync(m->d_pos, h, sizeof(int), cudaMemcpyHostToDevice, m->s));
    CPG_CUDA(cudaStreamSynchronize(m->s));
    return CPG_OK;
}

extern "C" int cpg_qwen3_step(cpg_qwen3 *m, int id, int *next_id) {
    CPG_REQUIRE(m && id >= 0 && id < m->V, "cpg_qwen3_step: bad argument");
    *m->h_next = id;
    CPG_CUDA(cudaMemcpyAsync(m->d_ids, m->h_next, sizeof(int), cudaMemcpyHostToDevice, m->s));
    const int rc = qwen3_step_device(m, nullptr, 0);
    if (rc) return rc;
    return qwen3_read_next(m, next_id);
}

extern "C" int cpg_qwen3_generate(cpg_qwen3 *m, const int *prompt, int n_prompt, int n_new, int *out_ids) {
    CPG_REQUIRE(m && prompt && out_ids && n_new >= 0, "cpg_qwen3_generate: bad argument");
    int next = 0;
    int rc = cpg_qwen3_prefill(m, prompt, n_prompt, &next);
    if (rc) return rc;
    out_ids[0] = next;
    // the argmax stays on the device: each step embeds the previous one and records it at
    // d_out[position - prompt]; the ids come back once at the end
    for (int i = 1; i <= n_new; ++i) {
        rc = qwen3_step_device(m, m->d_out, n_prompt);
        if (rc) return rc;
    }
    if (n_new > 0) {
        CPG_CUDA(cudaMemcpyAsync(out_ids + 1, m->d_out + 1, sizeof(int) * (size_t)n_new, cudaMemcpyDeviceToHost, m->s));
        CPG_CUDA(cudaStreamSynchronize(m->s));
    }
    return CPG_OK;
}

extern "C" const float *cpg_qwen3_logits(const cpg_qwen3 *m) { return m ? m->logits : nullptr; }
extern "C" void *cpg_qwen3_stream(const cpg_qwen3 *m) { return m ? (void *)m->s : nullptr; }
extern "C" int cpg_qwen3_position(const cpg_qwen3 *m) { return m ? m->pos : -1; }

// ---------------------------------------------------------------------------------------------
// Several sequences at once (continuous batching). The reference engine decodes one sequence
// (engine/api/cachepotato.h:12-16); here n_slots sequences share the model's weights, each with
// its own KV cache and position, and a step embeds one new token per named slot and runs them
// through every layer as one batch: the projections and the MoE block see T = n tokens (the
// batched expert kernel reads each routed expert once for all of them), the attention of token t
// reads only its own slot's cache. Per sequence this is the greedy loop of cp_chat
// (cachepotato.c:315-378). Everything runs on the model's stream and scratch rows, so a batch
// and the model's own sequence never run at the same time.
struct cpg_qwen3_batch {
    cpg_qwen3 *m = nullptr;
    int S = 0, C = 0;
    float *kv = nullptr;                 // L × 2 × S × C × KD
    int *slot_pos = nullptr;             // (S) device positions
    std::vector<int> pos;                // host copies
    int *tok_slot = nullptr, *tok_pos = nullptr, *d_next = nullptr, *d_step = nullptr;
    int *d_out = nullptr;                // (C, S) ids of a generate call, step-major
    int *h_buf = nullptr;                // pinned staging: 2S ints
    float *logits = nullptr, *am_v = nullptr, *as_part = nullptr;
    int *am_i = nullptr, *as_cnt = nullptr;
    int last_rows = 0;
    std::vector<cudaGraphExec_t> graphs; // one step of n sequences, by n
};

static void batch_free(cpg_qwen3_batch *b) {
    for (cudaGraphExec_t g : b->graphs)
        if (g) cudaGraphExecDestroy(g);
    cudaFree(b->kv); cudaFree(b->slot_pos); cudaFree(b->tok_slot); cudaFree(b->tok_pos);
    cudaFree(b->d_next); cudaFree(b->d_step); cudaFree(b->d_out); cudaFree(b->logits); cudaFree(b->am_v);
    cudaFree(b->am_i); cudaFree(b->as_part); cudaFree(b->as_cnt);
    if (b->h_buf) cudaFreeHost(b->h_buf);
    delete b;
}

extern "C" int cpg_qwen3_batch_create(cpg_qwen3 *m, int n_slots, int max_ctx, cpg_qwen3_batch **out) {
    CPG_REQUIRE(m && out, "cpg_qwen3_batch_create: null argument");
    *out = nullptr;
    CPG_REQUIRE(n_slots >= 1 && n_slots <= m->max_ctx,
                "cpg_qwen3_batch_create: n_slots %d (1..the model's max_ctx %d)", n_slots, m->max_ctx);
    CPG_REQUIRE(max_ctx >= 1 && max_ctx <= m->max_ctx,
                "cpg_qwen3_batch_create: max_ctx %d (1..the model's max_ctx %d)", max_ctx, m->max_ctx);
    cpg_qwen3_batch *b = new cpg_qwen3_batch();
    b->m = m;
    b->S = n_slots;
    b->C = max_ctx;
    b->pos.assign(n_slots, -1);
    b->graphs.assign(n_slots + 1, nullptr);
    const size_t S = n_slots, C = max_ctx, KD = (size_t)m->KV * QW_HD;
    cudaError_t ce = cudaMalloc(&b->kv, (size_t)m->L * 2 * S * C * KD * sizeof(float));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->slot_pos, S * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->tok_slot, S * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->tok_pos, S * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->d_next, S * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->d_step, sizeof(int));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->d_out, C * S * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMallocHost(&b->h_buf, 2 * S * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->logits, S * (size_t)m->V * sizeof(float));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->am_v, S * AM_BLOCKS * sizeof(float));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->am_i, S * AM_BLOCKS * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->as_part, S * m->H * AS_SPLIT * (QW_HD + 2) * sizeof(float));
    if (ce == cudaSuccess) ce = cudaMalloc(&b->as_cnt, S * m->H * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMemsetAsync(b->as_cnt, 0, S * m->H * sizeof(int), m->s);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(b->slot_pos, 0, S * sizeof(int), m->s);
    if (ce == cudaSuccess)
        ce = cudaFuncSetAttribute(k_attention_group, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)attention_group_smem());
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(m->s);
    if (ce != cudaSuccess) {
        batch_free(b);
        return cuda_fail(ce, "cpg_qwen3_batch_create: allocation");
    }
    if (n_slots >= QW_DENSE_DEC_MIN_T && m->dn.attn.empty()) {
        const int rc = build_dense(m);
        if (rc) {
            batch_free(b);
            return rc;
        }
    }
    *out = b;
    return CPG_OK;
}

extern "C" void cpg_qwen3_batch_destroy(cpg_qwen3_batch *b) {
    if (b) {
        if (b->m) cudaStreamSynchronize(b->m->s);
        batch_free(b);
    }
}

extern "C" int cpg_qwen3_batch_prefill(cpg_qwen3_batch *b, int slot, const int *ids, int n, int *next_id) {
    CPG_REQUIRE(b && ids && n > 0, "cpg_qwen3_batch_prefill: bad argument");
    cpg_qwen3 *m = b->m;
    CPG_REQUIRE(slot >= 0 && slot < b->S, "cpg_qwen3_batch_prefill: slot %d of %d", slot, b->S);
    CPG_REQUIRE(n < b->C, "cpg_qwen3_batch_prefill: %d tokens leave no room in max_ctx %d", n, b->C);
    for (int t = 0; t < n; ++t)
        CPG_REQUIRE(ids[t] >= 0 && ids[t] < m->V, "cpg_qwen3_batch_prefill: id %d out of range", ids[t]);
    CPG_CUDA(cudaMemsetAsync(b->slot_pos + slot, 0, sizeof(int), m->s));
    CPG_CUDA(cudaMemcpyAsync(m->d_ids, ids, sizeof(int) * (size_t)n, cudaMemcpyHostToDevice, m->s));
    const QwSeq sq{b->kv, b->S, b->C, b->slot_pos + slot, slot, nullptr, nullptr, n, m->as_part, m->as_cnt,
                   b->logits, b->am_v, b->am_i, b->d_next, m->dn.attn.empty() ? nullptr : &m->dn};
    int rc = qwen3_enqueue(m, sq, n, m->s);
    if (rc) return rc;
    b->h_buf[0] = n;
    CPG_CUDA(cudaMemcpyAsync(b->slot_pos + slot, b->h_buf, sizeof(int), cudaMemcpyHostToDevice, m->s));
    CPG_CUDA(cudaMemcpyAsync(b->h_buf + 1, b->d_next, sizeof(int), cudaMemcpyDeviceToHost, m->s));
    CPG_CUDA(cudaStreamSynchronize(m->s));
    b->pos[slot] = n;
    b->last_rows = 1;
    if (next_id) *next_id = b->h_buf[1];
    return qwen3_status(m, "cpg_qwen3_batch_prefill");
}

// The slots of a step: distinct, prefilled, room for n_steps more positions each.
static int batch_check(cpg_qwen3_batch *b, const int *slots, int n, int n_steps, const char *fn) {
    CPG_REQUIRE(slots && n >= 1 && n <= b->S, "%s: %d sequences (1..%d)", fn, n, b->S);
    std::vector<char> seen(b->S, 0);
    for (int t = 0; t < n; ++t) {
        const int j = slots[t];
        CPG_REQUIRE(j >= 0 && j < b->S, "%s: slot %d of %d", fn, j, b->S);
        CPG_REQUIRE(!seen[j], "%s: slot %d named twice", fn, j);
        seen[j] = 1;
        CPG_REQUIRE(b->pos[j] >= 1, "%s: slot %d holds no sequence (prefill it first)", fn, j);
        CPG_REQUIRE(b->pos[j] + n_steps <= b->C, "%s: slot %d at position %d: %d more steps pass max_ctx %d", fn, j,
                    b->pos[j], n_steps, b->C);
    }
    return CPG_OK;
}

// n_steps steps of the named slots from ids (host, one per slot); each step's argmax is the
// next step's input. The step of n sequences is captured once (positions live on the device).
static int batch_run(cpg_qwen3_batch *b, const int *slots, const int *ids, int n, int n_steps) {
    cpg_qwen3 *m = b->m;
    for (int t = 0; t < n; ++t) {
        b->h_buf[t] = slots[t];
        b->h_buf[n + t] = ids[t];
    }
    CPG_CUDA(cudaMemcpyAsync(b->tok_slot, b->h_buf, sizeof(int) * n, cudaMemcpyHostToDevice, m->s));
    CPG_CUDA(cudaMemcpyAsync(m->d_ids, b->h_buf + n, sizeof(int) * n, cudaMemcpyHostToDevice, m->s));
    CPG_CUDA(cudaMemsetAsync(b->d_step, 0, sizeof(int), m->s));
    if (!b->graphs[n]) {
        const QwSeq sq{b->kv, b->S, b->C, nullptr, -1, b->tok_slot, b->tok_pos, 0, b->as_part, b->as_cnt,
                       b->logits, b->am_v, b->am_i, b->d_next, m->dn.attn.empty() ? nullptr : &m->dn};
        cudaGraph_t g = nullptr;
        CPG_CUDA(cudaStreamBeginCapture(m->s, cudaStreamCaptureModeThreadLocal));
        int rc = 0;
        k_batch_begin<<<1, 256, 0, m->s>>>(b->tok_slot, b->slot_pos, b->tok_pos, n);
        cudaError_t le = cudaGetLastError();
        if (le != cudaSuccess) rc = cuda_fail(le, "cpg_qwen3_batch: step launch");
        if (!rc) rc = qwen3_enqueue(m, sq, n, m->s);
        if (!rc) {
            k_batch_advance<<<1, 256, 0, m->s>>>(b->d_next, m->d_ids, b->tok_slot, b->slot_pos, n, b->d_out, b->d_step);
            le = cudaGetLastError();
            if (le != cudaSuccess) rc = cuda_fail(le, "cpg_qwen3_batch: step launch");
        }
        const cudaError_t ce = cudaStreamEndCapture(m->s, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (ce != cudaSuccess) return cuda_fail(ce, "cpg_qwen3_batch: step capture");
        const cudaError_t ie = cudaGraphInstantiate(&b->graphs[n], g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) return cuda_fail(ie, "cpg_qwen3_batch: step instantiate");
    }
    for (int i = 0; i < n_steps; ++i) CPG_CUDA(cudaGraphLaunch(b->graphs[n], m->s));
    for (int t = 0; t < n; ++t) b->pos[slots[t]] += n_steps;
    b->last_rows = n;
    return CPG_OK;
}

extern "C" int cpg_qwen3_batch_step(cpg_qwen3_batch *b, const int *slots, const int *ids, int n, int *next_ids) {
    CPG_REQUIRE(b && ids && next_ids, "cpg_qwen3_batch_step: null argument");
    int rc = batch_check(b, slots, n, 1, "cpg_qwen3_batch_step");
    for (int t = 0; !rc && t < n; ++t)
        CPG_REQUIRE(ids[t] >= 0 && ids[t] < b->m->V, "cpg_qwen3_batch_step: id %d out of range", ids[t]);
    if (!rc) rc = batch_run(b, slots, ids, n, 1);
    if (rc) return rc;
    CPG_CUDA(cudaMemcpyAsync(next_ids, b->d_out, sizeof(int) * n, cudaMemcpyDeviceToHost, b->m->s));
    CPG_CUDA(cudaStreamSynchronize(b->m->s));
    return qwen3_status(b->m, "cpg_qwen3_batch_step");
}

extern "C" int cpg_qwen3_batch_generate(cpg_qwen3_batch *b, const int *slots, const int *ids, int n, int n_steps,
                                        int *out_ids) {
    CPG_REQUIRE(b && ids && out_ids && n_steps >= 1, "cpg_qwen3_batch_generate: bad argument");
    int rc = batch_check(b, slots, n, n_steps, "cpg_qwen3_batch_generate");
    for (int t = 0; !rc && t < n; ++t)
        CPG_REQUIRE(ids[t] >= 0 && ids[t] < b->m->V, "cpg_qwen3_batch_generate: id %d out of range", ids[t]);
    if (!rc) rc = batch_run(b, slots, ids, n, n_steps);
    if (rc) return rc;
    CPG_CUDA(cudaMemcpyAsync(out_ids, b->d_out, sizeof(int) * (size_t)n * n_steps, cudaMemcpyDeviceToHost, b->m->s));
    CPG_CUDA(cudaStreamSynchronize(b->m->s));
    return qwen3_status(b->m, "cpg_qwen3_batch_generate");
}

extern "C" int cpg_qwen3_batch_position(const cpg_qwen3_batch *b, int slot) {
    return b && slot >= 0 && slot < b->S ? b->pos[slot] : -1;
}

extern "C" const float *cpg_qwen3_batch_logits(const cpg_qwen3_batch *b, int *rows) {
    if (rows) *rows = b ? b->last_rows : 0;
    return b ? b->logits : nullptr;
}
