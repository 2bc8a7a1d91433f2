// qwen3.cu — the whole Qwen3-MoE model on the device (SURVEY config 3): the attention half of
// qwen3_layer_kv (engine/blocks/qwen3_moe.c:110-167), the MoE half through cpg_moe_forward, and the
// model loop of cp_chat (engine/api/cachepotato.c:108-166, 315-378): embed_rows, run_layers,
// apply_head, greedy argmax.
//
// Per layer, for T new tokens at positions pos0..pos0+T-1:
//   k_rmsnorm       xn = RMSNorm(x, ln1)                                   kernels.c:408-413
//   cpg_matvec ×3   q = Wq·xn, k = Wk·xn, v = Wv·xn (k, v straight into the f32 KV cache)
//   k_qk_norm_rope  per-head RMSNorm of q and k (head_rmsnorm, qwen3_moe.c:44-49), then RoPE at
//                   each token's position (rope_apply_from, kernels.c:425-447)
//   k_attention     causal GQA: s = q·k / sqrt(hd), softmax, Σ s·v (qwen3_moe.c:135-155)
//   cpg_matvec      attn = Wo·ao
//   cpg_moe_forward RMSNorm(x + attn, ln2) → router → experts → x += attn + mlp (fused residual)
// Head: RMSNorm of the last position with final_norm, lm_head GEMV, k_argmax (first maximum wins).
// Head dimension 128 (one warp per head, four values per lane).
#include <math.h>

#include <vector>

#include "common.cuh"

namespace cpg {

constexpr int QW_HD = 128;

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
    __shared__ float s_red[8];
    const float *xr = x + (size_t)blockIdx.x * D;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < D; k += blockDim.x) ss = fmaf(xr[k], xr[k], ss);
    ss = block_sum(ss, s_red);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(ss, (float)D) + eps));
    float *o = out + (size_t)blockIdx.x * D;
    for (int k = threadIdx.x; k < D; k += blockDim.x) o[k] = __fmul_rn(__fmul_rn(xr[k], inv), g[k]);
}

// One warp per (token, head) of q (heads 0..H-1) and k (heads H..H+KV-1): head RMSNorm, then
// RoPE at position pos0 + t. Lane l holds elements l, l+32 (first half) and l+64, l+96 (their
// rotation partners). Products and sums are rounded one at a time, as the reference's ISO C.
__global__ void __launch_bounds__(256) k_qk_norm_rope(float *__restrict__ q, float *__restrict__ kc, int T, int pos0,
                                                       int H, int KV, const float *__restrict__ qn,
                                                       const float *__restrict__ kn, float theta, float eps) {
    const int lane = threadIdx.x & 31;
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nh = H + KV;
    if (w >= T * nh) return;
    const int t = w / nh, h = w - t * nh;
    const bool isq = h < H;
    float *v = isq ? q + ((size_t)t * H + h) * QW_HD : kc + ((size_t)(pos0 + t) * KV + (h - H)) * QW_HD;
    const float *g = isq ? qn : kn;
    float e[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = v[lane + 32 * i];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) ss = fmaf(e[i], e[i], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(ss, (float)QW_HD) + eps));
#pragma unroll
    for (int i = 0; i < 4; ++i) e[i] = __fmul_rn(__fmul_rn(e[i], inv), g[lane + 32 * i]);
    const float pos = (float)(pos0 + t);
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
    for (int i = 0; i < 4; ++i) v[lane + 32 * i] = e[i];
}

// Causal GQA attention (qwen3_moe.c:135-155), one block per (query token i, head h): scores over
// the n = pos0 + i + 1 cached positions, softmax (max, expf, sum, divide), then each thread one
// output element with the weighted sum over positions in order.
__global__ void __launch_bounds__(QW_HD) k_attention(const float *__restrict__ q, const float *__restrict__ kc,
                                                      const float *__restrict__ vc, int pos0, int H, int KV,
                                                      float *__restrict__ ao) {
    extern __shared__ float sc[];                        // (n) scores
    __shared__ float s_red[4];
    __shared__ float s_q[QW_HD];
    const int h = blockIdx.x, i = blockIdx.y;
    const int kh = h / (H / KV);
    const int n = pos0 + i + 1;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    s_q[threadIdx.x] = q[((size_t)i * H + h) * QW_HD + threadIdx.x];
    __syncthreads();
    const float scale = __fsqrt_rn((float)QW_HD);
    for (int j = warp; j < n; j += 4) {
        const float *kj = kc + ((size_t)j * KV + kh) * QW_HD;
        float s = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; ++e) s = fmaf(s_q[lane + 32 * e], kj[lane + 32 * e], s);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sc[j] = __fdiv_rn(s, scale);
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < n; j += blockDim.x) mx = fmaxf(mx, sc[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
    __syncthreads();
    float sum = 0.0f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const float ex = expf(__fsub_rn(sc[j], mx));
        sc[j] = ex;
        sum += ex;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) s_red[warp] = sum;
    __syncthreads();
    sum = (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]);
    for (int j = threadIdx.x; j < n; j += blockDim.x) sc[j] = __fdiv_rn(sc[j], sum);
    __syncthreads();
    float acc = 0.0f;
    const float *vp = vc + (size_t)kh * QW_HD + threadIdx.x;
    for (int j = 0; j < n; ++j) acc = __fadd_rn(acc, __fmul_rn(sc[j], vp[(size_t)j * KV * QW_HD]));
    ao[((size_t)i * H + h) * QW_HD + threadIdx.x] = acc;
}

// argmax with the first maximum winning (cachepotato.c:353-356): one block, NaN-free logits.
__global__ void __launch_bounds__(1024) k_argmax(const float *__restrict__ v, int n, int *out) {
    __shared__ float s_v[32];
    __shared__ int s_i[32];
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const float x = v[j];
        if (x > best) { best = x; bi = j; }                 // j ascends: ties keep the first
    }
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
        *out = bi;
    }
}

int matvec_launch(float *out, const float *x, cpg_tensor w, int n_in, int n_out, int T, cudaStream_t s);
int layer_dims(const cpg_moe_layer *L, int *D, int *F, int *E, int *K);

}  // namespace cpg

struct cpg_qwen3 {
    int D, H, KV, V, L, max_ctx;
    float theta, eps;
    cpg_tensor embed, lm_head;
    const float *final_norm;
    std::vector<cpg_qwen3_attn> attn;
    std::vector<const cpg_moe_layer *> moe;
    float *x = nullptr, *xn = nullptr, *q = nullptr, *ao = nullptr, *at = nullptr, *kv = nullptr, *logits = nullptr;
    int *d_ids = nullptr, *d_next = nullptr, *h_next = nullptr;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    int pos = 0;
    cudaStream_t s = nullptr;
};

using namespace cpg;

static void qwen3_free(cpg_qwen3 *m) {
    cudaFree(m->x); cudaFree(m->xn); cudaFree(m->q); cudaFree(m->ao); cudaFree(m->at); cudaFree(m->kv);
    cudaFree(m->logits); cudaFree(m->d_ids); cudaFree(m->d_next); cudaFree(m->ws);
    if (m->h_next) cudaFreeHost(m->h_next);
    if (m->s) cudaStreamDestroy(m->s);
    delete m;
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
    if (ce == cudaSuccess) ce = cudaMallocHost(&m->h_next, 4);
    if (ce == cudaSuccess) ce = cudaMalloc(&m->ws, m->ws_bytes);
    if (ce != cudaSuccess) {
        qwen3_free(m);
        return cuda_fail(ce, "cpg_qwen3_create: allocation");
    }
    *out = m;
    return CPG_OK;
}

extern "C" void cpg_qwen3_destroy(cpg_qwen3 *m) {
    if (m) qwen3_free(m);
}

// T tokens (ids already in m->d_ids[0..T)) at positions m->pos.. through embed, the layers and the
// head; the argmax lands in m->d_next.
static int qwen3_forward(cpg_qwen3 *m, int T) {
    CPG_REQUIRE(T > 0 && m->pos + T <= m->max_ctx, "cpg_qwen3: %d tokens at position %d exceed max_ctx %d", T, m->pos,
                m->max_ctx);
    cudaStream_t s = m->s;
    const int D = m->D, H = m->H, KV = m->KV, QD = H * QW_HD, KD = KV * QW_HD;
    const size_t C = (size_t)m->max_ctx;
    k_embed<<<T, 256, 0, s>>>((const uint8_t *)m->embed.p, m->embed.enc, m->d_ids, D, m->x);
    CPG_CUDA(cudaGetLastError());
    for (int l = 0; l < m->L; ++l) {
        const cpg_qwen3_attn &A = m->attn[l];
        float *kc = m->kv + (size_t)l * 2 * C * KD, *vc = kc + C * KD;
        k_rmsnorm<<<T, 256, 0, s>>>(m->x, A.ln1, D, m->eps, m->xn);
        CPG_CUDA(cudaGetLastError());
        int rc = matvec_launch(m->q, m->xn, A.wq, D, QD, T, s);
        if (!rc) rc = matvec_launch(kc + (size_t)m->pos * KD, m->xn, A.wk, D, KD, T, s);
        if (!rc) rc = matvec_launch(vc + (size_t)m->pos * KD, m->xn, A.wv, D, KD, T, s);
        if (rc) return rc;
        const int warps = T * (H + KV);
        k_qk_norm_rope<<<(warps + 7) / 8, 256, 0, s>>>(m->q, kc, T, m->pos, H, KV, A.q_norm, A.k_norm, m->theta,
                                                       m->eps);
        CPG_CUDA(cudaGetLastError());
        const size_t asmem = (size_t)(m->pos + T) * sizeof(float);
        CPG_REQUIRE(asmem <= 160 * 1024, "cpg_qwen3: context %d too long for the attention kernel", m->pos + T);
        if (asmem > 48 * 1024)
            CPG_CUDA(cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)asmem));
        k_attention<<<dim3(H, T), QW_HD, asmem, s>>>(m->q, kc, vc, m->pos, H, KV, m->ao);
        CPG_CUDA(cudaGetLastError());
        rc = matvec_launch(m->at, m->ao, A.wo, QD, D, T, s);
        if (rc) return rc;
        rc = cpg_moe_forward(m->moe[l], m->x, m->at, T, nullptr, m->x, nullptr, nullptr, nullptr, m->ws, m->ws_bytes, s);
        if (rc) return rc;
    }
    float *xl = m->x + (size_t)(T - 1) * D;
    k_rmsnorm<<<1, 256, 0, s>>>(xl, m->final_norm, D, m->eps, m->xn);
    CPG_CUDA(cudaGetLastError());
    int rc = matvec_launch(m->logits, m->xn, m->lm_head, D, m->V, 1, s);
    if (rc) return rc;
    k_argmax<<<1, 1024, 0, s>>>(m->logits, m->V, m->d_next);
    CPG_CUDA(cudaGetLastError());
    m->pos += T;
    return CPG_OK;
}

static int qwen3_read_next(cpg_qwen3 *m, int *next_id) {
    CPG_CUDA(cudaMemcpyAsync(m->h_next, m->d_next, 4, cudaMemcpyDeviceToHost, m->s));
    CPG_CUDA(cudaStreamSynchronize(m->s));
    if (next_id) *next_id = *m->h_next;
    return CPG_OK;
}

extern "C" int cpg_qwen3_prefill(cpg_qwen3 *m, const int *ids, int T, int *next_id) {
    CPG_REQUIRE(m && ids && T > 0, "cpg_qwen3_prefill: bad argument");
    CPG_REQUIRE(T <= m->max_ctx, "cpg_qwen3_prefill: %d tokens > max_ctx %d", T, m->max_ctx);
    for (int t = 0; t < T; ++t) CPG_REQUIRE(ids[t] >= 0 && ids[t] < m->V, "cpg_qwen3_prefill: id %d out of range", ids[t]);
    m->pos = 0;
    CPG_CUDA(cudaMemcpyAsync(m->d_ids, ids, sizeof(int) * (size_t)T, cudaMemcpyHostToDevice, m->s));
    const int rc = qwen3_forward(m, T);
    if (rc) return rc;
    return qwen3_read_next(m, next_id);
}

extern "C" int cpg_qwen3_step(cpg_qwen3 *m, int id, int *next_id) {
    CPG_REQUIRE(m && id >= 0 && id < m->V, "cpg_qwen3_step: bad argument");
    CPG_CUDA(cudaMemcpyAsync(m->d_ids, &id, sizeof(int), cudaMemcpyHostToDevice, m->s));
    const int rc = qwen3_forward(m, 1);
    if (rc) return rc;
    return qwen3_read_next(m, next_id);
}

extern "C" int cpg_qwen3_generate(cpg_qwen3 *m, const int *prompt, int n_prompt, int n_new, int *out_ids) {
    CPG_REQUIRE(m && prompt && out_ids && n_new >= 0, "cpg_qwen3_generate: bad argument");
    int next = 0;
    int rc = cpg_qwen3_prefill(m, prompt, n_prompt, &next);
    if (rc) return rc;
    out_ids[0] = next;
    for (int i = 1; i <= n_new; ++i) {
        // the argmax stays on the device: the next step embeds it directly
        CPG_CUDA(cudaMemcpyAsync(m->d_ids, m->d_next, 4, cudaMemcpyDeviceToDevice, m->s));
        rc = qwen3_forward(m, 1);
        if (rc) return rc;
        rc = qwen3_read_next(m, &next);
        if (rc) return rc;
        out_ids[i] = next;
    }
    return CPG_OK;
}

extern "C" const float *cpg_qwen3_logits(const cpg_qwen3 *m) { return m ? m->logits : nullptr; }
extern "C" void *cpg_qwen3_stream(const cpg_qwen3 *m) { return m ? (void *)m->s : nullptr; }
extern "C" int cpg_qwen3_position(const cpg_qwen3 *m) { return m ? m->pos : -1; }
