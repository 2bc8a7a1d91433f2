/* cpg_oracle.c — CPU restatement of the CachePotato Qwen3-MoE expert path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels, never the product. See
 * cpg_oracle.h for who may call it and what pins it. Compiled with -ffp-contract=off so that,
 * like the reference's ISO C11 build (Makefile:2, -std=c11), no multiply-add is fused.
 */
#define _POSIX_C_SOURCE 200809L
#include "cpg_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* fp16 bits -> f32, subnormals renormalised, inf/NaN preserved: engine/kernels/kernels.c:109-130 */
float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            /* value = m * 2^-24: normalise so the leading one becomes implicit */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            bits = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float r;
    memcpy(&r, &bits, sizeof r);
    return r;
}

/* f32 -> fp16 bits, round to nearest even (numpy's astype(np.float16) rule). */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    uint32_t a = x & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);       /* NaN */
    if (a >= 0x47800000u) return (uint16_t)(sign | 0x7C00u);      /* >= 2^16 (or inf) */
    if (a >= 0x38800000u) {                                        /* normal half: >= 2^-14 */
        uint32_t mant = a & 0x7FFFFFu;
        uint32_t h = (((a >> 23) - 112u) << 10) | (mant >> 13);
        uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;    /* carry may reach inf */
        return (uint16_t)(sign | h);
    }
    if (a < 0x33000000u) return sign;                              /* below 2^-25 */
    uint32_t ex = a >> 23;                                         /* 102..112 */
    uint32_t mant = (a & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126u - ex;                                    /* 14..24 */
    uint32_t h = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

static float group_scale(const uint8_t *blk) {
    return orc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
}

/* engine/kernels/kernels.c:143-151 */
void orc_q8_dequant_row(const uint8_t *blocks, float *out, long n) {
    for (long g = 0; g < n / 32; g++) {
        const uint8_t *blk = blocks + g * 34;
        float d = group_scale(blk);
        for (int i = 0; i < 32; i++) out[g * 32 + i] = (float)(int8_t)blk[2 + i] * d;
    }
}

static int nib(int v) { return v > 7 ? v - 16 : v; }

/* engine/kernels/kernels.c:463-477: byte k holds element k (low nibble) and k+16 (high) */
void orc_q4_dequant_row(const uint8_t *blocks, float *out, long n) {
    for (long g = 0; g < n / 32; g++) {
        const uint8_t *blk = blocks + g * 18;
        float d = group_scale(blk);
        for (int k = 0; k < 16; k++) {
            out[g * 32 + k] = (float)nib(blk[2 + k] & 0x0F) * d;
            out[g * 32 + k + 16] = (float)nib(blk[2 + k] >> 4) * d;
        }
    }
}

/* ---------------------------------------------------------------- encoders */

static float group_amax(const float *x) {
    float a = 0.0f;
    for (int i = 0; i < 32; i++) {
        float v = fabsf(x[i]);
        if (v > a) a = v;
    }
    return a;
}

/* format/q8.py:35-58: d = amax/127 in f32, stored as fp16 (RNE); q = clip(rint(x/d), ±127). */
static void q8_encode_groups(const float *x, long g0, long g1, uint8_t *out) {
    for (long g = g0; g < g1; g++) {
        const float *v = x + g * 32;
        uint8_t *blk = out + g * 34;
        float amax = group_amax(v);
        float d = amax > 0.0f ? amax / 127.0f : 0.0f;
        uint16_t dh = orc_f32_to_f16(d);
        float dq = orc_f16_to_f32(dh);
        blk[0] = (uint8_t)(dh & 0xFF);
        blk[1] = (uint8_t)(dh >> 8);
        for (int i = 0; i < 32; i++) {
            int q = 0;
            if (dq > 0.0f) {
                float r = rintf(v[i] / dq);
                q = r < -127.0f ? -127 : r > 127.0f ? 127 : (int)r;
            }
            blk[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

/* format/q4.py:30-57: d = amax/8 stored as fp16 (RNE) first; q = clip(rint(x/d), -8, 7);
   byte k = (q[k] & 0xF) | (q[k+16] & 0xF) << 4. */
static void q4_encode_groups(const float *x, long g0, long g1, uint8_t *out) {
    for (long g = g0; g < g1; g++) {
        const float *v = x + g * 32;
        uint8_t *blk = out + g * 18;
        float amax = group_amax(v);
        /* amax/8 is exact in f32 and f64 alike, so the f64 detour of q4.py:42-44 changes nothing */
        uint16_t dh = orc_f32_to_f16(amax > 0.0f ? amax / 8.0f : 0.0f);
        float dq = orc_f16_to_f32(dh);
        int q[32];
        for (int i = 0; i < 32; i++) {
            q[i] = 0;
            if (dq > 0.0f) {
                float r = rintf(v[i] / dq);
                q[i] = r < -8.0f ? -8 : r > 7.0f ? 7 : (int)r;
            }
        }
        blk[0] = (uint8_t)(dh & 0xFF);
        blk[1] = (uint8_t)(dh >> 8);
        for (int k = 0; k < 16; k++)
            blk[2 + k] = (uint8_t)((q[k] & 0xF) | ((q[k + 16] & 0xF) << 4));
    }
}

typedef struct {
    void (*fn)(const float *, long, long, uint8_t *);
    const float *x;
    long g0, g1;
    uint8_t *out;
} EncJob;

static void *enc_thread(void *p) {
    EncJob *j = p;
    j->fn(j->x, j->g0, j->g1, j->out);
    return NULL;
}

static void encode_parallel(void (*fn)(const float *, long, long, uint8_t *),
                            const float *x, long n, uint8_t *out, int nthreads) {
    long ng = n / 32;
    if (nthreads <= 1 || ng < 4096) { fn(x, 0, ng, out); return; }
    if (nthreads > 256) nthreads = 256;
    pthread_t tid[256];
    EncJob job[256];
    int joined[256];
    long chunk = (ng + nthreads - 1) / nthreads;
    for (int t = 0; t < nthreads; t++) {
        long g0 = t * chunk, g1 = g0 + chunk < ng ? g0 + chunk : ng;
        joined[t] = 0;
        if (g0 >= g1) continue;
        job[t] = (EncJob){fn, x, g0, g1, out};
        if (pthread_create(&tid[t], NULL, enc_thread, &job[t]) == 0) joined[t] = 1;
        else fn(x, g0, g1, out);                 /* no thread: do the slice here */
    }
    for (int t = 0; t < nthreads; t++)
        if (joined[t]) pthread_join(tid[t], NULL);
}

void orc_quantize_q8_0(const float *x, long n, uint8_t *out, int nthreads) {
    encode_parallel(q8_encode_groups, x, n, out, nthreads);
}

void orc_quantize_q4_0(const float *x, long n, uint8_t *out, int nthreads) {
    encode_parallel(q4_encode_groups, x, n, out, nthreads);
}

/* ---------------------------------------------------------------- matvec */

/* engine/kernels/kernels.c:90-94 (serial path; the threaded path splits rows, same order) */
void orc_matmul_wx(float *out, const float *x, const float *w, int n_in, int n_out) {
    for (int i = 0; i < n_out; i++) {
        float acc = 0.0f;
        for (int k = 0; k < n_in; k++) acc += w[(size_t)i * n_in + k] * x[k];
        out[i] = acc;
    }
}

/* engine/kernels/kernels.c:386-395 (scalar Q8_0 row loop) */
void orc_matmul_wx_q8(float *out, const float *x, const uint8_t *w, int n_in, int n_out) {
    const int ng = n_in / 32;
    for (int i = 0; i < n_out; i++) {
        const uint8_t *row = w + (size_t)i * ng * 34;
        float acc = 0.0f;
        for (int g = 0; g < ng; g++) {
            float d = group_scale(row + (size_t)g * 34);
            const int8_t *q = (const int8_t *)(row + (size_t)g * 34 + 2);
            for (int j = 0; j < 32; j++) acc += ((float)q[j] * d) * x[g * 32 + j];
        }
        out[i] = acc;
    }
}

/* engine/kernels/kernels.c:524-539 (scalar Q4_0 row loop) */
void orc_matmul_wx_q4(float *out, const float *x, const uint8_t *w, int n_in, int n_out) {
    const int ng = n_in / 32;
    for (int i = 0; i < n_out; i++) {
        const uint8_t *row = w + (size_t)i * ng * 18;
        float acc = 0.0f;
        for (int g = 0; g < ng; g++) {
            float d = group_scale(row + (size_t)g * 18);
            const uint8_t *q = row + (size_t)g * 18 + 2;
            for (int k = 0; k < 16; k++) {
                acc += ((float)nib(q[k] & 0x0F) * d) * x[g * 32 + k];
                acc += ((float)nib(q[k] >> 4) * d) * x[g * 32 + k + 16];
            }
        }
        out[i] = acc;
    }
}

/* engine/blocks/qwen3_moe.c:36-40 */
void orc_mm(const void *w, int enc, float *out, const float *x, int n_in, int n_out) {
    if (enc == ORC_ENC_Q4) orc_matmul_wx_q4(out, x, (const uint8_t *)w, n_in, n_out);
    else if (enc == ORC_ENC_Q8) orc_matmul_wx_q8(out, x, (const uint8_t *)w, n_in, n_out);
    else orc_matmul_wx(out, x, (const float *)w, n_in, n_out);
}

/* ---------------------------------------------------------------- elementwise */

/* engine/kernels/kernels.c:408-413 */
void orc_rmsnorm(float *out, const float *x, const float *g, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * inv * g[i];
}

/* engine/kernels/kernels.c:20-26 */
void orc_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; i++) { x[i] = expf(x[i] - mx); sum += x[i]; }
    for (int i = 0; i < n; i++) x[i] /= sum;
}

/* engine/kernels/kernels.c:416 */
float orc_silu(float x) { return x / (1.0f + expf(-x)); }

/* ---------------------------------------------------------------- router + experts */

/* engine/blocks/qwen3_moe.c:180-197 */
void orc_route(const void *wgate, int wgate_enc, const float *xn, int d_model, int n_experts,
               int topk, float *logits, float *probs, int *idx, float *wt) {
    orc_mm(wgate, wgate_enc, logits, xn, d_model, n_experts);
    memcpy(probs, logits, sizeof(float) * (size_t)n_experts);
    orc_softmax(probs, n_experts);
    for (int j = 0; j < topk; j++) {          /* strict '>', lower id wins ties (184-194) */
        int best = -1;
        for (int e = 0; e < n_experts; e++) {
            int taken = 0;
            for (int p = 0; p < j; p++) if (idx[p] == e) { taken = 1; break; }
            if (taken) continue;
            if (best < 0 || probs[e] > probs[best]) best = e;
        }
        idx[j] = best;
    }
    float sum = 0.0f;                         /* norm_topk_prob (195-197) */
    for (int j = 0; j < topk; j++) sum += probs[idx[j]];
    for (int j = 0; j < topk; j++) wt[j] = probs[idx[j]] / sum;
}

static void expert_swiglu(const void *const *exp, int enc, int e, int d_model, int d_exp,
                          const float *xn, float *gu, float *hh, float *y) {
    /* engine/blocks/qwen3_moe.c:217-220 */
    orc_mm(exp[(size_t)e * 3 + 0], enc, gu, xn, d_model, d_exp);
    orc_mm(exp[(size_t)e * 3 + 1], enc, hh, xn, d_model, d_exp);
    for (int i = 0; i < d_exp; i++) gu[i] = orc_silu(gu[i]) * hh[i];
    orc_mm(exp[(size_t)e * 3 + 2], enc, y, gu, d_exp, d_model);
}

int orc_qwen3_moe(const float *ln2, const void *wgate, int wgate_enc,
                  const void *const *exp, int exp_enc,
                  int d_model, int d_exp, int n_experts, int topk, float eps,
                  const float *x, const float *attn, int T,
                  float *mlp, float *router, int *topk_idx, float *wt, float *xn_out) {
    const int D = d_model, F = d_exp, E = n_experts, K = topk;
    int mx = F > D ? F : D;
    float *hh = malloc(sizeof(float) * (size_t)mx);
    float *gu = malloc(sizeof(float) * (size_t)mx);
    float *y = malloc(sizeof(float) * (size_t)D);
    float *xn = malloc(sizeof(float) * (size_t)D);
    float *logits = malloc(sizeof(float) * (size_t)E);
    float *probs = malloc(sizeof(float) * (size_t)E);
    int *idx = malloc(sizeof(int) * (size_t)K);
    float *w = malloc(sizeof(float) * (size_t)K);
    int rc = 0;
    if (!hh || !gu || !y || !xn || !logits || !probs || !idx || !w) { rc = -1; goto done; }
    for (int t = 0; t < T; t++) {
        /* qwen3_moe.c:178-179 */
        for (int j = 0; j < D; j++)
            hh[j] = x[(size_t)t * D + j] + (attn ? attn[(size_t)t * D + j] : 0.0f);
        orc_rmsnorm(xn, hh, ln2, D, eps);
        if (xn_out) memcpy(xn_out + (size_t)t * D, xn, sizeof(float) * (size_t)D);
        orc_route(wgate, wgate_enc, xn, D, E, K, logits, probs, idx, w);
        if (router) memcpy(router + (size_t)t * E, logits, sizeof(float) * (size_t)E);
        for (int j = 0; j < K; j++) {
            if (topk_idx) topk_idx[(size_t)t * K + j] = idx[j];
            if (wt) wt[(size_t)t * K + j] = w[j];
            expert_swiglu(exp, exp_enc, idx[j], D, F, xn, gu, hh, y);
            for (int i = 0; i < D; i++) mlp[(size_t)t * D + i] += w[j] * y[i];   /* 221 */
        }
    }
done:
    free(hh); free(gu); free(y); free(xn); free(logits); free(probs); free(idx); free(w);
    return rc;
}

int orc_moe_apply(const void *const *exp, int exp_enc, int d_model, int d_exp,
                  const float *xn, int T, int topk, const int *idx, const float *wt,
                  float *mlp) {
    const int D = d_model, F = d_exp;
    int mx = F > D ? F : D;
    float *hh = malloc(sizeof(float) * (size_t)mx);
    float *gu = malloc(sizeof(float) * (size_t)mx);
    float *y = malloc(sizeof(float) * (size_t)D);
    if (!hh || !gu || !y) { free(hh); free(gu); free(y); return -1; }
    for (int t = 0; t < T; t++) {
        for (int j = 0; j < topk; j++) {
            expert_swiglu(exp, exp_enc, idx[(size_t)t * topk + j], D, F, xn + (size_t)t * D,
                          gu, hh, y);
            float w = wt[(size_t)t * topk + j];
            for (int i = 0; i < D; i++) mlp[(size_t)t * D + i] += w * y[i];
        }
    }
    free(hh); free(gu); free(y);
    return 0;
}

/* ---------------------------------------------------------------- synthetic data */

static uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

typedef struct { float *out; long i0, i1; uint64_t seed; float std; } FillJob;

static void fill_range(float *out, long i0, long i1, uint64_t seed, float std) {
    /* pair p = (2p, 2p+1) is one Box-Muller draw keyed by p; i0 is even except at n's end */
    for (long i = i0 & ~1L; i < i1; i += 2) {
        uint64_t r = splitmix64(seed * 0xD1B54A32D192ED03ull + (uint64_t)(i >> 1));
        float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);             /* (0,1) */
        float u2 = (float)(r & 0xFFFFFFull) * (1.0f / 16777216.0f);             /* [0,1) */
        float rad = sqrtf(-2.0f * logf(u1)) * std;
        float s, c;
        s = sinf(6.28318530718f * u2);
        c = cosf(6.28318530718f * u2);
        if (i >= i0) out[i] = rad * c;
        if (i + 1 < i1) out[i + 1] = rad * s;
    }
}

static void *fill_thread(void *p) {
    FillJob *j = p;
    fill_range(j->out, j->i0, j->i1, j->seed, j->std);
    return NULL;
}

void orc_fill_normal(float *out, long n, uint64_t seed, float std, int nthreads) {
    if (nthreads <= 1 || n < (1L << 16)) { fill_range(out, 0, n, seed, std); return; }
    if (nthreads > 256) nthreads = 256;
    pthread_t tid[256];
    FillJob job[256];
    int joined[256];
    long chunk = ((n + nthreads - 1) / nthreads + 1) & ~1L;
    for (int t = 0; t < nthreads; t++) {
        long i0 = t * chunk, i1 = i0 + chunk < n ? i0 + chunk : n;
        joined[t] = 0;
        if (i0 >= i1) continue;
        job[t] = (FillJob){out, i0, i1, seed, std};
        if (pthread_create(&tid[t], NULL, fill_thread, &job[t]) == 0) joined[t] = 1;
        else fill_range(out, i0, i1, seed, std);
    }
    for (int t = 0; t < nthreads; t++)
        if (joined[t]) pthread_join(tid[t], NULL);
}
