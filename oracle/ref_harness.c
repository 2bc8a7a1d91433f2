/* ref_harness.c — drives the UNMODIFIED CachePotato engine (compiled from its own sources into
 * oracle/_ref/libcpref.so by oracle/Makefile) on in-memory synthetic layers.
 *
 * TEST INFRASTRUCTURE ONLY: the reference side of the parity tests and the CPU baseline the
 * benchmark times. This file is ours; the engine sources it links are the reference's, read in
 * place and never copied.
 *
 * refh_qwen3_moe builds a QW3Layer (engine/blocks/qwen3_moe.h:21-69) whose attention half is
 * all-zero f32 weights with one query and one KV head of width 2: q = k = v = 0 exactly, so the
 * attention output is exactly 0 and the layer's MoE half (qwen3_moe.c:170-223) sees hh = x.
 * It then calls the reference's qwen3_layer_kv as run_layers does (engine/api/cachepotato.c:149-166).
 */
#include "blocks/qwen3_moe.h"
#include "kernels/kernels.h"
#include "kernels/parallel.h"

#include <stdlib.h>
#include <string.h>

int refh_init_threads(int n) { return cp_threads_init(n, 0); }
int refh_threads(void) { return cp_threads(); }

#define REFH_HD 2

int refh_qwen3_moe(const float *ln2, const float *wgate, const void *const *exp, int exp_enc,
                   int D, int F, int E, int K, float eps,
                   const float *x, int T, float *mlp, float *router, int *topk_idx) {
    QW3Layer m;
    memset(&m, 0, sizeof m);
    m.d_model = D; m.n_heads = 1; m.n_kv = 1; m.head_dim = REFH_HD;
    m.d_exp = F; m.n_experts = E; m.topk = K; m.vocab = 0;
    m.rope_theta = 1000000.0f; m.rms_eps = eps;

    float *zeros = calloc((size_t)REFH_HD * D * 2 + 2 * REFH_HD, sizeof(float));
    float *ones = malloc(sizeof(float) * (size_t)D);
    QW3T *tab = calloc((size_t)E * 3, sizeof(QW3T));
    if (!zeros || !ones || !tab) { free(zeros); free(ones); free(tab); return -2; }
    for (int i = 0; i < D; i++) ones[i] = 1.0f;
    float *hd_ones = zeros + (size_t)REFH_HD * D * 2;
    hd_ones[0] = hd_ones[1] = hd_ones[2] = hd_ones[3] = 1.0f;

    m.ln1 = ones;
    m.ln2 = ln2;
    m.q_norm = hd_ones;
    m.k_norm = hd_ones + REFH_HD;
    m.Wq.p = zeros; m.Wk.p = zeros; m.Wv.p = zeros;          /* (2, D) each, all zero */
    m.Wo.p = zeros + (size_t)REFH_HD * D;                    /* (D, 2), all zero */
    m.Wq.enc = m.Wk.enc = m.Wv.enc = m.Wo.enc = QW3_ENC_F32;
    m.Wgate.p = wgate; m.Wgate.enc = QW3_ENC_F32;
    for (int i = 0; i < E * 3; i++) { tab[i].p = exp[i]; tab[i].enc = exp_enc; }
    m.exp = tab;

    QW3KV kv;
    QW3Out o;
    int rc = -2;
    if (qwen3_kv_alloc(&kv, &m, T) == 0) {
        if (qwen3_layer_alloc(&o, &m, T) == 0) {
            rc = qwen3_layer_kv(&m, x, T, 0, &kv, &o);
            if (rc == 0) {
                if (mlp) memcpy(mlp, o.mlp, sizeof(float) * (size_t)T * D);
                if (router) memcpy(router, o.router, sizeof(float) * (size_t)T * E);
                if (topk_idx) memcpy(topk_idx, o.topk_idx, sizeof(int) * (size_t)T * K);
            }
            qwen3_layer_free(&o);
        }
        qwen3_kv_free(&kv);
    }
    free(zeros); free(ones); free(tab);
    return rc;
}

/* Externally routed experts through the reference's own qwen3_mm and silu: the expert loop of
   qwen3_moe.c:199-222 with the routing decided by the caller (prefill / expert-parallel
   workloads draw their token->expert assignment directly). */
int refh_moe_apply(const void *const *exp, int exp_enc, int D, int F, const float *xn, int T,
                   int K, const int *idx, const float *wt, float *mlp) {
    int mx = F > D ? F : D;
    float *gu = malloc(sizeof(float) * (size_t)mx);
    float *hh = malloc(sizeof(float) * (size_t)mx);
    if (!gu || !hh) { free(gu); free(hh); return -2; }
    for (int t = 0; t < T; t++) {
        const float *xt = xn + (size_t)t * D;
        for (int j = 0; j < K; j++) {
            const int e = idx[(size_t)t * K + j];
            QW3T wg = { exp[(size_t)e * 3 + 0], exp_enc };
            QW3T wu = { exp[(size_t)e * 3 + 1], exp_enc };
            QW3T wd = { exp[(size_t)e * 3 + 2], exp_enc };
            qwen3_mm(&wg, gu, xt, D, F);
            qwen3_mm(&wu, hh, xt, D, F);
            for (int i = 0; i < F; i++) gu[i] = silu(gu[i]) * hh[i];
            qwen3_mm(&wd, hh, gu, F, D);
            const float w = wt[(size_t)t * K + j];
            for (int i = 0; i < D; i++) mlp[(size_t)t * D + i] += w * hh[i];
        }
    }
    free(gu); free(hh);
    return 0;
}

/* A whole model, prompt then greedy decode, with the engine's own functions in the order cp_chat
   uses them (engine/api/cachepotato.c:315-378): embed_rows (108-133: q8/q4_dequant_row of the
   token's row), run_layers (149-166: qwen3_layer_kv per layer, then x += attn + mlp), apply_head
   (135-147: rmsnorm of the last position, lm_head through qwen3_mm), argmax with the first
   maximum winning (353-356). The prompt runs in one pass at position 0; then n_new single-token
   steps, each feeding the previous argmax. out_ids receives n_new + 1 ids (the argmax after the
   prompt and after every step); out_logits the logits of the last step. Per-layer tensors come
   as arrays of L pointers; exp holds L * E * 3 expert pointers. */
static void refh_embed(const void *embed, int enc, int id, float *x, int D) {
    if (enc == QW3_ENC_Q8) q8_dequant_row((const uint8_t *)embed + (size_t)id * (size_t)(D / 32) * 34, x, D);
    else if (enc == QW3_ENC_Q4) q4_dequant_row((const uint8_t *)embed + (size_t)id * (size_t)(D / 32) * 18, x, D);
    else memcpy(x, (const float *)embed + (size_t)id * D, sizeof(float) * (size_t)D);
}

static int refh_argmax(const float *v, int n) {
    int best = 0;
    for (int j = 1; j < n; j++) if (v[j] > v[best]) best = j;
    return best;
}

int refh_qwen3_generate(int D, int H, int KV, int HD, int F, int E, int K, int V, int L, float theta, float eps,
                        const void *embed, int embed_enc, const void *lm_head, int head_enc, const float *final_norm,
                        const void *const *ln1, const void *const *ln2, const void *const *qn, const void *const *kn,
                        const void *const *wq, const void *const *wk, const void *const *wv, const void *const *wo,
                        int attn_enc, const void *const *wgate, const void *const *exp, int exp_enc,
                        const int *prompt, int n_prompt, int n_new, int *out_ids, float *out_logits) {
    const int cap = n_prompt + n_new;
    QW3Layer *ls = calloc((size_t)L, sizeof(QW3Layer));
    QW3KV *kv = calloc((size_t)L, sizeof(QW3KV));
    QW3T *tab = calloc((size_t)L * E * 3, sizeof(QW3T));
    float *x = malloc(sizeof(float) * (size_t)n_prompt * D);
    float *logits = malloc(sizeof(float) * (size_t)V);
    int rc = -2;
    if (!ls || !kv || !tab || !x || !logits) goto out;
    for (int l = 0; l < L; l++) {
        QW3Layer *m = &ls[l];
        m->d_model = D; m->n_heads = H; m->n_kv = KV; m->head_dim = HD;
        m->d_exp = F; m->n_experts = E; m->topk = K; m->vocab = V;
        m->rope_theta = theta; m->rms_eps = eps;
        m->ln1 = ln1[l]; m->ln2 = ln2[l]; m->q_norm = qn[l]; m->k_norm = kn[l];
        m->Wq.p = wq[l]; m->Wk.p = wk[l]; m->Wv.p = wv[l]; m->Wo.p = wo[l];
        m->Wq.enc = m->Wk.enc = m->Wv.enc = m->Wo.enc = attn_enc;
        m->Wgate.p = wgate[l]; m->Wgate.enc = QW3_ENC_F32;
        for (int i = 0; i < E * 3; i++) {
            tab[(size_t)l * E * 3 + i].p = exp[(size_t)l * E * 3 + i];
            tab[(size_t)l * E * 3 + i].enc = exp_enc;
        }
        m->exp = tab + (size_t)l * E * 3;
        if (qwen3_kv_alloc(&kv[l], m, cap)) goto out;
    }
    QW3T head = { lm_head, head_enc };
    int pos = 0, T = n_prompt;
    const int *ids = prompt;
    int cur = 0;
    for (int step = 0; step <= n_new; step++) {
        for (int t = 0; t < T; t++) refh_embed(embed, embed_enc, step == 0 ? ids[t] : cur, x + (size_t)t * D, D);
        for (int l = 0; l < L; l++) {
            QW3Out o;
            if (qwen3_layer_alloc(&o, &ls[l], T)) goto out;
            if (qwen3_layer_kv(&ls[l], x, T, pos, &kv[l], &o)) { qwen3_layer_free(&o); goto out; }
            for (size_t i = 0; i < (size_t)T * D; i++) x[i] += o.attn[i] + o.mlp[i];
            qwen3_layer_free(&o);
        }
        float *xl = x + (size_t)(T - 1) * D;
        rmsnorm(xl, xl, final_norm, D, eps);
        qwen3_mm(&head, logits, xl, D, V);
        cur = refh_argmax(logits, V);
        out_ids[step] = cur;
        pos += T;
        T = 1;
    }
    if (out_logits) memcpy(out_logits, logits, sizeof(float) * (size_t)V);
    rc = 0;
out:
    if (kv) for (int l = 0; l < L; l++) qwen3_kv_free(&kv[l]);
    free(ls); free(kv); free(tab); free(x); free(logits);
    return rc;
}

/* A CPW1 v4 file through the reference's OWN loader: qwen3_map_ex with no pager (the weights
   are read from the mapping, engine/blocks/qwen3_moe.c:318-459) and qwen3_bind_layer per layer,
   as cp_open binds them (engine/api/cachepotato.c:262-283), then the generate loop above with
   embed_rows' chunked-table lookup (cachepotato.c:108-133). out_ids gets n_new + 1 ids, out_meta
   {n_layers, d_model, vocab, n_experts, topk, d_exp}. */
int refh_v4_generate(const char *path, const int *prompt, int n_prompt, int n_new, int *out_ids,
                     float *out_logits, int *out_meta) {
    QW3Layer base;
    if (qwen3_map_ex(&base, path, QW3_BUDGET_NONE)) return -1;
    if (qwen3_bind_layer(&base, 0)) return -2;
    const int L = base.n_layers, D = base.d_model, V = base.vocab, E = base.n_experts;
    const int cap = n_prompt + n_new;
    QW3Layer *ls = calloc((size_t)L, sizeof(QW3Layer));
    QW3KV *kv = calloc((size_t)L, sizeof(QW3KV));
    float *x = malloc(sizeof(float) * (size_t)n_prompt * D);
    float *logits = malloc(sizeof(float) * (size_t)V);
    int rc = -3;
    if (!ls || !kv || !x || !logits) goto out;
    for (int l = 0; l < L; l++) {
        ls[l] = base;                                   /* tables of 128 experts, as qwen3_map_ex
                                                           allocates them: qwen3_bind_layer clears 128 */
        ls[l].exp = calloc((size_t)(E > 128 ? E : 128) * 3, sizeof(QW3T));
        ls[l].exp_owned = 0;
        ls[l].reg_exp = calloc((size_t)(E > 128 ? E : 128), sizeof(int));
        if (!ls[l].exp || !ls[l].reg_exp || qwen3_bind_layer(&ls[l], l)) goto out;
        if (qwen3_kv_alloc(&kv[l], &ls[l], cap)) goto out;
    }
    if (out_meta) {
        out_meta[0] = L; out_meta[1] = D; out_meta[2] = V;
        out_meta[3] = E; out_meta[4] = base.topk; out_meta[5] = ls[0].d_exp;
    }
    {
        const size_t q8_row = (size_t)(D / 32) * 34, q4_row = (size_t)(D / 32) * 18;
        int pos = 0, T = n_prompt, cur = 0;
        for (int step = 0; step <= n_new; step++) {
            for (int t = 0; t < T; t++) {
                int row = step == 0 ? prompt[t] : cur;
                const void *eb = base.embed.p;
                if (base.embed_chunks > 0 && base.embed_rows > 0) {
                    int c = row / base.embed_rows, r = row - c * base.embed_rows;
                    if (c >= base.embed_chunks) { c = base.embed_chunks - 1; r = row - c * base.embed_rows; }
                    eb = base.embed_chunk_ptr[c];
                    row = r;
                }
                float *xt = x + (size_t)t * D;
                if (base.embed.enc == QW3_ENC_Q8) q8_dequant_row((const uint8_t *)eb + (size_t)row * q8_row, xt, D);
                else if (base.embed.enc == QW3_ENC_Q4) q4_dequant_row((const uint8_t *)eb + (size_t)row * q4_row, xt, D);
                else memcpy(xt, (const float *)eb + (size_t)row * D, sizeof(float) * (size_t)D);
            }
            for (int l = 0; l < L; l++) {
                QW3Out o;
                if (qwen3_layer_alloc(&o, &ls[l], T)) goto out;
                if (qwen3_layer_kv(&ls[l], x, T, pos, &kv[l], &o)) { qwen3_layer_free(&o); goto out; }
                for (size_t i = 0; i < (size_t)T * D; i++) x[i] += o.attn[i] + o.mlp[i];
                qwen3_layer_free(&o);
            }
            float *xl = x + (size_t)(T - 1) * D;
            rmsnorm(xl, xl, base.final_norm, D, base.rms_eps);
            qwen3_mm(&base.lm_head, logits, xl, D, V);
            cur = refh_argmax(logits, V);
            out_ids[step] = cur;
            pos += T;
            T = 1;
        }
    }
    if (out_logits) memcpy(out_logits, logits, sizeof(float) * (size_t)V);
    rc = 0;
out:
    if (ls)
        for (int l = 0; l < L; l++) {
            free(ls[l].exp);
            free(ls[l].reg_exp);
            if (kv) qwen3_kv_free(&kv[l]);
        }
    free(ls); free(kv); free(x); free(logits);
    return rc;
}
