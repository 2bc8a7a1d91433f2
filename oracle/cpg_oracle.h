/* cpg_oracle.h — CPU restatement of the CachePotato Qwen3-MoE expert path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA path is compared against; it is
 * never the thing measured or shipped. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference legs may load it.
 *
 * Every function restates the reference algorithm in plain scalar C11 and names the reference
 * file:line it follows (paths relative to the CachePotato project root). Pinned by:
 *   - the reference's own decoder KATs (tools/verify_q4_decode.py:48-55,
 *     tools/verify_q8_decode.py:48-58), re-generated as tests/golden/ fixtures;
 *   - outputs of the reference engine itself, compiled from its sources into oracle/_ref/
 *     (tests/golden/make_golden.py).
 */
#ifndef CPG_ORACLE_H
#define CPG_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* encodings, same codes as QW3_ENC_* (engine/blocks/qwen3_moe.h:15-17) */
#define ORC_ENC_F32 0
#define ORC_ENC_Q8  8
#define ORC_ENC_Q4  4

float orc_f16_to_f32(uint16_t h);                 /* kernels.c:109-130 */
uint16_t orc_f32_to_f16(float f);                 /* numpy astype(float16): RNE */

/* decoders: kernels.c:143-151 (Q8_0), kernels.c:463-477 (Q4_0) */
void orc_q8_dequant_row(const uint8_t *blocks, float *out, long n);
void orc_q4_dequant_row(const uint8_t *blocks, float *out, long n);

/* encoders: format/q8.py:35-58 (encode_q8_0), format/q4.py:30-57 (encode_q4_0).
   n must be a multiple of 32. nthreads <= 1 runs serially. */
void orc_quantize_q8_0(const float *x, long n, uint8_t *out, int nthreads);
void orc_quantize_q4_0(const float *x, long n, uint8_t *out, int nthreads);

/* Synthetic N(0, std^2) fill, counter-based (splitmix64 -> Box-Muller) so any slice can be
   generated independently and in parallel; element i depends only on (seed, i). Test-data
   generator only: it restates nothing from the reference. */
void orc_fill_normal(float *out, long n, uint64_t seed, float std, int nthreads);

/* W·x, W row-major (n_out, n_in): kernels.c:84-95 (f32), 386-395 (Q8 scalar),
   524-539 (Q4 scalar). Scalar summation order of the reference's 1-thread path. */
void orc_matmul_wx(float *out, const float *x, const float *w, int n_in, int n_out);
void orc_matmul_wx_q8(float *out, const float *x, const uint8_t *w, int n_in, int n_out);
void orc_matmul_wx_q4(float *out, const float *x, const uint8_t *w, int n_in, int n_out);
void orc_mm(const void *w, int enc, float *out, const float *x, int n_in, int n_out); /* qwen3_moe.c:36-40 */

void orc_rmsnorm(float *out, const float *x, const float *g, int n, float eps); /* kernels.c:408-413 */
void orc_softmax(float *x, int n);                                              /* kernels.c:20-26 */
float orc_silu(float x);                                                        /* kernels.c:416 */

/* router: logits = Wgate·xn, softmax, strict-'>' top-k (lower id wins ties), renormalise.
   qwen3_moe.c:180-197. probs (n_experts) is scratch/out. */
void orc_route(const void *wgate, int wgate_enc, const float *xn, int d_model, int n_experts,
               int topk, float *logits, float *probs, int *idx, float *wt);

/* The MoE half of qwen3_layer_kv (qwen3_moe.c:170-223) for T tokens:
   hh = x + attn; xn = rmsnorm(hh, ln2); route; for each selected expert j in selection order:
   g = Wg·xn, u = Wu·xn, h = silu(g)·u, y = Wd·h, mlp += wt_j·y.
   exp[e*3+kind] are weight pointers (kind 0 gate, 1 up, 2 down), all of encoding exp_enc.
   attn may be NULL (treated as zero). mlp is ACCUMULATED (caller zeroes), as in the reference.
   router (T, n_experts), topk_idx (T, topk), wt (T, topk), xn_out (T, d_model) may be NULL. */
int orc_qwen3_moe(const float *ln2, const void *wgate, int wgate_enc,
                  const void *const *exp, int exp_enc,
                  int d_model, int d_exp, int n_experts, int topk, float eps,
                  const float *x, const float *attn, int T,
                  float *mlp, float *router, int *topk_idx, float *wt, float *xn_out);

/* Externally routed experts (no router): for token t and slot j, expert idx[t*topk+j] with
   weight wt[t*topk+j] applied to xn[t]; mlp[t] += sum_j wt·Wd·(silu(Wg·xn)·(Wu·xn)), j in
   order. The expert loop of qwen3_moe.c:199-222 without the routing above it. */
int orc_moe_apply(const void *const *exp, int exp_enc, int d_model, int d_exp,
                  const float *xn, int T, int topk, const int *idx, const float *wt,
                  float *mlp);

#ifdef __cplusplus
}
#endif
#endif
