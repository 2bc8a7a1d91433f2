/* cpg.h — C ABI of cachepotato_b200: the Qwen3-MoE expert hot path of CachePotato on B200.
 *
 * Plain C: pointers, sizes and int status codes; no CUDA or torch types. `stream` arguments
 * are a cudaStream_t passed as void* (NULL = the legacy default stream). Device pointers are
 * CUDA global memory; "host" entry points take ordinary host memory and are synchronous.
 *
 * Status codes: every int-returning entry returns CPG_OK (0) or a negative CPG_E* code and
 * leaves a message for cpg_last_error(). The drop-ins with the reference's void signatures
 * report failures on stderr and through cpg_last_error(), as the reference reports through
 * stderr (engine/kernels/kernels.h has no error channel).
 *
 * Each declaration names the reference interface it replaces (paths relative to the
 * CachePotato source tree).
 */
#ifndef CPG_H
#define CPG_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CPG_OK        0
#define CPG_EINVAL   (-1)   /* bad argument or unsupported shape */
#define CPG_ECUDA    (-2)   /* a CUDA runtime call failed */
#define CPG_ETIMEOUT (-3)   /* a bounded device-side wait ran out (status word set) */
#define CPG_ENOMEM   (-4)   /* device or pinned allocation failed */
#define CPG_ENCCL    (-5)   /* collective failure (expert-parallel path) */
#define CPG_ESTATE   (-6)   /* call out of order (e.g. store not open) */

/* Tensor encodings: the same codes as QW3_ENC_* (engine/blocks/qwen3_moe.h:15-17). */
#define CPG_ENC_F32 0
#define CPG_ENC_Q8  8       /* Q8_0: 34-byte group = fp16 scale + 32 int8 (format/SPEC.md) */
#define CPG_ENC_Q4  4       /* Q4_0: 18-byte group = fp16 scale + 16 bytes of nibbles */

/* A weight tensor: pointer + encoding. Mirrors QW3T (engine/blocks/qwen3_moe.h:19). */
typedef struct { const void *p; int enc; } cpg_tensor;

/* Message of the last failure on this host thread ("" if none). */
const char *cpg_last_error(void);
/* Library version, major*10000 + minor*100 + patch. */
int cpg_version(void);

/* ============================================================== kernel drop-ins (host)
 * Same signatures and meaning as engine/kernels/kernels.h:17,21-24 and kernels.c:368 /
 * kernels.c:514: out = W·x with W row-major (n_out, n_in) in the given encoding, n_in % 32 == 0,
 * out OVERWRITTEN. Host pointers, synchronous. When `w` lies inside the range mirrored by
 * cpg_store_open_v4 the resident device copy is used (translated by offset, like
 * pager_region_get); otherwise the rows are copied to the device for the call. */
void cpg_matmul_wx(float *out, const float *x, const float *w, int n_in, int n_out);       /* kernels.c:84 */
void cpg_matmul_wx_q8(float *out, const float *x, const uint8_t *w, int n_in, int n_out);  /* kernels.c:368 */
void cpg_matmul_wx_q4(float *out, const float *x, const uint8_t *w, int n_in, int n_out);  /* kernels.c:514 */
/* Bit-exact decoders: kernels.c:143 (Q8_0) and kernels.c:463 (Q4_0); n % 32 == 0. */
void cpg_q8_dequant_row(const uint8_t *blocks, float *out, int n);
void cpg_q4_dequant_row(const uint8_t *blocks, float *out, int n);

/* ============================================================== device-pointer kernels */
/* Decode n values (n % 32 == 0) of a Q4_0/Q8_0 block stream, bit-exact with kernels.c:143/463. */
int cpg_dequant(float *out, const uint8_t *blocks, int enc, long n, void *stream);
/* Encode n f32 values (n % 32 == 0) to Q4_0/Q8_0 blocks, bit-exact with format/q4.py:30-57 and
   format/q8.py:35-58 (the reference's encoders). */
int cpg_quantize(uint8_t *blocks, const float *x, int enc, long n, void *stream);
/* T independent products out[t] = W·x[t], x (T, n_in) and out (T, n_out) row-major f32,
   f32 accumulation (kernels.c:84-95 / 287-396 / 480-540 arithmetic). Replaces qwen3_mm
   (engine/blocks/qwen3_moe.c:36-40) for device-resident tensors. */
int cpg_matvec(float *out, const float *x, cpg_tensor w, int n_in, int n_out, int T, void *stream);

/* ============================================================== region store
 * HBM-resident replacement for the pager's region table (engine/pager/pager.h:51-66).
 * One store per process and device, like the pager (pager.c:195-214). The whole data section
 * of a mapped CPW1 v4 file is copied to HBM once, through pinned staging buffers; region ids
 * are region-table indices exactly as pager_add_region hands them out. */
int cpg_store_open_v4(const void *map_base, size_t map_len, size_t data_off);          /* pager_open_v4 */
/* An empty store of `bytes` bytes (synthetic workloads); fill it through cpg_store_base(). */
int cpg_store_open(size_t bytes);
int cpg_store_add_region(size_t off, size_t len, int is_expert);                       /* pager_add_region: id or <0 */
const void *cpg_store_region_get(int id);                                             /* pager_region_get: device address */
/* Device address of a host pointer inside the mirrored mapping, NULL if outside. */
const void *cpg_store_translate(const void *host_ptr);
void *cpg_store_base(void);
size_t cpg_store_bytes(void);
typedef struct { long regions, expert_regions; long resident_bytes; long h2d_bytes; } cpg_store_totals_t;
int cpg_store_totals(cpg_store_totals_t *out);                                         /* pager_totals */
void cpg_store_close(void);
/* The loader's region digest check, on the device: region i's CRC-32 (IEEE, zlib.crc32, the
 * digest format/v4_writer.py:235-250 stores as a u64 in the region table) against digests[i],
 * for all n regions added (n must equal their count). CPG_OK, or CPG_EINVAL with *first_bad =
 * the lowest mismatching region id (-1 otherwise; first_bad may be NULL). Synchronous. */
int cpg_store_verify(const uint64_t *digests, int n, int *first_bad);
/* CRC-32 (IEEE, zlib.crc32) of n bytes of device memory; synchronous on `stream`. */
int cpg_crc32(const void *dev, size_t n, uint32_t *out, void *stream);

/* ============================================================== MoE block
 * The MoE half of qwen3_layer_kv (engine/blocks/qwen3_moe.c:169-223) plus the residual add of
 * run_layers (engine/api/cachepotato.c:157-159):
 *   hh = x + attn; xn = rmsnorm(hh, ln2, eps); logits = Wgate·xn; p = softmax(logits);
 *   top-k by strict '>' (lower id wins ties), wt = p[idx] / sum(p[idx]);
 *   for j in selection order: mlp += wt_j · Wd_e·(silu(Wg_e·xn) · (Wu_e·xn)).
 * Expert GEMVs run on tensor cores with exact Q4/Q8 integers and the f32 activations carried
 * as fp16 hi + lo halves, fp32 scales and accumulation; the block output matches the f32
 * reference within max|d|/max|ref| <= 1e-5. */
typedef struct {
    int d_model;              /* 2048 for Qwen3-30B-A3B; multiple of 256 */
    int d_exp;                /* 768; multiple of 256 */
    int n_experts;            /* 128; <= 256 */
    int topk;                 /* 8; <= 32 */
    float rms_eps;            /* 1e-6 */
    const float *ln2;         /* device (d_model) */
    cpg_tensor wgate;         /* device (n_experts, d_model), CPG_ENC_F32 */
    const cpg_tensor *experts;/* HOST array (n_experts*3) of DEVICE tensors, [e*3+kind], kind
                                 0 gate (d_exp,d_model), 1 up (d_exp,d_model), 2 down
                                 (d_model,d_exp); one encoding (Q4 or Q8) for all of them.
                                 Mirrors QW3Layer.exp (qwen3_moe.h:28-34). */
} cpg_moe_desc;

typedef struct cpg_moe_layer cpg_moe_layer;

/* Routing agreement under ties, on the device: the rule of tools/check_qwen3_baseline.py:39-72
 * (models/qwen3-30b-a3b/MODEL.md section 6). logits (T, E) f32, topk (T, K) int ids, wt (T, K)
 * f32, all device; E <= 256, K <= 32. p = softmax(logits) in float64, thr = its K-th largest;
 * a token's ids (as a set) are a valid top-K if every chosen p >= thr - 1e-12 and exactly the
 * experts with p > thr + 1e-12 are chosen among those above it. Writes stats[3] = {invalid
 * tokens, valid tokens resolved by a tie, first invalid token or -1} and errs[2] = {max
 * |sum(w) - 1|, max |w - p[ids] / sum(p[ids])|}. Synchronous on `stream`. */
int cpg_route_check(const float *logits, const int *topk, const float *wt, int T, int E, int K,
                    int *stats, double *errs, void *stream);

/* Validate a layer and upload its expert table (qwen3_bind_layer, qwen3_moe.c:462-586).
 * Also builds the small-batch expert kernels' copy of the expert matrices, regrouped into
 * 16-row x 256-value tiles (same bytes per matrix, device memory owned by the layer): the
 * matrices must hold their final values when the layer is created, as the reference's
 * mapped model file does. Synchronises the device. */
int cpg_moe_layer_create(const cpg_moe_desc *desc, cpg_moe_layer **out);
void cpg_moe_layer_destroy(cpg_moe_layer *layer);
/* Scratch bytes one forward of up to max_T tokens needs (the caller allocates it). */
size_t cpg_moe_workspace_bytes(const cpg_moe_layer *layer, int max_T);

/* One MoE block on device memory, enqueued on `stream` (no allocation, no host sync).
 *   x (T,d_model) in; attn (T,d_model) or NULL (= zero);
 *   mlp (T,d_model) or NULL: ACCUMULATED (+=), as QW3Out.mlp (qwen3_moe.h:73), caller zeroes;
 *   x_out (T,d_model) or NULL: x + (attn + mlp), mlp being the accumulated value above (the
 *     residual of run_layers); may alias x;
 *   topk_idx (T,topk) int, wt (T,topk), router (T,n_experts) logits: optional outputs.
 * The status word in the workspace records device-side timeouts; read it with
 * cpg_moe_check(). A one-token forward (T = 1) runs the whole block in one cooperative launch
 * (one CTA per SM, grid-wide barriers through two counters the layer owns): one-token forwards
 * of the same layer must not overlap on the GPU (serialise them on one stream, or with events). */
int cpg_moe_forward(const cpg_moe_layer *layer, const float *x, const float *attn, int T,
                    float *mlp, float *x_out, int *topk_idx, float *wt, float *router,
                    void *ws, size_t ws_bytes, void *stream);
/* Synchronise `stream` and return CPG_OK, or CPG_ETIMEOUT if a bounded wait in the last
   forward on this workspace gave up. */
int cpg_moe_check(const void *ws, void *stream);

/* cpg_moe_forward without a caller workspace, for callers that cannot allocate device memory
 * where they run the block (an engine whose host program owns all device memory through its
 * own pool, a decode loop that may not stall on the allocator). No counterpart in the reference (its CPU engine mallocs
 * scratch per call, qwen3_moe.c:98-108). Scratch comes from a fixed 8 MiB array in the
 * library's device image (enough for 64 tokens of a Qwen3-30B-A3B layer); larger T is rejected
 * with CPG_EINVAL. Allocates nothing. The first call on a device looks up the array's address
 * once. All calls share the array: calls that overlap on the
 * GPU race, so serialise them (one stream, or events). Device-side timeouts are recorded in the
 * array and not reported here; use cpg_moe_forward + cpg_moe_check when they must be read. */
int cpg_moe_forward_noalloc(const cpg_moe_layer *layer, const float *x, const float *attn, int T,
                            float *mlp, float *x_out, int *topk_idx, float *wt, float *router,
                            void *stream);

/* ============================================================== prefill: routed experts
 * The expert loop of qwen3_moe.c:199-222 with the routing supplied by the caller (prefill
 * batches whose token->expert assignment is drawn directly, the receive side of expert
 * parallelism): for every token t and slot j, mlp[t] += wt[t,j] · Wd·(silu(Wg·xn[t]) · (Wu·xn[t]))
 * with e = topk_idx[t,j], slots added in order j = 0..topk-1. xn (T,d_model) f32 device, already
 * normalised; topk_idx (T,topk) int; wt (T,topk) f32; mlp (T,d_model) accumulated. Tokens are
 * sorted by expert (deterministically, tokens ascending) and each expert's tokens run through a
 * grouped GEMM on the tcgen05 tensor cores: Q4_0 weights decoded to fp16 (q·d rounded once),
 * fp16 activations, fp32 accumulation in tensor memory. Q4_0 experts; d_exp % 128 == 0. */
size_t cpg_moe_apply_workspace_bytes(const cpg_moe_layer *layer, int max_T);
int cpg_moe_apply(const cpg_moe_layer *layer, const float *xn, int T, const int *topk_idx,
                  const float *wt, float *mlp, void *ws, size_t ws_bytes, void *stream);
/* Synchronise; CPG_EINVAL if an expert id was outside [0, n_experts) (those slots contributed
   zero), CPG_ETIMEOUT if a bounded device wait gave up. */
int cpg_moe_apply_check(const void *ws, void *stream);
/* cpg_moe_apply with CUDA events around its phases; synchronises and writes phase_ms[4]:
   token sort, gate/up GEMM, down GEMM, combine (milliseconds). */
int cpg_moe_apply_profile(const cpg_moe_layer *layer, const float *xn, int T, const int *topk_idx,
                          const float *wt, float *mlp, void *ws, size_t ws_bytes, void *stream,
                          float *phase_ms);
/* The same experts over R fp16 rows (R, d_model) with per-row slot lists: slot_expert (R, topk)
   holds a local expert id or -1 for an empty slot, slot_wt (R, topk) its weight. out (R, d_model)
   f32 is overwritten with sum over the row's valid slots of wt·expert(row), in slot order. This
   is the receive side of cpg_moe_ep; workspace: cpg_moe_apply_workspace_bytes(layer, R). */
int cpg_moe_apply_rows(const cpg_moe_layer *layer, const void *rows_f16, int R, const int *slot_expert,
                       const float *slot_wt, float *out, void *ws, size_t ws_bytes, void *stream);

/* ============================================================== expert parallelism (NCCL)
 * Batched MoE layers with the experts sharded across the GPUs of one node: rank r owns experts
 * [r·E_l, (r+1)·E_l), where E_l = n_experts of the local layer it passes, and T tokens of the
 * batch (the same T on every rank). No counterpart in the reference (single-host engine).
 * One process per GPU; NCCL is resolved at run time from the process or the system library.
 * cpg_ep_unique_id on one rank, shared with the others by the caller (128 bytes), then
 * cpg_ep_create on every rank with the device current. */
typedef struct cpg_ep cpg_ep;
int cpg_ep_unique_id(void *out128);
/* Creates the communicator non-blocking where NCCL offers it (ncclCommInitRankConfig with
   blocking = 0): a peer that never joins ends in CPG_ETIMEOUT after the rank's deadline (120 s,
   or CPG_EP_TIMEOUT_MS from the environment), with the communicator aborted, not in a hang. */
int cpg_ep_create(int nranks, int rank, const void *unique_id128, cpg_ep **out);
/* Frees the communicator after its outstanding work (bounded by the deadline, then aborted). */
void cpg_ep_destroy(cpg_ep *ep);
/* The host deadline (milliseconds) for this rank's asynchronous NCCL steps and cpg_ep_wait. */
int cpg_ep_set_timeout(cpg_ep *ep, int timeout_ms);
/* ncclCommAbort: NCCL ends this rank's collectives in flight and frees the communicator; every
   later call on `ep` returns CPG_ENCCL (destroy still frees the handle). For a caller that
   learned on the host that a peer is gone (a heartbeat or store), before its next launch. */
int cpg_ep_abort(cpg_ep *ep);
/* Wait (polling, bounded by the deadline) until `stream` has finished this rank's EP work.
   CPG_OK; CPG_ENCCL if NCCL reported an asynchronous error; CPG_ETIMEOUT if the stream was not
   done by the deadline (a peer stopped taking part). Both abort the communicator first, so
   the stream drains. */
int cpg_ep_wait(cpg_ep *ep, void *stream);
size_t cpg_ep_workspace_bytes(const cpg_ep *ep, const cpg_moe_layer *local_layer, int T);
/* mlp[t] += sum_j wt[t,j] · expert_{topk_idx[t,j]}(xn[t]) with global expert ids, the experts
 * computed on their owners: each token's row travels once per owner (fp16), each owner returns
 * one f32 row per token combining that token's slots on it in slot order, and the source adds
 * the owners' rows in ascending rank. Collective: every rank calls it in the same order.
 * Every argument is checked before the first collective (a rejected call posts no transfer).
 * Returns CPG_ENCCL on an NCCL error, after which the communicator is aborted (no open group,
 * no peer left waiting on a transfer this rank will not post). */
int cpg_moe_ep(cpg_ep *ep, const cpg_moe_layer *local_layer, const float *xn, int T, const int *topk_idx,
               const float *wt, float *mlp, void *ws, size_t ws_bytes, void *stream);
/* cpg_moe_ep with CUDA events around its phases; waits (cpg_ep_wait) and writes phase_ms[5]:
   plan + pack, dispatch, owner experts, return, combine (milliseconds). */
int cpg_moe_ep_profile(cpg_ep *ep, const cpg_moe_layer *local_layer, const float *xn, int T,
                       const int *topk_idx, const float *wt, float *mlp, void *ws, size_t ws_bytes,
                       void *stream, float *phase_ms);
/* Synchronise; CPG_EINVAL if an expert id was outside [0, nranks·E_l) (those slots contributed
   zero); CPG_ETIMEOUT if a bounded device wait in the owner's expert GEMMs gave up. */
int cpg_moe_ep_check(const void *ws, void *stream);

/* ============================================================== the whole model (config 3)
 * A Qwen3-MoE model on one device: embed_rows, run_layers (attention half of qwen3_layer_kv,
 * qwen3_moe.c:110-167, then the MoE half through cpg_moe_forward), apply_head and the greedy
 * argmax of cp_chat (engine/api/cachepotato.c:108-166, 315-378). Tensors are device pointers;
 * head_dim must be 128. The model owns an f32 KV cache of max_ctx positions per layer. */
typedef struct {
    const float *ln1, *q_norm, *k_norm;      /* (d_model), (head_dim), (head_dim) */
    cpg_tensor wq, wk, wv, wo;               /* (n_heads·hd, d), (n_kv·hd, d) ×2, (d, n_heads·hd) */
} cpg_qwen3_attn;
typedef struct {
    int d_model, n_heads, n_kv, head_dim, vocab, n_layers, max_ctx;
    float rope_theta, rms_eps;
    cpg_tensor embed, lm_head;               /* (vocab, d_model), Q8_0 or Q4_0 / any encoding */
    const float *final_norm;
    const cpg_qwen3_attn *attn;              /* n_layers */
    cpg_moe_layer *const *moe;               /* n_layers */
} cpg_qwen3_desc;
typedef struct cpg_qwen3 cpg_qwen3;
int cpg_qwen3_create(const cpg_qwen3_desc *d, cpg_qwen3 **out);
void cpg_qwen3_destroy(cpg_qwen3 *m);
/* The prompt (host ids) in one pass at position 0 (the cache restarts); *next_id = argmax of
   the last position's logits (first maximum wins). */
int cpg_qwen3_prefill(cpg_qwen3 *m, const int *ids, int T, int *next_id);
/* One token at the next position. */
int cpg_qwen3_step(cpg_qwen3 *m, int id, int *next_id);
/* T more prompt tokens (host ids) at the current position, in one pass, keeping what the cache
   holds (a conversation's next turn, cachepotato.c:336-346); *next_id = argmax after the last. */
int cpg_qwen3_append(cpg_qwen3 *m, const int *ids, int T, int *next_id);
/* Move the position back to pos (<= the current one); later tokens overwrite the cache from
   there (cp_reset / a restarted conversation). */
int cpg_qwen3_rewind(cpg_qwen3 *m, int pos);
/* Prefill, then n_new steps each feeding the previous argmax; out_ids gets n_new + 1 ids. */
int cpg_qwen3_generate(cpg_qwen3 *m, const int *prompt, int n_prompt, int n_new, int *out_ids);
const float *cpg_qwen3_logits(const cpg_qwen3 *m);   /* device (vocab) f32, last position */
void *cpg_qwen3_stream(const cpg_qwen3 *m);
int cpg_qwen3_position(const cpg_qwen3 *m);

/* ------------------------------------------- several sequences at once (continuous batching)
 * The reference decodes one sequence per engine (engine/api/cachepotato.h:12-16). A batch holds
 * n_slots sequences over one model's weights, each with its own f32 KV cache of max_ctx
 * positions (≤ the model's max_ctx; n_slots ≤ the model's max_ctx). A sequence enters a slot
 * with cpg_qwen3_batch_prefill (its prompt from position 0, replacing what the slot held); a
 * step then takes one new token for each slot it names, so sequences join and leave between
 * steps. Per sequence the ids are those of cpg_qwen3_generate on the same prompt (the greedy
 * loop of cp_chat, cachepotato.c:315-378). Runs on the model's stream and scratch: do not use
 * the model's own sequence (cpg_qwen3_prefill/step) concurrently from another thread; its KV
 * cache and position are left untouched. */
typedef struct cpg_qwen3_batch cpg_qwen3_batch;
int cpg_qwen3_batch_create(cpg_qwen3 *m, int n_slots, int max_ctx, cpg_qwen3_batch **out);
void cpg_qwen3_batch_destroy(cpg_qwen3_batch *b);
/* n < max_ctx prompt ids into `slot`; *next_id = argmax of the last position's logits. */
int cpg_qwen3_batch_prefill(cpg_qwen3_batch *b, int slot, const int *ids, int n, int *next_id);
/* One step: slots[0..n) distinct prefilled slots, ids[t] the new token of slots[t];
   next_ids[t] its argmax. */
int cpg_qwen3_batch_step(cpg_qwen3_batch *b, const int *slots, const int *ids, int n, int *next_ids);
/* n_steps steps of the same slots, each feeding the previous argmax; out_ids (n_steps, n),
   step-major. */
int cpg_qwen3_batch_generate(cpg_qwen3_batch *b, const int *slots, const int *ids, int n, int n_steps,
                             int *out_ids);
int cpg_qwen3_batch_position(const cpg_qwen3_batch *b, int slot);   /* -1: empty slot */
/* Device logits of the last call, *rows rows of vocab f32: a step's rows in its slot order; a
   prefill's one row. */
const float *cpg_qwen3_batch_logits(const cpg_qwen3_batch *b, int *rows);

/* ============================================================== decode loop (host buffers)
 * A context owns a stream, a workspace and device activation buffers on one device. */
typedef struct cpg_ctx cpg_ctx;
int cpg_ctx_create(int device, int max_T, const cpg_moe_layer *shape, cpg_ctx **out);
void cpg_ctx_destroy(cpg_ctx *ctx);
void *cpg_ctx_stream(cpg_ctx *ctx);
/* The MoE half of run_layers (engine/api/cachepotato.c:149-166) over L layers, host in and
 * out: x (T,d_model) in HOST memory is updated in place, x += mlp_l for l = 0..L-1 (the
 * attention half is the caller's). Copies x to the device, runs the layers (replayed from a
 * CUDA graph after the first call with the same layers and T), copies x back; synchronous.
 * topk_out (L,T,topk) host int, optional. */
int cpg_run_moe_layers(cpg_ctx *ctx, cpg_moe_layer *const *layers, int L, float *x, int T,
                       int *topk_out);
/* The same L layers on the context's device activations cpg_ctx_x(ctx) (T, d_model), enqueued
 * on cpg_ctx_stream(ctx) without copies or synchronisation (device-resident decode). */
int cpg_ctx_run(cpg_ctx *ctx, cpg_moe_layer *const *layers, int L, int T);
float *cpg_ctx_x(cpg_ctx *ctx);
/* (L, T, topk) device ids of the last run. */
int *cpg_ctx_topk(cpg_ctx *ctx);
/* Phase timing: when enabled, the decode graph records CUDA events around the router,
 * gate/up, down and combine launches of every layer; cpg_ctx_phase_ms sums each phase over
 * the layers of the last run (synchronises the stream). Batches whose gate/up items outnumber
 * the SMs run gate/up and down in one launch: its time is the gate/up phase and the down
 * phase is then ~0. */
int cpg_ctx_profile(cpg_ctx *ctx, int enable);
int cpg_ctx_phase_ms(cpg_ctx *ctx, float *ms4);

#ifdef __cplusplus
}
#endif
#endif
