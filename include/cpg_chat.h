#ifndef CPG_CHAT_H
#define CPG_CHAT_H
/* cpg_chat.h — the reference engine's public API (engine/api/cachepotato.h:24-90) served by
 * the GPU: libcachepotato_b200.so exports the same functions with the same types, so the
 * reference's front-ends (the C chat, the Rust CLI through cli/src/ffi.rs) link it in place of
 * the CPU engine. The model step runs on the device (cpg_qwen3: embed, attention, MoE block,
 * head, greedy argmax); the CPW1 v4 file is copied to HBM once and its region digests are
 * checked on the device; the conversation's KV cache stays on the device between turns.
 *
 * Tokenisation is the reference's own module (engine/tokenizers: tokenizer_load,
 * tokenizer_qwen_load_unicode, tokenizer_qwen_encode, tokenizer_free), linked by the program
 * that links this library; it is outside the GPU path.
 *
 * Differences from the CPU engine: there is no pager (the whole file is resident in HBM), so
 * budget_mb is accepted but only CP_BUDGET_AUTO's memory check is not applied; threads and
 * pin_cores do not apply (cp_get_stats reports threads = 0, budget_mb = -1 and zero pager
 * counters). ONE MODEL PER PROCESS, as in the reference. */
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct cp_model cp_model;

#define CP_BUDGET_AUTO 0L
#define CP_BUDGET_ENV  (-2L)
#define CP_BUDGET_NONE (-1L)

typedef struct {                /* cachepotato.h:33-39 */
    long budget_mb;
    int threads;
    int pin_cores;
    int max_ctx;                /* 0 = 2048 tokens */
    const char *tokenizer_dir;  /* NULL = next to the model, its tokenizer/ folder, weights/ */
} cp_options;

void cp_options_default(cp_options *opt);                                            /* cachepotato.h:42 */
cp_model *cp_open(const char *model_path, const cp_options *opt, char *err, size_t errlen); /* :45 */
void cp_close(cp_model *m);                                                          /* :46 */

typedef int (*cp_token_fn)(const char *bytes, size_t len, void *user);               /* :51 */
typedef enum { CP_STOP_EOS = 0, CP_STOP_MAX_TOKENS, CP_STOP_CONTEXT, CP_STOP_CALLER } cp_stop;

typedef struct {                /* cachepotato.h:55-62 */
    int prompt_tokens;
    int context_tokens;
    int generated_tokens;
    int context_reset;
    double prefill_s, decode_s;
    cp_stop stop;
} cp_turn;

int cp_chat(cp_model *m, const char *user_msg, int max_new,
            cp_token_fn on_token, void *user, cp_turn *turn);                        /* :68-69 */
void cp_reset(cp_model *m);                                                          /* :72 */

typedef struct {                /* cachepotato.h:74-83 */
    int n_layers, d_model, n_experts, topk, vocab, max_ctx;
    int threads;
    long budget_mb;
    long long file_bytes;
    long hits, misses, evictions;
    long long bytes_fetched, resident_bytes;
} cp_stats;

void cp_get_stats(const cp_model *m, cp_stats *out);                                 /* :85 */
int  cp_physical_cores(void);                                                        /* :88 */
long cp_mem_available_mb(void);                                                      /* :89 */
long cp_auto_budget_mb(long long model_file_bytes);                                  /* :90 */

#ifdef __cplusplus
}
#endif
#endif
