// cp_chat.cpp — the reference engine's public API (engine/api/cachepotato.h) over the GPU model:
// cp_open maps a CPW1 v4 file, walks its tables (qwen3_map_ex / qwen3_bind_layer,
// engine/blocks/qwen3_moe.c:318-586), copies the data section into the HBM region store once,
// checks every region's digest on the device and binds the whole model (cpg_qwen3) from the
// resident copy; cp_chat runs a conversation turn as the reference does (cachepotato.c:315-378):
// the ChatML fragment is appended at the conversation's position, the first token comes from the
// fragment's last position, then greedy steps until <|im_end|>, max_new, the context limit or the
// callback; the emitted token always goes through the forward pass. Host code only: every
// forward runs in libcpg_b200.so.
//
// Tokenisation is the reference's own module (engine/tokenizers/tokenizer.h), linked by the
// program that links this library; its Tokenizer layout is declared here to read token bytes.
#include <fcntl.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "cpg.h"
#include "cpg_chat.h"

// ---- the tokenizer module of the integrating build (engine/tokenizers/tokenizer.h:10-29) ----
struct CpTokMerge {
    uint64_t key;
    uint32_t out, rank;
};
struct CpTokenizer {
    uint32_t n_vocab, n_merges;
    char **vocab;
    uint16_t *vocab_len;
    int32_t byte_id[256];
    CpTokMerge *merges;
};
extern "C" int tokenizer_load(CpTokenizer *t, const char *path);
extern "C" void tokenizer_free(CpTokenizer *t);
extern "C" int tokenizer_qwen_load_unicode(const char *path);
extern "C" int tokenizer_qwen_encode(const CpTokenizer *t, const char *text, int *ids, int max_ids);

namespace {

constexpr int kImEnd = 151645;                       // <|im_end|> (cachepotato.c:28)
constexpr int kDefaultCtx = 2048;
constexpr const char *kTokFile = "qwen2.5-tokenizer.bin", *kUniFile = "qwen2.5-unicode.bin";
constexpr uint32_t kMagic = 0x34575043u, kVersion = 4;
constexpr int kKindAttn = 0x10, kKindMoe = 0x20, kRegionExpert = 1;
constexpr int kTopK = 8;                             // qwen3_moe.c:397-401 fixes top-k and eps
constexpr float kEps = 1e-6f;

bool g_opened = false;                               // one model per process, as the reference

double now_s() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

void set_err(char *err, size_t n, const char *fmt, ...) {
    if (!err || !n) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, n, fmt, ap);
    va_end(ap);
}

// ---- CPW1 v4 tables (format/SPEC.md; little-endian, packed) ----
struct V4Tensor {
    int enc = -1;
    std::vector<uint32_t> dims;
    uint64_t off = 0, nbytes = 0;
};
struct V4Block {
    int kind = 0;
    std::vector<uint32_t> params;
};
struct V4Region {
    uint64_t off = 0, len = 0, digest = 0;
    uint32_t lo = 0, hi = 0;
    int kind = 0;
};

class Reader {
  public:
    Reader(const uint8_t *b, size_t n, size_t pos) : b_(b), n_(n), p_(pos) {}
    template <class T>
    T take() {
        T v{};
        if (p_ + sizeof(T) > n_) { ok_ = false; return v; }
        memcpy(&v, b_ + p_, sizeof(T));
        p_ += sizeof(T);
        return v;
    }
    std::string str() {
        const uint16_t len = take<uint16_t>();
        if (p_ + len > n_) { ok_ = false; return {}; }
        std::string s(reinterpret_cast<const char *>(b_ + p_), len);
        p_ += len;
        return s;
    }
    bool ok() const { return ok_; }

  private:
    const uint8_t *b_;
    size_t n_, p_;
    bool ok_ = true;
};

struct V4File {
    const uint8_t *map = nullptr;
    size_t size = 0;
    uint64_t off_data = 0;
    std::vector<int> encodings;
    std::vector<V4Tensor> tensors;
    std::unordered_map<std::string, int> by_name;
    std::vector<V4Block> blocks;
    std::vector<V4Region> regions;
    int n_layers = 0;

    bool parse(std::string &why) {
        if (size < 72) { why = "file too short"; return false; }
        Reader h(map, size, 0);
        const uint32_t magic = h.take<uint32_t>(), version = h.take<uint32_t>();
        h.take<uint32_t>();
        h.take<uint32_t>();
        if (magic != kMagic || version != kVersion) { why = "not a CPW1 v4 file"; return false; }
        const uint32_t n_tens = h.take<uint32_t>(), n_blk = h.take<uint32_t>(), n_reg = h.take<uint32_t>(),
                       n_enc = h.take<uint32_t>();
        const uint64_t off_enc = h.take<uint64_t>(), off_tens = h.take<uint64_t>(), off_blk = h.take<uint64_t>(),
                       off_reg = h.take<uint64_t>();
        off_data = h.take<uint64_t>();
        Reader r(map, size, off_enc);
        for (uint32_t i = 0; i < n_enc; ++i) {
            r.take<uint32_t>();
            const uint8_t kind = r.take<uint8_t>(), scalar = r.take<uint8_t>();
            r.take<uint16_t>();
            r.take<uint16_t>();
            r.take<uint8_t>();
            r.take<uint8_t>();
            r.take<uint8_t>();
            r.str();
            encodings.push_back(kind == 0 ? CPG_ENC_F32 : scalar == 3 ? CPG_ENC_Q8 : scalar == 4 ? CPG_ENC_Q4 : -1);
        }
        Reader t(map, size, off_tens);
        if (t.take<uint32_t>() != n_tens) { why = "tensor table count differs from the header"; return false; }
        for (uint32_t i = 0; i < n_tens && t.ok(); ++i) {
            V4Tensor x;
            const std::string name = t.str();
            const uint32_t eidx = t.take<uint32_t>();
            const uint8_t nd = t.take<uint8_t>();
            for (int d = 0; d < nd; ++d) x.dims.push_back(t.take<uint32_t>());
            x.off = t.take<uint64_t>();
            x.nbytes = t.take<uint64_t>();
            t.take<uint32_t>();
            t.take<uint16_t>();
            x.enc = eidx < encodings.size() ? encodings[eidx] : -1;
            by_name[name] = (int)tensors.size();
            tensors.push_back(x);
        }
        Reader b(map, size, off_blk);
        if (b.take<uint32_t>() != n_blk) { why = "block table count differs from the header"; return false; }
        for (uint32_t i = 0; i < n_blk && b.ok(); ++i) {
            V4Block x;
            x.kind = b.take<uint8_t>();
            b.take<uint32_t>();
            const uint8_t nref = b.take<uint8_t>();
            for (int k = 0; k < nref; ++k) b.take<uint32_t>();
            const uint8_t npar = b.take<uint8_t>();
            for (int k = 0; k < npar; ++k) x.params.push_back(b.take<uint32_t>());
            if (x.kind == kKindAttn) ++n_layers;
            blocks.push_back(x);
        }
        Reader g(map, size, off_reg);
        if (g.take<uint32_t>() != n_reg) { why = "region table count differs from the header"; return false; }
        for (uint32_t i = 0; i < n_reg && g.ok(); ++i) {
            V4Region x;
            x.off = g.take<uint64_t>();
            x.len = g.take<uint64_t>();
            x.lo = g.take<uint32_t>();
            x.hi = g.take<uint32_t>();
            x.kind = g.take<uint8_t>();
            g.take<uint16_t>();
            g.take<uint32_t>();
            g.take<uint32_t>();
            x.digest = g.take<uint64_t>();
            regions.push_back(x);
        }
        if (!(r.ok() && t.ok() && b.ok() && g.ok())) { why = "truncated tables"; return false; }
        return true;
    }
    const V4Tensor *find(const std::string &name) const {
        auto it = by_name.find(name);
        return it == by_name.end() ? nullptr : &tensors[it->second];
    }
    // bytes a region's digest covers: its tensors including each one's 64-byte alignment padding
    uint64_t digest_len(const V4Region &r) const {
        if (r.hi == 0 || r.hi > tensors.size()) return r.len;
        const V4Tensor &last = tensors[r.hi - 1];
        uint64_t end = last.off + last.nbytes;
        end += (64 - end % 64) % 64;
        return end - r.off;
    }
};

bool file_exists(const std::string &p) { return access(p.c_str(), R_OK) == 0; }

bool find_tokenizer(const char *model_path, const char *dir, std::string &out) {
    std::string mdir = model_path;
    const size_t slash = mdir.rfind('/');
    mdir = slash == std::string::npos ? std::string(".") : mdir.substr(0, slash);
    std::vector<std::string> cand;
    if (dir) cand.push_back(dir);
    else cand = {mdir + "/tokenizer", mdir, "weights"};
    for (const std::string &c : cand)
        if (file_exists(c + "/" + kTokFile) && file_exists(c + "/" + kUniFile)) { out = c; return true; }
    return false;
}

}  // namespace

struct cp_model {
    V4File f;
    int fd = -1;
    int L = 0, D = 0, V = 0, E = 0, K = 0, max_ctx = 0, hist = 0;
    long long file_bytes = 0;
    CpTokenizer tk{};
    bool tk_loaded = false, store_open = false;
    std::vector<cpg_moe_layer *> moe;
    cpg_qwen3 *model = nullptr;
    std::vector<int> turn;
};

extern "C" void cp_options_default(cp_options *opt) {
    memset(opt, 0, sizeof *opt);
    opt->budget_mb = CP_BUDGET_AUTO;
    opt->pin_cores = -1;
}

extern "C" void cp_close(cp_model *m) {
    if (!m) return;
    if (m->model) cpg_qwen3_destroy(m->model);
    for (cpg_moe_layer *l : m->moe) cpg_moe_layer_destroy(l);
    if (m->store_open) cpg_store_close();
    if (m->f.map) munmap(const_cast<uint8_t *>(m->f.map), m->f.size);
    if (m->fd >= 0) close(m->fd);
    if (m->tk_loaded) tokenizer_free(&m->tk);
    delete m;
}

static cp_model *open_fail(cp_model *m, char *err, size_t errlen, const char *fmt, const char *arg) {
    set_err(err, errlen, fmt, arg);
    cp_close(m);
    return nullptr;
}

extern "C" cp_model *cp_open(const char *model_path, const cp_options *opt_in, char *err, size_t errlen) {
    cp_options opt;
    if (opt_in) opt = *opt_in;
    else cp_options_default(&opt);
    if (g_opened) {
        set_err(err, errlen, "one model per process: the region store is process-global");
        return nullptr;
    }
    struct stat st;
    if (!model_path || stat(model_path, &st) != 0) {
        set_err(err, errlen, "cannot open model file %s", model_path ? model_path : "(null)");
        return nullptr;
    }
    std::string tdir;
    if (!find_tokenizer(model_path, opt.tokenizer_dir, tdir)) {
        set_err(err, errlen, "tokenizer files (%s, %s) not found %s%s", kTokFile, kUniFile,
                opt.tokenizer_dir ? "in " : "next to the model, in its tokenizer/ folder or in weights/",
                opt.tokenizer_dir ? opt.tokenizer_dir : "");
        return nullptr;
    }
    cp_model *m = new cp_model();
    m->max_ctx = opt.max_ctx > 0 ? opt.max_ctx : kDefaultCtx;
    m->file_bytes = (long long)st.st_size;
    if (tokenizer_qwen_load_unicode((tdir + "/" + kUniFile).c_str()) ||
        tokenizer_load(&m->tk, (tdir + "/" + kTokFile).c_str()))
        return open_fail(m, err, errlen, "cannot load tokenizer from %s", tdir.c_str());
    m->tk_loaded = true;
    g_opened = true;

    // the file: mapped read-only, tables walked, data section copied into HBM once
    m->fd = open(model_path, O_RDONLY);
    if (m->fd < 0) return open_fail(m, err, errlen, "cannot open model file %s", model_path);
    void *mp = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, m->fd, 0);
    if (mp == MAP_FAILED) return open_fail(m, err, errlen, "cannot map %s", model_path);
    m->f.map = static_cast<const uint8_t *>(mp);
    m->f.size = (size_t)st.st_size;
    std::string why;
    if (!m->f.parse(why)) return open_fail(m, err, errlen, "cannot map the model (%s)", why.c_str());
    V4File &f = m->f;
    if (cpg_store_open_v4(f.map, f.size, f.off_data) != CPG_OK)
        return open_fail(m, err, errlen, "region store: %s", cpg_last_error());
    m->store_open = true;
    for (size_t i = 0; i < f.regions.size(); ++i) {
        const V4Region &rg = f.regions[i];
        if (cpg_store_add_region(rg.off, rg.len, rg.kind == kRegionExpert) != (int)i)
            return open_fail(m, err, errlen, "region store: %s", cpg_last_error());
    }
    // every region's digest on the device (format/v4_writer.py:235-250)
    bool whole = true;
    std::vector<uint64_t> digests;
    for (const V4Region &rg : f.regions) {
        whole = whole && f.digest_len(rg) == rg.len;
        digests.push_back(rg.digest);
    }
    const uint8_t *base = static_cast<const uint8_t *>(cpg_store_base());
    if (whole) {
        int bad = -1;
        if (cpg_store_verify(digests.data(), (int)digests.size(), &bad) != CPG_OK)
            return open_fail(m, err, errlen, "region digest mismatch: %s", cpg_last_error());
    } else {
        for (const V4Region &rg : f.regions) {
            uint32_t crc = 0;
            if (cpg_crc32(base + rg.off, f.digest_len(rg), &crc, nullptr) != CPG_OK || crc != rg.digest)
                return open_fail(m, err, errlen, "region digest mismatch: %s", "a region's CRC-32 differs");
        }
    }

    // the model's shape (qwen3_map_ex) and its layers (qwen3_bind_layer)
    const V4Block *attn_blk = nullptr, *moe_blk = nullptr;
    for (const V4Block &b : f.blocks) {
        if (b.kind == kKindAttn && !attn_blk) attn_blk = &b;
        if (b.kind == kKindMoe && !moe_blk) moe_blk = &b;
    }
    m->L = f.n_layers;
    const V4Tensor *fn = f.find("final_norm"), *head = f.find("lm_head"), *wg0 = f.find("expert.0.0.Wg");
    if (!attn_blk || attn_blk->params.size() < 4 || m->L <= 0 || !fn || !head || !wg0)
        return open_fail(m, err, errlen, "cannot map %s (not a CPW1 v4 Qwen3 file?)", model_path);
    const int H = (int)attn_blk->params[0], KVH = (int)attn_blk->params[1], HD = (int)attn_blk->params[2];
    float theta;
    memcpy(&theta, &attn_blk->params[3], sizeof theta);
    m->D = (int)fn->dims[0];
    m->E = moe_blk && !moe_blk->params.empty() ? (int)moe_blk->params[0] : 0;
    if (m->E <= 0) {
        const V4Tensor *wg = f.find("Wgate.0");
        m->E = wg ? (int)wg->dims[0] : 0;
    }
    m->K = moe_blk && moe_blk->params.size() > 1 ? (int)moe_blk->params[1] : kTopK;
    const int F = (int)wg0->dims[0];
    // embed: one tensor, or row chunks embed.0, embed.1, ... back to back in the data section
    const V4Tensor *emb = f.find("embed");
    m->V = 0;
    if (emb) {
        m->V = (int)emb->dims[0];
    } else {
        for (int c = 0;; ++c) {
            const V4Tensor *ch = f.find("embed." + std::to_string(c));
            if (!ch) break;
            if (c == 0) emb = ch;
            else {
                const V4Tensor *prev = f.find("embed." + std::to_string(c - 1));
                if (prev->off + prev->nbytes != ch->off)
                    return open_fail(m, err, errlen, "%s: embed chunks are not contiguous", model_path);
            }
            m->V += (int)ch->dims[0];
        }
    }
    if (!emb || m->V <= 0) return open_fail(m, err, errlen, "%s: no embed table", model_path);
    auto dev = [&](const V4Tensor *t) { return static_cast<const void *>(base + t->off); };
    std::vector<cpg_qwen3_attn> attn((size_t)m->L);
    m->moe.assign((size_t)m->L, nullptr);
    for (int l = 0; l < m->L; ++l) {
        const std::string s = "." + std::to_string(l);
        const V4Tensor *ln1 = f.find("ln1" + s), *qn = f.find("q_norm" + s), *kn = f.find("k_norm" + s),
                       *wq = f.find("Wq" + s), *wk = f.find("Wk" + s), *wv = f.find("Wv" + s), *wo = f.find("Wo" + s),
                       *ln2 = f.find("ln2" + s), *wgate = f.find("Wgate" + s);
        if (!ln1 || !qn || !kn || !wq || !wk || !wv || !wo || !ln2 || !wgate)
            return open_fail(m, err, errlen, "bind layer %s failed", std::to_string(l).c_str());
        attn[l] = cpg_qwen3_attn{static_cast<const float *>(dev(ln1)), static_cast<const float *>(dev(qn)),
                                 static_cast<const float *>(dev(kn)), cpg_tensor{dev(wq), wq->enc},
                                 cpg_tensor{dev(wk), wk->enc}, cpg_tensor{dev(wv), wv->enc},
                                 cpg_tensor{dev(wo), wo->enc}};
        std::vector<cpg_tensor> ex((size_t)m->E * 3);
        static const char *kinds[3] = {"Wg", "Wu", "Wd"};
        for (int e = 0; e < m->E; ++e)
            for (int k = 0; k < 3; ++k) {
                const V4Tensor *t = f.find("expert" + s + "." + std::to_string(e) + "." + kinds[k]);
                if (!t) return open_fail(m, err, errlen, "bind layer %s failed (expert tensor)", std::to_string(l).c_str());
                ex[(size_t)e * 3 + k] = cpg_tensor{dev(t), t->enc};
            }
        cpg_moe_desc md{m->D, F, m->E, m->K, kEps, static_cast<const float *>(dev(ln2)),
                        cpg_tensor{dev(wgate), wgate->enc}, ex.data()};
        if (cpg_moe_layer_create(&md, &m->moe[l]) != CPG_OK)
            return open_fail(m, err, errlen, "bind layer: %s", cpg_last_error());
    }
    cpg_qwen3_desc qd{};
    qd.d_model = m->D;
    qd.n_heads = H;
    qd.n_kv = KVH;
    qd.head_dim = HD;
    qd.vocab = m->V;
    qd.n_layers = m->L;
    qd.max_ctx = m->max_ctx;
    qd.rope_theta = theta;
    qd.rms_eps = kEps;
    qd.embed = cpg_tensor{dev(emb), emb->enc};
    qd.lm_head = cpg_tensor{dev(head), head->enc};
    qd.final_norm = static_cast<const float *>(dev(fn));
    qd.attn = attn.data();
    qd.moe = m->moe.data();
    if (cpg_qwen3_create(&qd, &m->model) != CPG_OK)
        return open_fail(m, err, errlen, "model: %s", cpg_last_error());
    m->turn.resize((size_t)m->max_ctx);
    return m;
}

extern "C" void cp_reset(cp_model *m) {
    if (m) m->hist = 0;
}

extern "C" int cp_chat(cp_model *m, const char *user_msg, int max_new, cp_token_fn on_token, void *user,
                       cp_turn *out) {
    if (!m || !user_msg) return -1;
    cp_turn t;
    memset(&t, 0, sizeof t);
    const int MAX_CTX = m->max_ctx;
    if (m->hist > MAX_CTX - max_new - 64) {
        m->hist = 0;
        t.context_reset = 1;
    }
    // the turn's ChatML fragment, appended to the conversation (the same text as
    // cachepotato.c:332-334, so the same tokens)
    std::string prompt = "<|im_start|>user\n";
    prompt += user_msg;
    prompt += " /no_think<|im_end|>\n<|im_start|>assistant\n";
    const int Tn = tokenizer_qwen_encode(&m->tk, prompt.c_str(), m->turn.data(), MAX_CTX - m->hist - 8);
    if (Tn <= 0) return -2;
    const int pos0 = m->hist;
    m->hist += Tn;
    t.prompt_tokens = Tn;

    const double t0 = now_s();
    // the device cache holds positions [0, pos0) of this conversation (the model's position is
    // never behind hist): continue from there
    int next = 0;
    if (cpg_qwen3_rewind(m->model, pos0) != CPG_OK) return -3;
    if (cpg_qwen3_append(m->model, m->turn.data(), Tn, &next) != CPG_OK) return -3;
    const double t1 = now_s();
    int pos = m->hist, produced = 0, stop_req = 0, rc = 0;
    t.stop = CP_STOP_EOS;
    const double t2 = now_s();
    for (;;) {
        const int best = next;                          // greedy, first maximum (cachepotato.c:353-356)
        if (best == kImEnd) { t.stop = CP_STOP_EOS; break; }
        if (produced >= max_new) { t.stop = CP_STOP_MAX_TOKENS; break; }
        if (pos >= MAX_CTX - 1) { t.stop = CP_STOP_CONTEXT; break; }
        if (on_token && best >= 0 && (uint32_t)best < m->tk.n_vocab)
            stop_req = on_token(m->tk.vocab[best], m->tk.vocab_len[best], user);
        if (pos < MAX_CTX - 2) m->hist = pos + 1;
        // the emitted token always goes through the forward pass, even when the caller stops
        // here, so the cache holds every token hist counts
        if (cpg_qwen3_step(m->model, best, &next) != CPG_OK) { rc = -3; break; }
        ++pos;
        ++produced;
        if (stop_req) { t.stop = CP_STOP_CALLER; break; }
    }
    const double t3 = now_s();
    t.generated_tokens = produced;
    t.context_tokens = m->hist;
    t.prefill_s = t1 - t0;
    t.decode_s = t3 - t2;
    if (out) *out = t;
    return rc;
}

extern "C" void cp_get_stats(const cp_model *m, cp_stats *s) {
    memset(s, 0, sizeof *s);
    if (!m) return;
    s->n_layers = m->L;
    s->d_model = m->D;
    s->n_experts = m->E;
    s->topk = m->K;
    s->vocab = m->V;
    s->max_ctx = m->max_ctx;
    s->threads = 0;
    s->budget_mb = -1;
    s->file_bytes = m->file_bytes;
}

extern "C" int cp_physical_cores(void) {
    // distinct (physical id, core id) pairs of /proc/cpuinfo, else the online processors
    FILE *f = fopen("/proc/cpuinfo", "r");
    std::vector<std::pair<int, int>> seen;
    if (f) {
        char line[256];
        int pkg = 0;
        while (fgets(line, sizeof line, f)) {
            int v;
            if (sscanf(line, "physical id : %d", &v) == 1) pkg = v;
            else if (sscanf(line, "core id : %d", &v) == 1) {
                bool dup = false;
                for (const auto &p : seen) dup = dup || (p.first == pkg && p.second == v);
                if (!dup) seen.emplace_back(pkg, v);
            }
        }
        fclose(f);
    }
    if (!seen.empty()) return (int)seen.size();
    const long c = sysconf(_SC_NPROCESSORS_ONLN);
    return c > 0 ? (int)c : 1;
}

extern "C" long cp_mem_available_mb(void) {
    FILE *f = fopen("/proc/meminfo", "r");
    if (!f) return -1;
    char line[256];
    long kb = -1;
    while (fgets(line, sizeof line, f))
        if (sscanf(line, "MemAvailable: %ld kB", &kb) == 1) break;
    fclose(f);
    return kb < 0 ? -1 : kb / 1024;
}

extern "C" long cp_auto_budget_mb(long long model_file_bytes) {
    // MemAvailable less 2 GB of headroom, capped at the file, at least 2 GB (cachepotato.c:82-95)
    const long headroom_mb = 2048, min_mb = 2048;
    const long avail = cp_mem_available_mb();
    if (avail < 0) return -1;
    long b = avail - headroom_mb;
    const long file_mb = (long)(model_file_bytes / (1024 * 1024)) + 1;
    if (model_file_bytes > 0 && b > file_mb) b = file_mb;
    return b < min_mb ? -1 : b;
}
