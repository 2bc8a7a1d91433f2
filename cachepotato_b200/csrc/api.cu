// api.cu — the C ABI around the kernels: error reporting, the HBM region store (the pager's
// replacement), the kernels.h drop-ins with host pointers, and the host-buffer decode loop.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace cpg {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char *what) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? CPG_ENOMEM : CPG_ECUDA;
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

int smem_optin() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 227 * 1024;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || n <= 0)
            n = 227 * 1024;
        cached[dev] = n;
    }
    return cached[dev];
}

int allow_max_smem(const void *kernel) {
    cudaFuncAttributes fa;
    CPG_CUDA(cudaFuncGetAttributes(&fa, kernel));
    CPG_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  smem_optin() - (int)fa.sharedSizeBytes));
    return CPG_OK;
}

int matvec_launch(float *out, const float *x, cpg_tensor w, int n_in, int n_out, int T, cudaStream_t s);

// ------------------------------------------------------------------ region store
// One per process (the pager is process-global too, pager.c:195-214).
struct Region { size_t off, len; int is_expert; };
struct Store {
    std::mutex mu;
    uint8_t *dev = nullptr;          // device copy of the data section
    size_t bytes = 0;
    const uint8_t *host = nullptr;   // mirrored host range (map_base + data_off), or null
    std::vector<Region> regions;
    long h2d = 0;
};
static Store g_store;

static int store_alloc(size_t bytes) {
    if (g_store.dev) {
        set_error("region store already open (one per process, like the pager)");
        return CPG_ESTATE;
    }
    if (bytes == 0) bytes = 256;
    CPG_CUDA(cudaMalloc((void **)&g_store.dev, bytes));
    g_store.bytes = bytes;
    g_store.regions.clear();
    g_store.h2d = 0;
    return CPG_OK;
}

// Copy a host range to the device through two pinned bounce buffers on one stream, so the
// memcpy into one buffer overlaps the DMA out of the other (the source may be a file mapping,
// which cannot be registered as pinned memory in general).
static int upload(uint8_t *dst, const uint8_t *src, size_t bytes) {
    const size_t CH = 64u << 20;
    void *pin[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    cudaStream_t s = nullptr;
    int rc = CPG_OK;
    cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaMallocHost(&pin[i], CH);
    for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
    for (size_t o = 0, k = 0; e == cudaSuccess && o < bytes; o += CH, ++k) {
        const size_t n = bytes - o < CH ? bytes - o : CH;
        const int b = (int)(k & 1);
        if (k >= 2) e = cudaEventSynchronize(ev[b]);
        if (e != cudaSuccess) break;
        memcpy(pin[b], src + o, n);
        e = cudaMemcpyAsync(dst + o, pin[b], n, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaEventRecord(ev[b], s);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) rc = cuda_fail(e, "region store upload");
    for (int i = 0; i < 2; ++i) {
        if (ev[i]) cudaEventDestroy(ev[i]);
        if (pin[i]) cudaFreeHost(pin[i]);
    }
    if (s) cudaStreamDestroy(s);
    return rc;
}

// ------------------------------------------------------------------ context (decode loop)
}  // namespace cpg

struct cpg_ctx {
    int device = 0;
    int max_T = 0;
    int D = 0, K = 0;
    cudaStream_t stream = nullptr;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    float *x = nullptr;              // (max_T, D) device activations
    int *topk = nullptr;             // (L, max_T, K) device, grown on demand
    size_t topk_cap = 0;
    cudaGraphExec_t graph = nullptr; // cached decode graph
    std::vector<const cpg_moe_layer *> graph_layers;
    int graph_T = 0;
    bool graph_profiled = false;
    bool profile = false;            // record 5 events per layer inside the graph
    std::vector<cudaEvent_t> ev;     // (L, 5)
};

using namespace cpg;

extern "C" const char *cpg_last_error(void) { return g_err; }
extern "C" int cpg_version(void) { return 100; }

extern "C" int cpg_store_open(size_t bytes) {
    std::lock_guard<std::mutex> lk(g_store.mu);
    int rc = store_alloc(bytes);
    if (rc == CPG_OK) g_store.host = nullptr;
    return rc;
}

extern "C" int cpg_store_open_v4(const void *map_base, size_t map_len, size_t data_off) {
    CPG_REQUIRE(map_base && data_off <= map_len, "cpg_store_open_v4: bad mapping (len %zu, data_off %zu)", map_len, data_off);
    std::lock_guard<std::mutex> lk(g_store.mu);
    const size_t n = map_len - data_off;
    int rc = store_alloc(n);
    if (rc != CPG_OK) return rc;
    rc = upload(g_store.dev, (const uint8_t *)map_base + data_off, n);
    if (rc != CPG_OK) {
        cudaFree(g_store.dev);
        g_store.dev = nullptr;
        g_store.bytes = 0;
        return rc;
    }
    g_store.host = (const uint8_t *)map_base + data_off;
    g_store.h2d = (long)n;
    return CPG_OK;
}

extern "C" int cpg_store_add_region(size_t off, size_t len, int is_expert) {
    std::lock_guard<std::mutex> lk(g_store.mu);
    if (!g_store.dev) {
        set_error("cpg_store_add_region: store not open");
        return CPG_ESTATE;
    }
    CPG_REQUIRE(off <= g_store.bytes && len <= g_store.bytes - off,
                "cpg_store_add_region: region [%zu, +%zu) outside the %zu-byte store", off, len, g_store.bytes);
    g_store.regions.push_back(Region{off, len, is_expert});
    return (int)g_store.regions.size() - 1;
}

extern "C" const void *cpg_store_region_get(int id) {
    std::lock_guard<std::mutex> lk(g_store.mu);
    if (!g_store.dev || id < 0 || id >= (int)g_store.regions.size()) {
        set_error("cpg_store_region_get: no region %d", id);
        return nullptr;
    }
    return g_store.dev + g_store.regions[id].off;
}

extern "C" const void *cpg_store_translate(const void *host_ptr) {
    std::lock_guard<std::mutex> lk(g_store.mu);
    const uint8_t *p = (const uint8_t *)host_ptr;
    if (!g_store.host || p < g_store.host || p >= g_store.host + g_store.bytes) return nullptr;
    return g_store.dev + (p - g_store.host);
}

extern "C" void *cpg_store_base(void) { return g_store.dev; }
extern "C" size_t cpg_store_bytes(void) { return g_store.bytes; }

extern "C" int cpg_store_totals(cpg_store_totals_t *out) {
    CPG_REQUIRE(out, "cpg_store_totals: null");
    std::lock_guard<std::mutex> lk(g_store.mu);
    memset(out, 0, sizeof *out);
    out->regions = (long)g_store.regions.size();
    for (const Region &r : g_store.regions) out->expert_regions += r.is_expert ? 1 : 0;
    out->resident_bytes = (long)g_store.bytes;
    out->h2d_bytes = g_store.h2d;
    return CPG_OK;
}

namespace cpg {
int crc32_regions(const std::vector<const uint8_t *> &base, const std::vector<unsigned long long> &len,
                  uint32_t *out, cudaStream_t s);
}

// The v4 loader's digest check (format/v4_writer.py:235-250 writes zlib.crc32 of each region's
// bytes as a u64; the loader compares at open): every region's CRC-32 computed in HBM.
extern "C" int cpg_store_verify(const uint64_t *digests, int n, int *first_bad) {
    CPG_REQUIRE(digests || n == 0, "cpg_store_verify: null digests");
    if (first_bad) *first_bad = -1;
    std::lock_guard<std::mutex> lk(g_store.mu);
    if (!g_store.dev) {
        set_error("cpg_store_verify: store not open");
        return CPG_ESTATE;
    }
    CPG_REQUIRE(n == (int)g_store.regions.size(), "cpg_store_verify: %d digests for %zu regions", n,
                g_store.regions.size());
    std::vector<const uint8_t *> b(n);
    std::vector<unsigned long long> l(n);
    for (int i = 0; i < n; ++i) {
        b[i] = g_store.dev + g_store.regions[i].off;
        l[i] = g_store.regions[i].len;
    }
    std::vector<uint32_t> crc(n > 0 ? n : 1);
    const int rc = crc32_regions(b, l, crc.data(), nullptr);
    if (rc != CPG_OK) return rc;
    for (int i = 0; i < n; ++i) {
        if ((uint64_t)crc[i] != digests[i]) {
            if (first_bad) *first_bad = i;
            set_error("cpg_store_verify: region %d: CRC-32 %08x, file digest %016llx", i, crc[i],
                      (unsigned long long)digests[i]);
            return CPG_EINVAL;
        }
    }
    return CPG_OK;
}

extern "C" void cpg_store_close(void) {
    std::lock_guard<std::mutex> lk(g_store.mu);
    if (g_store.dev) cudaFree(g_store.dev);
    g_store.dev = nullptr;
    g_store.bytes = 0;
    g_store.host = nullptr;
    g_store.regions.clear();
    g_store.h2d = 0;
}

// ------------------------------------------------------------------ kernels.h drop-ins
namespace {

// Resolve `w` (host) to device memory: the store's resident copy when `w` lies in the mirrored
// mapping, otherwise a temporary upload of the rows this call reads.
struct DevWeights {
    const void *dev = nullptr;
    void *owned = nullptr;
    ~DevWeights() { if (owned) cudaFree(owned); }
};

int resolve(const void *w, size_t bytes, DevWeights &out) {
    if (const void *d = cpg_store_translate(w)) {
        const uint8_t *h = (const uint8_t *)w;
        if (h + bytes <= g_store.host + g_store.bytes) { out.dev = d; return CPG_OK; }
    }
    CPG_CUDA(cudaMalloc(&out.owned, bytes));
    CPG_CUDA(cudaMemcpy(out.owned, w, bytes, cudaMemcpyHostToDevice));
    out.dev = out.owned;
    return CPG_OK;
}

int host_matvec(float *out, const float *x, const void *w, int enc, int n_in, int n_out) {
    g_err[0] = 0;                    // void drop-ins: an empty message after the call = success
    CPG_REQUIRE(out && x && w && n_in > 0 && n_out > 0, "matmul_wx: bad arguments");
    DevWeights dw;
    int rc = resolve(w, (size_t)row_bytes(enc, n_in) * n_out, dw);
    if (rc) return rc;
    float *dx = nullptr, *dy = nullptr;
    CPG_CUDA(cudaMalloc(&dx, sizeof(float) * n_in));
    cudaError_t e = cudaMalloc(&dy, sizeof(float) * n_out);
    if (e == cudaSuccess) e = cudaMemcpy(dx, x, sizeof(float) * n_in, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        rc = matvec_launch(dy, dx, cpg_tensor{dw.dev, enc}, n_in, n_out, 1, nullptr);
        if (rc == CPG_OK) e = cudaMemcpy(out, dy, sizeof(float) * n_out, cudaMemcpyDeviceToHost);
    }
    cudaFree(dx);
    cudaFree(dy);
    if (e != cudaSuccess) return cuda_fail(e, "matmul_wx");
    return rc;
}

int host_dequant(const uint8_t *blocks, float *out, int n, int enc) {
    g_err[0] = 0;
    CPG_REQUIRE(blocks && out && n >= 0 && n % 32 == 0, "dequant_row: bad arguments");
    if (n == 0) return CPG_OK;
    DevWeights dw;
    int rc = resolve(blocks, (size_t)(n / 32) * group_bytes(enc), dw);
    if (rc) return rc;
    float *dy = nullptr;
    CPG_CUDA(cudaMalloc(&dy, sizeof(float) * n));
    rc = cpg_dequant(dy, (const uint8_t *)dw.dev, enc, n, nullptr);
    cudaError_t e = rc == CPG_OK ? cudaMemcpy(out, dy, sizeof(float) * n, cudaMemcpyDeviceToHost) : cudaSuccess;
    cudaFree(dy);
    if (e != cudaSuccess) return cuda_fail(e, "dequant_row");
    return rc;
}

void report(int rc, const char *fn) {
    if (rc != CPG_OK) fprintf(stderr, "%s: %s\n", fn, cpg_last_error());
}

}  // namespace

extern "C" void cpg_matmul_wx(float *out, const float *x, const float *w, int n_in, int n_out) {
    report(host_matvec(out, x, w, CPG_ENC_F32, n_in, n_out), "cpg_matmul_wx");
}
extern "C" void cpg_matmul_wx_q8(float *out, const float *x, const uint8_t *w, int n_in, int n_out) {
    report(host_matvec(out, x, w, CPG_ENC_Q8, n_in, n_out), "cpg_matmul_wx_q8");
}
extern "C" void cpg_matmul_wx_q4(float *out, const float *x, const uint8_t *w, int n_in, int n_out) {
    report(host_matvec(out, x, w, CPG_ENC_Q4, n_in, n_out), "cpg_matmul_wx_q4");
}
extern "C" void cpg_q8_dequant_row(const uint8_t *blocks, float *out, int n) {
    report(host_dequant(blocks, out, n, CPG_ENC_Q8), "cpg_q8_dequant_row");
}
extern "C" void cpg_q4_dequant_row(const uint8_t *blocks, float *out, int n) {
    report(host_dequant(blocks, out, n, CPG_ENC_Q4), "cpg_q4_dequant_row");
}

// ------------------------------------------------------------------ decode loop
namespace cpg {
int layer_dims(const cpg_moe_layer *L, int *D, int *F, int *E, int *K);
int moe_forward_impl(const cpg_moe_layer *L, const float *x, const float *attn, int T, float *mlp,
                     float *x_out, int *topk_idx, float *wt, float *router, void *ws, size_t ws_bytes,
                     cudaStream_t s, cudaEvent_t *ev);
}

extern "C" int cpg_ctx_create(int device, int max_T, const cpg_moe_layer *shape, cpg_ctx **out) {
    CPG_REQUIRE(out && shape && max_T > 0, "cpg_ctx_create: bad arguments");
    *out = nullptr;
    CPG_CUDA(cudaSetDevice(device));
    int D, F, E, K;
    int rc = cpg::layer_dims(shape, &D, &F, &E, &K);
    if (rc) return rc;
    cpg_ctx *c = new cpg_ctx();
    c->device = device;
    c->max_T = max_T;
    c->D = D;
    c->K = K;
    c->ws_bytes = cpg_moe_workspace_bytes(shape, max_T);
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&c->ws, c->ws_bytes);
    if (e == cudaSuccess) e = cudaMemset(c->ws, 0, c->ws_bytes);
    if (e == cudaSuccess) e = cudaMalloc((void **)&c->x, sizeof(float) * (size_t)max_T * D);
    if (e != cudaSuccess) {
        cpg_ctx_destroy(c);
        return cuda_fail(e, "cpg_ctx_create");
    }
    *out = c;
    return CPG_OK;
}

extern "C" void cpg_ctx_destroy(cpg_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->graph) cudaGraphExecDestroy(c->graph);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (cudaEvent_t e : c->ev) cudaEventDestroy(e);
    cudaFree(c->ws);
    cudaFree(c->x);
    cudaFree(c->topk);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

extern "C" void *cpg_ctx_stream(cpg_ctx *c) { return c ? (void *)c->stream : nullptr; }

static int enqueue_layers(cpg_ctx *c, cpg_moe_layer *const *layers, int L, int T) {
    for (int l = 0; l < L; ++l) {
        int *tk = c->topk ? c->topk + (size_t)l * T * c->K : nullptr;
        int rc = moe_forward_impl(layers[l], c->x, nullptr, T, nullptr, c->x, tk, nullptr, nullptr,
                                  c->ws, c->ws_bytes, c->stream, c->profile ? &c->ev[(size_t)l * 5] : nullptr);
        if (rc) return rc;
    }
    return CPG_OK;
}

// Make sure the cached graph runs exactly these layers at this T (re-capture otherwise).
static int prepare_graph(cpg_ctx *c, cpg_moe_layer *const *layers, int L, int T) {
    CPG_REQUIRE(c && layers && L > 0 && T > 0 && T <= c->max_T, "decode loop: bad arguments (T=%d, L=%d)", T, L);
    CPG_CUDA(cudaSetDevice(c->device));
    const size_t need_topk = (size_t)L * T * c->K;
    if (c->topk_cap < need_topk) {
        if (c->graph) { cudaGraphExecDestroy(c->graph); c->graph = nullptr; }
        cudaFree(c->topk);
        c->topk = nullptr;
        c->topk_cap = 0;
        CPG_CUDA(cudaMalloc((void **)&c->topk, sizeof(int) * need_topk));
        c->topk_cap = need_topk;
    }
    if (c->profile && c->ev.size() < (size_t)L * 5) {
        if (c->graph) { cudaGraphExecDestroy(c->graph); c->graph = nullptr; }
        while (c->ev.size() < (size_t)L * 5) {
            cudaEvent_t e;
            CPG_CUDA(cudaEventCreate(&e));
            c->ev.push_back(e);
        }
    }
    bool same = c->graph && c->graph_T == T && (int)c->graph_layers.size() == L && c->graph_profiled == c->profile;
    for (int l = 0; same && l < L; ++l) same = c->graph_layers[l] == layers[l];
    if (same) return CPG_OK;
    if (c->graph) { cudaGraphExecDestroy(c->graph); c->graph = nullptr; }
    cudaGraph_t g = nullptr;
    CPG_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_layers(c, layers, L, T);
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (rc) { if (g) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return cuda_fail(e, "decode graph capture");
    e = cudaGraphInstantiate(&c->graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { c->graph = nullptr; return cuda_fail(e, "decode graph instantiate"); }
    c->graph_layers.assign(layers, layers + L);
    c->graph_T = T;
    c->graph_profiled = c->profile;
    return CPG_OK;
}

extern "C" int cpg_run_moe_layers(cpg_ctx *c, cpg_moe_layer *const *layers, int L, float *x, int T,
                                  int *topk_out) {
    CPG_REQUIRE(x, "cpg_run_moe_layers: null x");
    int rc = prepare_graph(c, layers, L, T);
    if (rc) return rc;
    const size_t xb = sizeof(float) * (size_t)T * c->D;
    CPG_CUDA(cudaMemcpyAsync(c->x, x, xb, cudaMemcpyHostToDevice, c->stream));
    CPG_CUDA(cudaGraphLaunch(c->graph, c->stream));
    CPG_CUDA(cudaMemcpyAsync(x, c->x, xb, cudaMemcpyDeviceToHost, c->stream));
    if (topk_out)
        CPG_CUDA(cudaMemcpyAsync(topk_out, c->topk, sizeof(int) * (size_t)L * T * c->K,
                                 cudaMemcpyDeviceToHost, c->stream));
    return cpg_moe_check(c->ws, c->stream);
}

extern "C" int cpg_ctx_run(cpg_ctx *c, cpg_moe_layer *const *layers, int L, int T) {
    int rc = prepare_graph(c, layers, L, T);
    if (rc) return rc;
    CPG_CUDA(cudaGraphLaunch(c->graph, c->stream));
    return CPG_OK;
}

extern "C" float *cpg_ctx_x(cpg_ctx *c) { return c ? c->x : nullptr; }
extern "C" int *cpg_ctx_topk(cpg_ctx *c) { return c ? c->topk : nullptr; }

extern "C" int cpg_ctx_profile(cpg_ctx *c, int enable) {
    CPG_REQUIRE(c, "cpg_ctx_profile: null context");
    c->profile = enable != 0;
    return CPG_OK;
}

extern "C" int cpg_ctx_phase_ms(cpg_ctx *c, float *ms4) {
    CPG_REQUIRE(c && ms4, "cpg_ctx_phase_ms: null argument");
    CPG_REQUIRE(c->graph && c->graph_profiled, "cpg_ctx_phase_ms: the last decode graph was not profiled");
    CPG_CUDA(cudaStreamSynchronize(c->stream));
    for (int p = 0; p < 4; ++p) ms4[p] = 0.0f;
    for (size_t l = 0; l < c->graph_layers.size(); ++l)
        for (int p = 0; p < 4; ++p) {
            float ms = 0.0f;
            CPG_CUDA(cudaEventElapsedTime(&ms, c->ev[l * 5 + p], c->ev[l * 5 + p + 1]));
            ms4[p] += ms;
        }
    return CPG_OK;
}
