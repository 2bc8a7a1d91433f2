// noalloc.cu — the MoE block without a caller workspace, for callers that cannot allocate.
//
// Some callers of this library cannot call cudaMalloc at the point where they run the MoE
// block: a C engine embedded in a host program that owns every byte of device memory through
// its own pool, or a latency-critical decode loop that may not stall on the allocator. cpg_moe_forward_noalloc serves them from a scratch array that is part
// of the library's own device image: nothing is allocated per call.
//
// The array is fixed in size (kStaticScratchBytes, 8 MiB: 64 tokens of a Qwen3-30B-A3B layer
// need about 6.3 MB), every GPU that loads the library holds it until the process exits, and all
// calls share it.
#include <mutex>

#include "common.cuh"

namespace cpg {

int moe_forward_impl(const cpg_moe_layer *L, const float *x, const float *attn, int T, float *mlp,
                     float *x_out, int *topk_idx, float *wt, float *router, void *ws, size_t ws_bytes,
                     cudaStream_t s, cudaEvent_t *ev);

constexpr size_t kStaticScratchBytes = 8u << 20;

// Device-side scratch. In host code this name is only a stand-in for the symbol, not a device
// address: the address is looked up with cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
static void *g_scratch_addr[kMaxDevices];
static std::mutex g_scratch_mu;

// Device address of the scratch array on the current device, looked up once per device.
static int static_scratch(void **out) {
    int dev = 0;
    CPG_CUDA(cudaGetDevice(&dev));
    CPG_REQUIRE(dev >= 0 && dev < kMaxDevices, "cpg_moe_forward_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        CPG_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return CPG_OK;
}

}  // namespace cpg

using namespace cpg;

extern "C" int cpg_moe_forward_noalloc(const cpg_moe_layer *layer, const float *x, const float *attn,
                                       int T, float *mlp, float *x_out, int *topk_idx, float *wt,
                                       float *router, void *stream) {
    CPG_REQUIRE(layer && T > 0, "cpg_moe_forward_noalloc: null layer or T=%d", T);
    const size_t need = cpg_moe_workspace_bytes(layer, T);
    CPG_REQUIRE(need > 0 && need <= kStaticScratchBytes,
                "cpg_moe_forward_noalloc: T=%d needs %zu bytes of scratch, the built-in scratch holds %zu "
                "(use cpg_moe_forward with a caller workspace for larger batches)",
                T, need, kStaticScratchBytes);
    void *ws = nullptr;
    const int rc = static_scratch(&ws);
    if (rc) return rc;
    return moe_forward_impl(layer, x, attn, T, mlp, x_out, topk_idx, wt, router, ws, kStaticScratchBytes,
                            (cudaStream_t)stream, nullptr);
}
