// ep.cu — expert parallelism for batched MoE layers across the GPUs of one node.
//
// The reference engine has no counterpart (it runs the expert loop token by token on one host,
// engine/blocks/qwen3_moe.c:199-222); the layout follows the partitioning the batched configs
// call for: rank r owns experts [r·E_l, (r+1)·E_l) (E_l = n_experts of its local layer) and T
// tokens of the batch (the same T on every rank). Per layer:
//   k_ep_plan       per owner: which local tokens have a slot there, their position in the send
//                   buffer (tokens ascending), and per-slot metadata (local expert id or -1, weight)
//   k_ep_pack_rows  each token's normalised row as fp16, once per owner that needs it
//   NCCL            send/recv of rows + metadata to every owner (fixed capacity of T rows per
//                   peer, so no counts round trip and no host synchronisation)
//   apply_rows      the owner's tcgen05 grouped GEMMs over all received rows; each row's slots
//                   combined in selection order into one f32 partial row
//   NCCL            the partial rows back to their sources
//   k_ep_combine    mlp[t] += the partial rows of t's owners, ascending owner rank
// NCCL comes from the process (a torch process already holds it) or from the system library,
// resolved at run time, so the library itself links no NCCL.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <mutex>

#include "common.cuh"

namespace cpg {

int layer_dims(const cpg_moe_layer *L, int *D, int *F, int *E, int *K);

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;   // optional: non-blocking init
    decltype(&ncclCommGetAsyncError) async_error = nullptr;          // optional
    decltype(&ncclCommAbort) abort = nullptr;                        // optional
    decltype(&ncclCommFinalize) finalize = nullptr;                  // optional
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclGetErrorString) err_str = nullptr;
    bool ok = false;
};

static const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
        api.init_rank = (decltype(api.init_rank))dlsym(h, "ncclCommInitRank");
        api.init_rank_config = (decltype(api.init_rank_config))dlsym(h, "ncclCommInitRankConfig");
        api.async_error = (decltype(api.async_error))dlsym(h, "ncclCommGetAsyncError");
        api.abort = (decltype(api.abort))dlsym(h, "ncclCommAbort");
        api.finalize = (decltype(api.finalize))dlsym(h, "ncclCommFinalize");
        api.destroy = (decltype(api.destroy))dlsym(h, "ncclCommDestroy");
        api.group_start = (decltype(api.group_start))dlsym(h, "ncclGroupStart");
        api.group_end = (decltype(api.group_end))dlsym(h, "ncclGroupEnd");
        api.send = (decltype(api.send))dlsym(h, "ncclSend");
        api.recv = (decltype(api.recv))dlsym(h, "ncclRecv");
        api.err_str = (decltype(api.err_str))dlsym(h, "ncclGetErrorString");
        api.ok = api.get_unique_id && api.init_rank && api.destroy && api.group_start && api.group_end && api.send &&
                 api.recv && api.err_str;
    });
    return api;
}

#define CPG_NCCL(call)                                                                            \
    do {                                                                                          \
        const ncclResult_t r_ = (call);                                                           \
        if (r_ != ncclSuccess && r_ != ncclInProgress) {                                          \
            ::cpg::set_error("%s: %s", #call, nccl().err_str(r_));                                \
            return CPG_ENCCL;                                                                     \
        }                                                                                         \
    } while (0)

constexpr int EP_PLAN_THREADS = 1024;
constexpr int EP_MAX_K = 32;

// One message per peer and direction. Out: T records of RS bytes per owner, record q =
// [fp16 row (D halves) | K local expert ids | K weights | padding to 16 B]; back: T f32 rows.
struct EpWs {
    size_t status, send, recv, pos, out_rows, back, apply, total;
    size_t rs;                              // record bytes
};

static size_t al(size_t v) { return (v + 255) / 256 * 256; }

static EpWs ep_layout(int G, int T, int D, int K, size_t apply_bytes) {
    EpWs w{};
    size_t o = 0;
    const size_t R = (size_t)G * T;
    w.rs = ((size_t)D * sizeof(__half) + (size_t)K * 8 + 15) / 16 * 16;
    w.status = o; o = al(o + 16 * sizeof(int));
    w.send = o; o = al(o + R * w.rs);
    w.recv = o; o = al(o + R * w.rs);
    w.pos = o; o = al(o + (size_t)T * G * sizeof(int));
    w.out_rows = o; o = al(o + R * D * sizeof(float));
    w.back = o; o = al(o + R * D * sizeof(float));
    w.apply = o; o = al(o + apply_bytes);
    w.total = o;
    return w;
}

// Block-wide exclusive scan of 0/1 flags (EP_PLAN_THREADS threads); returns the prefix of this
// thread and writes the block total to *total.
__device__ __forceinline__ int block_excl_scan(int flag, int *s_warp, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const unsigned ball = __ballot_sync(0xffffffffu, flag);
    const int in_warp = __popc(ball & ((1u << lane) - 1u));
    if (lane == 0) s_warp[warp] = __popc(ball);
    __syncthreads();
    if (warp == 0) {
        int v = lane < nw ? s_warp[lane] : 0;
        int inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += n;
        }
        if (lane < nw) s_warp[lane] = inc - v;
        if (lane == 31) s_warp[32] = inc;
    }
    __syncthreads();
    const int r = s_warp[warp] + in_warp;
    *total = s_warp[32];
    __syncthreads();
    return r;
}

// One block per owner rank p: send positions (tokens ascending) and per-slot metadata into the
// records' tails (record r of the out buffer at send + r·rs; ids at byte 2D, weights after them).
__global__ void __launch_bounds__(EP_PLAN_THREADS) k_ep_plan(int T, int K, int G, int E_l, int D, const int *__restrict__ idx,
                                                              const float *__restrict__ wt, int *__restrict__ pos,
                                                              uint8_t *__restrict__ send, size_t rs, int *status) {
    __shared__ int s_warp[33];
    const int p = blockIdx.x;
    const int E_tot = E_l * G;
    int base = 0;
    for (int t0 = 0; t0 < T; t0 += blockDim.x) {
        const int t = t0 + threadIdx.x;
        int flag = 0;
        if (t < T)
            for (int j = 0; j < K; ++j) {
                const int e = idx[(size_t)t * K + j];
                if (e < 0 || e >= E_tot) {
                    if (p == 0) atomicExch(status, ST_BAD_ITEM);
                    continue;
                }
                flag |= (e / E_l == p);
            }
        int tot;
        const int r = block_excl_scan(flag, s_warp, &tot);
        if (t < T) {
            const int q = base + r;
            pos[(size_t)t * G + p] = flag ? q : -1;
            if (flag) {
                uint8_t *rec = send + ((size_t)p * T + q) * rs + (size_t)D * sizeof(__half);
                int *ide = reinterpret_cast<int *>(rec);
                float *w8 = reinterpret_cast<float *>(rec) + K;
                for (int j = 0; j < K; ++j) {
                    const int e = idx[(size_t)t * K + j];
                    const bool mine = e >= 0 && e < E_tot && e / E_l == p;
                    ide[j] = mine ? e - p * E_l : -1;
                    w8[j] = mine ? wt[(size_t)t * K + j] : 0.0f;
                }
            }
        }
        base += tot;
    }
    // capacity rows past the last token carry no slots
    for (size_t i = (size_t)base * K + threadIdx.x; i < (size_t)T * K; i += blockDim.x) {
        uint8_t *rec = send + ((size_t)p * T + i / K) * rs + (size_t)D * sizeof(__half);
        reinterpret_cast<int *>(rec)[i % K] = -1;
        reinterpret_cast<float *>(rec)[K + i % K] = 0.0f;
    }
}

// One warp per token: its row as fp16 into the record of every owner that needs it.
__global__ void __launch_bounds__(256) k_ep_pack_rows(int T, int D, int G, const float *__restrict__ xn,
                                                       const int *__restrict__ pos, uint8_t *__restrict__ send, size_t rs) {
    const int lane = threadIdx.x & 31;
    for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < T; t += (gridDim.x * blockDim.x) >> 5) {
        const float4 *src = reinterpret_cast<const float4 *>(xn + (size_t)t * D);
        for (int i = lane; i < D / 8; i += 32) {
            const float4 a = src[2 * i], b = src[2 * i + 1];
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
            const uint4 v = make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                                       *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
            for (int p = 0; p < G; ++p) {
                const int q = __ldg(pos + (size_t)t * G + p);
                if (q >= 0) reinterpret_cast<uint4 *>(send + ((size_t)p * T + q) * rs)[i] = v;
            }
        }
    }
}

// mlp[t] += partial rows of t's owners in ascending owner rank (one rounding per add).
__global__ void __launch_bounds__(256) k_ep_combine(int T, int D, int G, const int *__restrict__ pos,
                                                     const float *__restrict__ back, float *mlp) {
    const int n4 = T * D / 4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        const int t = (i * 4) / D, k = i * 4 - t * D;
        float4 acc = reinterpret_cast<const float4 *>(mlp)[i];
        for (int p = 0; p < G; ++p) {
            const int q = __ldg(pos + (size_t)t * G + p);
            if (q < 0) continue;
            const float4 v = __ldg(reinterpret_cast<const float4 *>(back + ((size_t)p * T + q) * D + k));
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        reinterpret_cast<float4 *>(mlp)[i] = acc;
    }
}

}  // namespace cpg

struct cpg_ep {
    int G, rank, device;
    ncclComm_t comm;
    bool nonblocking;      // communicator created with config.blocking = 0
    bool aborted;          // ncclCommAbort was called: every later call fails with CPG_ENCCL
    int timeout_ms;        // host deadline for NCCL's asynchronous steps (init, group launch, wait)
};

using namespace cpg;

namespace cpg {

// Monotonic milliseconds.
static double now_ms() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

// Abort the communicator (NCCL stops its kernels in flight and frees the communicator); every
// later call on this handle returns CPG_ENCCL. Peers blocked on this rank see their own
// collectives fail or time out instead of waiting for ever.
static void ep_abort(cpg_ep *ep) {
    if (ep->aborted) return;
    ep->aborted = true;
    if (nccl().abort) nccl().abort(ep->comm);
}

// A non-blocking communicator finishes init and group launches in the background: poll its
// state until it leaves ncclInProgress, giving up (and aborting) at the host deadline.
static int ep_settle(cpg_ep *ep, const char *what) {
    if (!ep->nonblocking || !nccl().async_error) return CPG_OK;
    const double t0 = now_ms();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = nccl().async_error(ep->comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return CPG_OK;
        if (st != ncclInProgress) {
            set_error("%s: %s", what, nccl().err_str(st));
            ep_abort(ep);
            return CPG_ENCCL;
        }
        const double waited = now_ms() - t0;
        if (waited > ep->timeout_ms) {
            set_error("%s: not complete after %d ms (communicator aborted)", what, ep->timeout_ms);
            ep_abort(ep);
            return CPG_ETIMEOUT;
        }
        // the stream's next work waits for this: poll without sleeping for the first 2 ms (a
        // sleep overshoots by tens of microseconds, which the GPU would idle), then back off
        if (waited > 2.0) {
            const timespec ns = {0, 20000};
            nanosleep(&ns, nullptr);
        }
    }
}

// One grouped send/recv round. On any failure the group is still closed (a group left open
// would swallow the caller's next NCCL calls) and the communicator is aborted, so no peer keeps
// waiting on a transfer this rank will never post.
struct P2P { void *buf; size_t count; ncclDataType_t type; int peer; bool send; };
static int ep_group(cpg_ep *ep, const P2P *ops, int n, cudaStream_t s, const char *what) {
    const NcclApi &api = nccl();
    ncclResult_t r = api.group_start();
    int failed = -1;
    if (r == ncclSuccess || r == ncclInProgress) {
        for (int i = 0; i < n; ++i) {
            r = ops[i].send ? api.send(ops[i].buf, ops[i].count, ops[i].type, ops[i].peer, ep->comm, s)
                            : api.recv(ops[i].buf, ops[i].count, ops[i].type, ops[i].peer, ep->comm, s);
            if (r != ncclSuccess && r != ncclInProgress) { failed = i; break; }
        }
    }
    const ncclResult_t re = api.group_end();
    if (failed >= 0 || (r != ncclSuccess && r != ncclInProgress) || (re != ncclSuccess && re != ncclInProgress)) {
        set_error("%s: %s", what, api.err_str(failed >= 0 || (r != ncclSuccess && r != ncclInProgress) ? r : re));
        ep_abort(ep);
        return CPG_ENCCL;
    }
    return ep_settle(ep, what);
}

static int ep_timeout_default() {
    const char *e = getenv("CPG_EP_TIMEOUT_MS");
    const int v = e ? atoi(e) : 0;
    return v > 0 ? v : 120000;
}

}  // namespace cpg

extern "C" int cpg_ep_unique_id(void *out) {
    CPG_REQUIRE(out, "cpg_ep_unique_id: null output");
    if (!nccl().ok) {
        set_error("NCCL is not available (libnccl.so.2 not found in the process or on the library path)");
        return CPG_ENCCL;
    }
    ncclUniqueId id;
    CPG_NCCL(nccl().get_unique_id(&id));
    memcpy(out, &id, sizeof(id));
    return CPG_OK;
}

extern "C" int cpg_ep_create(int nranks, int rank, const void *unique_id, cpg_ep **out) {
    CPG_REQUIRE(out && unique_id, "cpg_ep_create: null argument");
    *out = nullptr;
    CPG_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, "cpg_ep_create: rank %d of %d", rank, nranks);
    if (!nccl().ok) {
        set_error("NCCL is not available (libnccl.so.2 not found in the process or on the library path)");
        return CPG_ENCCL;
    }
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof(id));
    cpg_ep *ep = new cpg_ep();
    ep->G = nranks;
    ep->rank = rank;
    ep->timeout_ms = ep_timeout_default();
    cudaGetDevice(&ep->device);
    ncclResult_t r;
    if (nccl().init_rank_config && nccl().async_error && nccl().abort) {
        // non-blocking: a peer that never joins ends in CPG_ETIMEOUT here, not a hung process
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        r = nccl().init_rank_config(&ep->comm, nranks, id, rank, &cfg);
        ep->nonblocking = true;
    } else {
        r = nccl().init_rank(&ep->comm, nranks, id, rank);
    }
    if (r != ncclSuccess && r != ncclInProgress) {
        set_error("ncclCommInitRank: %s", nccl().err_str(r));
        if (ep->nonblocking && ep->comm) nccl().abort(ep->comm);
        delete ep;
        return CPG_ENCCL;
    }
    const int rc = ep_settle(ep, "ncclCommInitRankConfig");
    if (rc) {
        delete ep;          // ep_settle aborted (and freed) the communicator
        return rc;
    }
    *out = ep;
    return CPG_OK;
}

extern "C" void cpg_ep_destroy(cpg_ep *ep) {
    if (!ep) return;
    if (!ep->aborted) {
        if (ep->nonblocking) {
            // finish outstanding work first (bounded), then free; a stuck peer ends in an abort
            bool ok = ep_settle(ep, "cpg_ep_destroy") == CPG_OK;
            if (ok && nccl().finalize) {
                const ncclResult_t r = nccl().finalize(ep->comm);
                ok = (r == ncclSuccess || r == ncclInProgress) && ep_settle(ep, "ncclCommFinalize") == CPG_OK;
                if (!ok) ep_abort(ep);
            }
            if (ok) nccl().destroy(ep->comm);
        } else {
            nccl().destroy(ep->comm);
        }
    }
    delete ep;
}

extern "C" int cpg_ep_abort(cpg_ep *ep) {
    CPG_REQUIRE(ep, "cpg_ep_abort: null handle");
    ep_abort(ep);
    return CPG_OK;
}

extern "C" int cpg_ep_set_timeout(cpg_ep *ep, int timeout_ms) {
    CPG_REQUIRE(ep && timeout_ms > 0, "cpg_ep_set_timeout: null handle or timeout %d ms", timeout_ms);
    ep->timeout_ms = timeout_ms;
    return CPG_OK;
}

extern "C" int cpg_ep_wait(cpg_ep *ep, void *stream) {
    CPG_REQUIRE(ep, "cpg_ep_wait: null handle");
    if (ep->aborted) {
        set_error("cpg_ep_wait: the communicator was aborted");
        return CPG_ENCCL;
    }
    cudaStream_t s = (cudaStream_t)stream;
    const double t0 = now_ms();
    for (;;) {
        const cudaError_t ce = cudaStreamQuery(s);
        if (ce == cudaSuccess) return ep_settle(ep, "cpg_ep_wait");
        if (ce != cudaErrorNotReady) return cuda_fail(ce, "cpg_ep_wait: stream");
        if (nccl().async_error) {
            ncclResult_t st = ncclSuccess;
            nccl().async_error(ep->comm, &st);
            if (st != ncclSuccess && st != ncclInProgress) {
                set_error("cpg_ep_wait: %s (communicator aborted)", nccl().err_str(st));
                ep_abort(ep);
                return CPG_ENCCL;
            }
        }
        if (now_ms() - t0 > ep->timeout_ms) {
            // a peer stopped taking part: abort, which ends this rank's NCCL kernels in flight
            set_error("cpg_ep_wait: stream not done after %d ms (communicator aborted)", ep->timeout_ms);
            ep_abort(ep);
            return CPG_ETIMEOUT;
        }
        const timespec ns = {0, 50000};
        nanosleep(&ns, nullptr);
    }
}

extern "C" size_t cpg_ep_workspace_bytes(const cpg_ep *ep, const cpg_moe_layer *local_layer, int T) {
    int D, F, E, K;
    if (!ep || !local_layer || T <= 0 || layer_dims(local_layer, &D, &F, &E, &K) != CPG_OK) return 0;
    return ep_layout(ep->G, T, D, K, cpg_moe_apply_workspace_bytes(local_layer, ep->G * T)).total;
}

namespace cpg {
int apply_validate(const cpg_moe_layer *layer, int T, size_t ws_bytes);
// rows_f16: R fp16 rows xstride halves apart; row r's slot ids / weights at + r·istride.
int apply_rows_impl(const cpg_moe_layer *layer, const void *rows_f16, int xstride, int R, const int *slot_expert,
                    const float *slot_wt, int istride, float *out, void *ws, size_t ws_bytes, cudaStream_t s);

// ev: null, or 6 events recorded before plan/pack, dispatch, owner experts, return, combine and
// after the combine.
static int ep_impl(cpg_ep *ep, const cpg_moe_layer *local_layer, const float *xn, int T, const int *topk_idx,
                   const float *wt, float *mlp, void *ws, size_t ws_bytes, cudaStream_t s, cudaEvent_t *ev) {
    CPG_REQUIRE(ep && local_layer && xn && topk_idx && wt && mlp && ws, "cpg_moe_ep: null argument");
    CPG_REQUIRE(T > 0, "cpg_moe_ep: T=%d", T);
    if (ep->aborted) {
        set_error("cpg_moe_ep: the communicator was aborted");
        return CPG_ENCCL;
    }
    int D, F, E_l, K;
    int rc = layer_dims(local_layer, &D, &F, &E_l, &K);
    if (rc) return rc;
    CPG_REQUIRE(K <= EP_MAX_K, "cpg_moe_ep: topk %d > %d", K, EP_MAX_K);
    const int G = ep->G, me = ep->rank;
    CPG_REQUIRE(G <= 64, "cpg_moe_ep: at most 64 ranks");
    const size_t apply_bytes = cpg_moe_apply_workspace_bytes(local_layer, G * T);
    const EpWs W = ep_layout(G, T, D, K, apply_bytes);
    CPG_REQUIRE(ws_bytes >= W.total, "cpg_moe_ep: workspace %zu < %zu bytes", ws_bytes, W.total);
    CPG_REQUIRE((((uintptr_t)xn | (uintptr_t)mlp | (uintptr_t)ws) & 15) == 0, "cpg_moe_ep: 16-byte alignment");
    // everything the owner step can reject, checked before the first collective
    rc = apply_validate(local_layer, G * T, apply_bytes);
    if (rc) return rc;
    uint8_t *w = (uint8_t *)ws;
    int *status = (int *)(w + W.status);
    if (ev) CPG_CUDA(cudaEventRecord(ev[0], s));
    CPG_CUDA(cudaMemsetAsync(status, 0, 16 * sizeof(int), s));
    int *pos = (int *)(w + W.pos);
    k_ep_plan<<<G, EP_PLAN_THREADS, 0, s>>>(T, K, G, E_l, D, topk_idx, wt, pos, w + W.send, W.rs, status);
    CPG_CUDA(cudaGetLastError());
    int pgrid = (T + 7) / 8;
    if (pgrid > sm_count() * 8) pgrid = sm_count() * 8;
    k_ep_pack_rows<<<pgrid, 256, 0, s>>>(T, D, G, xn, pos, w + W.send, W.rs);
    CPG_CUDA(cudaGetLastError());

    // dispatch: one message of T records to every other owner through NCCL; this rank's own
    // share is a device copy
    const size_t msg_b = (size_t)T * W.rs;
    if (ev) CPG_CUDA(cudaEventRecord(ev[1], s));
    CPG_CUDA(cudaMemcpyAsync(w + W.recv + me * msg_b, w + W.send + me * msg_b, msg_b, cudaMemcpyDeviceToDevice, s));
    if (G > 1) {
        P2P ops[2 * 64];
        int n = 0;
        for (int p = 0; p < G; ++p) {
            if (p == me) continue;
            ops[n++] = {w + W.send + p * msg_b, msg_b, ncclUint8, p, true};
            ops[n++] = {w + W.recv + p * msg_b, msg_b, ncclUint8, p, false};
        }
        rc = ep_group(ep, ops, n, s, "cpg_moe_ep dispatch");
        if (rc) return rc;
    }

    // the owner's experts over every received row (empty slots are -1); arguments were checked
    // above, so only a CUDA launch failure can end it here: the communicator is aborted then,
    // which fails the peers' return exchange instead of leaving it waiting
    if (ev) CPG_CUDA(cudaEventRecord(ev[2], s));
    const uint8_t *meta = w + W.recv + (size_t)D * sizeof(__half);
    rc = apply_rows_impl(local_layer, w + W.recv, (int)(W.rs / sizeof(__half)), G * T, (const int *)meta,
                         (const float *)meta + K, (int)(W.rs / sizeof(int)), (float *)(w + W.out_rows), w + W.apply,
                         apply_bytes, s);
    if (rc) {
        ep_abort(ep);
        return rc;
    }
    // the owner step's status word (bounded device waits) next to this call's own
    CPG_CUDA(cudaMemcpyAsync(status + 1, w + W.apply, sizeof(int), cudaMemcpyDeviceToDevice, s));

    // return: one partial row per (token, owner); this rank's own rows by a device copy
    const size_t out_n = (size_t)T * D;
    if (ev) CPG_CUDA(cudaEventRecord(ev[3], s));
    CPG_CUDA(cudaMemcpyAsync((float *)(w + W.back) + me * out_n, (float *)(w + W.out_rows) + me * out_n,
                             out_n * sizeof(float), cudaMemcpyDeviceToDevice, s));
    if (G > 1) {
        P2P ops[2 * 64];
        int n = 0;
        for (int p = 0; p < G; ++p) {
            if (p == me) continue;
            ops[n++] = {(float *)(w + W.out_rows) + p * out_n, out_n, ncclFloat32, p, true};
            ops[n++] = {(float *)(w + W.back) + p * out_n, out_n, ncclFloat32, p, false};
        }
        rc = ep_group(ep, ops, n, s, "cpg_moe_ep return");
        if (rc) return rc;
    }

    if (ev) CPG_CUDA(cudaEventRecord(ev[4], s));
    int cgrid = (T * D / 4 + 255) / 256;
    if (cgrid > sm_count() * 8) cgrid = sm_count() * 8;
    k_ep_combine<<<cgrid, 256, 0, s>>>(T, D, G, pos, (const float *)(w + W.back), mlp);
    CPG_CUDA(cudaGetLastError());
    if (ev) CPG_CUDA(cudaEventRecord(ev[5], s));
    return CPG_OK;
}
}  // namespace cpg

extern "C" int cpg_moe_ep(cpg_ep *ep, const cpg_moe_layer *local_layer, const float *xn, int T, const int *topk_idx,
                          const float *wt, float *mlp, void *ws, size_t ws_bytes, void *stream) {
    return ep_impl(ep, local_layer, xn, T, topk_idx, wt, mlp, ws, ws_bytes, (cudaStream_t)stream, nullptr);
}

extern "C" int cpg_moe_ep_profile(cpg_ep *ep, const cpg_moe_layer *local_layer, const float *xn, int T,
                                  const int *topk_idx, const float *wt, float *mlp, void *ws, size_t ws_bytes,
                                  void *stream, float *phase_ms) {
    CPG_REQUIRE(phase_ms, "cpg_moe_ep_profile: null phase_ms");
    cudaEvent_t ev[6] = {};
    for (int i = 0; i < 6; ++i) {
        const cudaError_t ce = cudaEventCreate(&ev[i]);
        if (ce != cudaSuccess) {
            for (int j = 0; j < i; ++j) cudaEventDestroy(ev[j]);
            return cuda_fail(ce, "cpg_moe_ep_profile: event");
        }
    }
    int rc = ep_impl(ep, local_layer, xn, T, topk_idx, wt, mlp, ws, ws_bytes, (cudaStream_t)stream, ev);
    if (rc == CPG_OK) rc = cpg_ep_wait(ep, stream);
    for (int i = 0; rc == CPG_OK && i < 5; ++i) {
        const cudaError_t e2 = cudaEventElapsedTime(&phase_ms[i], ev[i], ev[i + 1]);
        if (e2 != cudaSuccess) rc = cuda_fail(e2, "cpg_moe_ep_profile: elapsed time");
    }
    for (int i = 0; i < 6; ++i) cudaEventDestroy(ev[i]);
    return rc;
}

extern "C" int cpg_moe_ep_check(const void *ws, void *stream) {
    CPG_REQUIRE(ws, "cpg_moe_ep_check: null workspace");
    int st[2] = {0, 0};
    CPG_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    CPG_CUDA(cudaMemcpy(st, ws, sizeof(st), cudaMemcpyDeviceToHost));
    if (st[0] == ST_BAD_ITEM) {
        set_error("cpg_moe_ep: expert id outside [0, n_ranks * local experts) (those slots contributed zero)");
        return CPG_EINVAL;
    }
    if (st[1] != ST_OK) {
        set_error("cpg_moe_ep: a bounded device wait in the owner's expert GEMMs gave up (status %d)", st[1]);
        return CPG_ETIMEOUT;
    }
    return CPG_OK;
}
