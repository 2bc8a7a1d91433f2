// common.cuh — shared host/device helpers for the cachepotato_b200 kernels (sm_100a).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <utility>

#include "cpg.h"

namespace cpg {

// ------------------------------------------------------------------ host error plumbing
void set_error(const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);

#define CPG_CUDA(call)                                              \
    do {                                                            \
        cudaError_t e_ = (call);                                    \
        if (e_ != cudaSuccess) return ::cpg::cuda_fail(e_, #call);  \
    } while (0)

#define CPG_REQUIRE(cond, ...)                                      \
    do {                                                            \
        if (!(cond)) {                                              \
            ::cpg::set_error(__VA_ARGS__);                          \
            return CPG_EINVAL;                                      \
        }                                                           \
    } while (0)

int sm_count();
// Largest dynamic shared memory a block may opt into on this device (227 KB on B200).
int smem_optin();
// Raise a kernel's dynamic shared-memory limit to the device maximum minus its static shared
// memory (never lowered, so launches sized for one layer cannot be broken by a later, smaller one).
int allow_max_smem(const void *kernel);

inline long group_bytes(int enc) { return enc == CPG_ENC_Q4 ? 18 : enc == CPG_ENC_Q8 ? 34 : 0; }
inline long row_bytes(int enc, long n_in) {
    return enc == CPG_ENC_F32 ? 4 * n_in : (n_in / 32) * group_bytes(enc);
}

// Launch with programmatic dependent launch: the kernel may start while the previous kernel on
// the stream drains; it must call pdl_wait() before touching anything that kernel produces.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl for a kernel whose CTAs run in thread-block clusters of `cluster_x` along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                      int cluster_x, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ device helpers

// Cluster-wide barrier (hardware; every CTA of a cluster is resident together, so it ends):
// memory operations before it, global ones included, are visible to the cluster after it.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ int cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return (int)r;
}
__device__ __forceinline__ int cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return (int)r;
}

// Wait until the grid this one depends on has completed and its writes are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Let the next kernel on the stream start launching (it still waits in pdl_wait()).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// fp16 bits -> f32 by bit manipulation, NaN payloads and subnormals preserved exactly as
// the reference decoder does (engine/kernels/kernels.c:109-130).
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int sh = __clz(m) - 21;                 // shifts until bit 10 is set
            bits = sign | ((uint32_t)(113 - sh) << 23) | (((m << sh) & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    return __uint_as_float(bits);
}

// Device status word codes (workspace word 0).
enum : int { ST_OK = 0, ST_TIMEOUT_FULL = 1, ST_TIMEOUT_EMPTY = 2, ST_BAD_ITEM = 3 };

// Bounded waits: a healthy wait lasts microseconds; a wait that reaches kWaitLimitNs (2 s of
// %globaltimer) gives up, records a status code and lets the kernel return, so no GPU hangs.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done) : "r"(addr), "r"(parity) : "memory");
    return done != 0;
}

// Bounded wait for the phase with the given parity to complete. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    uint32_t addr = smem_u32(bar);
    if (mbar_try_wait(addr, parity)) return true;
    uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(addr, parity)) return true;
        if ((i & 63u) == 0 && global_ns() - t0 > kWaitLimitNs) return false;
    }
}

// 1D bulk copy global -> shared through the TMA engine, completing on an mbarrier.
// dst, src 16-byte aligned; bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// 16-byte asynchronous copy global -> shared on the load/store path (L2 only, no L1 line).
// dst and src 16-byte aligned.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// One arrival on the barrier once every earlier cp.async of this thread has landed (counts as
// one of the arrivals the barrier was initialised with).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// Close this thread's current group of cp.async copies / wait until at most N groups are pending.
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// D = A·B + C, m16n8k16, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                          const float c[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
          "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// Two f32 values as fp16 hi and lo halves (hi = fp16(v), lo = fp16(v - hi); v - hi is exact in
// f32), packed as half2 words {a, b}: hi + lo keeps about 22 significant bits of v for |v| in
// fp16's normal range (the lo half's absolute error is at most 2^-25 below it).
__device__ __forceinline__ void split_half2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
__device__ __forceinline__ void split_half(float v, __half &hi, __half &lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

// (a & b) ^ c in one LOP3.
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// (a0, a1) = fma(d, (s0, s1), (a0, a1)) as one packed f32x2 instruction (sm_100): each lane is
// an IEEE fma with round to nearest, the same value fmaf gives.
__device__ __forceinline__ void fma2_f32(float &a0, float &a1, float d, float s0, float s1) {
    asm("{\n\t.reg .b64 A, B, C;\n\t"
        "mov.b64 A, {%0, %1};\n\t"
        "mov.b64 B, {%2, %2};\n\t"
        "mov.b64 C, {%3, %4};\n\t"
        "fma.rn.f32x2 A, B, C, A;\n\t"
        "mov.b64 {%0, %1}, A;\n\t}"
        : "+f"(a0), "+f"(a1) : "f"(d), "f"(s0), "f"(s1));
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

}  // namespace cpg
