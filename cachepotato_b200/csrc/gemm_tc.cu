// gemm_tc.cu — grouped expert GEMM on the 5th-generation tensor cores (tcgen05), for prefill and
// other large batches where each expert sees many tokens.
//
// Per tile: 256 weight rows (gate 128 + up 128 of one expert, or 256 rows of its down matrix) ×
// 128 tokens of that expert, K streamed 64 values per stage. Eight math warps decode Q4_0
// groups straight from the v4 rows in global memory into fp16 (q·d rounded once to fp16) in
// shared memory, in the K-major no-swizzle canonical layout the tensor core reads, and stage the
// tokens' fp16 activation rows beside them. One thread issues tcgen05.mma (M=128, N=128, K=16,
// fp16 × fp16 → fp32 in TMEM) twice per K step, one per 128-row half, and commits each stage to
// an mbarrier that frees it. The epilogue reads the accumulators with tcgen05.ld:
//   gate/up: h = silu(g)·u (engine/blocks/qwen3_moe.c:217-219), fp16, one row per (token, slot);
//   down:    y per (token, slot) in fp32, combined in selection order by k_combine.
// Every mbarrier wait is bounded; a timeout records a status code and all roles leave together.
#include <math.h>

#include "gemm_tc.cuh"

namespace cpg {

constexpr int TC_BM = 128;                  // rows per MMA (one TMEM lane per row)
constexpr int TC_BN = 128;                  // tokens per tile (MMA N, TMEM columns per half)
constexpr int TC_BK = 64;                   // K per stage (4 MMAs of K=16)
constexpr int TC_STAGES = 3;
constexpr int TC_MATH_WARPS = 8;
constexpr int TC_THREADS = (2 + TC_MATH_WARPS) * 32;   // warp 0: TMEM owner, warp 1: MMA issuer
constexpr int TC_A_BYTES = 2 * TC_BM * TC_BK * 2;      // 32 KB: two 128-row halves, fp16
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;          // 16 KB
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES;
constexpr int TC_SBO = (TC_BK / 8) * 128;              // bytes between 8-row core-matrix groups
constexpr int TC_LBO = 128;                            // bytes between 8-column core matrices
constexpr int TC_TMEM_COLS = 2 * TC_BN;                // two fp32 accumulators of 128 columns
constexpr int TC_MAX_E = 256;

// ---------------------------------------------------------------- tcgen05 wrappers
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // SM100 shared-memory matrix descriptor, K-major, no swizzle: start, LBO, SBO in 16-byte
    // units, version 1 (bit 46), base offset 0, layout type 0.
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// kind::f16 instruction descriptor: fp32 accumulate, fp16 A and B, both K-major, M=128, N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Bounded wait that also honours the CTA-wide abort flag.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status,
                                        int code) {
    if (*abort_flag) return false;
    if (mbar_wait(bar, parity)) return true;
    *abort_flag = 1;
    atomicCAS(status, ST_OK, code);
    return false;
}

// Q4_0 group pair (36 bytes, 4-byte aligned) of one row -> 64 fp16 values q*d in K order,
// as 8 chunks of 8 values (16 bytes each).
__device__ __forceinline__ void q4_pair_to_f16(const uint32_t *src, uint4 (&out)[8]) {
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = __ldg(src + i);
    const uint32_t d0 = w[0] & 0xFFFFu, d1 = w[4] >> 16;
    const uint32_t s0 = d0 | (d0 << 16), s1 = d1 | (d1 << 16);
    // quant bytes of group j: w0[2..3], w1..w3, w4[0..1]; of group j+1: w5..w8
    const uint32_t qa[4] = {__byte_perm(w[0], w[1], 0x5432), __byte_perm(w[1], w[2], 0x5432),
                            __byte_perm(w[2], w[3], 0x5432), __byte_perm(w[3], w[4], 0x5432)};
    const uint32_t qb[4] = {w[5], w[6], w[7], w[8]};
    const uint32_t k1032 = 0x64086408u, k1_16 = 0x2C002C00u, km72 = 0xD480D480u;
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
        const uint32_t *q = grp ? qb : qa;
        const uint32_t sc = grp ? s1 : s0;
        uint32_t lo[8], hi[8];                 // element pairs (2i, 2i+1) of the low / high nibbles
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            const uint32_t x = __byte_perm(q[wi], 0, 0x3120);          // [b0, b2, b1, b3]
            const uint32_t x2 = x >> 8;
            lo[2 * wi] = hsub2_u32(lop3_and_xor(x, 0x000F000Fu, 0x64086408u), k1032);
            lo[2 * wi + 1] = hsub2_u32(lop3_and_xor(x2, 0x000F000Fu, 0x64086408u), k1032);
            hi[2 * wi] = hfma2_u32(lop3_and_xor(x, 0x00F000F0u, 0x64806480u), k1_16, km72);
            hi[2 * wi + 1] = hfma2_u32(lop3_and_xor(x2, 0x00F000F0u, 0x64806480u), k1_16, km72);
        }
        // scale (one rounding to fp16 per weight)
        uint32_t v[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(v[i]) : "r"(lo[i]), "r"(sc));
            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(v[8 + i]) : "r"(hi[i]), "r"(sc));
        }
        // elements 0..15 = low nibbles of bytes 0..15, 16..31 = high nibbles
        out[grp * 4 + 0] = make_uint4(v[0], v[1], v[2], v[3]);
        out[grp * 4 + 1] = make_uint4(v[4], v[5], v[6], v[7]);
        out[grp * 4 + 2] = make_uint4(v[8], v[9], v[10], v[11]);
        out[grp * 4 + 3] = make_uint4(v[12], v[13], v[14], v[15]);
    }
}

// canonical K-major no-swizzle offset of the 16-byte chunk (row r, chunk c) in a tile
__device__ __forceinline__ uint32_t canon_off(int r, int c) {
    return (uint32_t)((r >> 3) * TC_SBO + c * TC_LBO + (r & 7) * 16);
}

template <int KIND>
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(TcArgs a) {
    // The runtime places dynamic shared memory after the static variables, 16-byte aligned only,
    // so the operand tiles are moved up to the next 1024-byte boundary here (the launch adds the
    // slack). The declaration states 16 so that the compiler cannot assume more and fold this away.
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t *const smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __shared__ uint64_t full_bar[TC_STAGES], empty_bar[TC_STAGES], acc_full, acc_empty, drain_bar;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    __shared__ int4 s_act[TC_MAX_E + 1];
    __shared__ const uint8_t *s_ptr[TC_MAX_E][2];
    __shared__ int s_tpre[TC_MAX_E + 1];        // token tiles before active expert u
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K_in = KIND == 0 ? a.D : a.F;
    const int n_rows = KIND == 0 ? a.F : a.D;
    const int MT = KIND == 0 ? n_rows / TC_BM : n_rows / (2 * TC_BM);   // row tiles per expert
    const int KST = K_in / TC_BK;                                         // K stages per tile
    const long rowbytes = (long)(K_in / 32) * 18;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; ++s) {
            mbar_init(&full_bar[s], TC_MATH_WARPS * 32);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&acc_full, 1);
        mbar_init(&acc_empty, TC_MATH_WARPS * 32);
        mbar_init(&drain_bar, 1);
        fence_mbar_init();
        s_abort = 0;
    }
    if (warp == 0) {                                   // TMEM: 256 fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&s_tmem)), "r"(TC_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    const int U = *a.n_active;
    for (int u = threadIdx.x; u <= U; u += blockDim.x) {
        s_act[u] = a.act[u];
        if (u < U) {
            s_ptr[u][0] = a.act_ptr[3 * u + (KIND == 0 ? 0 : 2)];
            s_ptr[u][1] = a.act_ptr[3 * u + 1];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int u = 0; u < U; ++u) {
            s_tpre[u] = acc;
            acc += (s_act[u].z + TC_BN - 1) / TC_BN;
        }
        s_tpre[U] = acc;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int total = MT * s_tpre[U];
    volatile int *abort_flag = &s_abort;
    const uint32_t sbase = smem_u32(smem);

    // tile -> (active expert u, row tile m, token tile n); token tiles innermost so the tiles of
    // one weight block run back to back and its second read hits L2
    auto decode = [&](int tile, int &u, int &m, int &n) {
        int lo = 0, hi = U;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (MT * s_tpre[mid] <= tile) lo = mid; else hi = mid;
        }
        u = lo;
        const int ntn = s_tpre[u + 1] - s_tpre[u];
        const int local = tile - MT * s_tpre[u];
        m = local / ntn;
        n = local - m * ntn;
    };

    if (warp == 1) {
        // ---------------- MMA issuer (one thread)
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(TC_BM, TC_BN);
            int it = 0, ti = 0;
            for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++ti) {
                if (ti > 0 && !tc_wait(&acc_empty, (uint32_t)(ti - 1) & 1u, abort_flag, a.status, ST_TIMEOUT_EMPTY)) break;
                tc_fence_after();
                bool ok = true;
                for (int ks = 0; ks < KST; ++ks, ++it) {
                    const int st = it % TC_STAGES;
                    if (!tc_wait(&full_bar[st], (uint32_t)(it / TC_STAGES) & 1u, abort_flag, a.status, ST_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = sbase + st * TC_STAGE_BYTES, sb = sa + TC_A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; ++kk) {
                        const uint64_t bdesc = umma_desc(sb + kk * 2 * TC_LBO, TC_LBO, TC_SBO);
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const uint64_t adesc = umma_desc(sa + h * (TC_BM / 8) * TC_SBO + kk * 2 * TC_LBO, TC_LBO, TC_SBO);
                            umma_f16(tmem + h * TC_BN, adesc, bdesc, idesc, (ks | kk) ? 1u : 0u);
                        }
                    }
                    umma_commit(&empty_bar[st]);           // frees the stage when these MMAs finish
                }
                if (!ok) break;
                umma_commit(&acc_full);                    // accumulators complete
            }
            // drain: wait (bounded) until every MMA this thread issued has finished
            umma_commit(&drain_bar);
            mbar_wait(&drain_bar, 0);
        }
    } else if (warp >= 2) {
        // ---------------- math warps: decode weights, stage tokens, epilogue
        const int mt = threadIdx.x - 64;                   // 0..255
        const int quad = warp & 3;                         // TMEM lane quadrant this warp may access
        const int colhalf = (warp - 2) >> 2;               // epilogue columns [64*colhalf, +64)
        int it = 0, ti = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++ti) {
            int u, m, n;
            decode(tile, u, m, n);
            const int4 ex = s_act[u];
            const int off = ex.y + n * TC_BN;
            const int cnt = min(TC_BN, ex.z - n * TC_BN);
            // this thread's weight row (one of 256) and token half-row
            const int r = mt;                              // A row 0..255
            const uint8_t *wrow;
            if (KIND == 0) wrow = s_ptr[u][r >> 7] + (size_t)(m * TC_BM + (r & 127)) * rowbytes;
            else wrow = s_ptr[u][0] + (size_t)(m * 2 * TC_BM + r) * rowbytes;
            const int bt = mt >> 1, bhalf = mt & 1;         // token row bt, chunks 4*bhalf..+3
            const __half *brow = nullptr;
            if (bt < cnt) {
                const int p = off + bt;
                brow = KIND == 0 ? a.bsrc + (size_t)(a.pairs[p] / a.K) * a.D : a.bsrc + (size_t)p * a.F;
            }
            bool ok = true;
            for (int ks = 0; ks < KST; ++ks, ++it) {
                const int st = it % TC_STAGES;
                if (it >= TC_STAGES &&
                    !tc_wait(&empty_bar[st], (uint32_t)(it / TC_STAGES - 1) & 1u, abort_flag, a.status, ST_TIMEOUT_EMPTY)) {
                    ok = false;
                    break;
                }
                uint8_t *sa = smem + st * TC_STAGE_BYTES, *sb = sa + TC_A_BYTES;
                uint4 v[8];
                q4_pair_to_f16(reinterpret_cast<const uint32_t *>(wrow + (size_t)ks * 36), v);
                const int hr = r >> 7, rr = r & 127;       // half, row within half
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<uint4 *>(sa + hr * (TC_BM / 8) * TC_SBO + canon_off(rr, c)) = v[c];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int cc = bhalf * 4 + c;
                    uint4 bv = make_uint4(0, 0, 0, 0);
                    if (brow) bv = __ldg(reinterpret_cast<const uint4 *>(brow + ks * TC_BK + cc * 8));
                    *reinterpret_cast<uint4 *>(sb + canon_off(bt, cc)) = bv;
                }
                fence_async_smem();                        // generic-proxy writes -> tensor core
                mbar_arrive(&full_bar[st]);
            }
            if (!__all_sync(0xffffffffu, ok)) break;
            // epilogue: wait for the accumulators, read this warp's 32 rows (tcgen05.ld is
            // warp-collective, so the whole warp decides together)
            const bool got = tc_wait(&acc_full, (uint32_t)ti & 1u, abort_flag, a.status, ST_TIMEOUT_FULL);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const int row = quad * 32 + lane;              // accumulator row (TMEM lane)
            for (int c0 = colhalf * 64; c0 < colhalf * 64 + 64; c0 += 32) {
                float g[32], w2[32];
                tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c0, g);
                tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + TC_BN + c0, w2);
                if (KIND == 0) {
                    const int feat = m * TC_BM + row;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int col = c0 + j;
                        if (col < cnt) {
                            const float gv = g[j];
                            const float h = gv / (1.0f + expf(-gv)) * w2[j];   // silu(g)*u
                            a.h_out[(size_t)(off + col) * a.F + feat] = __float2half_rn(h);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int col = c0 + j;
                        if (col < cnt) {
                            float *yr = a.y_out + (size_t)a.pairs[off + col] * a.D + m * 2 * TC_BM;
                            yr[row] = g[j];
                            yr[TC_BM + row] = w2[j];
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty);
        }
    }
    // all roles leave here (a timeout anywhere raised the abort flag, every wait is bounded)
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
    }
}

int gemm_tc_launch(int kind, const TcArgs &a, int max_tiles, cudaStream_t s) {
    auto *k = kind == 0 ? k_gemm_tc<0> : k_gemm_tc<1>;
    const size_t smem = (size_t)TC_STAGES * TC_STAGE_BYTES + 1024;
    CPG_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int grid = sm_count();
    if (max_tiles < grid) grid = max_tiles > 0 ? max_tiles : 1;
    k<<<grid, TC_THREADS, smem, s>>>(a);
    CPG_CUDA(cudaGetLastError());
    return CPG_OK;
}

}  // namespace cpg
