// gemm_tc.cu — grouped expert GEMM on the 5th-generation tensor cores (tcgen05), for prefill and
// other large batches where each expert sees many tokens.
//
// Per tile: 256 weight rows (gate 128 + up 128 of one expert, or 256 rows of its down matrix) ×
// up to 256 tokens of that expert (MMA N = the tile's token count rounded up to 16), K streamed 32
// values per stage through four stages. Roles (one CTA per SM):
//   warp 0      owns the TMEM allocation; one thread loads raw Q4_0 rows into a two-slot
//               shared-memory ring with 2D tensor TMA boxes of 128 rows × 144 bytes (eight stages
//               of K) over each expert matrix: two requests per group, where one small copy per
//               row queued 256 requests on the copy engine and starved the tensor core
//   warp 1      one thread issues tcgen05.mma (M=128, N≤256, K=16, fp16 × fp16 → fp32 in TMEM),
//               twice per K step (one per 128-row half), and commits each stage to the mbarrier
//               that frees it
//   warps 2, 3  one thread each loads the token tile of every other stage with a 2D tensor TMA
//               (64-byte swizzle, a 128- or 256-row box) from the expert-sorted fp16 activation
//               rows (one issuing warp's copies are served one after another, ~500 cycles each)
//   warps 4-19  decode the raw rows from shared memory into fp16 (q·d rounded once) in the
//               K-major no-swizzle canonical layout, two threads per row (one takes quant bytes
//               0-7 of each group = K chunks 0 and 2, the other bytes 8-15 = chunks 1 and 3, so
//               both write the same stage), then run the epilogue from TMEM:
//                 gate/up: h = silu(g)·u (engine/blocks/qwen3_moe.c:217-219), fp16 per pair
//                 down:    y per (token, slot) in fp32, combined in selection order by k_combine
// Kind 2 (dense) serves the whole model's attention projections on a prompt: one group of all
// tokens in 128-token tiles, each tile one of three passes (W_hi·x_hi, W_hi·x_lo, W_lo·x_hi, with
// both operands split exactly into two fp16 terms), each pass writing its own f32 plane.
// Every mbarrier wait is bounded; a timeout records a status code, all roles leave together, and
// the copy engines' last transfers are waited for (bounded) before the CTA exits.
#include <cuda.h>
#include <math.h>

#include <mutex>
#include <vector>

#include "gemm_tc.cuh"

namespace cpg {

constexpr int TC_BM = 128;                  // rows per MMA (one TMEM lane per row)
constexpr int TC_BN = 256;                  // tokens per tile (MMA N at most, TMEM columns per half)
constexpr int TC_BN_SMALL = 128;            // token box for tiles of at most 128 tokens
constexpr int TC_BK = 32;                   // K per stage (one Q4_0 group; 2 MMAs of K=16 per half)
constexpr int TC_STAGES = 4;
constexpr int TC_ROWS = 2 * TC_BM;          // weight rows per tile
constexpr int TC_GRP = 8;                   // K stages per raw group
constexpr int TC_RAW_ROW = 144;             // bytes per row per raw group: four Q4_0 group pairs
constexpr int TC_RAW_BYTES = TC_ROWS * TC_RAW_ROW;                  // 36 KB per raw slot
constexpr int TC_RAW_SLOTS = 2;
constexpr int TC_A_BYTES = TC_ROWS * TC_BK * 2;                     // 16 KB: two 128-row halves
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;                       // 16 KB
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES;
constexpr int TC_STAGE0 = TC_RAW_SLOTS * TC_RAW_BYTES;              // operand stages follow the raw ring
constexpr int TC_SMEM = TC_STAGE0 + TC_STAGES * TC_STAGE_BYTES;     // 200 KB (+1 KB alignment slack)
constexpr int TC_MATH_WARPS = 16;               // two threads per weight row
constexpr int TC_B_WARPS = 2;                   // token-tile producers: warps 2, 3
constexpr int TC_FIRST_MATH = 2 + TC_B_WARPS;
constexpr int TC_THREADS = (TC_FIRST_MATH + TC_MATH_WARPS) * 32;
constexpr int TC_SBO = (TC_BK / 8) * 128;   // no-swizzle A: bytes between 8-row core-matrix groups
constexpr int TC_LBO = 128;                 // no-swizzle A: bytes between 8-column core matrices
constexpr int TC_TMEM_COLS = 2 * TC_BN;     // two fp32 accumulators of 256 columns (all of TMEM)
constexpr int TC_MAX_E = 256;
static_assert(TC_STAGE0 % 1024 == 0 && TC_STAGE_BYTES % 1024 == 0 && TC_A_BYTES % 1024 == 0,
              "operand tiles must stay 1024-byte aligned");

// ---------------------------------------------------------------- tcgen05 / TMA wrappers
// SM100 shared-memory matrix descriptor, K-major, no swizzle: start, LBO, SBO in 16-byte units,
// version 1 (bit 46), base offset 0, layout type 0.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// K-major, 64-byte swizzle (the layout a SWIZZLE_64B tensor TMA writes): rows of 64 bytes,
// 8-row groups 512 bytes apart (SBO), LBO unused (1), layout type 4. Advancing K by 16 fp16
// values inside the 64-byte row moves the start address by 32 bytes.
__device__ __forceinline__ uint64_t umma_desc_sw64(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(512 >> 4) << 32) | (1ull << 46) |
           (4ull << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, fp16 A and B, both K-major, M, N.
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

// 2D tensor TMA load (no multicast) of the box at (x, y) into shared memory, completing on bar.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

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

// Q4_0 group pair (36 bytes as 9 words: scale d0 + 16 quant bytes, scale d1 + 16 quant bytes)
// -> 64 fp16 values q*d in K order, as 8 chunks of 8 values (16 bytes each).
__device__ __forceinline__ void q4_pair_to_f16(const uint32_t *w, uint4 (&out)[8]) {
    const uint32_t d0 = w[0] & 0xFFFFu, d1 = w[4] >> 16;
    const uint32_t s0 = d0 | (d0 << 16), s1 = d1 | (d1 << 16);
    // quant bytes of the first group: w0[2..3], w1..w3, w4[0..1]; of the second: w5..w8
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

// Eight quant bytes of one Q4_0 group (u0 = bytes 0..3, u1 = bytes 4..7 of the caller's half) and
// its fp16 scale (duplicated in both halves of sc) -> the low-nibble values (8 consecutive K) and
// the high-nibble values (the 8 values 16 further on), each as one 16-byte chunk of q·d in fp16.
// low: the residual q·d − fp16(q·d) instead (one fused multiply-add, exact in fp16 while it is
// not below the subnormal range), the second half of a weight split into two fp16 terms.
__device__ __forceinline__ void q4_half_group(uint32_t u0, uint32_t u1, uint32_t sc, uint4 &lo_chunk, uint4 &hi_chunk,
                                              bool low = false) {
    const uint32_t k1032 = 0x64086408u, k1_16 = 0x2C002C00u, km72 = 0xD480D480u;
    const uint32_t q[2] = {u0, u1};
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int wi = 0; wi < 2; ++wi) {
        const uint32_t x = __byte_perm(q[wi], 0, 0x3120);              // [b0, b2, b1, b3]
        const uint32_t x2 = x >> 8;
        lo[2 * wi] = hsub2_u32(lop3_and_xor(x, 0x000F000Fu, 0x64086408u), k1032);
        lo[2 * wi + 1] = hsub2_u32(lop3_and_xor(x2, 0x000F000Fu, 0x64086408u), k1032);
        hi[2 * wi] = hfma2_u32(lop3_and_xor(x, 0x00F000F0u, 0x64806480u), k1_16, km72);
        hi[2 * wi + 1] = hfma2_u32(lop3_and_xor(x2, 0x00F000F0u, 0x64806480u), k1_16, km72);
    }
    uint32_t v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(v[i]) : "r"(lo[i]), "r"(sc));
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(v[4 + i]) : "r"(hi[i]), "r"(sc));
    }
    if (low) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(v[i]) : "r"(lo[i]), "r"(sc), "r"(v[i] ^ 0x80008000u));
            asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(v[4 + i]) : "r"(hi[i]), "r"(sc), "r"(v[4 + i] ^ 0x80008000u));
        }
    }
    lo_chunk = make_uint4(v[0], v[1], v[2], v[3]);
    hi_chunk = make_uint4(v[4], v[5], v[6], v[7]);
}

// canonical K-major no-swizzle offset of the 16-byte chunk (row r, chunk c) in a 128-row half
__device__ __forceinline__ uint32_t canon_off(int r, int c) {
    return (uint32_t)((r >> 3) * TC_SBO + c * TC_LBO + (r & 7) * 16);
}

template <int KIND>
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(const TcArgs a, const __grid_constant__ CUtensorMap tmap_b,
                                                       const __grid_constant__ CUtensorMap tmap_b_small) {
    // The runtime places dynamic shared memory after the static variables, 16-byte aligned only,
    // so the tiles are moved up to the next 1024-byte boundary here (the launch adds the slack).
    // The declaration states 16 so that the compiler cannot assume more and fold this away.
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t *const smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __shared__ uint64_t raw_full[TC_RAW_SLOTS], raw_empty[TC_RAW_SLOTS];
    __shared__ uint64_t a_full[TC_STAGES], b_full[TC_STAGES], empty_bar[TC_STAGES];
    __shared__ uint64_t acc_full, acc_empty, drain_bar;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    __shared__ int4 s_act[TC_MAX_E + 1];
    __shared__ int s_tpre[TC_MAX_E + 1];        // token tiles before active expert u
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K_in = KIND == 0 ? a.D : a.F;
    const int n_rows = KIND == 0 ? a.F : a.D;
    const int MT = KIND == 0 ? n_rows / TC_BM : n_rows / TC_ROWS;   // row tiles per expert
    // KIND 2 (dense projections): three passes, each its own tiles and output plane,
    // W_hi·x_hi, W_hi·x_lo, W_lo·x_hi, where x = x_hi + x_lo (the token rows hold [x_hi | x_lo])
    // and W_hi + W_lo = q·d exactly; 128-token tiles, for more CTAs on short prompts
    constexpr int NPASS = KIND == 2 ? 3 : 1;
    constexpr int BN = KIND == 2 ? TC_BN_SMALL : TC_BN;             // tokens per tile
    const int KST = K_in / TC_BK;                                   // K stages per tile
    const int NG = KST / TC_GRP;                                    // raw groups per tile
    constexpr int NMATH = TC_MATH_WARPS * 32;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_RAW_SLOTS; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], NMATH);
        }
        for (int s = 0; s < TC_STAGES; ++s) {
            mbar_init(&a_full[s], NMATH);
            mbar_init(&b_full[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&acc_full, 1);
        mbar_init(&acc_empty, NMATH);
        mbar_init(&drain_bar, 1);
        fence_mbar_init();
        s_abort = 0;
    }
    if (warp == 0) {                                   // TMEM: 512 fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&s_tmem)), "r"(TC_TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    const int U = *a.n_active;
    for (int u = threadIdx.x; u <= U; u += blockDim.x) s_act[u] = a.act[u];
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int u = 0; u < U; ++u) {
            s_tpre[u] = acc;
            acc += (s_act[u].z + BN - 1) / BN;
        }
        s_tpre[U] = acc;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int per_pass = MT * s_tpre[U];
    const int total = per_pass * NPASS;
    volatile int *abort_flag = &s_abort;
    const uint32_t sbase = smem_u32(smem);

    // tile -> (active expert u, row tile m, token tile n); token tiles innermost so the tiles of
    // one weight block run back to back and its later reads hit L2
    auto decode = [&](int tile, int &u, int &m, int &n, int &pass) {
        pass = NPASS > 1 ? tile / per_pass : 0;
        tile -= pass * per_pass;
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

    if (warp == 0) {
        // ---------------- raw weight producer (one thread): two 128-row boxes per group
        if (lane == 0) {
            const CUtensorMap *maps = reinterpret_cast<const CUtensorMap *>(a.wmaps);
            int git = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
                int u, m, n, pass;
                decode(tile, u, m, n, pass);
                const int e = s_act[u].x;
                const CUtensorMap *m0 = maps + 3 * e + (KIND == 0 ? 0 : 2);
                const CUtensorMap *m1 = KIND == 0 ? maps + 3 * e + 1 : m0;
                const int y0 = KIND == 0 ? m * TC_BM : m * TC_ROWS;
                const int y1 = KIND == 0 ? m * TC_BM : m * TC_ROWS + TC_BM;
                for (int g = 0; g < NG; ++g, ++git) {
                    const int slot = git % TC_RAW_SLOTS;
                    if (git >= TC_RAW_SLOTS &&
                        !tc_wait(&raw_empty[slot], (uint32_t)(git / TC_RAW_SLOTS - 1) & 1u, abort_flag, a.status, ST_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    uint8_t *dst = smem + slot * TC_RAW_BYTES;
                    mbar_arrive_expect_tx(&raw_full[slot], TC_RAW_BYTES);
                    tma_load_2d(dst, m0, g * TC_RAW_ROW, y0, &raw_full[slot]);
                    tma_load_2d(dst + TC_BM * TC_RAW_ROW, m1, g * TC_RAW_ROW, y1, &raw_full[slot]);
                }
            }
            // the last groups' copies must land before the CTA may exit (bounded)
            for (int q = git > TC_RAW_SLOTS ? git - TC_RAW_SLOTS : 0; q < git; ++q)
                mbar_wait(&raw_full[q % TC_RAW_SLOTS], (uint32_t)(q / TC_RAW_SLOTS) & 1u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (one thread)
        if (lane == 0) {
            int it = 0, ti = 0;
            for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++ti) {
                int u, m, n, pass;
                decode(tile, u, m, n, pass);
                const int cnt = min(BN, s_act[u].z - n * BN);
                const uint32_t idesc = umma_idesc_f16(TC_BM, (cnt + 15) & ~15);
                if (ti > 0 && !tc_wait(&acc_empty, (uint32_t)(ti - 1) & 1u, abort_flag, a.status, ST_TIMEOUT_EMPTY)) break;
                tc_fence_after();
                bool ok = true;
                for (int ks = 0; ks < KST; ++ks, ++it) {
                    const int st = it % TC_STAGES;
                    const uint32_t par = (uint32_t)(it / TC_STAGES) & 1u;
                    if (!tc_wait(&b_full[st], par, abort_flag, a.status, ST_TIMEOUT_FULL) ||
                        !tc_wait(&a_full[st], par, abort_flag, a.status, ST_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = sbase + TC_STAGE0 + st * TC_STAGE_BYTES, sb = sa + TC_A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; ++kk) {
                        const uint64_t bdesc = umma_desc_sw64(sb + kk * 32);
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
    } else if (warp < TC_FIRST_MATH) {
        // ---------------- token-tile producers (one thread per warp): 2D tensor TMA per stage,
        // stages dealt round-robin over TC_B_WARPS warps (a warp's copies are served one at a
        // time, ~500 cycles each on B200 whatever their size, so one warp cannot feed a stage
        // per MMA stage time)
        if (lane == 0) {
            const int bw = warp - 2;
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < total; tile += gridDim.x) {
                int u, m, n, pass;
                decode(tile, u, m, n, pass);
                const int row0 = s_act[u].y + n * BN;
                const bool small = s_act[u].z - n * BN <= TC_BN_SMALL;
                const CUtensorMap *bmap = small ? &tmap_b_small : &tmap_b;
                const uint32_t bbytes = small ? TC_B_BYTES / 2 : TC_B_BYTES;
                for (int ks = 0; ks < KST; ++ks, ++it) {
                    if (it % TC_B_WARPS != bw) continue;
                    const int st = it % TC_STAGES;
                    if (it >= TC_STAGES &&
                        !tc_wait(&empty_bar[st], (uint32_t)(it / TC_STAGES - 1) & 1u, abort_flag, a.status, ST_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&b_full[st], bbytes);
                    // KIND 2: x_hi in passes 0 and 2, x_lo (columns K_in..2K_in) in pass 1
                    const int bx = ks * TC_BK + (KIND == 2 && pass == 1 ? K_in : 0);
                    tma_load_2d(smem + TC_STAGE0 + st * TC_STAGE_BYTES + TC_A_BYTES, bmap, bx, row0, &b_full[st]);
                }
            }
            for (int q = it > TC_STAGES ? it - TC_STAGES : 0; q < it; ++q)
                if (q % TC_B_WARPS == bw) mbar_wait(&b_full[q % TC_STAGES], (uint32_t)(q / TC_STAGES) & 1u);
        }
    } else {
        // ---------------- math warps: decode weights into the A operand, epilogue
        // a warp decodes 16 rows: lanes 0-15 the byte half 0 of each, lanes 16-31 half 1, so each
        // 8-lane phase of a 16-byte store covers 8 consecutive rows (conflict-free)
        const int wrow = ((warp - TC_FIRST_MATH) << 4) | (lane & 15);   // weight row of the tile
        const int hb = lane >> 4;                          // quant bytes 0-7 or 8-15 of each group
        const int quad = warp & 3;                         // TMEM lane quadrant this warp may access
        const int colq = (warp - TC_FIRST_MATH) >> 2;      // epilogue columns [64*colq, +64)
        const int hr = wrow >> 7, rr = wrow & 127;         // half, row within half
        int it = 0, git = 0, ti = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++ti) {
            int u, m, n, pass;
            decode(tile, u, m, n, pass);
            const int4 ex = s_act[u];
            const int off = ex.y + n * BN;
            const int cnt = min(BN, ex.z - n * BN);
            bool ok = true;
            for (int g = 0; g < NG && ok; ++g, ++git) {
                const int slot = git % TC_RAW_SLOTS;
                if (!tc_wait(&raw_full[slot], (uint32_t)(git / TC_RAW_SLOTS) & 1u, abort_flag, a.status, ST_TIMEOUT_FULL)) {
                    ok = false;
                    break;
                }
                // per group pair: scales (words 0, 4), and this half's quant words
                uint32_t w[TC_GRP / 2][6];
                const uint32_t *src = reinterpret_cast<const uint32_t *>(smem + slot * TC_RAW_BYTES + wrow * TC_RAW_ROW);
#pragma unroll
                for (int j = 0; j < TC_GRP / 2; ++j) {
                    const uint32_t *pw = src + 9 * j;
                    w[j][0] = pw[0];
                    w[j][1] = pw[2];
                    w[j][2] = pw[4];
                    w[j][3] = pw[1 + 2 * hb];
                    w[j][4] = pw[5 + 2 * hb];
                    w[j][5] = pw[6 + 2 * hb];
                }
#pragma unroll
                for (int j = 0; j < TC_GRP / 2; ++j) {     // group pair j -> stages it+2j, it+2j+1
                    const int i0 = it + 2 * j, i1 = i0 + 1;
                    const int st0 = i0 % TC_STAGES, st1 = i1 % TC_STAGES;
                    // each stage waits for its own previous use (a pair of stages straddles the
                    // first pass through the ring if the stage count is odd)
                    if ((i0 >= TC_STAGES &&
                         !tc_wait(&empty_bar[st0], (uint32_t)(i0 / TC_STAGES - 1) & 1u, abort_flag, a.status, ST_TIMEOUT_EMPTY)) ||
                        (i1 >= TC_STAGES &&
                         !tc_wait(&empty_bar[st1], (uint32_t)(i1 / TC_STAGES - 1) & 1u, abort_flag, a.status, ST_TIMEOUT_EMPTY))) {
                        ok = false;
                        break;
                    }
                    const uint32_t w0 = w[j][0], w2 = w[j][1], w4 = w[j][2];
                    const uint32_t d0 = w0 & 0xFFFFu, d1 = w4 >> 16;
                    // group 0: bytes 0..7 (half 0) are w0[2..3], w1, w2[0..1]; bytes 8..15 (half 1)
                    // are w2[2..3], w3, w4[0..1]; group 1: words 5,6 (half 0) or 7,8 (half 1)
                    const uint32_t u0 = hb ? __byte_perm(w2, w[j][3], 0x5432) : __byte_perm(w0, w[j][3], 0x5432);
                    const uint32_t u1 = hb ? __byte_perm(w[j][3], w4, 0x5432) : __byte_perm(w[j][3], w2, 0x5432);
                    uint4 l0, h0, l1, h1;
                    const bool low = KIND == 2 && pass == 2;      // W_lo in the third pass
                    q4_half_group(u0, u1, d0 | (d0 << 16), l0, h0, low);
                    q4_half_group(w[j][4], w[j][5], d1 | (d1 << 16), l1, h1, low);
                    uint8_t *sa0 = smem + TC_STAGE0 + st0 * TC_STAGE_BYTES + hr * (TC_BM / 8) * TC_SBO;
                    uint8_t *sa1 = smem + TC_STAGE0 + st1 * TC_STAGE_BYTES + hr * (TC_BM / 8) * TC_SBO;
                    *reinterpret_cast<uint4 *>(sa0 + canon_off(rr, hb)) = l0;
                    *reinterpret_cast<uint4 *>(sa0 + canon_off(rr, 2 + hb)) = h0;
                    *reinterpret_cast<uint4 *>(sa1 + canon_off(rr, hb)) = l1;
                    *reinterpret_cast<uint4 *>(sa1 + canon_off(rr, 2 + hb)) = h1;
                    fence_async_smem();                    // generic-proxy writes -> tensor core
                    mbar_arrive(&a_full[st0]);
                    mbar_arrive(&a_full[st1]);
                }
                // The slot is released only after all its stages are decoded: the TMA engine
                // (async proxy) refills it, and a release right after the shared-memory loads let
                // the refill overtake them (corrupted rows measured on B200).
                mbar_arrive(&raw_empty[slot]);
                it += TC_GRP;
            }
            if (!__all_sync(0xffffffffu, ok)) break;
            // epilogue: wait for the accumulators, read this warp's 32 rows (tcgen05.ld is
            // warp-collective, so the whole warp decides together)
            const bool got = tc_wait(&acc_full, (uint32_t)ti & 1u, abort_flag, a.status, ST_TIMEOUT_FULL);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const int row = quad * 32 + lane;              // accumulator row (TMEM lane)
            for (int c0 = colq * (BN / 4); c0 < colq * (BN / 4) + BN / 4 && c0 < cnt; c0 += 32) {
                float g[32], w2[32];
                tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c0, g);
                tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + TC_BN + c0, w2);
                if (KIND == 0) {
                    const int feat = m * TC_BM + row;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int col = c0 + j;
                        if (col < cnt) {
                            // silu(g)*u with the fast exponential and division: h is rounded to
                            // fp16 next, so their few-ulp error stays far below that rounding
                            const float gv = g[j];
                            const float h = __fdividef(gv, 1.0f + __expf(-gv)) * w2[j];
                            a.h_out[(size_t)(off + col) * a.F + feat] = __float2half_rn(h);
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int col = c0 + j;
                        if (col < cnt) {
                            float *yr = a.y_out + (KIND == 2 ? pass * a.pass_stride : 0) +
                                        (size_t)a.pairs[off + col] * a.D + m * TC_ROWS;
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

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int build_row_maps(const uint8_t *const *h_ptrs, int E, int D, int F, int wenc, int rows_gu, int rows_dn,
                   void **d_maps) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled is unavailable from the driver");
        return CPG_ECUDA;
    }
    const int gb = wenc == CPG_ENC_Q4 ? 18 : 34;
    // a box is 256 K values of each row: 8 groups (144 B for Q4_0 as bytes, 272 B for Q8_0 as
    // 16-bit elements, since a box dimension holds at most 256 elements)
    const int esz = wenc == CPG_ENC_Q4 ? 1 : 2;
    CUtensorMap *h = (CUtensorMap *)malloc(sizeof(CUtensorMap) * 3 * (size_t)E);
    CPG_REQUIRE(h != nullptr, "host allocation failed");
    for (int i = 0; i < 3 * E; ++i) {
        const int kind = i % 3;                               // 0 gate, 1 up: (F, D); 2 down: (D, F)
        const int n_in = kind == 2 ? F : D, n_out = kind == 2 ? D : F;
        const cuuint64_t rb = (cuuint64_t)(n_in / 32) * gb;
        const cuuint64_t dims[2] = {rb / esz, (cuuint64_t)n_out};
        const cuuint64_t strides[1] = {rb};
        const cuuint32_t box[2] = {(cuuint32_t)(8 * gb / esz), (cuuint32_t)(kind == 2 ? rows_dn : rows_gu)};
        const cuuint32_t estr[2] = {1, 1};
        const CUresult r = enc(&h[i], esz == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
                               const_cast<uint8_t *>(h_ptrs[i]), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            free(h);
            set_error("tensor map of expert %d kind %d failed (%d)", i / 3, kind, (int)r);
            return CPG_ECUDA;
        }
    }
    void *d = nullptr;
    cudaError_t ce = cudaMalloc(&d, sizeof(CUtensorMap) * 3 * (size_t)E);
    if (ce == cudaSuccess) ce = cudaMemcpy(d, h, sizeof(CUtensorMap) * 3 * (size_t)E, cudaMemcpyHostToDevice);
    free(h);
    if (ce != cudaSuccess) {
        cudaFree(d);
        return cuda_fail(ce, "tensor map upload");
    }
    *d_maps = d;
    return CPG_OK;
}

int gemm_tc_build_weight_maps(const uint8_t *const *h_ptrs, int E, int D, int F, void **d_maps) {
    return build_row_maps(h_ptrs, E, D, F, CPG_ENC_Q4, TC_BM, TC_BM, d_maps);
}

int gemm_tc_dense_maps(const uint8_t *const *w, const int *rows, const int *k, int n, void **d_maps) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled is unavailable from the driver");
        return CPG_ECUDA;
    }
    std::vector<CUtensorMap> h((size_t)3 * n);
    for (int i = 0; i < n; ++i) {
        CPG_REQUIRE(rows[i] % TC_ROWS == 0 && k[i] % (TC_BK * TC_GRP) == 0,
                    "dense GEMM: a %d x %d matrix is not a multiple of %d x %d", rows[i], k[i], TC_ROWS, TC_BK * TC_GRP);
        const cuuint64_t rb = (cuuint64_t)(k[i] / 32) * 18;              // Q4_0 row bytes
        const cuuint64_t dims[2] = {rb, (cuuint64_t)rows[i]};
        const cuuint64_t strides[1] = {rb};
        const cuuint32_t box[2] = {(cuuint32_t)TC_RAW_ROW, (cuuint32_t)TC_BM};
        const cuuint32_t estr[2] = {1, 1};
        const CUresult r = enc(&h[(size_t)3 * i + 2], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(w[i]), dims,
                               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            set_error("dense GEMM: tensor map of matrix %d failed (%d)", i, (int)r);
            return CPG_ECUDA;
        }
        h[(size_t)3 * i] = h[(size_t)3 * i + 1] = h[(size_t)3 * i + 2];   // only entry 3i+2 is read
    }
    void *d = nullptr;
    cudaError_t ce = cudaMalloc(&d, sizeof(CUtensorMap) * h.size());
    if (ce == cudaSuccess) ce = cudaMemcpy(d, h.data(), sizeof(CUtensorMap) * h.size(), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        cudaFree(d);
        return cuda_fail(ce, "dense GEMM: tensor map upload");
    }
    *d_maps = d;
    return CPG_OK;
}

// y = p0 + p1 + p2 over the three planes of the passes, in that order.
__global__ void k_sum3(const float4 *__restrict__ p, size_t n4, float4 *__restrict__ y) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 a = p[i], b = p[n4 + i], c = p[2 * n4 + i];
        y[i] = make_float4((a.x + b.x) + c.x, (a.y + b.y) + c.y, (a.z + b.z) + c.z, (a.w + b.w) + c.w);
    }
}

int gemm_tc_dense(const void *maps, const int4 *tab, const int *n_active, const int *iota, const __half *x16, int T,
                  int rows, int k, float *y, float *planes, int *status, cudaStream_t s) {
    TcArgs a{};
    a.n_active = n_active;
    a.act = tab;
    a.wmaps = maps;
    a.pairs = iota;
    a.D = rows;
    a.F = k;
    a.K = 1;
    a.y_out = planes;
    a.pass_stride = (size_t)T * rows;
    a.status = status;
    const int rc = gemm_tc_launch(2, a, x16, T, 3 * (rows / TC_ROWS) * ((T + TC_BN_SMALL - 1) / TC_BN_SMALL), s);
    if (rc) return rc;
    const size_t n4 = (size_t)T * rows / 4;
    k_sum3<<<(int)(n4 / 256 + 1 < 1184 ? n4 / 256 + 1 : 1184), 256, 0, s>>>((const float4 *)planes, n4, (float4 *)y);
    CPG_CUDA(cudaGetLastError());
    return CPG_OK;
}

int gemm_tc_launch(int kind, const TcArgs &a, const __half *b, int b_rows, int max_tiles, cudaStream_t s) {
    const int kdim = kind == 0 ? a.D : a.F;
    const int bdim = kind == 2 ? 2 * kdim : kdim;                   // [x_hi | x_lo] for kind 2
    CPG_REQUIRE(kdim % (TC_BK * TC_GRP) == 0, "grouped GEMM: K=%d must be a multiple of %d", kdim, TC_BK * TC_GRP);
    CPG_REQUIRE(((uintptr_t)b & 15) == 0, "grouped GEMM: token rows must be 16-byte aligned");
    EncodeTiledFn enc = encode_tiled();
    if (!enc) {
        set_error("grouped GEMM: cuTensorMapEncodeTiled is unavailable from the driver");
        return CPG_ECUDA;
    }
    CUtensorMap map[2];
    const cuuint64_t dims[2] = {(cuuint64_t)bdim, (cuuint64_t)b_rows};
    const cuuint64_t strides[1] = {(cuuint64_t)bdim * 2};
    const cuuint32_t estr[2] = {1, 1};
    for (int i = 0; i < 2; ++i) {
        const cuuint32_t box[2] = {TC_BK, (cuuint32_t)(i == 0 ? TC_BN : TC_BN_SMALL)};
        const CUresult r = enc(&map[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(b), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            set_error("grouped GEMM: cuTensorMapEncodeTiled failed (%d)", (int)r);
            return CPG_ECUDA;
        }
    }
    auto *k = kind == 0 ? k_gemm_tc<0> : kind == 1 ? k_gemm_tc<1> : k_gemm_tc<2>;
    const size_t smem = (size_t)TC_SMEM + 1024;
    CPG_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int grid = sm_count();
    if (max_tiles < grid) grid = max_tiles > 0 ? max_tiles : 1;
    k<<<grid, TC_THREADS, smem, s>>>(a, map[0], map[1]);
    CPG_CUDA(cudaGetLastError());
    return CPG_OK;
}

}  // namespace cpg
