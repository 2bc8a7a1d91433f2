// expert_tile.cuh — the decode tile layout of expert matrices and its register decoders,
// shared by the expert kernels (moe.cu) and the one-token layer kernel (moe_one.cu).
#pragma once
#include "common.cuh"
#include "layout.cuh"

namespace cpg {

constexpr int EX_KSL = 256;       // values per K slice of a decode tile (eight 32-value groups)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// The reference's top-k scan (engine/blocks/qwen3_moe.c:184-194) by one warp over probabilities
// held PL per lane (expert lane + 32 i): for each slot j the scan starts from the lowest-id
// expert not yet taken and moves only to a strictly larger probability, so ties keep the lower
// id, a NaN never wins, and a NaN first candidate stays selected. Returns the ids and their
// probabilities in selection order (valid on every lane).
template <int PL, int MAXK>
__device__ __forceinline__ void warp_topk(const float (&p)[PL], int E, int K, int (&sel_e)[MAXK],
                                          float (&sel_p)[MAXK]) {
    const int lane = threadIdx.x & 31;
    uint32_t taken = 0;                       // bit i: expert lane + 32 i already selected
    for (int j = 0; j < K && j < MAXK; ++j) {
        float bv = -1.0f;                     // probabilities are >= 0 (or NaN)
        int be = 0x7fffffff, first = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < PL; ++i) {
            const int e = lane + 32 * i;
            if (e < E && !((taken >> i) & 1u)) {
                if (e < first) first = e;
                if (p[i] > bv) { bv = p[i]; be = e; }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {     // larger probability wins, equal: lower id
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            const int of = __shfl_xor_sync(0xffffffffu, first, o);
            if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
            if (of < first) first = of;
        }
        // the scan's starting point keeps the slot if its probability is NaN (nothing compares
        // larger) or if no number beat it
        float mine = 0.0f;                    // this lane's value in the first candidate's column
#pragma unroll
        for (int i = 0; i < PL; ++i)
            if (i == (first >> 5)) mine = p[i];
        const float pf = __shfl_sync(0xffffffffu, mine, first & 31);
        if (first < E && (isnan(pf) || be >= E)) { be = first; bv = pf; }
        if ((be & 31) == lane && be < E) taken |= 1u << (be >> 5);
        sel_p[j] = bv;
        sel_e[j] = be;
    }
}

// Softmax over the E logits of one token, strict-'>' top-k (larger probability first, lower id on ties) and
// renormalisation (qwen3_moe.c:181-197; softmax kernels.c:20-26), by the whole CTA. Warp 0
// computes the probabilities into shared memory; thread e then counts the rank of expert e,
// #{e' : p' > p, or p' == p and e' < e}, and the experts of rank < K fill the K slots in rank
// order: the reference scan's result without its K sequential passes (the loops stay short:
// this code runs once per launch, so its instruction fetch is part of the latency). A NaN
// probability makes ranks meaningless; warp 0 then runs the scan itself (warp_topk, which
// reproduces the reference's NaN behaviour). logits: global memory, or shared memory with
// LOGITS_SMEM; s_p: 16-byte aligned shared memory for MAXE + MAXK floats (MAXE a multiple of
// four); sel_e, sel_w: K ids and weights, in shared or global memory. Every thread of the CTA
// calls it.
template <int MAXE, int MAXK, bool LOGITS_SMEM = false>
__device__ void select_topk(const float *logits, int E, int K, int *sel_e, float *sel_w, float *s_p) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int PL = MAXE / 32;
    __shared__ int s_nan;
    if (warp == 0) {
        float p[PL];
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < PL; ++i) {
            const int e = lane + 32 * i;
            p[i] = e < E ? (LOGITS_SMEM ? logits[e] : __ldcg(logits + e)) : -INFINITY;
            mx = fmaxf(mx, p[i]);
        }
        mx = warp_max(mx);
        float sum = 0.0f;
#pragma unroll 1
        for (int i = 0; i < PL; ++i) {
            const int e = lane + 32 * i;
            p[i] = e < E ? expf(p[i] - mx) : 0.0f;
            sum += p[i];
        }
        sum = warp_sum(sum);
        bool nan = false;
#pragma unroll 1
        for (int i = 0; i < PL; ++i) {
            const int e = lane + 32 * i;
            p[i] = __fdiv_rn(p[i], sum);
            if (e < E) {
                s_p[e] = p[i];
                nan |= isnan(p[i]);
            }
        }
        nan = __any_sync(0xffffffffu, nan);
        if (lane == 0) s_nan = nan;
        if (lane < ((E + 3) & ~3) - E) s_p[E + lane] = -INFINITY;     // the rank loop's padding
        if (nan) {
            float sp[MAXK];
            int se[MAXK];
            warp_topk<PL, MAXK>(p, E, K, se, sp);
            if (lane == 0)
                for (int j = 0; j < K; ++j) {
                    sel_e[j] = se[j];
                    s_p[MAXE + j] = sp[j];
                }
        }
    }
    __syncthreads();
    if (!s_nan) {
        // rank of expert e: the probabilities read four at a time (s_p is 16-byte aligned and
        // padded with -inf up to a multiple of four, which never counts)
        const int E4 = (E + 3) >> 2;
        for (int e = tid; e < E; e += blockDim.x) {
            const float pe = s_p[e];
            int r = 0;
#pragma unroll 4
            for (int f4 = 0; f4 < E4; ++f4) {
                const float4 q = reinterpret_cast<const float4 *>(s_p)[f4];
                const int f = 4 * f4;
                r += (q.x > pe || (q.x == pe && f < e)) ? 1 : 0;
                r += (q.y > pe || (q.y == pe && f + 1 < e)) ? 1 : 0;
                r += (q.z > pe || (q.z == pe && f + 2 < e)) ? 1 : 0;
                r += (q.w > pe || (q.w == pe && f + 3 < e)) ? 1 : 0;
            }
            if (r < K) {
                sel_e[r] = e;
                s_p[MAXE + r] = pe;
            }
        }
        __syncthreads();
    }
    if (tid < K) {                                       // qwen3_moe.c:195-197: the sum in selection
        float s = 0.0f;                                  // order (every thread the same), one division each
        for (int j = 0; j < K; ++j) s += s_p[MAXE + j];
        sel_w[tid] = __fdiv_rn(s_p[MAXE + tid], s);
    }
    __syncthreads();
}

template <int ENC>
__device__ __forceinline__ void load_pair_words(const uint32_t *row, int P, int t, uint32_t &w1,
                                                uint32_t &w2, uint32_t &w3, uint32_t &w4, float &d0,
                                                float &d1) {
    if (ENC == CPG_ENC_Q4) {
        const uint32_t *s = row + P * 9;
        const uint32_t wa = s[1 + t], w0 = s[0], wq = s[4], wb = s[5 + t];
        w1 = t == 3 ? __byte_perm(w0, wq, 0x5432) : wa;
        w2 = wb;
        w3 = 0; w4 = 0;
        d0 = __half2float(__ushort_as_half((unsigned short)(w0 & 0xFFFFu)));
        d1 = __half2float(__ushort_as_half((unsigned short)(wq >> 16)));
    } else {
        const uint32_t *s = row + P * 17;
        const uint32_t wa = s[1 + t], wb = s[5 + t], w0 = s[0], w8 = s[8], wc = s[9 + t], wd = s[13 + t];
        w1 = wa;
        w2 = t == 3 ? __byte_perm(w0, w8, 0x5432) : wb;
        w3 = wc;
        w4 = wd;
        d0 = __half2float(__ushort_as_half((unsigned short)(w0 & 0xFFFFu)));
        d1 = __half2float(__ushort_as_half((unsigned short)(w8 >> 16)));
    }
}

// Q4 word -> two k16 steps of one row: {lo(b0),lo(b2)}, {hi(b0),hi(b2)}, {lo(b1),lo(b3)}, {hi(b1),hi(b3)}
__device__ __forceinline__ void q4_word(uint32_t w, uint32_t &sA0, uint32_t &sA2, uint32_t &sB0, uint32_t &sB2) {
    const uint32_t k1032 = 0x64086408u, k1_16 = 0x2C002C00u, km72 = 0xD480D480u;
    const uint32_t w2 = w >> 8;
    sA0 = hsub2_u32(lop3_and_xor(w, 0x000F000Fu, 0x64086408u), k1032);
    sA2 = hfma2_u32(lop3_and_xor(w, 0x00F000F0u, 0x64806480u), k1_16, km72);
    sB0 = hsub2_u32(lop3_and_xor(w2, 0x000F000Fu, 0x64086408u), k1032);
    sB2 = hfma2_u32(lop3_and_xor(w2, 0x00F000F0u, 0x64806480u), k1_16, km72);
}

// Q8 word -> one k16 step of one row: {b0,b1}, {b2,b3}
__device__ __forceinline__ void q8_word(uint32_t w, uint32_t &s0, uint32_t &s2) {
    const uint32_t x = w ^ 0x80808080u, k1152 = 0x64806480u;
    s0 = hsub2_u32(__byte_perm(x, 0x64646464u, 0x4140), k1152);
    s2 = hsub2_u32(__byte_perm(x, 0x64646464u, 0x4342), k1152);
}

// Decode tile layout of one expert matrix (R rows, Kd values), built once per layer: tile (s, rt)
// covers rows [16rt, 16rt + 16) and values [256s, 256s + 256) and sits at byte (s·R/16 + rt)·TB,
// TB = 16 rows × 8 groups × group bytes, so the row tiles of one K slice are contiguous (one bulk
// copy per matrix and stage). An expert's gate and up matrices form one interleaved matrix of
// 2·d_exp rows: its tile rt holds gate rows [8rt, 8rt + 8) as tile rows 0-7 and the same up rows as
// tile rows 8-15, so one MMA row pair (g, g + 8) is feature 8rt + g of both matrices. Inside a
// tile, for group pair P and lane l = 4g + t of the warp that consumes it:
//   Q4: 16 B at (32P + l)·16 = row g's two words for this lane, then row g+8's two words;
//   Q8: 16 B at (32P + l)·16 = row g's four words; row g+8's at 2048 + (32P + l)·16;
// then the scales: row g's eight fp16 group scales at DB + 32g, row g+8's at DB + 32g + 16
// (DB = 2048 for Q4, 4096 for Q8). The words are the raw group bytes (load_pair_words), regrouped
// so that a lane's share of a pair is one aligned 16-byte load; the bytes per tile are unchanged.
template <int ENC>
struct ExTile {
    static constexpr int GB = ENC == CPG_ENC_Q4 ? 18 : 34;
    static constexpr int TB = 16 * 8 * GB;                    // bytes per tile
    static constexpr int DB = ENC == CPG_ENC_Q4 ? 2048 : 4096; // scale block offset
};

// Lane `lane`'s share of building one decode tile from raw rows: src = the raw row that becomes
// tile row 0 and src8 the one that becomes tile row 8, both at the tile's K slice (row stride
// rowb bytes; src8 = src + 8·rowb for 16 consecutive rows of one matrix), dst = the tile. Every
// lane of a warp writes its words of the four group pairs; lanes t = 0, 1 of each quad also write
// the scales of rows g, g + 8.
template <int ENC>
__device__ __forceinline__ void tile_build_lane(const uint8_t *src, const uint8_t *src8, size_t rowb, uint8_t *dst,
                                                int lane) {
    using X = ExTile<ENC>;
    const int g = lane >> 2, t = lane & 3;
    const uint32_t *rg = reinterpret_cast<const uint32_t *>(src + g * rowb);
    const uint32_t *r8 = reinterpret_cast<const uint32_t *>(src8 + g * rowb);
    for (int P = 0; P < 4; ++P) {
        uint32_t a1, a2, a3, a4, b1, b2, b3, b4;
        float d0, d1;
        load_pair_words<ENC>(rg, P, t, a1, a2, a3, a4, d0, d1);
        load_pair_words<ENC>(r8, P, t, b1, b2, b3, b4, d0, d1);
        if (ENC == CPG_ENC_Q4) {
            *reinterpret_cast<uint4 *>(dst + (P * 32 + lane) * 16) = make_uint4(a1, a2, b1, b2);
        } else {
            *reinterpret_cast<uint4 *>(dst + (P * 32 + lane) * 16) = make_uint4(a1, a2, a3, a4);
            *reinterpret_cast<uint4 *>(dst + 2048 + (P * 32 + lane) * 16) = make_uint4(b1, b2, b3, b4);
        }
    }
    if (t < 2) {                                               // lane t = 0: row g, t = 1: row g + 8
        const uint8_t *row = (t ? src8 : src) + g * rowb;
        uint32_t w[4];
        for (int j = 0; j < 4; ++j)
            w[j] = (uint32_t)*reinterpret_cast<const uint16_t *>(row + 2 * j * X::GB) |
                   ((uint32_t)*reinterpret_cast<const uint16_t *>(row + (2 * j + 1) * X::GB) << 16);
        *reinterpret_cast<uint4 *>(dst + X::DB + g * 32 + t * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Decoded fragments of pair P of a tile for this lane.
template <int ENC>
__device__ __forceinline__ void tile_frags(const uint8_t *tp, int P, int lane, uint32_t (&fr)[4][4]) {
    const uint4 w = *reinterpret_cast<const uint4 *>(tp + (P * 32 + lane) * 16);
    if (ENC == CPG_ENC_Q4) {
        q4_word(w.x, fr[0][0], fr[0][2], fr[1][0], fr[1][2]);
        q4_word(w.y, fr[2][0], fr[2][2], fr[3][0], fr[3][2]);
        q4_word(w.z, fr[0][1], fr[0][3], fr[1][1], fr[1][3]);
        q4_word(w.w, fr[2][1], fr[2][3], fr[3][1], fr[3][3]);
    } else {
        const uint4 v = *reinterpret_cast<const uint4 *>(tp + 2048 + (P * 32 + lane) * 16);
        q8_word(w.x, fr[0][0], fr[0][2]);
        q8_word(w.y, fr[1][0], fr[1][2]);
        q8_word(w.z, fr[2][0], fr[2][2]);
        q8_word(w.w, fr[3][0], fr[3][2]);
        q8_word(v.x, fr[0][1], fr[0][3]);
        q8_word(v.y, fr[1][1], fr[1][3]);
        q8_word(v.z, fr[2][1], fr[2][3]);
        q8_word(v.w, fr[3][1], fr[3][3]);
    }
}

// The fragments of one group (hf = 0: group 2P, 1: group 2P + 1) of pair P: fr[0..1] or fr[2..3]
// of tile_frags.
template <int ENC>
__device__ __forceinline__ void group_frags(const uint8_t *tp, int P, int hf, int lane, uint32_t (&fh)[2][4]) {
    const uint4 w = *reinterpret_cast<const uint4 *>(tp + (P * 32 + lane) * 16);
    if (ENC == CPG_ENC_Q4) {
        q4_word(hf ? w.y : w.x, fh[0][0], fh[0][2], fh[1][0], fh[1][2]);
        q4_word(hf ? w.w : w.z, fh[0][1], fh[0][3], fh[1][1], fh[1][3]);
    } else {
        const uint4 v = *reinterpret_cast<const uint4 *>(tp + 2048 + (P * 32 + lane) * 16);
        q8_word(hf ? w.z : w.x, fh[0][0], fh[0][2]);
        q8_word(hf ? w.w : w.y, fh[1][0], fh[1][2]);
        q8_word(hf ? v.z : v.x, fh[0][1], fh[0][3]);
        q8_word(hf ? v.w : v.y, fh[1][1], fh[1][3]);
    }
}

}  // namespace cpg
