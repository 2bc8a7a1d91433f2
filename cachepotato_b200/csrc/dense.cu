// dense.cu — W·x for a batch of up to 64 token rows on the tensor cores at the reference's f32
// accuracy: the attention projections and the lm_head of a step of several sequences (the
// matmul_wx_q4 / matmul_wx_q8 calls of qwen3_layer_kv and apply_head, engine/kernels/
// kernels.c:368-396, 514-540, one row of x per sequence).
//
// The weights are read from a decode tile copy of the matrix (the layout of expert_tile.cuh:
// 16 rows × 256 values per tile, K slice major), built once; the activations are prepared once
// per step as fp16 hi + lo halves in the decode K permutation, laid out slice by slice:
//     xh[s][t] = hi(x_t[256s .. 256s + 255]) (512 B), 16 B gap, lo(...) (512 B), 16 B gap
// so that one bulk copy brings a K slice of every token. A CTA owns a band of 64 rows and one
// range of K slices (split K when the bands alone leave SMs idle): one producer thread copies
// the band's four tiles and the tokens' slice per stage (2-8 stages, as many as fit), eight consumer warps
// (four 16-row groups × two halves of the tokens) decode Q4_0 / Q8_0 in registers into
// mma.sync.m16n8k16 with the tokens' hi and lo halves in neighbouring N columns, scale each
// group's partial sums in fp32 and add hi + lo at the end, as the batched expert kernel does.
// Split-K partial rows go to planes; the band's last CTA adds them in range order (deterministic).
#include <algorithm>

#include "common.cuh"
#include "expert_tile.cuh"

namespace cpg {

constexpr int DN_CW = 8;                          // consumer warps
constexpr int DN_THREADS = (DN_CW + 1) * 32;
constexpr int DN_ROWS = 64;                       // rows per band
constexpr int DN_MAXT = 64;                       // token rows per launch
constexpr int DN_LOFF = EX_KSL * 2 + 16;          // a token slice's lo half
constexpr int DN_BROW = 2 * DN_LOFF;              // one token's slice
constexpr int DN_MAX_STAGES = 8;                  // ring depth: as many stages as fit, at most 8

__constant__ Perm64 c_perm_dense[2] = {kPermQ4, kPermQ8};

struct DenseSeg {
    const uint8_t *tiles;
    float *out;                                   // (T, rows)
    int rows;
};
struct DenseArgs {
    DenseSeg seg[3];
    int band0[4];                                 // first band of each segment; band0[nseg] = all
    int row0[4];                                  // first row of each segment in the planes
    int nseg, rows_all;
    const uint8_t *xh;
    int T, K, spc;                                // spc: K slices per split
    float *planes;                                // split K: (splits, T, rows_all)
    int *counters;                                // split K: one per band, zero between launches
    int *status;
    int stages;                                   // ring depth (<= DN_MAX_STAGES)
};

// One K slice of one 16-row tile against ntw ≤ 8 eight-column tiles of tokens (bs: this lane's
// first B word; TS bytes from one column tile to the next). One group at a time: its two k16
// steps accumulate into a fresh sum that is scaled by the group's fp32 scale, as the reference
// applies d per group (kernels.c:368-396).
template <int ENC>
__device__ __forceinline__ void dense_slice(const uint8_t *tp, int lane, const uint8_t *bs, int ntw,
                                            float (&acc)[8][4]) {
    using X = ExTile<ENC>;
    constexpr int TS = 4 * DN_BROW;
    const uint2 *sc = reinterpret_cast<const uint2 *>(tp + X::DB + (lane >> 2) * 32);
#pragma unroll
    for (int P = 0; P < 4; ++P) {
        const uint2 sg = sc[P >> 1], s8 = sc[2 + (P >> 1)];
        const uint32_t dg = P & 1 ? sg.y : sg.x, d8 = P & 1 ? s8.y : s8.x;
        const float2 fg = __half22float2(*reinterpret_cast<const __half2 *>(&dg));
        const float2 f8 = __half22float2(*reinterpret_cast<const __half2 *>(&d8));
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            uint32_t fh[2][4];
            group_frags<ENC>(tp, P, hf, lane, fh);
            const float d0 = hf ? fg.y : fg.x, d1 = hf ? f8.y : f8.x;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                if (nt < ntw) {
                    const uint4 bq = *reinterpret_cast<const uint4 *>(bs + nt * TS + P * 128 + hf * 16);
                    const float z[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    float sj[4];
                    mma_16816(sj, fh[0], bq.x, bq.y, z);
                    mma_16816(sj, fh[1], bq.z, bq.w, sj);
                    fma2_f32(acc[nt][0], acc[nt][1], d0, sj[0], sj[1]);
                    fma2_f32(acc[nt][2], acc[nt][3], d1, sj[2], sj[3]);
                }
            }
        }
    }
}

template <int ENC>
__global__ void __launch_bounds__(DN_THREADS, 1) k_dense_dec(const DenseArgs a) {
    using X = ExTile<ENC>;
    extern __shared__ uint8_t dn_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dn_raw) + 127) & ~uintptr_t(127));
    __shared__ __align__(8) uint64_t full[DN_MAX_STAGES], empty[DN_MAX_STAGES];
    const int NST = a.stages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int band = blockIdx.x, kidx = blockIdx.y;
    int sg = 0;                                           // the segment (static indices only)
#pragma unroll
    for (int i = 1; i < 3; ++i)
        if (i < a.nseg && band >= a.band0[i]) sg = i;
    const DenseSeg seg = sg == 0 ? a.seg[0] : sg == 1 ? a.seg[1] : a.seg[2];
    const int rb = band - (sg == 0 ? a.band0[0] : sg == 1 ? a.band0[1] : a.band0[2]);
    const int row0 = sg == 0 ? a.row0[0] : sg == 1 ? a.row0[1] : a.row0[2];
    const int R = seg.rows, T = a.T;
    const int NS = a.K / EX_KSL;
    const int s0 = kidx * a.spc, s1 = min(NS, s0 + a.spc);
    // a stage holds the token slices rounded up to four (the B fragments of a column tile read
    // four tokens whatever T is; the columns past T are never written out)
    const uint32_t wbytes = 4 * X::TB, abytes = (uint32_t)T * DN_BROW;
    const size_t stage = ((size_t)wbytes + (size_t)((T + 3) & ~3) * DN_BROW + 127) & ~size_t(127);
    if (tid == 0) {
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], DN_CW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();                                           // xh from the preparing kernel
    pdl_launch_dependents();

    if (warp == DN_CW) {                                  // ---------------- producer
        if (lane != 0) return;
        int issued = 0;
        for (int s = s0; s < s1; ++s, ++issued) {
            const int i = s - s0, st = i % NST;
            if (i >= NST && !mbar_wait(&empty[st], (uint32_t)(i / NST - 1) & 1u)) {
                atomicCAS(a.status, ST_OK, ST_TIMEOUT_EMPTY);
                break;
            }
            uint8_t *dst = smem + st * stage;
            mbar_arrive_expect_tx(&full[st], wbytes + abytes);
            bulk_g2s(dst, seg.tiles + ((size_t)s * (R / 16) + (size_t)rb * 4) * X::TB, wbytes, &full[st]);
            bulk_g2s(dst + wbytes, a.xh + (size_t)s * abytes, abytes, &full[st]);
        }
        for (int k = 1; k <= NST && issued - k >= 0; ++k) {         // copies in flight land first
            const int j = issued - k;
            mbar_wait(&full[j % NST], (uint32_t)(j / NST) & 1u);
        }
        return;
    }

    // ---------------- consumers: warp w owns rows 16·(w & 3) .. + 15 of the band and tokens
    // 32·(w >> 2) .. + 31. MMA column 8·nt + c holds token 4·nt + c/2 of the half, its hi half
    // for even c, lo for odd c; acc[nt][0] + acc[nt][1] is token 4·nt + t at row g,
    // acc[nt][2] + acc[nt][3] at row g + 8.
    const int rg = warp & 3, hh = warp >> 2;
    const int g = lane >> 2, t = lane & 3;
    const int nt_all = (T + 3) >> 2;
    const int ntw = max(0, min(8, nt_all - 8 * hh));
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[nt][c] = 0.0f;
    bool ok = true;
    for (int s = s0; s < s1; ++s) {
        const int i = s - s0, st = i % NST;
        if (!mbar_wait(&full[st], (uint32_t)(i / NST) & 1u)) {
            if (lane == 0) atomicCAS(a.status, ST_OK, ST_TIMEOUT_FULL);
            ok = false;
            break;
        }
        const uint8_t *sb = smem + st * stage;
        if (ntw > 0)
            dense_slice<ENC>(sb + rg * X::TB, lane,
                             sb + wbytes + (size_t)(32 * hh + (g >> 1)) * DN_BROW + (g & 1) * DN_LOFF + t * 32, ntw, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    // a warp whose wait gave up (status recorded) writes nothing but still meets the barriers below
    const int r = rb * DN_ROWS + rg * 16 + g;                 // rows r, r + 8 of the segment
    const int splits = gridDim.y;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
        const int tok = 32 * hh + 4 * nt + t;
        if (!ok || nt >= ntw || tok >= T) continue;
        float *o = splits > 1 ? a.planes + ((size_t)kidx * T + tok) * a.rows_all + row0 : seg.out + (size_t)tok * R;
        o[r] = acc[nt][0] + acc[nt][1];
        o[r + 8] = acc[nt][2] + acc[nt][3];
    }
    if (splits == 1) return;
    // split K: the last CTA of the band to finish adds the ranges' partial rows in range order
    __shared__ int s_last;
    __threadfence();
    named_bar_sync(1, DN_CW * 32);
    if (tid == 0) s_last = atomicAdd(a.counters + band, 1) == splits - 1;
    named_bar_sync(1, DN_CW * 32);
    if (!s_last) return;
    __threadfence();
    const size_t plane = (size_t)T * a.rows_all;
    for (int i = tid; i < T * DN_ROWS; i += DN_CW * 32) {
        const int tok = i / DN_ROWS, rr = rb * DN_ROWS + i % DN_ROWS;
        const float *p = a.planes + (size_t)tok * a.rows_all + row0 + rr;
        float v = __ldcg(p);
        for (int k = 1; k < splits; ++k) v += __ldcg(p + k * plane);
        seg.out[(size_t)tok * R + rr] = v;
    }
    if (tid == 0) a.counters[band] = 0;                       // ready for the next launch
}

// Token rows x (T, K) f32 -> xh (the layout above) for weights of encoding enc, optionally through
// rmsnorm with gain first (kernels.c:408-413: inv = 1 / sqrt(Σx²/K + eps), (x·inv)·g). Block
// (token, K slice), 128 threads, two positions each; with a gain every block of the token forms
// the row's sum of squares itself (8-16 KB from L2) rather than waiting for another.
__global__ void __launch_bounds__(128) k_dense_act(const float *__restrict__ x, int T, int K, const float *__restrict__ gain,
                                                    float eps, int enc, uint8_t *__restrict__ xh) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float s_red[4];
    const int tok = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
    const float *xr = x + (size_t)tok * K;
    float inv = 1.0f;
    if (gain) {
        const float4 *x4 = reinterpret_cast<const float4 *>(xr);
        float ss = 0.0f;
        for (int c = tid; c < K / 4; c += 128) {
            const float4 v = __ldg(x4 + c);
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) s_red[tid >> 5] = ss;
        __syncthreads();
        const float tot = (s_red[0] + s_red[1]) + (s_red[2] + s_red[3]);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(tot, (float)K) + eps));
    }
    const Perm64 &pm = c_perm_dense[enc == CPG_ENC_Q4 ? 0 : 1];
    const int q = 2 * tid;                                       // positions q, q + 1 of the slice
    const int e0 = s * EX_KSL + (q & ~63) + pm.pos_to_elem[q & 63];
    const int e1 = s * EX_KSL + (q & ~63) + pm.pos_to_elem[(q + 1) & 63];
    float v0 = __ldg(xr + e0), v1 = __ldg(xr + e1);
    if (gain) {
        v0 = __fmul_rn(__fmul_rn(v0, inv), __ldg(gain + e0));
        v1 = __fmul_rn(__fmul_rn(v1, inv), __ldg(gain + e1));
    }
    uint32_t hi, lo;
    split_half2(v0, v1, hi, lo);
    uint8_t *dst = xh + ((size_t)s * T + tok) * DN_BROW;
    *reinterpret_cast<uint32_t *>(dst + 2 * q) = hi;
    *reinterpret_cast<uint32_t *>(dst + DN_LOFF + 2 * q) = lo;
}

// The decode tiles of one R × K matrix (K slice major), one thread per (tile, lane).
template <int ENC>
__global__ void k_tile_matrix(const uint8_t *__restrict__ src, int R, int K, uint8_t *__restrict__ out) {
    using X = ExTile<ENC>;
    const int RT = R / 16;
    const long n = (long)RT * (K / EX_KSL) * 32;
    const size_t rowb = (size_t)K / 32 * X::GB;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const long q = i >> 5;
        const int s = (int)(q / RT), rt = (int)(q - (long)s * RT);
        const uint8_t *t0 = src + (size_t)rt * 16 * rowb + (size_t)s * 8 * X::GB;
        tile_build_lane<ENC>(t0, t0 + 8 * rowb, rowb, out + (size_t)q * X::TB, lane);
    }
}

// ------------------------------------------------------------------ host side

bool dense_ok(int enc, int rows, int k) {
    return (enc == CPG_ENC_Q4 || enc == CPG_ENC_Q8) && rows > 0 && rows % DN_ROWS == 0 && k > 0 && k % EX_KSL == 0;
}

size_t dense_act_bytes(int T, int K) { return (size_t)(K / EX_KSL) * T * DN_BROW; }

int dense_build(const void *w, int enc, int rows, int k, uint8_t **tiles, cudaStream_t s) {
    CPG_REQUIRE(dense_ok(enc, rows, k), "dense tiles: a %d x %d matrix of encoding %d", rows, k, enc);
    const size_t bytes = (size_t)rows * k / 32 * (enc == CPG_ENC_Q4 ? 18 : 34);
    uint8_t *p = nullptr;
    CPG_CUDA(cudaMalloc(&p, bytes));
    const long threads = (long)(rows / 16) * (k / EX_KSL) * 32;
    const int grid = (int)std::min<long>((threads + 255) / 256, 148L * 16);
    if (enc == CPG_ENC_Q4)
        k_tile_matrix<CPG_ENC_Q4><<<grid, 256, 0, s>>>((const uint8_t *)w, rows, k, p);
    else
        k_tile_matrix<CPG_ENC_Q8><<<grid, 256, 0, s>>>((const uint8_t *)w, rows, k, p);
    const cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(ce, "dense tiles: build");
    }
    *tiles = p;
    return CPG_OK;
}

int dense_prep(const float *x, int T, int K, const float *gain, float eps, int enc, uint8_t *xh, cudaStream_t s) {
    CPG_REQUIRE(T >= 1 && T <= DN_MAXT && K % EX_KSL == 0, "dense: %d rows of %d values", T, K);
    CPG_CUDA(launch_pdl(k_dense_act, dim3(T, K / EX_KSL), dim3(128), 0, s, x, T, K, gain, eps, enc, xh));
    return CPG_OK;
}

// y_i = W_i · x for nseg ≤ 3 matrices of one encoding and width K (tiles from dense_build),
// x prepared by dense_prep for that encoding. Split K needs planes (room for planes_floats f32)
// and n_counters zeroed ints (at least the bands).
int dense_run(const uint8_t *const *tiles, const int *rows, float *const *outs, int nseg, int enc, int K,
              const uint8_t *xh, int T, float *planes, size_t planes_floats, int *counters, int n_counters,
              int *status, cudaStream_t s) {
    CPG_REQUIRE(nseg >= 1 && nseg <= 3 && T >= 1 && T <= DN_MAXT, "dense: %d matrices, %d rows", nseg, T);
    DenseArgs a{};
    a.nseg = nseg;
    a.xh = xh;
    a.T = T;
    a.K = K;
    a.planes = planes;
    a.counters = counters;
    a.status = status;
    int bands = 0, rall = 0;
    for (int i = 0; i < nseg; ++i) {
        CPG_REQUIRE(dense_ok(enc, rows[i], K), "dense: a %d x %d matrix", rows[i], K);
        a.seg[i] = DenseSeg{tiles[i], outs[i], rows[i]};
        a.band0[i] = bands;
        a.row0[i] = rall;
        bands += rows[i] / DN_ROWS;
        rall += rows[i];
    }
    a.band0[nseg] = bands;
    a.row0[nseg] = rall;
    a.rows_all = rall;
    // split K while the CTAs still fit one wave (a CTA's stages take most of an SM's shared
    // memory: one CTA per SM), as far as the planes allow; measured at 64 tokens: 2-3 waves of
    // short two-slice CTAs took 38 us for q, k, v of a Qwen3 layer
    const int NS = K / EX_KSL, sms = sm_count();
    int splits = bands >= sms || bands > n_counters ? 1 : std::max(1, std::min(NS, sms / bands));
    while (splits > 1 && (size_t)splits * T * rall > planes_floats) --splits;
    a.spc = (NS + splits - 1) / splits;
    splits = (NS + a.spc - 1) / a.spc;
    const uint32_t tb = enc == CPG_ENC_Q4 ? ExTile<CPG_ENC_Q4>::TB : ExTile<CPG_ENC_Q8>::TB;
    const size_t stage = ((size_t)4 * tb + (size_t)((T + 3) & ~3) * DN_BROW + 127) & ~size_t(127);   // as the kernel
    // as deep a ring as fits: a step of a few sequences has small stages (the weight tiles and a
    // few token slices), and the copies in flight per SM are what bounds it
    const int fit = (int)(((size_t)smem_optin() - 4096 - 128) / stage);
    a.stages = std::max(2, std::min(DN_MAX_STAGES, fit));
    const size_t smem = a.stages * stage + 128;
    const void *k = enc == CPG_ENC_Q4 ? (const void *)k_dense_dec<CPG_ENC_Q4> : (const void *)k_dense_dec<CPG_ENC_Q8>;
    const int rc = allow_max_smem(k);
    if (rc) return rc;
    if (enc == CPG_ENC_Q4)
        CPG_CUDA(launch_pdl(k_dense_dec<CPG_ENC_Q4>, dim3(bands, splits), dim3(DN_THREADS), smem, s, a));
    else
        CPG_CUDA(launch_pdl(k_dense_dec<CPG_ENC_Q8>, dim3(bands, splits), dim3(DN_THREADS), smem, s, a));
    return CPG_OK;
}

}  // namespace cpg
