// crc.cu — CRC-32 of device memory: the CPW1 v4 region digest (format/v4_writer.py:235-250:
// zlib.crc32 over exactly the region's bytes, stored as u64; the loader verifies it at open,
// engine/core/weights_v4.c:30-50), computed where the regions live, in HBM.
//
// The CRC is the reflected IEEE 802.3 polynomial 0xEDB88320 with register init ~0 and a final
// inversion (zlib's convention). Work splits into pieces computed in parallel and combined
// exactly: for a register state s and bytes B, the update is affine,
//   R(B, s) = R(B, 0) ^ Z_|B|(s),
// where Z_n is the linear map "feed n zero bytes" (a 32 x 32 matrix over GF(2)). So
//   R(A || B, 0) = Z_|B|(R(A, 0)) ^ R(B, 0),
// and a whole region is ~R(M, ~0) = ~(Z_|M|(~0) ^ R(M, 0)).
// Z_n for any n is the product of the matrices Z_{2^k} for the bits of n (64 matrices, built on
// the host by squaring Z_1). Bytes are fed with the slice-by-4 tables (four 256-entry tables;
// table k maps a byte to its CRC followed by k zero bytes), a published table method.
#include <string.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace cpg {

constexpr int CRC_THREADS = 128;
constexpr int CRC_PIECE = 516;           // bytes per thread: 129 words, so the threads' word reads
                                         // of the staged segment fall in distinct banks
constexpr int CRC_SEG = CRC_THREADS * CRC_PIECE;   // bytes per CTA (66,048)
constexpr int CRC_SMEM = CRC_SEG + 16;   // the segment, staged from its 16-byte-aligned start

__constant__ uint32_t c_crc_tab[4][256];
__constant__ uint32_t c_crc_zero[64][32];   // [k][i]: Z_{2^k}(1 << i)
__constant__ uint32_t c_crc_zseg[4][256];   // [k][b]: Z_{CRC_SEG}(b << 8k), one segment of zeros

// v -> M v over GF(2), M given by its 32 columns.
__device__ __forceinline__ uint32_t gf2_apply(const uint32_t *col, uint32_t v) {
    uint32_t r = 0;
#pragma unroll 8
    for (int i = 0; i < 32; ++i)
        if ((v >> i) & 1u) r ^= col[i];
    return r;
}

// Z_n(v): the register after n zero bytes.
__device__ uint32_t crc_zeros(uint32_t v, unsigned long long n) {
    for (int k = 0; n != 0 && k < 64; ++k, n >>= 1)
        if (n & 1ull) v = gf2_apply(c_crc_zero[k], v);
    return v;
}

// R(bytes, s) with the tables and the bytes in shared memory.
__device__ uint32_t crc_bytes(const uint32_t (*t)[256], uint32_t s, const uint8_t *p, size_t n) {
    while (n != 0 && ((uintptr_t)p & 3u)) {
        s = (s >> 8) ^ t[0][(s ^ *p++) & 0xFFu];
        --n;
    }
    const uint32_t *w = reinterpret_cast<const uint32_t *>(p);
    for (; n >= 4; n -= 4) {
        s ^= *w++;
        s = t[3][s & 0xFFu] ^ t[2][(s >> 8) & 0xFFu] ^ t[1][(s >> 16) & 0xFFu] ^ t[0][s >> 24];
    }
    p = reinterpret_cast<const uint8_t *>(w);
    while (n-- != 0) s = (s >> 8) ^ t[0][(s ^ *p++) & 0xFFu];
    return s;
}

struct CrcJob {
    const uint8_t *const *base;          // (n) region starts
    const unsigned long long *len;       // (n) region lengths
    const int *seg0;                     // (n + 1) first segment of each region
    int n;
    uint32_t *raw;                       // (segments) R(segment, 0)
    uint32_t *crc;                       // (n) results
};

// One CTA per segment: the segment staged in shared memory by coalesced loads (16-byte loads
// inside it, byte loads for its unaligned ends: nothing outside the segment is read), then
// R(segment, 0) from its 128 pieces, combined pairwise in a tree.
__global__ void __launch_bounds__(CRC_THREADS) k_crc_segments(CrcJob j) {
    extern __shared__ __align__(16) uint8_t sb[];
    __shared__ uint32_t t[4][256];
    __shared__ uint32_t r[CRC_THREADS];
    __shared__ unsigned long long plen[CRC_THREADS];
    for (int i = threadIdx.x; i < 4 * 256; i += CRC_THREADS) t[i >> 8][i & 255] = c_crc_tab[i >> 8][i & 255];
    int lo = 0, hi = j.n;                                   // region: last with seg0 <= blockIdx.x
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (j.seg0[mid] <= (int)blockIdx.x) lo = mid; else hi = mid;
    }
    const unsigned long long s0 = (unsigned long long)(blockIdx.x - j.seg0[lo]) * CRC_SEG;
    const unsigned long long L = j.len[lo];
    const unsigned long long seg_len = L - s0 < (unsigned long long)CRC_SEG ? L - s0 : CRC_SEG;
    const unsigned long long p0 = (unsigned long long)threadIdx.x * CRC_PIECE;
    const unsigned long long n = p0 < seg_len ? (seg_len - p0 < CRC_PIECE ? seg_len - p0 : CRC_PIECE) : 0;
    const uint8_t *g0 = j.base[lo] + s0;                    // the segment in global memory
    const int sh = (int)((uintptr_t)g0 & 15u);              // smem byte of global byte g0 + i: sh + i
    const int head = (int)min((unsigned long long)((16 - sh) & 15), seg_len);
    const int nb = (int)((seg_len - head) / 16);
    const int tail0 = head + nb * 16;
    for (int i = threadIdx.x; i < head; i += CRC_THREADS) sb[sh + i] = g0[i];
    const uint4 *gv = reinterpret_cast<const uint4 *>(g0 + head);
    uint4 *sv = reinterpret_cast<uint4 *>(sb + sh + head);
    for (int i = threadIdx.x; i < nb; i += CRC_THREADS) sv[i] = __ldg(gv + i);
    for (int i = tail0 + threadIdx.x; i < (int)seg_len; i += CRC_THREADS) sb[sh + i] = g0[i];
    __syncthreads();
    r[threadIdx.x] = crc_bytes(t, 0u, sb + sh + p0, (size_t)n);
    plen[threadIdx.x] = n;
    __syncthreads();
    for (int step = 1; step < CRC_THREADS; step <<= 1) {   // pieces [i, i + 2 step) -> i
        const int i = threadIdx.x * 2 * step;
        if (i + step < CRC_THREADS) {
            r[i] = crc_zeros(r[i], plen[i + step]) ^ r[i + step];
            plen[i] += plen[i + step];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) j.raw[blockIdx.x] = r[0];
}

// One CTA per region: each thread folds a contiguous range of the region's segments from state 0
// (a whole segment of zeros is four byte-table lookups), the ranges combine in a tree, and the
// initial register ~0 enters at the end: R(M, ~0) = Z_|M|(~0) ^ R(M, 0); the CRC is its inverse.
constexpr int CRC_FOLD_THREADS = 256;
__global__ void __launch_bounds__(CRC_FOLD_THREADS) k_crc_fold(CrcJob j) {
    __shared__ uint32_t zt[4][256];
    __shared__ uint32_t r[CRC_FOLD_THREADS];
    __shared__ unsigned long long pl[CRC_FOLD_THREADS];
    for (int i = threadIdx.x; i < 4 * 256; i += CRC_FOLD_THREADS) zt[i >> 8][i & 255] = c_crc_zseg[i >> 8][i & 255];
    __syncthreads();
    const int g = blockIdx.x;
    const unsigned long long L = j.len[g];
    const int sb = j.seg0[g], ns = j.seg0[g + 1] - sb;
    const int a = (int)((long long)ns * threadIdx.x / CRC_FOLD_THREADS);
    const int b = (int)((long long)ns * (threadIdx.x + 1) / CRC_FOLD_THREADS);
    uint32_t acc = 0;
    unsigned long long bytes = 0;
    for (int s = a; s < b; ++s) {
        const unsigned long long off = (unsigned long long)s * CRC_SEG;
        const unsigned long long n = L - off < (unsigned long long)CRC_SEG ? L - off : CRC_SEG;
        acc = n == (unsigned long long)CRC_SEG
                  ? zt[0][acc & 0xFFu] ^ zt[1][(acc >> 8) & 0xFFu] ^ zt[2][(acc >> 16) & 0xFFu] ^ zt[3][acc >> 24]
                  : crc_zeros(acc, n);
        acc ^= j.raw[sb + s];
        bytes += n;
    }
    r[threadIdx.x] = acc;
    pl[threadIdx.x] = bytes;
    __syncthreads();
    for (int step = 1; step < CRC_FOLD_THREADS; step <<= 1) {
        const int i = threadIdx.x * 2 * step;
        if (i + step < CRC_FOLD_THREADS) {
            r[i] = crc_zeros(r[i], pl[i + step]) ^ r[i + step];
            pl[i] += pl[i + step];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) j.crc[g] = ~(crc_zeros(0xFFFFFFFFu, pl[0]) ^ r[0]);
}

static int crc_tables_ready() {
    static std::once_flag once;
    static int rc = CPG_OK;
    std::call_once(once, [] {
        uint32_t tab[4][256];
        for (uint32_t b = 0; b < 256; ++b) {
            uint32_t c = b;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? (c >> 1) ^ 0xEDB88320u : c >> 1;
            tab[0][b] = c;
        }
        for (int k = 1; k < 4; ++k)
            for (int b = 0; b < 256; ++b) tab[k][b] = (tab[k - 1][b] >> 8) ^ tab[0][tab[k - 1][b] & 0xFFu];
        static uint32_t zero[64][32];
        for (int i = 0; i < 32; ++i) {                      // Z_1: one zero byte
            const uint32_t v = 1u << i;
            zero[0][i] = (v >> 8) ^ tab[0][v & 0xFFu];
        }
        for (int k = 1; k < 64; ++k)                        // Z_{2^k} = Z_{2^(k-1)} squared
            for (int i = 0; i < 32; ++i) {
                uint32_t v = zero[k - 1][i], r = 0;
                for (int b = 0; b < 32; ++b)
                    if ((v >> b) & 1u) r ^= zero[k - 1][b];
                zero[k][i] = r;
            }
        static uint32_t zseg[4][256];                       // Z_{CRC_SEG}: the product over its bits
        uint32_t col[32];
        for (int i = 0; i < 32; ++i) {
            uint32_t v = 1u << i;
            for (int k = 0; k < 64; ++k) {
                if (!((unsigned long long)CRC_SEG >> k & 1ull)) continue;
                uint32_t r = 0;
                for (int bb = 0; bb < 32; ++bb)
                    if ((v >> bb) & 1u) r ^= zero[k][bb];
                v = r;
            }
            col[i] = v;
        }
        for (int k = 0; k < 4; ++k)
            for (uint32_t b = 0; b < 256; ++b) {
                const uint32_t v = b << (8 * k);
                uint32_t r = 0;
                for (int bb = 0; bb < 32; ++bb)
                    if ((v >> bb) & 1u) r ^= col[bb];
                zseg[k][b] = r;
            }
        cudaError_t e = cudaMemcpyToSymbol(c_crc_tab, tab, sizeof(tab));
        if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_crc_zero, zero, sizeof(zero));
        if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_crc_zseg, zseg, sizeof(zseg));
        if (e != cudaSuccess) rc = cuda_fail(e, "CRC tables");
    });
    return rc;
}

// CRC-32 of n regions of device memory (synchronous on `s`).
int crc32_regions(const std::vector<const uint8_t *> &base, const std::vector<unsigned long long> &len,
                  uint32_t *out, cudaStream_t s) {
    const int n = (int)base.size();
    if (n == 0) return CPG_OK;
    int rc = crc_tables_ready();
    if (rc != CPG_OK) return rc;
    std::vector<int> seg0(n + 1, 0);
    for (int i = 0; i < n; ++i) {
        const unsigned long long segs = (len[i] + CRC_SEG - 1) / CRC_SEG;
        CPG_REQUIRE((unsigned long long)seg0[i] + segs < (1ull << 31), "CRC: too many bytes in one call");
        seg0[i + 1] = seg0[i] + (int)segs;
    }
    const int nseg = seg0[n];
    // one device block: bases | lengths | seg0 | raw | crc
    const size_t b_base = sizeof(void *) * n, b_len = sizeof(unsigned long long) * n, b_seg = sizeof(int) * (n + 1);
    const size_t o_len = b_base, o_seg = o_len + b_len, o_raw = (o_seg + b_seg + 15) / 16 * 16;
    const size_t o_crc = o_raw + sizeof(uint32_t) * (size_t)(nseg > 0 ? nseg : 1);
    const size_t total = o_crc + sizeof(uint32_t) * n;
    std::vector<uint8_t> h(o_raw);
    memcpy(h.data(), base.data(), b_base);
    memcpy(h.data() + o_len, len.data(), b_len);
    memcpy(h.data() + o_seg, seg0.data(), b_seg);
    uint8_t *d = nullptr;
    CPG_CUDA(cudaMalloc((void **)&d, total));
    CrcJob j{reinterpret_cast<const uint8_t *const *>(d), reinterpret_cast<const unsigned long long *>(d + o_len),
             reinterpret_cast<const int *>(d + o_seg), n, reinterpret_cast<uint32_t *>(d + o_raw),
             reinterpret_cast<uint32_t *>(d + o_crc)};
    cudaError_t e = cudaMemcpyAsync(d, h.data(), o_raw, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && nseg > 0) {
        static const cudaError_t attr =
            cudaFuncSetAttribute(k_crc_segments, cudaFuncAttributeMaxDynamicSharedMemorySize, CRC_SMEM);
        e = attr;
        if (e == cudaSuccess) k_crc_segments<<<nseg, CRC_THREADS, CRC_SMEM, s>>>(j);
        if (e == cudaSuccess) e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        k_crc_fold<<<n, CRC_FOLD_THREADS, 0, s>>>(j);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d + o_crc, sizeof(uint32_t) * n, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(d);
    if (e != cudaSuccess) return cuda_fail(e, "CRC-32");
    return CPG_OK;
}

}  // namespace cpg

using namespace cpg;

extern "C" int cpg_crc32(const void *dev, size_t n, uint32_t *out, void *stream) {
    CPG_REQUIRE(out && (dev || n == 0), "cpg_crc32: null argument");
    if (n == 0) {
        *out = 0u;                                          // zlib.crc32(b"") == 0
        return CPG_OK;
    }
    std::vector<const uint8_t *> b{(const uint8_t *)dev};
    std::vector<unsigned long long> l{(unsigned long long)n};
    return crc32_regions(b, l, out, (cudaStream_t)stream);
}
