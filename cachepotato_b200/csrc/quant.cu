// quant.cu — Q4_0 / Q8_0 decode (bit-exact with the reference decoder) and encode (bit-exact
// with the reference encoders). One thread per 32-value group; both are HBM-streaming.
#include "common.cuh"

namespace cpg {

// (float)q * d with the host's (x86 SSE) NaN rules, so that decoding is bit-exact for every
// byte pattern, not only for finite scales: a NaN scale propagates quieted with its payload,
// and 0 * inf gives the default NaN 0xFFC00000 (the GPU would return its canonical NaN).
__device__ __forceinline__ float mul_hostnan(float q, float d) {
    const float v = __fmul_rn(q, d);
    if (!isnan(v)) return v;
    return isnan(d) ? __uint_as_float(__float_as_uint(d) | 0x00400000u) : __uint_as_float(0xFFC00000u);
}

// engine/kernels/kernels.c:143-151 (Q8_0) and 463-477 (Q4_0). The group scale is fp16 and the
// quantised value an integer, so q * d in fp32 is exact: there is one right answer.
template <int ENC>
__global__ void k_dequant(float *__restrict__ out, const uint8_t *__restrict__ blocks, long ngroups) {
    constexpr int GB = ENC == CPG_ENC_Q4 ? 18 : 34;
    for (long g = blockIdx.x * (long)blockDim.x + threadIdx.x; g < ngroups;
         g += (long)gridDim.x * blockDim.x) {
        const uint8_t *blk = blocks + g * GB;
        const float d = f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
        float4 *o = reinterpret_cast<float4 *>(out + g * 32);
        if (ENC == CPG_ENC_Q8) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = mul_hostnan((float)(int8_t)blk[2 + i], d);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
            float v[32];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int b = blk[2 + k];
                const int lo = (b & 0x0F) > 7 ? (b & 0x0F) - 16 : (b & 0x0F);
                const int hi = (b >> 4) > 7 ? (b >> 4) - 16 : (b >> 4);
                v[k] = mul_hostnan((float)lo, d);
                v[k + 16] = mul_hostnan((float)hi, d);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    }
}

// format/q4.py:30-57 and format/q8.py:35-58. The scale is rounded to fp16 FIRST (RNE) and the
// values are divided by the stored scale (IEEE fp32 division), rounded half-to-even, clipped.
template <int ENC>
__global__ void k_quantize(uint8_t *__restrict__ blocks, const float *__restrict__ x, long ngroups) {
    constexpr int GB = ENC == CPG_ENC_Q4 ? 18 : 34;
    for (long g = blockIdx.x * (long)blockDim.x + threadIdx.x; g < ngroups;
         g += (long)gridDim.x * blockDim.x) {
        float v[32];
        const float4 *src = reinterpret_cast<const float4 *>(x + g * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 f = src[i];
            v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) amax = fabsf(v[i]) > amax ? fabsf(v[i]) : amax;
        // Q4: amax/8 is exact; Q8: amax/127 is an fp32 division (numpy's float32 result)
        const float d = amax > 0.0f ? (ENC == CPG_ENC_Q4 ? amax * 0.125f : __fdiv_rn(amax, 127.0f)) : 0.0f;
        const uint32_t bits = (uint32_t)__half_as_ushort(__float2half_rn(d));
        const float dq = f16_bits_to_f32(bits);
        const float lo = ENC == CPG_ENC_Q4 ? -8.0f : -127.0f;
        const float hi = ENC == CPG_ENC_Q4 ? 7.0f : 127.0f;
        int q[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            int qi = 0;
            if (dq > 0.0f) {
                const float r = rintf(__fdiv_rn(v[i], dq));
                qi = (int)fminf(fmaxf(r, lo), hi);
            }
            q[i] = qi;
        }
        // the group as 16-bit words (groups are 2-byte aligned): scale, then payload bytes
        uint16_t *dst = reinterpret_cast<uint16_t *>(blocks + g * GB);
        dst[0] = (uint16_t)bits;
        if (ENC == CPG_ENC_Q8) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                dst[1 + i] = (uint16_t)((q[2 * i] & 0xFF) | ((q[2 * i + 1] & 0xFF) << 8));
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t b0 = (uint32_t)((q[2 * i] & 0xF) | ((q[2 * i + 16] & 0xF) << 4));
                const uint32_t b1 = (uint32_t)((q[2 * i + 1] & 0xF) | ((q[2 * i + 17] & 0xF) << 4));
                dst[1 + i] = (uint16_t)(b0 | (b1 << 8));
            }
        }
    }
}

static int grid_for(long n, int block) {
    long g = (n + block - 1) / block;
    long cap = (long)sm_count() * 16;
    return (int)(g < 1 ? 1 : g > cap ? cap : g);
}

}  // namespace cpg

using namespace cpg;

extern "C" int cpg_dequant(float *out, const uint8_t *blocks, int enc, long n, void *stream) {
    CPG_REQUIRE(out && blocks, "cpg_dequant: null pointer");
    CPG_REQUIRE(n >= 0 && n % 32 == 0, "cpg_dequant: n=%ld is not a multiple of 32", n);
    CPG_REQUIRE(enc == CPG_ENC_Q4 || enc == CPG_ENC_Q8, "cpg_dequant: encoding %d is not Q4/Q8", enc);
    CPG_REQUIRE(((uintptr_t)out & 15) == 0, "cpg_dequant: out must be 16-byte aligned");
    if (n == 0) return CPG_OK;
    const long ng = n / 32;
    cudaStream_t s = (cudaStream_t)stream;
    if (enc == CPG_ENC_Q4) k_dequant<CPG_ENC_Q4><<<grid_for(ng, 256), 256, 0, s>>>(out, blocks, ng);
    else k_dequant<CPG_ENC_Q8><<<grid_for(ng, 256), 256, 0, s>>>(out, blocks, ng);
    CPG_CUDA(cudaGetLastError());
    return CPG_OK;
}

extern "C" int cpg_quantize(uint8_t *blocks, const float *x, int enc, long n, void *stream) {
    CPG_REQUIRE(blocks && x, "cpg_quantize: null pointer");
    CPG_REQUIRE(n >= 0 && n % 32 == 0, "cpg_quantize: n=%ld is not a multiple of 32", n);
    CPG_REQUIRE(enc == CPG_ENC_Q4 || enc == CPG_ENC_Q8, "cpg_quantize: encoding %d is not Q4/Q8", enc);
    CPG_REQUIRE(((uintptr_t)x & 15) == 0 && ((uintptr_t)blocks & 1) == 0,
                "cpg_quantize: x must be 16-byte and blocks 2-byte aligned");
    if (n == 0) return CPG_OK;
    const long ng = n / 32;
    cudaStream_t s = (cudaStream_t)stream;
    if (enc == CPG_ENC_Q4) k_quantize<CPG_ENC_Q4><<<grid_for(ng, 128), 128, 0, s>>>(blocks, x, ng);
    else k_quantize<CPG_ENC_Q8><<<grid_for(ng, 128), 128, 0, s>>>(blocks, x, ng);
    CPG_CUDA(cudaGetLastError());
    return CPG_OK;
}
