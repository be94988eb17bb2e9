// mlq_convert.cu -- quantize / dequantize / bias kernels.
//
// These run the reference's per-block rules on the device, bit for bit:
//   quantizeToQ80   src/quant.cc:130-190
//   quantizeToQ40   src/quant.cc:228-302
//   dequantizeFrom* src/quant.cc:192-223, 304-345, 350-392
//   quantizeQtToQ80/Q40 (dequantize, then quantize) src/model.cc:94-149
//   addBiasInPlace  src/cuda_quant.cu:229-235 (the reference does it on the host)
// Every multiply, divide and add uses the explicit round-to-nearest
// intrinsics so nvcc cannot contract them into FMAs: the reference's stock
// x86 build rounds each operation separately.  The q4_1 quantizer has no
// reference counterpart (the reference has none); its rule is stated below.
#include <cuda_runtime.h>
#include <stdint.h>

#include "mlq_device.cuh"
#include "mlq_kernels.h"

namespace mlq {
namespace {

// fp32 -> fp16 bits with the reference encoder's rounding (src/quant.cc:32-70):
// keep 10 mantissa bits, add one unit when the next lower bit (bit 12 of the
// fp32 mantissa) is set -- round half up in magnitude, not to nearest even;
// the same rule after the shift for subnormal results; exponent overflow
// and NaN encode as +-Inf.
__device__ __forceinline__ uint32_t fp16_encode_ref(float v) {
    const uint32_t bits = __float_as_uint(v);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    int e = (int)((bits >> 23) & 0xffu) - 112;
    uint32_t man = bits & 0x7fffffu;
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t sh = (man | 0x800000u) >> (1 - e);
        if (sh & 0x1000u) sh += 0x2000u;
        return sign | (sh >> 13);
    }
    if (e >= 31) return sign | 0x7c00u;
    if (man & 0x1000u) {
        man += 0x2000u;
        if (man & 0x800000u) {
            man = 0;
            e += 1;
            if (e >= 31) return sign | 0x7c00u;
        }
    }
    return sign | ((uint32_t)e << 10) | (man >> 13);
}

__device__ __forceinline__ int clamp_i(int q, int lo, int hi) { return q < lo ? lo : (q > hi ? hi : q); }

// One block: `n` real values x[0..n) (the last block of a row may be
// short) -> the block's bytes o[0..BS).
template <int F>
__device__ __forceinline__ void quantize_block(const float* x, int n, uint8_t* o) {
    constexpr int BS = Fmt<F>::kBlockBytes;
    uint8_t blk[BS];
#pragma unroll
    for (int i = 0; i < BS; ++i) blk[i] = 0;
    if constexpr (F == kQ8_0 || F == kQ4_0) {
        float amax = 0.0f;
        for (int i = 0; i < n; ++i) {
            const float a = fabsf(x[i]);
            if (a > amax) amax = a;
        }
        if (amax > 0.0f) {
            const uint32_t dh = fp16_encode_ref(__fdiv_rn(amax, F == kQ8_0 ? 127.0f : 7.0f));
            blk[0] = (uint8_t)dh;
            blk[1] = (uint8_t)(dh >> 8);
            const float sd = half_bits_to_float(dh);
            const float id = sd == 0.0f ? 0.0f : __frcp_rn(sd);
            if constexpr (F == kQ8_0) {
                for (int i = 0; i < n; ++i) {
                    const int q = clamp_i((int)roundf(__fmul_rn(x[i], id)), -127, 127);
                    blk[2 + i] = (uint8_t)(int8_t)q;
                }
            } else {
                for (int j = 0; j < 16; ++j) {
                    const float v0 = j < n ? __fmul_rn(x[j], id) : 0.0f;
                    const float v1 = j + 16 < n ? __fmul_rn(x[j + 16], id) : 0.0f;
                    const int q0 = clamp_i((int)roundf(__fadd_rn(v0, 8.0f)), 0, 15);
                    const int q1 = clamp_i((int)roundf(__fadd_rn(v1, 8.0f)), 0, 15);
                    blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
                }
            }
        }
    } else {
        // q4_1 (no reference quantizer; this library's rule): d = (max-min)/15,
        // m = min, both through the reference's fp16 encoder; codes
        // round-half-away((x - m') * (1/d')) clamped to 0..15 against the
        // STORED d', m'; d' == 0 gives code 0; padding values get code 0.
        float mn = x[0], mx = x[0];
        for (int i = 1; i < n; ++i) {
            if (x[i] < mn) mn = x[i];
            if (x[i] > mx) mx = x[i];
        }
        const uint32_t dh = fp16_encode_ref(__fdiv_rn(__fsub_rn(mx, mn), 15.0f));
        const uint32_t mh = fp16_encode_ref(mn);
        blk[0] = (uint8_t)dh;
        blk[1] = (uint8_t)(dh >> 8);
        blk[2] = (uint8_t)mh;
        blk[3] = (uint8_t)(mh >> 8);
        const float sd = half_bits_to_float(dh);
        const float sm = half_bits_to_float(mh);
        const float id = sd == 0.0f ? 0.0f : __frcp_rn(sd);
        for (int j = 0; j < 16; ++j) {
            const int q0 = j < n ? clamp_i((int)roundf(__fmul_rn(__fsub_rn(x[j], sm), id)), 0, 15) : 0;
            const int q1 = j + 16 < n ? clamp_i((int)roundf(__fmul_rn(__fsub_rn(x[j + 16], sm), id)), 0, 15) : 0;
            blk[4 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
#pragma unroll
    for (int i = 0; i < BS; ++i) o[i] = blk[i];
}

// One thread per block.
template <int F>
__global__ void quantize_kernel(const float* __restrict__ src, long long rows, int cols,
                                uint8_t* __restrict__ out) {
    const int bpr = (cols + kQK - 1) / kQK;
    const long long nblk = rows * bpr;
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblk;
         b += (long long)gridDim.x * blockDim.x) {
        const long long r = b / bpr;
        const int kb = (int)(b % bpr);
        quantize_block<F>(src + r * cols + (long long)kb * kQK, min(kQK, cols - kb * kQK),
                          out + b * Fmt<F>::kBlockBytes);
    }
}

// Element e of a block, the reference's dequantized value:
// d*q (q8_0), d*(q-8) (q4_0), d*q + m (q4_1), each operation rounded.
template <int F>
__device__ __forceinline__ float dequant_value(const uint8_t* blk, int e) {
    const float d = half_bits_to_float((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
    if constexpr (F == kQ8_0) {
        return __fmul_rn(d, (float)(int8_t)blk[2 + e]);
    } else if constexpr (F == kQ4_0) {
        const int q = e < 16 ? (blk[2 + e] & 15) : (blk[2 + e - 16] >> 4);
        return __fmul_rn(d, (float)(q - 8));
    } else {
        const float m = half_bits_to_float((uint32_t)blk[2] | ((uint32_t)blk[3] << 8));
        const int q = e < 16 ? (blk[4 + e] & 15) : (blk[4 + e - 16] >> 4);
        return __fadd_rn(__fmul_rn(d, (float)q), m);
    }
}

// Blocks of format S -> blocks of format D, one thread per block: the
// reference's quantizedTensorToF32 (dequantizeFrom*) then quantizeTo*
// (src/model.cc:94-149), fused -- the fp32 values never leave registers.
template <int S, int D>
__global__ void transcode_kernel(const uint8_t* __restrict__ src, long long rows, int cols,
                                 uint8_t* __restrict__ out) {
    const int bpr = (cols + kQK - 1) / kQK;
    const long long nblk = rows * bpr;
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblk;
         b += (long long)gridDim.x * blockDim.x) {
        const int kb = (int)(b % bpr);
        const int n = min(kQK, cols - kb * kQK);
        const uint8_t* blk = src + b * Fmt<S>::kBlockBytes;
        float v[kQK];
#pragma unroll
        for (int e = 0; e < kQK; ++e) v[e] = e < n ? dequant_value<S>(blk, e) : 0.0f;
        quantize_block<D>(v, n, out + b * Fmt<D>::kBlockBytes);
    }
}

// One thread per output value: w = d*q (q8_0), d*(q-8) (q4_0), d*q + m (q4_1).
template <int F>
__global__ void dequantize_kernel(const uint8_t* __restrict__ in, long long rows, int cols,
                                  float* __restrict__ dst) {
    constexpr int BS = Fmt<F>::kBlockBytes;
    const int bpr = (cols + kQK - 1) / kQK;
    const long long n = rows * cols;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long r = idx / cols;
        const int k = (int)(idx % cols);
        dst[idx] = dequant_value<F>(in + (r * bpr + k / kQK) * BS, k % kQK);
    }
}

__global__ void add_bias_kernel(float* __restrict__ y, const float* __restrict__ bias, int rows,
                                int cols) {
    const long long n = (long long)rows * cols;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], bias[i % cols]);
}

__global__ void swiglu_kernel(float* __restrict__ h, const float* __restrict__ u, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        h[i] = silu_mul(h[i], u[i]);
}

int grid_for(long long n, int block) {
    long long g = (n + block - 1) / block;
    if (g > 148LL * 32) g = 148LL * 32;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace

cudaError_t launch_quantize(int fmt, const float* src, long long rows, int cols, uint8_t* blocks,
                            cudaStream_t stream) {
    const long long nblk = rows * ((cols + kQK - 1) / kQK);
    const int grid = grid_for(nblk, 128);
    switch (fmt) {
        case kQ8_0: quantize_kernel<kQ8_0><<<grid, 128, 0, stream>>>(src, rows, cols, blocks); break;
        case kQ4_0: quantize_kernel<kQ4_0><<<grid, 128, 0, stream>>>(src, rows, cols, blocks); break;
        case kQ4_1: quantize_kernel<kQ4_1><<<grid, 128, 0, stream>>>(src, rows, cols, blocks); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequantize(int fmt, const uint8_t* blocks, long long rows, int cols, float* dst,
                              cudaStream_t stream) {
    const int grid = grid_for(rows * cols, 256);
    switch (fmt) {
        case kQ8_0: dequantize_kernel<kQ8_0><<<grid, 256, 0, stream>>>(blocks, rows, cols, dst); break;
        case kQ4_0: dequantize_kernel<kQ4_0><<<grid, 256, 0, stream>>>(blocks, rows, cols, dst); break;
        case kQ4_1: dequantize_kernel<kQ4_1><<<grid, 256, 0, stream>>>(blocks, rows, cols, dst); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_transcode(int src_fmt, const uint8_t* src, int dst_fmt, uint8_t* dst, long long rows, int cols,
                             cudaStream_t stream) {
    const long long nblk = rows * ((cols + kQK - 1) / kQK);
    const int grid = grid_for(nblk, 128);
#define MLQ_TC(S, D)                                                                           \
    if (src_fmt == S && dst_fmt == D) {                                                        \
        transcode_kernel<S, D><<<grid, 128, 0, stream>>>(src, rows, cols, dst);                \
        return cudaGetLastError();                                                             \
    }
    MLQ_TC(kQ8_0, kQ4_0) MLQ_TC(kQ8_0, kQ4_1) MLQ_TC(kQ4_0, kQ8_0)
    MLQ_TC(kQ4_0, kQ4_1) MLQ_TC(kQ4_1, kQ8_0) MLQ_TC(kQ4_1, kQ4_0)
#undef MLQ_TC
    return cudaErrorInvalidValue;
}

cudaError_t launch_add_bias(float* y, const float* bias, int rows, int cols, cudaStream_t stream) {
    add_bias_kernel<<<grid_for((long long)rows * cols, 256), 256, 0, stream>>>(y, bias, rows, cols);
    return cudaGetLastError();
}

cudaError_t launch_swiglu(float* h, const float* u, long long n, cudaStream_t stream) {
    swiglu_kernel<<<grid_for(n, 256), 256, 0, stream>>>(h, u, n);
    return cudaGetLastError();
}

}  // namespace mlq
