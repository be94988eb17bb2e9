// mlq_kernels.h -- host-side launch interface of the mlq kernels (internal).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mlq {

// Arguments of the streaming GEMV (mlq_gemv.cu).
struct GemvArgs {
    const uint8_t* w;        // packed blocks, row-major [out][bpr]
    const float* x;          // [M][in]
    float* y;                // [M][y_stride]
    int out, in, M;          // M <= the launch's tokens-per-pass
    int bpr;                 // blocks per row
    int gpr;                 // lane-groups per row (bpr / blocks per group)
    int ktiles;              // ceil(gpr / 32)
    int nstages;             // pipeline depth (set by the dispatcher)
    int y_stride;            // row stride of y in floats
    long long row_bytes;     // bpr * block bytes
    long long total_bytes;   // out * row_bytes
    int* err;                // device error flag
};

// Tokens per pass for `rows_left` remaining rows of x: 1, 2, 4 or 8.
int gemv_tokens_per_pass(int rows_left);

// Streaming GEMV, tokens-per-pass `mt` in {1,2,4,8}; `grid` CTAs (one per
// SM), `smem_budget` bytes of dynamic shared memory at most.
cudaError_t launch_gemv_stream(int fmt, GemvArgs args, int mt, int grid, int smem_budget,
                               cudaStream_t stream);

// Any-alignment fallback GEMV (one warp per output row).
cudaError_t launch_gemv_generic(int fmt, const uint8_t* w, const float* x, float* y, int out,
                                int in, int M, int bpr, cudaStream_t stream);

// Quantize fp32 [rows][cols] -> blocks, reference rules (mlq_convert.cu).
cudaError_t launch_quantize(int fmt, const float* src, long long rows, int cols, uint8_t* blocks,
                            cudaStream_t stream);

// Blocks -> fp32 [rows][cols], reference rules (mlq_convert.cu).
cudaError_t launch_dequantize(int fmt, const uint8_t* blocks, long long rows, int cols, float* dst,
                              cudaStream_t stream);

// y[r][c] += bias[c] for r < rows, c < cols.
cudaError_t launch_add_bias(float* y, const float* bias, int rows, int cols, cudaStream_t stream);

}  // namespace mlq
