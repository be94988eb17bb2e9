// ref_gpu.cu -- the REFERENCE's own CUDA quant kernels, launchable on a
// given stream, for timing them beside this library's kernels.
//
// TEST / BASELINE INFRASTRUCTURE ONLY.  oracle/Makefile (target `refgpu`)
// compiles this file, which textually includes the reference's unmodified
// src/cuda_quant.cu (read in place; its kernels live in an anonymous
// namespace, so they are launched from this translation unit), together with
// the reference sources that file links against, for sm_100a into
// oracle/_ref/libref_gpu.so.  bench.py times it as the GPU baseline (the
// reference's q80/q40/q41LinearKernel, src/cuda_quant.cu:78-182) on the same
// device weights and x as the library's own kernels.
//
// refgpu_linear launches exactly what cudaQ{80,40,41}LinearDeviceInput
// (src/cuda_quant.cu:333-361, 411-439, 489-517) launches -- the same kernel,
// grid and block -- minus that entry point's per-call cudaMalloc of y and
// its shape checks (the caller passes y).
#include REF_CUDA_QUANT

extern "C" int refgpu_linear(int fmt, const float* x, const void* w, float* y, int rows, int in_features,
                             int out_features, void* stream) {
    using namespace mini_llama;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int bpr = (in_features + 31) / 32;
    switch (fmt) {
        case 8:
            q80LinearKernel<<<q80Grid(out_features, rows), quantBlock(), 0, s>>>(
                x, static_cast<const BlockQ80*>(w), y, rows, in_features, out_features, bpr);
            break;
        case 2:
            q40LinearKernel<<<quantGrid(out_features, rows), quantBlock(), 0, s>>>(
                x, static_cast<const BlockQ40*>(w), y, rows, in_features, out_features, bpr);
            break;
        case 3:
            q41LinearKernel<<<quantGrid(out_features, rows), quantBlock(), 0, s>>>(
                x, static_cast<const BlockQ41*>(w), y, rows, in_features, out_features, bpr);
            break;
        default:
            return -1;
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
