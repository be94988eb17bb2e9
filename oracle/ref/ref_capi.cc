// ref_capi.cc -- a C entry layer over the REFERENCE's own CPU quant code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together
// with the reference's unmodified src/quant.cc, src/threadpool.cc,
// src/tensor.cc, src/quantized_tensor.cc, src/ops.cc and
// src/matmul_dispatch.cc (read in place from the reference checkout) into
// oracle/_ref/libref_*.so.  tests/golden/make_golden.py uses it to produce
// golden vectors, the CPU tests use it (when present) to pin the oracle, and
// bench.py --impl reference times it as the reference's CPU baseline.
//
// Functions wrapped (reference include/mini_llama/quant.h):
//   quantizeToQ80 / quantizeToQ40          quant.h:265, 275
//   dequantizeFromQ80 / Q40 / Q41          quant.h:269, 279, 285
//   linearQ80 / linearQ40 / linearQ41      quant.h:293-298
//   ThreadPool::setThreadCount             threadpool.h:39
//   swiGlu (silu(gate) * up)               ops.h:35-36
#include <cstdint>
#include <cstring>
#include <vector>

#include "mini_llama/ops.h"
#include "mini_llama/quant.h"
#include "mini_llama/quantized_tensor.h"
#include "mini_llama/tensor.h"
#include "mini_llama/threadpool.h"

using namespace mini_llama;

namespace {

Tensor makeMatrix(const float* data, int rows, int cols) {
    // rows == 0 means "1-D tensor of cols elements" (the reference keys the
    // output rank off the input rank, quant.cc:449-451).
    Tensor t(rows == 0 ? std::vector<int>{cols} : std::vector<int>{rows, cols}, 0.0f);
    std::memcpy(t.data.data(), data, t.data.size() * sizeof(float));
    return t;
}

template <typename Block>
std::vector<Block> toBlocks(const void* p, size_t n) {
    std::vector<Block> v(n);
    std::memcpy(v.data(), p, n * sizeof(Block));
    return v;
}

}  // namespace

extern "C" {

int ref_block_bytes(int fmt) {
    switch (fmt) {
        case 8: return static_cast<int>(sizeof(BlockQ80));
        case 2: return static_cast<int>(sizeof(BlockQ40));
        case 3: return static_cast<int>(sizeof(BlockQ41));
    }
    return 0;
}

void ref_set_threads(int n) { ThreadPool::setThreadCount(n > 0 ? static_cast<size_t>(n) : 0); }

int ref_get_threads(void) { return static_cast<int>(ThreadPool::getThreadCount()); }

// Returns the number of blocks written (fmt 8 = q8_0, 2 = q4_0).
long long ref_quantize(int fmt, const float* src, int rows, int cols, void* out) {
    Tensor t = makeMatrix(src, rows, cols);
    if (fmt == 8) {
        auto b = quantizeToQ80(t);
        std::memcpy(out, b.data(), b.size() * sizeof(BlockQ80));
        return static_cast<long long>(b.size());
    }
    if (fmt == 2) {
        auto b = quantizeToQ40(t);
        std::memcpy(out, b.data(), b.size() * sizeof(BlockQ40));
        return static_cast<long long>(b.size());
    }
    return -1;
}

int ref_dequantize(int fmt, const void* blocks, size_t nblocks, int rows, int cols, float* dst) {
    std::vector<int> shape = rows == 0 ? std::vector<int>{cols} : std::vector<int>{rows, cols};
    Tensor y;
    if (fmt == 8) y = dequantizeFromQ80(toBlocks<BlockQ80>(blocks, nblocks), shape);
    else if (fmt == 2) y = dequantizeFromQ40(toBlocks<BlockQ40>(blocks, nblocks), shape);
    else if (fmt == 3) y = dequantizeFromQ41(toBlocks<BlockQ41>(blocks, nblocks), shape);
    else return -1;
    std::memcpy(dst, y.data.data(), y.data.size() * sizeof(float));
    return static_cast<int>(y.data.size() == 0 ? -1 : 0);
}

// x is [xrows, in] (xrows == 0: 1-D x of length in); y receives [xrows, out].
int ref_linear(int fmt, const float* x, int xrows, int in, const void* blocks, size_t nblocks,
               int out, float* y) {
    Tensor xt = makeMatrix(x, xrows, in);
    std::vector<int> wshape{out, in};
    Tensor r;
    if (fmt == 8) r = linearQ80(xt, toBlocks<BlockQ80>(blocks, nblocks), wshape);
    else if (fmt == 2) r = linearQ40(xt, toBlocks<BlockQ40>(blocks, nblocks), wshape);
    else if (fmt == 3) r = linearQ41(xt, toBlocks<BlockQ41>(blocks, nblocks), wshape);
    else return -1;
    if (r.data.empty()) return -2;
    std::memcpy(y, r.data.data(), r.data.size() * sizeof(float));
    return 0;
}

// Same as ref_linear but the caller keeps the block vector alive between
// timed calls (no per-call copy of the weights), for the CPU baseline timer.
void* ref_blocks_new(int fmt, const void* blocks, size_t nblocks) {
    if (fmt == 8) return new std::vector<BlockQ80>(toBlocks<BlockQ80>(blocks, nblocks));
    if (fmt == 2) return new std::vector<BlockQ40>(toBlocks<BlockQ40>(blocks, nblocks));
    if (fmt == 3) return new std::vector<BlockQ41>(toBlocks<BlockQ41>(blocks, nblocks));
    return nullptr;
}

void ref_blocks_free(int fmt, void* h) {
    if (fmt == 8) delete static_cast<std::vector<BlockQ80>*>(h);
    else if (fmt == 2) delete static_cast<std::vector<BlockQ40>*>(h);
    else if (fmt == 3) delete static_cast<std::vector<BlockQ41>*>(h);
}

// h[i] = silu(gate[i]) * up[i] through the reference's swiGlu (1-D tensors).
int ref_swiglu(const float* gate, const float* up, int n, float* h) {
    Tensor g = makeMatrix(gate, 0, n);
    Tensor u = makeMatrix(up, 0, n);
    Tensor r = swiGlu(g, u);
    if (r.data.size() != static_cast<size_t>(n)) return -2;
    std::memcpy(h, r.data.data(), r.data.size() * sizeof(float));
    return 0;
}

int ref_linear_held(int fmt, const float* x, int xrows, int in, const void* handle, int out,
                    float* y) {
    Tensor xt = makeMatrix(x, xrows, in);
    std::vector<int> wshape{out, in};
    Tensor r;
    if (fmt == 8) r = linearQ80(xt, *static_cast<const std::vector<BlockQ80>*>(handle), wshape);
    else if (fmt == 2) r = linearQ40(xt, *static_cast<const std::vector<BlockQ40>*>(handle), wshape);
    else if (fmt == 3) r = linearQ41(xt, *static_cast<const std::vector<BlockQ41>*>(handle), wshape);
    else return -1;
    if (r.data.empty()) return -2;
    std::memcpy(y, r.data.data(), r.data.size() * sizeof(float));
    return 0;
}

}  // extern "C"
