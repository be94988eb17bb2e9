// Drop-in integration test: the reference's own C++ API and CPU code, with
// its GPU quant path replaced by mini-llama_b200/cpp/cuda_quant_mlq.cc +
// libmlq.so.  oracle/Makefile (target `dropin`) compiles this file against
// the reference's headers together with the reference's src/tensor.cc,
// quant.cc, threadpool.cc, ops.cc, matmul_dispatch.cc, quantized_tensor.cc,
// cuda_runtime.cc, cuda_tensor.cc and cuda_weight_upload.cc (read in place,
// never copied), so the calls below are exactly what the reference's
// callers make (src/forward.cc:190-225, tests/test_cuda.cc:679-809).
//
// Exit status 0 = all passed; 2 = no CUDA device (skipped).
#include <cmath>
#include <cstdio>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "mini_llama/cuda_quant.h"
#include "mini_llama/cuda_runtime.h"
#include "mini_llama/cuda_tensor.h"
#include "mini_llama/cuda_weight_upload.h"
#include "mini_llama/quant.h"
#include "mini_llama/threadpool.h"
#include "mlq_model_quant.h"

using namespace mini_llama;

namespace {

int g_failures = 0;

#define CHECK(cond)                                                              \
    do {                                                                         \
        if (!(cond)) {                                                           \
            std::fprintf(stderr, "  FAILED: %s (%s:%d)\n", #cond, __FILE__, __LINE__); \
            ++g_failures;                                                        \
            return;                                                              \
        }                                                                        \
    } while (0)

void fill(Tensor& t, float scale, float offset) {
    for (size_t i = 0; i < t.size(); ++i) t.data[i] = offset + scale * static_cast<float>(i);
}

// Max abs difference, divided by max(1, max|b|): the reference's 1e-4 checks
// hold only for sums taken in the CPU's order; this library sums in another
// fp32 order, so large outputs are compared relative to their magnitude.
float maxAbsDiff(const Tensor& a, const Tensor& b) {
    float m = 0.f, scale = 1.f;
    for (size_t i = 0; i < a.size(); ++i) {
        m = std::fmax(m, std::fabs(a.data[i] - b.data[i]));
        scale = std::fmax(scale, std::fabs(b.data[i]));
    }
    return m / scale;
}

// worst relative L2 error over the output vectors (rows)
double worstRelL2(const Tensor& y, const Tensor& ref, int cols) {
    double worst = 0.0;
    for (size_t r = 0; r < y.size() / cols; ++r) {
        double num = 0, den = 0;
        for (int c = 0; c < cols; ++c) {
            const double d = double(y.data[r * cols + c]) - ref.data[r * cols + c];
            num += d * d;
            den += double(ref.data[r * cols + c]) * ref.data[r * cols + c];
        }
        worst = std::fmax(worst, std::sqrt(num / std::fmax(den, 1e-60)));
    }
    return worst;
}

bool throwsRuntime(const std::function<void()>& fn) {
    try {
        fn();
    } catch (const std::runtime_error&) {
        return true;
    } catch (...) {
        return false;
    }
    return false;
}

std::vector<BlockQ41> makeQ41(int out, int in) {
    std::vector<BlockQ41> b(static_cast<size_t>(out) * ((in + 31) / 32));
    for (auto& blk : b) {
        blk.d = 0x3800;
        blk.m = 0x0000;
        for (int i = 0; i < 16; ++i) blk.qs[i] = static_cast<uint8_t>(((i * 3 + 1) & 15) | (((i * 5 + 2) & 15) << 4));
    }
    return b;
}

// tests/test_cuda.cc:679-710
void q80MatchesCpu() {
    Tensor w({4, 32}), x({32}), x2({2, 32}), bias({4});
    fill(w, 0.05f, -1.0f);
    fill(x, 0.1f, -0.4f);
    fill(x2, 0.07f, -0.3f);
    fill(bias, 0.2f, -0.1f);
    auto blocks = quantizeToQ80(w);
    CHECK(maxAbsDiff(cudaQ80Linear(x, blocks, w.shape), linearQ80(x, blocks, w.shape)) <= 1e-4f);
    Tensor cpu2 = linearQ80(x2, blocks, w.shape);
    for (int r = 0; r < 2; ++r)
        for (int c = 0; c < 4; ++c) cpu2.at2(r, c) += bias[c];
    Tensor gpu2 = cudaQ80Linear(x2, blocks, w.shape, &bias);
    CHECK(gpu2.shape == cpu2.shape);
    CHECK(maxAbsDiff(gpu2, cpu2) <= 1e-4f);
}

// tests/test_cuda.cc:712-743
void q40q41MatchCpu() {
    Tensor w({4, 32}), x({32});
    fill(w, 0.05f, -1.0f);
    fill(x, 0.1f, -0.4f);
    auto b40 = quantizeToQ40(w);
    CHECK(maxAbsDiff(cudaQ40Linear(x, b40, w.shape), linearQ40(x, b40, w.shape)) <= 1e-4f);
    auto b41 = makeQ41(4, 32);
    std::vector<int> shape{4, 32};
    CHECK(maxAbsDiff(cudaQ41Linear(x, b41, shape), linearQ41(x, b41, shape)) <= 1e-4f);
}

// tests/test_cuda.cc:745-774
void deviceVariants() {
    Tensor w({4, 32}), x({32});
    fill(w, 0.05f, -1.0f);
    fill(x, 0.1f, -0.4f);
    auto blocks = quantizeToQ80(w);
    Tensor host = cudaQ80Linear(x, blocks, w.shape);
    CudaDeviceBuffer w_dev(blocks.size() * sizeof(BlockQ80), 0);
    w_dev.upload(blocks.data(), blocks.size() * sizeof(BlockQ80));
    Tensor dw = cudaQ80LinearDeviceWeight(x, w_dev.data(), blocks.size(), w.shape, nullptr);
    CHECK(maxAbsDiff(dw, host) <= 1e-5f);
    CudaTensor x_dev = cudaTensorFromHost(x, 0);
    CudaTensor di = cudaQ80LinearDeviceInput(x_dev, w_dev.data(), blocks.size(), w.shape, 0);
    Tensor dih = di.download();
    CHECK(dih.shape == std::vector<int>({4}));
    CHECK(maxAbsDiff(dih, host) <= 1e-5f);
}

// tests/test_cuda.cc:776-809
void validation() {
    Tensor w({4, 32});
    fill(w, 0.05f, -1.0f);
    auto blocks = quantizeToQ80(w);
    Tensor x_bad({16});
    CHECK(throwsRuntime([&] { (void)cudaQ80Linear(x_bad, blocks, w.shape); }));
    auto short_blocks = blocks;
    short_blocks.pop_back();
    Tensor x({32});
    CHECK(throwsRuntime([&] { (void)cudaQ80Linear(x, short_blocks, w.shape); }));
    CHECK(throwsRuntime([&] { (void)cudaQ80LinearDeviceWeight(x, nullptr, blocks.size(), w.shape, nullptr); }));
    Tensor x3({1, 1, 32});
    CHECK(throwsRuntime([&] { (void)cudaQ80Linear(x3, blocks, w.shape); }));
}

// The forward.cc call pattern on real-sized weights: upload through the
// reference's uploadQ{80,40,41}LinearWeight (cuda_weight_upload.cc), then
// cudaQ*LinearDeviceInput on a device x, compared with the reference's CPU
// linearQ* within relative L2 1e-3 per output vector.
void forwardPattern() {
    struct Case { QuantType t; int out, in, rows; };
    const Case cases[] = {{QuantType::kQ80, 4864, 896, 1},
                          {QuantType::kQ40, 4608, 3584, 1},
                          {QuantType::kQ40, 3584, 18944, 4},
                          {QuantType::kQ41, 2048, 4096, 8}};
    for (const Case& c : cases) {
        Tensor w({c.out, c.in});
        for (size_t i = 0; i < w.size(); ++i) w.data[i] = 0.02f * std::sin(0.37f * static_cast<float>(i % 100003));
        Tensor x({c.rows, c.in});
        for (size_t i = 0; i < x.size(); ++i) x.data[i] = std::cos(0.11f * static_cast<float>(i % 9973));
        QuantizedTensor q;
        q.type = c.t;
        q.shape = {c.out, c.in};
        if (c.t == QuantType::kQ80) q.q8_0_data = quantizeToQ80(w);
        if (c.t == QuantType::kQ40) q.q4_0_data = quantizeToQ40(w);
        if (c.t == QuantType::kQ41) q.q4_1_data = makeQ41(c.out, c.in);
        CudaModelWeights storage;
        uploadLinearWeight(storage, q, "layers.0.w", 0);
        CHECK(storage.weights.size() == 1);
        const CudaUploadedWeight& cw = storage.weights[0];
        CudaTensor x_dev = cudaTensorFromHost(x, 0);
        CudaTensor y_dev;
        Tensor ref;
        if (c.t == QuantType::kQ80) {
            y_dev = cudaQ80LinearDeviceInput(x_dev, cw.buffer.data(), cw.block_count, cw.shape, 0);
            ref = linearQ80(x, q.q8_0_data, q.shape);
        } else if (c.t == QuantType::kQ40) {
            y_dev = cudaQ40LinearDeviceInput(x_dev, cw.buffer.data(), cw.block_count, cw.shape, 0);
            ref = linearQ40(x, q.q4_0_data, q.shape);
        } else {
            y_dev = cudaQ41LinearDeviceInput(x_dev, cw.buffer.data(), cw.block_count, cw.shape, 0);
            ref = linearQ41(x, q.q4_1_data, q.shape);
        }
        Tensor y = y_dev.download();
        CHECK(y.shape == ref.shape);
        const double err = worstRelL2(y, ref, c.out);
        std::printf("  forward pattern type=%d %dx%d rows=%d: worst rel-L2 %.3g\n",
                    static_cast<int>(c.t), c.out, c.in, c.rows, err);
        CHECK(err <= 1e-3);
    }
}

// The generate path quantizes after uploading (src/main.cc:559-564): the
// reference's uploadLinearWeight puts F32 and Q4_1 weights on the GPU, the
// host model is quantized with quantizeModelTo*'s per-tensor rule, and
// quantizeUploadedWeights brings the device copies along.  The device blocks
// must equal the reference's host quantization byte for byte, carry the new
// type (so forward.cc's lookup by name and type finds them), and feed
// cudaQ*LinearDeviceInput.
void quantizeAfterUpload() {
    const int out = 1000, in = 4096;
    Tensor w({out, in});
    for (size_t i = 0; i < w.size(); ++i) w.data[i] = 0.02f * std::sin(0.71f * static_cast<float>(i % 65537));
    QuantizedTensor f32;
    f32.type = QuantType::kF32;
    f32.shape = {out, in};
    f32.f32_data = w.data;
    QuantizedTensor q41;
    q41.type = QuantType::kQ41;
    q41.shape = {out, in};
    q41.q4_1_data = makeQ41(out, in);
    for (QuantType target : {QuantType::kQ80, QuantType::kQ40}) {
        CudaModelWeights storage;
        storage.device_id = 0;
        uploadLinearWeight(storage, f32, "layers.0.wq", 0);
        uploadLinearWeight(storage, q41, "layers.0.wk", 0);
        CHECK(storage.weights.size() == 2);
        quantizeUploadedWeights(storage, target);
        // the reference's host pass on the same tensors
        const Tensor from41 = dequantizeFromQ41(q41.q4_1_data, q41.shape);
        for (int k = 0; k < 2; ++k) {
            const CudaUploadedWeight& cw = storage.weights[k];
            CHECK(cw.type == target);
            const Tensor& src = k == 0 ? w : from41;
            std::vector<uint8_t> want;
            if (target == QuantType::kQ80) {
                auto b = quantizeToQ80(src);
                want.assign(reinterpret_cast<const uint8_t*>(b.data()),
                            reinterpret_cast<const uint8_t*>(b.data()) + b.size() * sizeof(BlockQ80));
            } else {
                auto b = quantizeToQ40(src);
                want.assign(reinterpret_cast<const uint8_t*>(b.data()),
                            reinterpret_cast<const uint8_t*>(b.data()) + b.size() * sizeof(BlockQ40));
            }
            CHECK(cw.buffer.bytes() == want.size());
            std::vector<uint8_t> got(want.size());
            cw.buffer.download(got.data(), got.size());
            CHECK(got == want);
            CHECK(cw.block_count == static_cast<size_t>(out) * (in / 32));
        }
        // the forward path on the re-quantized device weight
        Tensor x({2, in});
        for (size_t i = 0; i < x.size(); ++i) x.data[i] = std::cos(0.13f * static_cast<float>(i));
        CudaTensor x_dev = cudaTensorFromHost(x, 0);
        const CudaUploadedWeight& cw = storage.weights[0];
        Tensor y, ref;
        if (target == QuantType::kQ80) {
            y = cudaQ80LinearDeviceInput(x_dev, cw.buffer.data(), cw.block_count, cw.shape, 0).download();
            ref = linearQ80(x, quantizeToQ80(w), cw.shape);
        } else {
            y = cudaQ40LinearDeviceInput(x_dev, cw.buffer.data(), cw.block_count, cw.shape, 0).download();
            ref = linearQ40(x, quantizeToQ40(w), cw.shape);
        }
        const double err = worstRelL2(y, ref, out);
        std::printf("  quantize after upload, target type=%d: worst rel-L2 %.3g\n", static_cast<int>(target), err);
        CHECK(err <= 1e-3);
    }
}

}  // namespace

int main() {
    int devices = 0;
    try {
        devices = cudaRuntimeBuilt() ? cudaDeviceCount() : 0;
    } catch (const std::exception&) {
        devices = 0;  // no driver / no GPU on this machine
    }
    if (devices == 0) {
        std::printf("skip: no CUDA device\n");
        return 2;
    }
    std::printf("cudaQuantBuilt() = %d\n", cudaQuantBuilt() ? 1 : 0);
    const std::pair<const char*, void (*)()> tests[] = {
        {"cuda_q80_linear_matches_cpu", q80MatchesCpu},
        {"cuda_q40_q41_linear_match_cpu", q40q41MatchCpu},
        {"cuda_quant_device_variants", deviceVariants},
        {"cuda_quant_validation", validation},
        {"forward_linear_device_pattern", forwardPattern},
        {"quantize_uploaded_weights_after_upload", quantizeAfterUpload},
    };
    for (const auto& t : tests) {
        const int before = g_failures;
        try {
            t.second();
        } catch (const std::exception& e) {
            std::fprintf(stderr, "  EXCEPTION: %s\n", e.what());
            ++g_failures;
        }
        std::printf("[%s] %s\n", g_failures == before ? "PASS" : "FAIL", t.first);
    }
    return g_failures == 0 ? 0 : 1;
}
