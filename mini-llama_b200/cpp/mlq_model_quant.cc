// mlq_model_quant.cc -- quantizeUploadedWeights (mlq_model_quant.h) over the
// C ABI (mlq_quantize_model, include/mlq.h).  Compiled with the reference's
// headers into the caller's program, like cuda_quant_mlq.cc.
#include "mlq_model_quant.h"

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "mlq.h"

namespace mini_llama {
namespace {

int mlqType(QuantType t) {
    switch (t) {
        case QuantType::kF32: return 0;
        case QuantType::kQ80: return MLQ_Q8_0;
        case QuantType::kQ40: return MLQ_Q4_0;
        case QuantType::kQ41: return MLQ_Q4_1;
    }
    return -1;
}

}  // namespace

void quantizeUploadedWeights(CudaModelWeights& weights, QuantType target) {
    const int dst = mlqType(target);
    if (dst <= 0) throw std::runtime_error("quantizeUploadedWeights: target must be a block type");
    // new buffers first: on any failure the model keeps its current weights
    std::vector<size_t> which;
    std::vector<CudaDeviceBuffer> fresh;
    std::vector<mlq_quantize_op> ops;
    for (size_t i = 0; i < weights.weights.size(); ++i) {
        CudaUploadedWeight& w = weights.weights[i];
        if (!w.linear || w.type == target || w.shape.size() != 2 || w.buffer.empty()) continue;
        const int rows = w.shape[0], cols = w.shape[1];
        const size_t blocks = mlq_block_count(rows, cols);
        fresh.emplace_back(blocks * mlq_block_bytes(static_cast<mlq_format>(dst)), w.buffer.device_id());
        which.push_back(i);
        mlq_quantize_op op{};
        op.src_type = mlqType(w.type);
        op.src = w.buffer.data();
        op.dst_fmt = dst;
        op.dst = fresh.back().data();
        op.rows = rows;
        op.cols = cols;
        ops.push_back(op);
    }
    if (ops.empty()) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(weights.device_id);
    mlq_status st = mlq_quantize_model(ops.data(), static_cast<int>(ops.size()), nullptr);
    const cudaError_t e = st == MLQ_OK ? cudaDeviceSynchronize() : cudaSuccess;
    cudaSetDevice(prev);
    if (st != MLQ_OK) throw std::runtime_error(std::string("quantizeUploadedWeights: ") + mlq_last_error());
    if (e != cudaSuccess) throw std::runtime_error(std::string("quantizeUploadedWeights: ") + cudaGetErrorString(e));
    for (size_t k = 0; k < which.size(); ++k) {
        CudaUploadedWeight& w = weights.weights[which[k]];
        w.buffer = std::move(fresh[k]);
        w.type = target;
        w.block_count = mlq_block_count(w.shape[0], w.shape[1]);
    }
}

}  // namespace mini_llama
