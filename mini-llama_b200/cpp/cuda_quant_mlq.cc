// cuda_quant_mlq.cc -- drop-in implementation of the reference's
// include/mini_llama/cuda_quant.h on top of libmlq.so (include/mlq.h).
//
// A maintainer of the reference replaces src/cuda_quant.cu with this file
// and links libmlq.so; every caller (src/forward.cc:190-266,
// tests/test_cuda.cc:679-809) compiles unchanged.  It is C++17 host code
// only: no CUDA kernels, no CUDA headers -- the kernels live behind the C ABI.
//
// Behaviour kept from the reference (src/cuda_quant.cu):
//   * validation and its messages: rank of x, [out,in] weight shape,
//     non-empty dims, in-features match, block count (:188-227), null
//     weight pointer (:305-307), x on another device (:342-345);
//     every failure throws std::runtime_error;
//   * result rank follows x (:274-277); bias added on the host after the
//     download (:326-329);
//   * the host variants upload x / download y and are synchronous; the
//     DeviceInput variant allocates y (a CudaTensor) and is asynchronous on
//     the legacy default stream.
// Changed: the kernels, and no temporary device buffers per call for x/y in
// the host variants (libmlq keeps one staging buffer per device).
#include "mini_llama/cuda_quant.h"

#include <cstddef>
#include <stdexcept>
#include <string>
#include <vector>

#include "mlq.h"

namespace mini_llama {
namespace {

void throwIfError(mlq_status st) {
    if (st != MLQ_OK) throw std::runtime_error(mlq_last_error());
}

int inFeatures(const std::vector<int>& x_shape, const std::string& x_str, const char* caller) {
    if (x_shape.size() == 1) return x_shape[0];
    if (x_shape.size() == 2) return x_shape[1];
    throw std::runtime_error(std::string(caller) +
                             ": expected x shape [in_features] or [batch, in_features], got " + x_str);
}

struct Shape {
    int rows, in, out;
    bool one_d;
};

Shape checkShape(const std::vector<int>& x_shape, const std::string& x_str,
                 const std::vector<int>& w_shape, size_t block_count, const char* caller) {
    if (w_shape.size() != 2)
        throw std::runtime_error(std::string(caller) +
                                 ": expected weight shape [out_features, in_features]");
    const int in = inFeatures(x_shape, x_str, caller);
    if (in <= 0 || w_shape[0] <= 0 || w_shape[1] <= 0)
        throw std::runtime_error(std::string(caller) + ": empty tensors are not supported");
    if (w_shape[1] != in)
        throw std::runtime_error(std::string(caller) + ": dimension mismatch x=" + x_str + " weight=[" +
                                 std::to_string(w_shape[0]) + ", " + std::to_string(w_shape[1]) + "]");
    const size_t expected = mlq_block_count(w_shape[0], in);
    if (block_count != expected)
        throw std::runtime_error(std::string(caller) + ": block count mismatch: expected " +
                                 std::to_string(expected) + ", got " + std::to_string(block_count));
    Shape s;
    s.one_d = x_shape.size() == 1;
    s.rows = s.one_d ? 1 : x_shape[0];
    s.in = in;
    s.out = w_shape[0];
    return s;
}

std::vector<int> outShape(const Shape& s) {
    return s.one_d ? std::vector<int>{s.out} : std::vector<int>{s.rows, s.out};
}

Tensor deviceWeightLinear(mlq_format fmt, const char* caller, const Tensor& x, const void* w_dev,
                          size_t block_count, const std::vector<int>& w_shape, const Tensor* bias,
                          int device_id) {
    if (w_dev == nullptr) throw std::runtime_error(std::string(caller) + ": null weight pointer");
    const Shape s = checkShape(x.shape, x.shapeString(), w_shape, block_count, caller);
    Tensor y(outShape(s), 0.0f);
    throwIfError(mlq_linear_host(fmt, w_dev, block_count, s.out, s.in, x.data.data(), s.rows,
                                 bias ? bias->data.data() : nullptr, y.data.data(), device_id,
                                 nullptr));
    return y;
}

Tensor hostWeightLinear(mlq_format fmt, const char* caller, const Tensor& x, const void* blocks,
                        size_t block_count, const std::vector<int>& w_shape, const Tensor* bias,
                        int device_id) {
    const Shape s = checkShape(x.shape, x.shapeString(), w_shape, block_count, caller);
    Tensor y(outShape(s), 0.0f);
    throwIfError(mlq_linear_host_weight(fmt, blocks, block_count, s.out, s.in, x.data.data(), s.rows,
                                        bias ? bias->data.data() : nullptr, y.data.data(),
                                        device_id));
    return y;
}

CudaTensor deviceInputLinear(mlq_format fmt, const char* caller, const CudaTensor& x,
                             const void* w_dev, size_t block_count,
                             const std::vector<int>& w_shape, int device_id) {
    if (w_dev == nullptr) throw std::runtime_error(std::string(caller) + ": null weight pointer");
    if (x.deviceId() != device_id)
        throw std::runtime_error(std::string(caller) + ": input tensor on different CUDA device");
    const Shape s = checkShape(x.shape(), x.shapeString(), w_shape, block_count, caller);
    cudaSetDeviceId(device_id);
    CudaTensor y(outShape(s), device_id);
    throwIfError(mlq_linear(fmt, w_dev, block_count, s.out, s.in, static_cast<const float*>(x.data()),
                            s.rows, static_cast<float*>(y.data()), nullptr));
    return y;
}

}  // namespace

bool cudaQuantBuilt() { return mlq_built() == 1; }

// --- Q8_0 -------------------------------------------------------------------
Tensor cudaQ80Linear(const Tensor& x, const std::vector<BlockQ80>& weight,
                     const std::vector<int>& weight_shape, const Tensor* bias, int device_id) {
    return hostWeightLinear(MLQ_Q8_0, "cudaQ80Linear", x, weight.data(), weight.size(), weight_shape,
                            bias, device_id);
}
Tensor cudaQ80LinearDeviceWeight(const Tensor& x, const void* q8_0_device, size_t q8_0_block_count,
                                 const std::vector<int>& weight_shape, const Tensor* bias,
                                 int device_id) {
    return deviceWeightLinear(MLQ_Q8_0, "cudaQ80Linear", x, q8_0_device, q8_0_block_count,
                              weight_shape, bias, device_id);
}
CudaTensor cudaQ80LinearDeviceInput(const CudaTensor& x, const void* q8_0_device,
                                    size_t q8_0_block_count, const std::vector<int>& weight_shape,
                                    int device_id) {
    return deviceInputLinear(MLQ_Q8_0, "cudaQ80LinearDeviceInput", x, q8_0_device, q8_0_block_count,
                             weight_shape, device_id);
}

// --- Q4_0 -------------------------------------------------------------------
Tensor cudaQ40Linear(const Tensor& x, const std::vector<BlockQ40>& weight,
                     const std::vector<int>& weight_shape, const Tensor* bias, int device_id) {
    return hostWeightLinear(MLQ_Q4_0, "cudaQ40Linear", x, weight.data(), weight.size(), weight_shape,
                            bias, device_id);
}
Tensor cudaQ40LinearDeviceWeight(const Tensor& x, const void* q4_0_device, size_t q4_0_block_count,
                                 const std::vector<int>& weight_shape, const Tensor* bias,
                                 int device_id) {
    return deviceWeightLinear(MLQ_Q4_0, "cudaQ40Linear", x, q4_0_device, q4_0_block_count,
                              weight_shape, bias, device_id);
}
CudaTensor cudaQ40LinearDeviceInput(const CudaTensor& x, const void* q4_0_device,
                                    size_t q4_0_block_count, const std::vector<int>& weight_shape,
                                    int device_id) {
    return deviceInputLinear(MLQ_Q4_0, "cudaQ40LinearDeviceInput", x, q4_0_device, q4_0_block_count,
                             weight_shape, device_id);
}

// --- Q4_1 -------------------------------------------------------------------
Tensor cudaQ41Linear(const Tensor& x, const std::vector<BlockQ41>& weight,
                     const std::vector<int>& weight_shape, const Tensor* bias, int device_id) {
    return hostWeightLinear(MLQ_Q4_1, "cudaQ41Linear", x, weight.data(), weight.size(), weight_shape,
                            bias, device_id);
}
Tensor cudaQ41LinearDeviceWeight(const Tensor& x, const void* q4_1_device, size_t q4_1_block_count,
                                 const std::vector<int>& weight_shape, const Tensor* bias,
                                 int device_id) {
    return deviceWeightLinear(MLQ_Q4_1, "cudaQ41Linear", x, q4_1_device, q4_1_block_count,
                              weight_shape, bias, device_id);
}
CudaTensor cudaQ41LinearDeviceInput(const CudaTensor& x, const void* q4_1_device,
                                    size_t q4_1_block_count, const std::vector<int>& weight_shape,
                                    int device_id) {
    return deviceInputLinear(MLQ_Q4_1, "cudaQ41LinearDeviceInput", x, q4_1_device, q4_1_block_count,
                             weight_shape, device_id);
}

}  // namespace mini_llama
