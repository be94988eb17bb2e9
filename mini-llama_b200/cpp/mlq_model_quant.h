// mlq_model_quant.h -- model-level quantization of weights already resident
// on the GPU, for the reference's C++ integration layer.
//
// The reference quantizes a model on the host (quantizeModelToQ80 /
// quantizeModelToQ40, src/model.cc:110-149), and its generate path does so
// AFTER uploading the weights (src/main.cc:559-564): the device copies keep
// their old type, forwardLinearDevice's lookup by (name, type)
// (src/forward.cc:64-87, 198) misses them, and the CUDA quant path is never
// taken.  quantizeUploadedWeights re-quantizes the uploaded copies on the
// device (mlq_quantize_model) to the type the host model now has, so a
// caller that quantizes after upload calls it once, right after
// quantizeModelTo*, and the lookups hit.
#ifndef MLQ_MODEL_QUANT_H_
#define MLQ_MODEL_QUANT_H_

#include "mini_llama/cuda_weight_upload.h"
#include "mini_llama/quantized_tensor.h"

namespace mini_llama {

// Every linear weight of `weights` (2-D, F32 / Q8_0 / Q4_0 / Q4_1) becomes
// `target` (kQ80 or kQ40, as the reference's passes; kQ41 uses this
// library's q4_1 rule) in device memory: bit-identical to quantizing the
// host tensor with the reference's quantizeQtToQ80/Q40 and uploading it.
// Weights already of type `target`, and non-linear weights, stay as they
// are.  Throws std::runtime_error on failure (the weights are then
// unchanged).
void quantizeUploadedWeights(CudaModelWeights& weights, QuantType target);

}  // namespace mini_llama

#endif  // MLQ_MODEL_QUANT_H_
