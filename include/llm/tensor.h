// C++ façade over libllmgpu.so: the part of llm::Tensor (include/llm/tensor.h of the
// reference) that the training API exposes to its callers.
//
// In the reference a Tensor owns fp32 `data` and a mutable fp32 `grad` that the manual
// backward accumulates into (include/llm/tensor.h:29-30 there). Here the parameters live on
// the device; GPT::parameters() fills host Tensors with the current device values and
// gradients, and writes to `data` are sent back to the device before the next device call.
// The reference's tensor arithmetic (matmul, softmax, norms, ...) is not part of this
// surface: the training step runs as CUDA kernels behind the C ABI (include/llmgpu.h).
#pragma once
#include <cstddef>
#include <vector>

namespace llm {

struct Tensor {
    std::vector<size_t> shape;
    std::vector<float> data;
    mutable std::vector<float> grad;

    Tensor() = default;
    explicit Tensor(std::vector<size_t> shape_, float fill_value = 0.0f);

    size_t numel() const;
    size_t ndim() const { return shape.size(); }
    // row-major 2-D element access, as Tensor::operator()(i, j) of the reference
    float& operator()(size_t i, size_t j) { return data[i * shape[1] + j]; }
    float operator()(size_t i, size_t j) const { return data[i * shape[1] + j]; }
    void fill(float v);
    void zero_grad();
};

}  // namespace llm
