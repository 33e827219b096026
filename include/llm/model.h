// C++ façade over libllmgpu.so: llm::Config and llm::GPT with the reference's names and
// argument meaning (include/llm/model.h:15-111 of the reference), backed by one device
// context of the C ABI (include/llmgpu.h).
//
// Kept from the reference: Config's fields and defaults; GPT(Config); forward (logits of
// every position); parameters() in the reference's order, with `data` and `grad`;
// num_parameters; zero_grad; tie_weights; save_binary / save_binary_atomic / load_binary in
// the reference's v3/v4 file layout; config().
// Not offered: the separate forward_with_hidden / backward pair (the device step fuses the
// forward, the loss gradient and the backward: Trainer::train_step), generation, the
// Mamba-state and GPU-weights helpers, and extend_context.
// Errors: where the reference asserts or prints, these throw std::runtime_error with the
// library's message (llmgpu_last_error).
#pragma once
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "llm/tensor.h"

struct llmgpu_ctx;

namespace llm {

enum class PosEncoding { Learned, Sinusoidal, RoPE };

struct Config {
    size_t vocab_size = 50257;
    size_t n_layers = 12;
    size_t n_heads = 12;
    size_t n_embd = 768;
    size_t block_size = 1024;
    float dropout = 0.0f;  // unused by the training step (the reference applies none either)
    bool bias = false;
    PosEncoding pos_encoding = PosEncoding::Learned;
    bool weight_tying = true;
    std::vector<float> dropout_per_layer;
    std::vector<float> weight_decay_per_layer;
    float rope_theta = 10000.0f;
    float rope_scaling = 1.0f;
    int rope_mode = 0;
    float yarn_alpha = 1.0f;
    float yarn_beta = 32.0f;
    bool deterministic = false;  // the device step is deterministic in any case
    bool use_rmsnorm = false;
    bool use_alibi = false;       // not read by GPT::forward_with_hidden; must stay false
    size_t sliding_window = 0;    // idem; must stay 0
    size_t global_every = 1;
    bool use_mamba = false;
    size_t d_inner = 0;
    size_t d_state = 16;
    size_t dt_rank = 0;
    size_t conv_kernel = 4;
    bool use_gpu_weights = false;  // ignored: the weights always live on the device
};

class GPT {
   public:
    // Creates the device context on the current CUDA device. `max_batch` sequences of up to
    // block_size tokens bound one step (the reference trains one sequence per call: 1).
    explicit GPT(const Config& config, size_t max_batch = 1);
    ~GPT();
    GPT(const GPT&) = delete;
    GPT& operator=(const GPT&) = delete;

    // tokens [T] -> logits [T, vocab_size] (GPT::forward, src/model.cpp:140-171)
    Tensor forward(const std::vector<int>& tokens) const;
    void zero_grad();

    void save_binary(const std::string& path) const;
    void save_binary_atomic(const std::string& path) const;
    void load_binary(const std::string& path);

    size_t num_parameters() const;
    // GPT::parameters() order (src/model.cpp:889-909): host copies of the device values and
    // of the last step's raw (pre-clip) gradients. Values written into `data` reach the
    // device before the next call that uses the parameters.
    std::vector<Tensor*> parameters();
    // The device keeps the tied head as the embedding itself; sends pending host writes.
    void tie_weights();
    const Config& config() const { return config_; }

    // The underlying C-ABI context (for calls the façade does not wrap).
    llmgpu_ctx* device_context() const { return ctx_; }
    // Sends host writes made through parameters() to the device (done before every device
    // call; public for callers that hand device_context() to C-ABI calls themselves).
    void sync_to_device() const;

   private:
    void pull_from_device() const;
    Config config_;
    llmgpu_ctx* ctx_ = nullptr;
    size_t max_batch_ = 1;
    mutable std::vector<Tensor> mirror_;
    mutable bool exposed_ = false;
};

}  // namespace llm
