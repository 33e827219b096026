// C++ façade (include/llm/*.h): the reference's llm::GPT / Trainer / AdamW / schedulers as
// thin host classes over the C ABI of include/llmgpu.h. Every device operation is one C-ABI
// call; a failing call throws std::runtime_error with the library's message.
#include <cmath>
#include <stdexcept>
#include <string>
#include <vector>

#include "llm/model.h"
#include "llm/optimizer.h"
#include "llm/scheduler.h"
#include "llm/tensor.h"
#include "llm/trainer.h"
#include "llmgpu.h"

namespace llm {

namespace {

[[noreturn]] void fail(const llmgpu_ctx* ctx, const std::string& what, long long rc) {
    throw std::runtime_error(what + " failed (" + std::to_string(rc) + "): " +
                             llmgpu_last_error(ctx));
}

void check(const llmgpu_ctx* ctx, const char* what, long long rc) {
    if (rc < 0) fail(ctx, what, rc);
}

}  // namespace

// ------------------------------------------------------------------------------- Tensor
Tensor::Tensor(std::vector<size_t> shape_, float fill_value) : shape(std::move(shape_)) {
    data.assign(numel(), fill_value);
}

size_t Tensor::numel() const {
    size_t n = 1;
    for (size_t d : shape) n *= d;
    return shape.empty() ? 0 : n;
}

void Tensor::fill(float v) { std::fill(data.begin(), data.end(), v); }

void Tensor::zero_grad() { grad.assign(data.size(), 0.0f); }

// ------------------------------------------------------------------------------- GPT
GPT::GPT(const Config& config, size_t max_batch) : config_(config), max_batch_(max_batch) {
    if (max_batch < 1) throw std::invalid_argument("GPT: max_batch must be at least 1");
    llmgpu_config c;
    llmgpu_config_default(&c);
    c.vocab_size = (int)config.vocab_size;
    c.n_layers = (int)config.n_layers;
    c.n_heads = (int)config.n_heads;
    c.n_embd = (int)config.n_embd;
    c.block_size = (int)config.block_size;
    c.weight_tying = config.weight_tying ? 1 : 0;
    c.use_rmsnorm = config.use_rmsnorm ? 1 : 0;
    c.use_mamba = config.use_mamba ? 1 : 0;
    c.d_inner = (int)config.d_inner;
    c.d_state = (int)config.d_state;
    c.dt_rank = (int)config.dt_rank;
    c.conv_kernel = (int)config.conv_kernel;
    c.rope_theta = config.rope_theta;
    c.pos_encoding = config.pos_encoding == PosEncoding::RoPE         ? LLMGPU_POS_ROPE
                     : config.pos_encoding == PosEncoding::Sinusoidal ? LLMGPU_POS_SINUSOIDAL
                                                                      : LLMGPU_POS_LEARNED;
    c.rope_scaling = config.rope_scaling;
    c.rope_mode = config.rope_mode;
    c.yarn_alpha = config.yarn_alpha;
    c.yarn_beta = config.yarn_beta;
    ctx_ = llmgpu_create(&c, (int)max_batch, (int)config.block_size, 0, 1, nullptr);
    if (!ctx_) throw std::runtime_error(std::string("GPT: ") + llmgpu_last_error(nullptr));
}

GPT::~GPT() {
    if (ctx_) llmgpu_destroy(ctx_);
}

void GPT::pull_from_device() const {
    const int n = llmgpu_num_params(ctx_);
    check(ctx_, "llmgpu_num_params", n);
    mirror_.resize((size_t)n);
    for (int i = 0; i < n; ++i) {
        char name[128];
        int64_t shape[4] = {0, 0, 0, 0};
        const int nd = llmgpu_param_info(ctx_, i, name, sizeof(name), shape);
        check(ctx_, "llmgpu_param_info", nd);
        Tensor& t = mirror_[(size_t)i];
        t.shape.assign(shape, shape + nd);
        t.data.resize(t.numel());
        t.grad.resize(t.numel());
        check(ctx_, "llmgpu_get_param",
              llmgpu_get_param(ctx_, i, t.data.data(), (int64_t)t.data.size()));
        check(ctx_, "llmgpu_get_grad",
              llmgpu_get_grad(ctx_, i, t.grad.data(), (int64_t)t.grad.size()));
    }
}

void GPT::sync_to_device() const {
    if (!exposed_) return;
    for (size_t i = 0; i < mirror_.size(); ++i)
        check(ctx_, "llmgpu_set_param",
              llmgpu_set_param(ctx_, (int)i, mirror_[i].data.data(),
                               (int64_t)mirror_[i].data.size()));
    exposed_ = false;
}

std::vector<Tensor*> GPT::parameters() {
    sync_to_device();
    pull_from_device();
    exposed_ = true;
    std::vector<Tensor*> out;
    out.reserve(mirror_.size());
    for (auto& t : mirror_) out.push_back(&t);
    return out;
}

size_t GPT::num_parameters() const { return llmgpu_num_parameters(ctx_); }

void GPT::zero_grad() {
    // the device step forms fresh gradients every optimizer step; host copies are cleared
    for (auto& t : mirror_) t.zero_grad();
}

void GPT::tie_weights() { sync_to_device(); }

Tensor GPT::forward(const std::vector<int>& tokens) const {
    sync_to_device();
    const size_t T = tokens.size(), V = config_.vocab_size;
    if (T == 0 || T > config_.block_size)
        throw std::invalid_argument("GPT::forward: sequence length outside [1, block_size]");
    Tensor logits({T, V});
    std::vector<int32_t> tok(tokens.begin(), tokens.end());
    check(ctx_, "llmgpu_forward_logits_all",
          llmgpu_forward_logits_all(ctx_, tok.data(), 1, (int)T, logits.data.data(),
                                    (int64_t)logits.data.size()));
    return logits;
}

void GPT::save_binary(const std::string& path) const {
    sync_to_device();
    check(ctx_, "llmgpu_save_binary", llmgpu_save_binary(ctx_, path.c_str()));
}

void GPT::save_binary_atomic(const std::string& path) const { save_binary(path); }

void GPT::load_binary(const std::string& path) {
    exposed_ = false;  // the file replaces any pending host writes
    check(ctx_, "llmgpu_load_binary", llmgpu_load_binary(ctx_, path.c_str()));
}

// ------------------------------------------------------------------------------- optimizers
void Optimizer::step(std::vector<Tensor*>&, const std::vector<Tensor>&) {
    throw std::logic_error(
        "llm::Optimizer::step: the AdamW update runs on the device inside Trainer::train_step");
}

Adam::Adam(float lr, float b1, float b2, float eps) : lr_(lr), b1_(b1), b2_(b2), eps_(eps) {}

AdamW::AdamW(float lr, float b1, float b2, float eps, float wd) : Adam(lr, b1, b2, eps), wd_(wd) {}

// ------------------------------------------------------------------------------- schedulers
CosineScheduler::CosineScheduler(float base_lr, int warmup, int max_iters)
    : base_lr_(base_lr), warmup_(warmup), max_iters_(max_iters) {}

CosineScheduler::CosineScheduler(float base_lr, int warmup, int max_iters, float min_lr, int cycles)
    : base_lr_(base_lr), warmup_(warmup), max_iters_(max_iters), min_lr_(min_lr),
      cycles_(cycles > 0 ? cycles : 1) {}

float CosineScheduler::get_lr(int step) {
    if (step < warmup_) return base_lr_ * (float)step / (float)(warmup_ > 0 ? warmup_ : 1);
    const int span = max_iters_ - warmup_;
    if (span <= 0) return min_lr_;
    float progress;
    if (cycles_ > 1) {
        int len = span / cycles_;
        if (len <= 0) len = span;
        progress = (float)((step - warmup_) % len) / (float)len;
    } else {
        progress = (float)(step - warmup_) / (float)span;
        if (progress > 1.0f) progress = 1.0f;
    }
    return min_lr_ + (base_lr_ - min_lr_) * 0.5f * (1.0f + std::cos(3.14159265f * progress));
}

StepScheduler::StepScheduler(float base_lr, int step_size, float gamma)
    : base_lr_(base_lr), step_size_(step_size), gamma_(gamma) {}

float StepScheduler::get_lr(int step) { return base_lr_ * std::pow(gamma_, step / step_size_); }

// ------------------------------------------------------------------------------- Trainer
Trainer::Trainer(GPT& model, const TrainConfig& cfg, Optimizer& optim, LRScheduler& sched)
    : model_(model), cfg_(cfg), optim_(optim), sched_(sched) {
    const Adam* adam = dynamic_cast<const Adam*>(&optim);
    if (!adam) throw std::invalid_argument("Trainer: the device step implements Adam / AdamW");
    if (cfg.allow_untrained_params)
        throw std::invalid_argument("Trainer: allow_untrained_params is not supported");
    llmgpu_ctx* ctx = model.device_context();
    check(ctx, "llmgpu_set_adamw",
          llmgpu_set_adamw(ctx, adam->get_lr(), adam->beta1(), adam->beta2(), adam->epsilon(),
                           adam->weight_decay()));
    check(ctx, "llmgpu_set_train",
          llmgpu_set_train(ctx, cfg.grad_clip,
                           (int)(cfg.grad_accum_steps < 1 ? 1 : cfg.grad_accum_steps),
                           cfg.label_smoothing));
    check(ctx, "llmgpu_set_loss_scale", llmgpu_set_loss_scale(ctx, cfg.loss_scale));
}

float Trainer::run(const std::vector<int>& tokens, int B, bool accum) {
    llmgpu_ctx* ctx = model_.device_context();
    model_.sync_to_device();
    if (B < 1 || tokens.empty() || tokens.size() % (size_t)B != 0)
        throw std::invalid_argument("Trainer: token count must be a positive multiple of B");
    const int T = (int)(tokens.size() / (size_t)B);
    // the learning rate of this optimizer step (src/trainer.cpp:115-117, 162-164)
    const float lr = sched_.get_lr(step_);
    check(ctx, "llmgpu_set_lr", llmgpu_set_lr(ctx, lr));
    std::vector<int32_t> tok(tokens.begin(), tokens.end());
    float loss = 0.0f, gnorm = 0.0f;
    int stepped = 1, rc;
    if (accum)
        rc = llmgpu_train_step_accum(ctx, tok.data(), B, T, &loss, &stepped);
    else
        rc = llmgpu_train_step(ctx, tok.data(), B, T, &loss, &gnorm);
    check(ctx, accum ? "llmgpu_train_step_accum" : "llmgpu_train_step", rc);
    if (accum) last_loss_ = loss;
    if (rc == LLMGPU_SKIPPED) {  // non-finite gradient (src/trainer.cpp:106-111, 151-156)
        ++skipped_;
        return loss;
    }
    if (stepped) {
        last_loss_ = loss;
        last_grad_norm_ = llmgpu_last_grad_norm(ctx);
        optim_.set_lr(lr);
    }
    return loss;
}

float Trainer::train_step(const std::vector<int>& batch) { return run(batch, 1, false); }

float Trainer::train_step_accum(const std::vector<int>& micro_batch) {
    return run(micro_batch, 1, true);
}

float Trainer::train_step_batch(const std::vector<int>& tokens, int B) {
    return run(tokens, B, false);
}

void Trainer::save_train_state(const std::string& prefix) {
    llmgpu_ctx* ctx = model_.device_context();
    model_.sync_to_device();
    check(ctx, "llmgpu_set_step", llmgpu_set_step(ctx, step_));
    check(ctx, "llmgpu_save_train_state", llmgpu_save_train_state(ctx, prefix.c_str()));
}

void Trainer::load_train_state(const std::string& prefix) {
    llmgpu_ctx* ctx = model_.device_context();
    check(ctx, "llmgpu_load_train_state", llmgpu_load_train_state(ctx, prefix.c_str()));
    step_ = llmgpu_step(ctx);
    skipped_ = llmgpu_skipped_steps(ctx);
}

void Trainer::snapshot_params() {
    last_good_.clear();
    for (Tensor* p : model_.parameters()) last_good_.push_back(p->data);
    has_snapshot_ = true;
}

bool Trainer::rollback_if_nonfinite(float loss) {
    if (std::isfinite(loss) || !has_snapshot_) return false;
    auto params = model_.parameters();
    for (size_t i = 0; i < params.size() && i < last_good_.size(); ++i)
        params[i]->data = last_good_[i];
    model_.sync_to_device();
    optim_.set_lr(optim_.get_lr() * 0.5f);
    return true;
}

}  // namespace llm
