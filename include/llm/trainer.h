// C++ façade over libllmgpu.so: llm::TrainConfig and llm::Trainer with the reference's
// names, constructor and step API (include/llm/trainer.h:10-76 of the reference). Each step
// is one call of the C ABI (llmgpu_train_step / llmgpu_train_step_accum): forward,
// cross-entropy, backward, non-finite skip, global-norm clip and AdamW on the device.
//
// Kept: TrainConfig's fields; Trainer(GPT&, const TrainConfig&, Optimizer&, LRScheduler&);
// train_step (one sequence, targets = inputs); train_step_accum (K = grad_accum_steps);
// the learning rate of every optimizer step is sched.get_lr(step()), set on the optimizer
// as the reference does; skipped_steps / step / set_step / last_loss / last_grad_norm;
// save_train_state / load_train_state (<prefix>.model.bin, .opt.bin, .json);
// snapshot_params / rollback_if_nonfinite.
// Extension: train_step_batch runs B sequences at once (= train_step_accum over them).
// Not offered: train(Dataset&) and evaluate(Dataset&) (the Dataset type is not part of this
// surface), allow_untrained_params and activation checkpointing (the device keeps the
// activations). Failures throw std::runtime_error with the library's message.
#pragma once
#include <string>
#include <vector>

#include "llm/model.h"
#include "llm/optimizer.h"
#include "llm/scheduler.h"

namespace llm {

struct TrainConfig {
    size_t batch_size = 32;
    size_t max_iters = 5000;
    size_t eval_interval = 500;
    float grad_clip = 1.0f;
    std::string checkpoint_dir = "checkpoints";
    size_t grad_accum_steps = 1;
    bool checkpointing = false;
    bool allow_untrained_params = false;  // must stay false: gradients are always real
    float label_smoothing = 0.0f;
    float loss_scale = 1.0f;
    bool deterministic = false;  // the device step is deterministic in any case
};

class Trainer {
   public:
    Trainer(GPT& model, const TrainConfig& cfg, Optimizer& optim, LRScheduler& sched);
    // One optimizer step over one sequence (src/trainer.cpp:37-124); returns its loss.
    float train_step(const std::vector<int>& batch);
    // Accumulates one micro-batch; every grad_accum_steps calls it averages, clips and steps
    // (src/trainer.cpp:127-169). Returns the micro-batch's loss.
    float train_step_accum(const std::vector<int>& micro_batch);
    // B sequences of tokens.size() / B tokens in one device step; returns the mean loss.
    float train_step_batch(const std::vector<int>& tokens, int B);

    void save_train_state(const std::string& prefix);
    void load_train_state(const std::string& prefix);
    int skipped_steps() const { return skipped_; }
    int step() const { return step_; }
    void set_step(int s) { step_ = s; }
    void snapshot_params();
    bool rollback_if_nonfinite(float loss);
    float last_loss() const { return last_loss_; }
    float last_grad_norm() const { return last_grad_norm_; }

   private:
    float run(const std::vector<int>& tokens, int B, bool accum);
    GPT& model_;
    TrainConfig cfg_;
    Optimizer& optim_;
    LRScheduler& sched_;
    int step_ = 0;
    int skipped_ = 0;
    float last_loss_ = 0.0f;
    float last_grad_norm_ = 0.0f;
    std::vector<std::vector<float>> last_good_;
    bool has_snapshot_ = false;
};

}  // namespace llm
