// C++ façade over libllmgpu.so: llm::Optimizer / Adam / AdamW with the reference's names,
// constructors and learning-rate accessors (include/llm/optimizer.h:8-76 of the reference).
//
// The update itself is the device AdamW that runs inside Trainer::train_step (decay of every
// tensor with ndim > 1 before the Adam update, bias corrections from the step counter, the
// same order as src/optimizer.cpp:13-48). An optimizer object here carries the
// hyper-parameters and the learning rate that the Trainer hands to the device; calling
// step() on host tensors directly throws, because the optimizer state lives on the device.
// Adam is AdamW without decay. SGD is not offered.
#pragma once
#include <vector>

#include "llm/tensor.h"

namespace llm {

class Optimizer {
   public:
    virtual ~Optimizer() = default;
    // Throws std::logic_error: the update runs on the device inside Trainer::train_step.
    virtual void step(std::vector<Tensor*>& params, const std::vector<Tensor>& grads);
    virtual void zero_grad() {}
    virtual void set_lr(float lr) = 0;
    virtual float get_lr() const = 0;
};

class Adam : public Optimizer {
   public:
    Adam(float lr = 1e-3f, float b1 = 0.9f, float b2 = 0.999f, float eps = 1e-8f);
    void set_lr(float lr) override { lr_ = lr; }
    float get_lr() const override { return lr_; }
    float beta1() const { return b1_; }
    float beta2() const { return b2_; }
    float epsilon() const { return eps_; }
    virtual float weight_decay() const { return 0.0f; }

   protected:
    float lr_, b1_, b2_, eps_;
};

class AdamW : public Adam {
   public:
    AdamW(float lr = 1e-3f, float b1 = 0.9f, float b2 = 0.999f, float eps = 1e-8f,
          float wd = 0.01f);
    float weight_decay() const override { return wd_; }

   private:
    float wd_;
};

}  // namespace llm
