// C++ façade over libllmgpu.so: llm::LRScheduler, CosineScheduler and StepScheduler with the
// reference's constructors and get_lr (include/llm/scheduler.h of the reference). get_lr is
// host arithmetic in float, evaluated the way src/scheduler.cpp evaluates it.
#pragma once

namespace llm {

class LRScheduler {
   public:
    virtual ~LRScheduler() = default;
    virtual float get_lr(int step) = 0;
};

// Linear warm-up to base_lr, then a cosine to min_lr over the rest of max_iters, optionally
// restarted `cycles` times (src/scheduler.cpp:13-28).
class CosineScheduler : public LRScheduler {
   public:
    CosineScheduler(float base_lr, int warmup, int max_iters);
    CosineScheduler(float base_lr, int warmup, int max_iters, float min_lr, int cycles = 1);
    float get_lr(int step) override;

   private:
    float base_lr_;
    int warmup_, max_iters_;
    float min_lr_ = 0.0f;
    int cycles_ = 1;
};

// base_lr * gamma^(step / step_size) (src/scheduler.cpp:29-33).
class StepScheduler : public LRScheduler {
   public:
    StepScheduler(float base_lr, int step_size, float gamma);
    float get_lr(int step) override;

   private:
    float base_lr_;
    int step_size_;
    float gamma_;
};

}  // namespace llm
