// A training program written against the reference's C++ API (llm::Config, llm::GPT,
// llm::AdamW, llm::CosineScheduler, llm::TrainConfig, llm::Trainer), compiled unchanged
// against the façade headers of include/llm/ and linked with libllmgpu.so.
//
// usage: train_tiny OUT_PREFIX TOKENS.i32 STEPS T [CKPT]
//   trains STEPS optimizer steps, one sequence of T tokens each (train_step), then writes
//   OUT_PREFIX.losses (float32 per step), OUT_PREFIX.lr, OUT_PREFIX.gnorm and
//   OUT_PREFIX.params (every parameter, parameters() order) and saves a train state.
// Exit status 3 with the library's message on stderr when the device cannot be used.
#include <cstdio>
#include <cstdlib>
#include <exception>
#include <fstream>
#include <string>
#include <vector>

#include "llm/model.h"
#include "llm/optimizer.h"
#include "llm/scheduler.h"
#include "llm/trainer.h"

static void dump(const std::string& path, const std::vector<float>& v) {
    std::ofstream o(path, std::ios::binary);
    o.write(reinterpret_cast<const char*>(v.data()), (std::streamsize)(v.size() * sizeof(float)));
}

int main(int argc, char** argv) {
    if (argc < 5) {
        std::fprintf(stderr, "usage: %s OUT_PREFIX TOKENS.i32 STEPS T [CKPT]\n", argv[0]);
        return 2;
    }
    const std::string out = argv[1];
    const int steps = std::atoi(argv[3]);
    const size_t T = std::strtoul(argv[4], nullptr, 10);
    try {
        llm::Config cfg;
        cfg.vocab_size = 256;
        cfg.n_layers = 2;
        cfg.n_heads = 4;
        cfg.n_embd = 128;
        cfg.block_size = 64;
        llm::GPT model(cfg);
        if (argc > 5) model.load_binary(argv[5]);
        llm::AdamW opt(3e-4f, 0.9f, 0.95f, 1e-8f, 0.1f);
        llm::CosineScheduler sched(3e-4f, 2, 10, 3e-5f);
        llm::TrainConfig tc;
        tc.grad_clip = 1.0f;
        llm::Trainer trainer(model, tc, opt, sched);

        std::ifstream in(argv[2], std::ios::binary);
        std::vector<int> tokens((size_t)steps * T);
        for (auto& t : tokens) {
            int32_t v = 0;
            in.read(reinterpret_cast<char*>(&v), 4);
            t = v;
        }
        std::vector<float> losses, lrs, gnorms;
        for (int s = 0; s < steps; ++s) {
            std::vector<int> seq(tokens.begin() + (long)(s * T), tokens.begin() + (long)((s + 1) * T));
            losses.push_back(trainer.train_step(seq));
            lrs.push_back(opt.get_lr());
            gnorms.push_back(trainer.last_grad_norm());
            trainer.set_step(trainer.step() + 1);
        }
        std::vector<float> flat;
        for (llm::Tensor* p : model.parameters()) flat.insert(flat.end(), p->data.begin(), p->data.end());
        dump(out + ".losses", losses);
        dump(out + ".lr", lrs);
        dump(out + ".gnorm", gnorms);
        dump(out + ".params", flat);
        trainer.save_train_state(out + ".state");
        std::printf("ok %d steps, last loss %.6f, %zu parameters\n", steps, losses.back(),
                    model.num_parameters());
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 3;
    }
    return 0;
}
