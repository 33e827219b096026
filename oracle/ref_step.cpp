// ORACLE — test infrastructure only (never part of the product path).
//
// Harness around the UNMODIFIED reference training step (sergiorandria/llm-cpp),
// linked from the reference's own sources by oracle/Makefile into oracle/_ref/.
// It loads a v3/v4 binary checkpoint (src/model.cpp:636-811) and a token file,
// runs `Trainer::train_step_accum` (src/trainer.cpp:127-169) with K = B
// micro-batches per optimizer step and a constant learning rate, and dumps:
//   losses.f32     loss of every micro-batch (src/loss.cpp:6-22), [steps*B]
//   grads.f32      raw mean gradient of the FIRST step (sum over micro-batches of
//                  p->grad divided by K, exactly as train_step_accum forms it
//                  before clipping), parameters() order (src/model.cpp:889-909)
//   params.f32     all parameters after the last step, parameters() order
//   gnorm.f32      Trainer::last_grad_norm() after each step
//   timing.txt     wall seconds per optimizer step
//
// usage: ref_step <ckpt.bin or -> <tokens.i32 or -> <B> <T> <outdir> [key=value ...]
//   "-" as checkpoint keeps the reference initialisation (vocab/layers/heads/embd/block keys);
//   "-" as token file draws seeded Zipf(1.1) ids (key seed).
//   keys: steps, lr, b1, b2, eps, wd, clip, tied (0/1), rmsnorm (0/1), mamba (0/1),
//         d_inner, d_state, dt_rank, conv_kernel, timing_only (0/1),
//         pos (0 learned, 1 sinusoidal, 2 RoPE), rope_theta, rope_scaling, rope_mode,
//         yarn_alpha, yarn_beta (Config fields of include/llm/model.h:25-33)
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <map>
#include <random>
#include <string>
#include <vector>

#include "llm/model.h"
#include "llm/optimizer.h"
#include "llm/scheduler.h"
#include "llm/trainer.h"

namespace {

struct ConstLR : llm::LRScheduler {
    float lr;
    explicit ConstLR(float v) : lr(v) {}
    float get_lr(int) override { return lr; }
};

bool read_header(const std::string& path, uint32_t& version, size_t (&hdr)[5], size_t (&mh)[4]) {
    std::ifstream in(path, std::ios::binary);
    if (!in) return false;
    uint32_t magic = 0;
    in.read((char*)&magic, 4);
    in.read((char*)&version, 4);
    if (magic != 0x4C4C4D00u) return false;
    for (auto& h : hdr) in.read((char*)&h, sizeof(size_t));
    if (version >= 4) {
        // skip the five top-level tensors (wte, wpe, ln_f gamma/beta, lm_head)
        for (int t = 0; t < 5; ++t) {
            uint64_t nd = 0, n = 0;
            in.read((char*)&nd, 8);
            in.seekg((std::streamoff)(8 * nd), std::ios::cur);
            in.read((char*)&n, 8);
            in.seekg((std::streamoff)(4 * n), std::ios::cur);
        }
        for (auto& h : mh) in.read((char*)&h, sizeof(size_t));
    }
    return (bool)in;
}

void dump(const std::string& path, const std::vector<float>& v) {
    std::ofstream o(path, std::ios::binary);
    o.write((const char*)v.data(), (std::streamsize)(v.size() * sizeof(float)));
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 6) {
        std::fprintf(stderr, "usage: %s ckpt tokens B T outdir [k=v...]\n", argv[0]);
        return 2;
    }
    std::string ckpt = argv[1], tokpath = argv[2], outdir = argv[5];
    const size_t B = std::strtoul(argv[3], nullptr, 10), T = std::strtoul(argv[4], nullptr, 10);
    std::map<std::string, std::string> kv;
    for (int i = 6; i < argc; ++i) {
        std::string s = argv[i];
        auto p = s.find('=');
        if (p != std::string::npos) kv[s.substr(0, p)] = s.substr(p + 1);
    }
    auto getf = [&](const char* k, double d) { return kv.count(k) ? std::atof(kv[k].c_str()) : d; };
    const int steps = (int)getf("steps", 1);
    const bool timing_only = getf("timing_only", 0) != 0;

    uint32_t version = 0;
    size_t hdr[5] = {0}, mh[4] = {0};
    const bool no_ckpt = (ckpt == "-");  // keep the reference constructors' initialisation
    if (no_ckpt) {
        version = getf("mamba", 0) != 0 ? 4 : 3;
        hdr[0] = (size_t)getf("vocab", 50257);
        hdr[1] = (size_t)getf("layers", 12);
        hdr[2] = (size_t)getf("heads", 12);
        hdr[3] = (size_t)getf("embd", 768);
        hdr[4] = (size_t)getf("block", 1024);
        mh[0] = (size_t)getf("d_inner", 0);
        mh[1] = (size_t)getf("d_state", 16);
        mh[2] = (size_t)getf("dt_rank", 0);
        mh[3] = (size_t)getf("conv_kernel", 4);
    } else if (!read_header(ckpt, version, hdr, mh)) {
        std::fprintf(stderr, "bad checkpoint %s\n", ckpt.c_str());
        return 3;
    }
    llm::Config c;
    c.vocab_size = hdr[0];
    c.n_layers = hdr[1];
    c.n_heads = hdr[2];
    c.n_embd = hdr[3];
    c.block_size = hdr[4];
    c.weight_tying = getf("tied", 1) != 0;
    c.use_rmsnorm = getf("rmsnorm", 0) != 0;
    c.use_mamba = version >= 4;
    const int pos = (int)getf("pos", 0);
    c.pos_encoding = pos == 2 ? llm::PosEncoding::RoPE
                   : pos == 1 ? llm::PosEncoding::Sinusoidal : llm::PosEncoding::Learned;
    c.rope_theta = (float)getf("rope_theta", 10000.0);
    c.rope_scaling = (float)getf("rope_scaling", 1.0);
    c.rope_mode = (int)getf("rope_mode", 0);
    c.yarn_alpha = (float)getf("yarn_alpha", 1.0);
    c.yarn_beta = (float)getf("yarn_beta", 32.0);
    if (c.use_mamba) {
        c.d_inner = mh[0];
        c.d_state = mh[1];
        c.dt_rank = mh[2];
        c.conv_kernel = mh[3];
    }
    llm::GPT model(c);
    if (!no_ckpt) model.load_binary(ckpt);

    std::vector<int> tokens(B * T * (size_t)steps);
    if (tokpath == "-") {
        // seeded Zipf(1.1) ids (rank k with probability ~ k^-1.1), when no token file is given
        std::mt19937_64 rng((uint64_t)getf("seed", 1234));
        std::vector<double> cdf(c.vocab_size);
        double acc = 0;
        for (size_t k = 0; k < c.vocab_size; ++k) cdf[k] = (acc += std::pow((double)(k + 1), -1.1));
        std::uniform_real_distribution<double> u(0.0, acc);
        for (auto& t : tokens)
            t = (int)(std::lower_bound(cdf.begin(), cdf.end(), u(rng)) - cdf.begin());
    } else {
        std::ifstream in(tokpath, std::ios::binary);
        std::vector<int32_t> raw;
        in.seekg(0, std::ios::end);
        size_t bytes = (size_t)in.tellg();
        in.seekg(0);
        raw.resize(bytes / 4);
        in.read((char*)raw.data(), (std::streamsize)bytes);
        if (raw.size() < B * T) {
            std::fprintf(stderr, "token file too short\n");
            return 4;
        }
        for (size_t i = 0; i < tokens.size(); ++i) tokens[i] = raw[i % raw.size()];
    }

    llm::TrainConfig tc;
    tc.grad_accum_steps = B;
    tc.grad_clip = (float)getf("clip", 1.0);
    llm::AdamW opt((float)getf("lr", 3e-4), (float)getf("b1", 0.9), (float)getf("b2", 0.95),
                   (float)getf("eps", 1e-8), (float)getf("wd", 0.1));
    ConstLR sched((float)getf("lr", 3e-4));
    llm::Trainer trainer(model, tc, opt, sched);

    std::vector<float> losses, gnorms, times, grads;
    auto params = model.parameters();
    std::vector<std::vector<float>> accum(params.size());
    for (size_t i = 0; i < params.size(); ++i) accum[i].assign(params[i]->data.size(), 0.0f);

    for (int s = 0; s < steps; ++s) {
        auto t0 = std::chrono::steady_clock::now();
        for (size_t b = 0; b < B; ++b) {
            std::vector<int> seq(tokens.begin() + (long)((s * B + b) * T),
                                 tokens.begin() + (long)((s * B + b + 1) * T));
            float loss = trainer.train_step_accum(seq);
            losses.push_back(loss);
            if (s == 0 && !timing_only) {
                // p->grad still holds this micro-batch's gradient (the optimizer
                // step of the last micro-batch does not touch it).
                for (size_t i = 0; i < params.size(); ++i) {
                    auto& g = params[i]->grad;
                    if (g.size() != params[i]->data.size()) continue;
                    for (size_t j = 0; j < g.size(); ++j) accum[i][j] += g[j];
                }
            }
        }
        auto t1 = std::chrono::steady_clock::now();
        times.push_back(std::chrono::duration<float>(t1 - t0).count());
        gnorms.push_back(trainer.last_grad_norm());
        trainer.set_step(trainer.step() + 1);
        if (s == 0 && !timing_only) {
            for (size_t i = 0; i < params.size(); ++i) {
                for (auto& v : accum[i]) v /= (float)B;
                grads.insert(grads.end(), accum[i].begin(), accum[i].end());
            }
        }
    }
    std::vector<float> pflat;
    for (auto* p : model.parameters()) pflat.insert(pflat.end(), p->data.begin(), p->data.end());
    dump(outdir + "/losses.f32", losses);
    dump(outdir + "/gnorm.f32", gnorms);
    if (!timing_only) {
        dump(outdir + "/grads.f32", grads);
        dump(outdir + "/params.f32", pflat);
    }
    {
        std::ofstream o(outdir + "/timing.txt");
        for (float t : times) o << t << "\n";
    }
    std::printf("ok steps=%d B=%zu T=%zu params=%zu loss0=%.6f\n", steps, B, T, pflat.size(),
                losses.empty() ? 0.0f : losses[0]);
    return 0;
}
