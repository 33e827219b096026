// ORACLE harness (test infrastructure only): drives the reference's own data-feed pieces
// (read in place from the reference tree and linked unmodified) and prints what they produce,
// for the parity tests of the host-side feed in llm-cpp_b200/python/llmgpu/feed.py.
//   ref_feed lr                      -> "lr base warmup max_iters min_lr cycles step value" lines
//   ref_feed data TEXT_FILE BS       -> "tokens ...", then "loader ..." / "prefetch ..." batches
//   ref_feed log OUT_FILE            -> MetricsLogger lines written to OUT_FILE
//   ref_feed pack TEXT_FILE BLOCK EOS RATIO -> pack_with_eos rows/masks, train_val_split sizes
//   ref_feed sample                  -> logits rows, then seeded sampler picks (src/sampling.cpp)
//   ref_feed rng                     -> draws of std::uniform_int_distribution and
//                                       std::discrete_distribution sharing one std::mt19937(42)
//   ref_feed generate CKPT TEMP TOPK TOPP REP N PROMPT... -> GPT::generate (src/model.cpp:393-474)
//                                       on a v3 checkpoint (tied, LayerNorm, learned positions)
// Calls: CosineScheduler::get_lr (src/scheduler.cpp:13-28), Dataset / DataLoader
// (src/dataset.cpp:41-84), PrefetchLoader (src/prefetch.cpp), MetricsLogger::log_step
// (src/logging.cpp:49-55).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <fstream>
#include <random>

#include "llm/dataset.h"
#include "llm/model.h"
#include "llm/logging.h"
#include "llm/prefetch.h"
#include "llm/sampling.h"
#include "llm/scheduler.h"

static void print_batch(const char* tag, const std::vector<int>& b) {
    std::printf("%s %zu", tag, b.size());
    for (int t : b) std::printf(" %d", t);
    std::printf("\n");
}

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    if (!std::strcmp(argv[1], "lr")) {
        struct Cfg { float base; int warmup, max_iters; float min_lr; int cycles; };
        const Cfg cfgs[] = {{3e-4f, 100, 1000, 0.f, 1}, {1e-3f, 0, 500, 1e-5f, 1},
                            {6e-4f, 50, 1050, 6e-5f, 4}, {1e-3f, 10, 10, 1e-4f, 1},
                            {2e-4f, 7, 93, 0.f, 3}};
        for (const Cfg& c : cfgs) {
            llm::CosineScheduler s(c.base, c.warmup, c.max_iters, c.min_lr, c.cycles);
            for (int step = 0; step <= c.max_iters + 20; step += (step < 120 ? 1 : 37))
                std::printf("lr %.9g %d %d %.9g %d %d %.9g\n", c.base, c.warmup, c.max_iters,
                            c.min_lr, c.cycles, step, s.get_lr(step));
        }
        const float bases[] = {3e-4f, 1e-2f};
        const int sizes[] = {1, 7, 100};
        const float gammas[] = {0.5f, 0.9f, 0.33f};
        for (float base : bases)
            for (int size : sizes)
                for (float gamma : gammas) {
                    llm::StepScheduler s(base, size, gamma);
                    for (int step = 0; step < 400; step += 13)
                        std::printf("steplr %.9g %d %.9g %d %.9g\n", base, size, gamma, step,
                                    s.get_lr(step));
                }
        return 0;
    }
    if (!std::strcmp(argv[1], "data") && argc >= 4) {
        const size_t bs = std::strtoul(argv[3], nullptr, 10);
        llm::Dataset ds(argv[2], bs);
        print_batch("tokens", ds.tokens());
        llm::DataLoader dl(ds, bs);
        while (dl.has_next()) {
            auto b = dl.next_batch();
            if (b.empty()) break;
            print_batch("loader", b[0]);
        }
        llm::PrefetchLoader pl(ds, bs, 2);
        while (true) {
            auto b = pl.next();
            if (b.empty()) break;
            print_batch("prefetch", b[0]);
        }
        return 0;
    }
    if (!std::strcmp(argv[1], "sample")) {
        // rows of logits from a fixed LCG (printed exactly), then the samplers' picks
        uint64_t st = 12345;
        auto rnd = [&]() {
            st = st * 6364136223846793005ull + 1442695040888963407ull;
            return (float)((double)(st >> 40) / (double)(1ull << 24)) * 8.0f - 4.0f;
        };
        const int V = 50;
        for (int r = 0; r < 6; ++r) {
            std::vector<float> l(V);
            for (auto& v : l) v = rnd();
            std::printf("logits");
            for (float v : l) std::printf(" %.9g", v);
            std::printf("\n");
            const float temps[] = {0.7f, 1.0f, 1.6f};
            for (float t : temps)
                for (uint64_t seed = 0; seed < 40; ++seed) {
                    std::printf("temp %d %.9g %llu %d\n", r, t, (unsigned long long)seed,
                                llm::sample_temperature_seeded(l, t, seed));
                    std::printf("topk %d %.9g %llu %d\n", r, t, (unsigned long long)seed,
                                llm::sample_top_k_seeded(l, 5 + (int)(seed % 7), t, seed));
                    std::printf("topp %d %.9g %llu %d\n", r, t, (unsigned long long)seed,
                                llm::sample_top_p_seeded(l, 0.5f + 0.01f * (float)seed, t, seed));
                }
            std::printf("greedy %d %d\n", r, llm::sample_greedy(l));
            const std::vector<int> gen = {3, 7, 7, 49, 0, 3, 3};
            auto rp = llm::apply_repetition_penalty(l, gen, 1.3f);
            auto fp = llm::apply_freq_presence(l, gen, 0.25f, 0.5f);
            std::printf("reppen");
            for (float v : rp) std::printf(" %.9g", v);
            std::printf("\nfreqpres");
            for (float v : fp) std::printf(" %.9g", v);
            std::printf("\n");
        }
        return 0;
    }
    if (!std::strcmp(argv[1], "rng")) {
        std::mt19937 rng(42);
        for (int i = 0; i < 400; ++i) {
            const int k = 1 + (int)((i * 7919u + 13u) % 5000u);
            if (i % 3 == 2) {
                std::vector<float> w(17);
                for (int j = 0; j < 17; ++j) w[j] = (float)((j * 31 + i) % 11 + 1);
                std::discrete_distribution<int> d(w.begin(), w.end());
                std::printf("disc %d %d\n", i, d(rng));
            } else {
                std::uniform_int_distribution<int> d(0, k - 1);
                std::printf("uni %d %d %d\n", i, k, d(rng));
            }
        }
        return 0;
    }
    if (!std::strcmp(argv[1], "generate") && argc >= 8) {
        std::ifstream in(argv[2], std::ios::binary);
        uint32_t magic = 0, version = 0;
        size_t hdr[5] = {0};
        in.read((char*)&magic, 4);
        in.read((char*)&version, 4);
        for (auto& h : hdr) in.read((char*)&h, sizeof(size_t));
        if (!in || magic != 0x4C4C4D00u) return 3;
        llm::Config c;
        c.vocab_size = hdr[0];
        c.n_layers = hdr[1];
        c.n_heads = hdr[2];
        c.n_embd = hdr[3];
        c.block_size = hdr[4];
        llm::GPT model(c);
        model.load_binary(argv[2]);
        std::vector<int> prompt;
        for (int i = 8; i < argc; ++i) prompt.push_back(std::atoi(argv[i]));
        auto out = model.generate(prompt, std::strtoul(argv[7], nullptr, 10),
                                  (float)std::atof(argv[3]), std::atoi(argv[4]),
                                  (float)std::atof(argv[5]), (float)std::atof(argv[6]));
        print_batch("gen", out);
        return 0;
    }
    if (!std::strcmp(argv[1], "pack") && argc >= 6) {
        llm::Dataset ds(argv[2], 0);
        auto packed = llm::pack_with_eos(ds.tokens(), std::strtoul(argv[3], nullptr, 10),
                                         std::atoi(argv[4]));
        for (size_t i = 0; i < packed.input.size(); ++i) {
            print_batch("row", packed.input[i]);
            print_batch("mask", packed.mask[i]);
        }
        std::vector<int> tr, va;
        llm::train_val_split(ds.tokens(), std::atof(argv[5]), 7, tr, va);
        print_batch("train", tr);
        print_batch("val", va);
        return 0;
    }
    if (!std::strcmp(argv[1], "log") && argc >= 3) {
        llm::MetricsLogger log(argv[2]);
        log.log_step(1, 2.3614869f, 10.60655f, 3e-4f, 0.8754321f, 756960.19f);
        log.log_step(20, 0.125f, 1.1331485f, 1.5e-5f, 12.5f, 1e-3f);
        log.log_step(300, 7.0f, 1096.6332f, 0.f, 0.f, 0.f);
        return 0;
    }
    return 2;
}
