// ORACLE harness — test infrastructure only, never part of the product.
//
// Runs the reference's own MoEFFN::forward (src/moe.cpp:23-62) and MoEFFN::aux_loss
// (src/moe.cpp:64-75), compiled unmodified from the reference sources by oracle/Makefile,
// on caller-given weights and inputs, to produce golden vectors for the MoE restatement.
// The reference keeps the gate and expert matrices private and offers no setter, so this
// harness opens the class's private section at include time to overwrite them after
// construction; no reference code is changed.
//
// usage: ref_moe <in.bin> <out.bin> C E k T coef
//   in.bin : float32 gate [C*E], W1 [E][C][4C], W2 [E][4C][C], x [T][C]
//   out.bin: float32 out [T][C], aux [1]
#include <cstdio>
#include <cstdlib>
#include <vector>

#define private public
#include "llm/moe.h"
#undef private

static bool read_all(const char* path, std::vector<float>& v) {
    FILE* f = std::fopen(path, "rb");
    if (!f) return false;
    const size_t n = std::fread(v.data(), sizeof(float), v.size(), f);
    std::fclose(f);
    return n == v.size();
}

int main(int argc, char** argv) {
    if (argc != 8) {
        std::fprintf(stderr, "usage: ref_moe in.bin out.bin C E k T coef\n");
        return 2;
    }
    const size_t C = std::strtoul(argv[3], nullptr, 10), E = std::strtoul(argv[4], nullptr, 10);
    const size_t k = std::strtoul(argv[5], nullptr, 10), T = std::strtoul(argv[6], nullptr, 10);
    const float coef = std::strtof(argv[7], nullptr);
    const size_t H = 4 * C;
    std::vector<float> in(C * E + 2 * E * C * H + T * C);
    if (!read_all(argv[1], in)) {
        std::fprintf(stderr, "cannot read %s\n", argv[1]);
        return 1;
    }
    llm::MoEFFN moe(C, llm::MoEConfig{E, k, 1.25f});
    const float* p = in.data();
    for (size_t i = 0; i < C * E; ++i) moe.gate_.data[i] = *p++;
    for (size_t e = 0; e < E; ++e)
        for (size_t i = 0; i < C * H; ++i) moe.experts_W1_[e].data[i] = *p++;
    for (size_t e = 0; e < E; ++e)
        for (size_t i = 0; i < H * C; ++i) moe.experts_W2_[e].data[i] = *p++;
    llm::Tensor x({T, C}, 0.0f);
    for (size_t i = 0; i < T * C; ++i) x.data[i] = *p++;
    llm::Tensor out = moe.forward(x);
    const float aux = moe.aux_loss(x, coef);
    FILE* f = std::fopen(argv[2], "wb");
    if (!f) return 1;
    std::fwrite(out.data.data(), sizeof(float), T * C, f);
    std::fwrite(&aux, sizeof(float), 1, f);
    std::fclose(f);
    return 0;
}
