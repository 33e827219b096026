// ORACLE harness (test infrastructure only): the reference's own GGUF F32 writer and reader
// (src/gguf.cpp save_gguf / load_gguf), driven through its GPT and binary checkpoint
// (src/model.cpp), for the parity tests of llm-cpp_b200/python/llmgpu/gguf.py.
//   ref_gguf save V L H C BLOCK TIED RMS CKPT_IN GGUF_OUT   checkpoint -> GGUF
//   ref_gguf load V L H C BLOCK TIED RMS GGUF_IN CKPT_OUT   GGUF -> checkpoint
//   ref_gguf quant V L H C BLOCK TIED RMS CKPT_IN GGUF_OUT QTYPE   save_gguf_quant
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "llm/gguf.h"
#include "llm/model.h"

int main(int argc, char** argv) {
    if (argc != 11 && !(argc == 12 && !std::strcmp(argv[1], "quant"))) return 2;
    llm::Config c;
    c.vocab_size = std::strtoul(argv[2], nullptr, 10);
    c.n_layers = std::strtoul(argv[3], nullptr, 10);
    c.n_heads = std::strtoul(argv[4], nullptr, 10);
    c.n_embd = std::strtoul(argv[5], nullptr, 10);
    c.block_size = std::strtoul(argv[6], nullptr, 10);
    c.weight_tying = std::atoi(argv[7]) != 0;
    c.use_rmsnorm = std::atoi(argv[8]) != 0;
    llm::GPT model(c);
    if (!std::strcmp(argv[1], "save")) {
        model.load_binary(argv[9]);
        return llm::save_gguf(model, argv[10]) ? 0 : 1;
    }
    if (!std::strcmp(argv[1], "quant")) {
        model.load_binary(argv[9]);
        return llm::save_gguf_quant(model, argv[10], std::atoi(argv[11])) ? 0 : 1;
    }
    if (!std::strcmp(argv[1], "load")) {
        if (!llm::load_gguf(model, argv[9])) return 1;
        model.save_binary(argv[10]);
        return 0;
    }
    return 2;
}
