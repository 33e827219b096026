// Device-resident GPT training step: parameter arena, activations, forward/backward
// orchestration over the sm_100a kernels, optimizer, checkpoints.
//
// Reference path (sergiorandria/llm-cpp): GPT::forward_with_hidden (src/model.cpp:144-171),
// cross-entropy (src/loss.cpp:6-40), GPT::backward (src/model.cpp:175-323) through
// TransformerBlock::backward (src/transformer.cpp:225-269), clip_by_global_norm and AdamW
// (src/optimizer.cpp:53-101), orchestrated like Trainer::train_step_accum
// (src/trainer.cpp:127-169).
//
// Differences of method (not of result): no recomputation (activations are kept), all B
// sequences of a step form one [B*T, C] activation matrix, GEMMs take bf16 operands with
// fp32 accumulation, and the weight gradients of a step are formed once for the whole batch.
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <thread>
#include <cstring>
#include <fcntl.h>
#include <fstream>
#include <random>
#include <unistd.h>

#include "mamba.cuh"
#include "model.h"
#include "moe.cuh"

namespace llmgpu {

// Ends the communicator for good (its kernels in flight return) and marks the context.
void abort_comm(Ctx* c) {
    if (c->nccl) ncclCommAbort(reinterpret_cast<ncclComm_t>(c->nccl));
    c->nccl = nullptr;
    c->comm_failed = true;
}

namespace {

#define CK(x)                                                                  \
    do {                                                                       \
        cudaError_t e_ = (x);                                                  \
        if (e_ != cudaSuccess) {                                               \
            c->err = std::string(#x) + ": " + cudaGetErrorString(e_);          \
            return LLMGPU_E_CUDA;                                              \
        }                                                                      \
    } while (0)
#define KC(x)                                                                  \
    do {                                                                       \
        int r_ = (x);                                                          \
        if (r_ != 0) {                                                         \
            c->err = std::string(#x) + " failed with status " + std::to_string(r_); \
            if (r_ <= -1000)                                                   \
                c->err += std::string(" (") +                                  \
                          cudaGetErrorName((cudaError_t)(-r_ - 1000)) + ")";   \
            return LLMGPU_E_CUDA;                                              \
        }                                                                      \
        c->launches++;                                                         \
    } while (0)

inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch())
        .count();
}


// The communicator is non-blocking: a call may return ncclInProgress, and the next call may
// only be made once ncclCommGetAsyncError reports success. Polls up to the context's timeout.
int nccl_settle(Ctx* c, ncclResult_t r, const char* what, double timeout_s) {
    const double deadline = now_s() + timeout_s;
    ncclComm_t comm = reinterpret_cast<ncclComm_t>(c->nccl);
    while (r == ncclInProgress) {
        if (now_s() > deadline) {
            c->err = std::string(what) + ": not finished after " + std::to_string(timeout_s) +
                     " s (a peer rank did not take part); communicator aborted";
            abort_comm(c);
            return LLMGPU_E_NCCL;
        }
        std::this_thread::yield();
        if (ncclCommGetAsyncError(comm, &r) != ncclSuccess) r = ncclSystemError;
    }
    if (r != ncclSuccess) {
        c->err = std::string(what) + ": " + ncclGetErrorString(r) + "; communicator aborted";
        abort_comm(c);
        return LLMGPU_E_NCCL;
    }
    return 0;
}

void add_param(Ctx* c, const std::string& name, std::vector<int64_t> shape) {
    Param p;
    p.name = name;
    p.shape = shape;
    p.numel = 1;
    for (auto d : shape) p.numel *= d;
    p.decay = shape.size() > 1 ? 1 : 0;  // AdamW::default_decay (include/llm/optimizer.h:70-72)
    p.cols = (int)shape.back();
    p.offset = c->n_floats;
    c->n_floats = align_up(c->n_floats + p.numel, 64);
    c->params.push_back(p);
}

// GPT::parameters() order (src/model.cpp:889-909), blocks per TransformerBlock::parameters
// (src/transformer.cpp:279-290) or MambaBlock::parameters (src/mamba.cpp:415-420).
void build_params(Ctx* c) {
    const auto& k = c->cfg;
    const int C = k.n_embd, V = k.vocab_size;
    c->i_wte = (int)c->params.size();
    add_param(c, "wte", {V, C});
    c->i_wpe = (int)c->params.size();
    add_param(c, "wpe", {k.block_size, C});
    c->i_lnfg = (int)c->params.size();
    add_param(c, "ln_f_gamma", {C});
    c->i_lnfb = (int)c->params.size();
    add_param(c, "ln_f_beta", {C});
    if (!k.weight_tying) {
        c->i_lm = (int)c->params.size();
        add_param(c, "lm_head", {C, V});
    }
    for (int l = 0; l < k.n_layers; ++l) {
        BlockIdx b;
        const std::string p = "blk" + std::to_string(l) + ".";
        auto idx = [&]() { return (int)c->params.size(); };
        if (k.use_mamba) {
            const int D = k.d_inner ? k.d_inner : 2 * C;
            const int N = k.d_state;
            const int R = k.dt_rank ? k.dt_rank : (C + 15) / 16;
            const int K = k.conv_kernel;
            b.norm_w = idx(); add_param(c, p + "norm_w", {C});
            b.in_proj = idx(); add_param(c, p + "in_proj", {2 * D, C});
            b.conv_w = idx(); add_param(c, p + "conv_w", {D, 1, K});
            b.conv_b = idx(); add_param(c, p + "conv_b", {D});
            b.x_proj = idx(); add_param(c, p + "x_proj", {R + 2 * N, D});
            b.dt_proj = idx(); add_param(c, p + "dt_proj", {D, R});
            b.a_log = idx(); add_param(c, p + "a_log", {D, N});
            b.dskip = idx(); add_param(c, p + "d", {D});
            b.out_proj = idx(); add_param(c, p + "out_proj", {C, D});
        } else {
            b.Wq = idx(); add_param(c, p + "Wq", {C, C});
            b.Wk = idx(); add_param(c, p + "Wk", {C, C});
            b.Wv = idx(); add_param(c, p + "Wv", {C, C});
            b.Wo = idx(); add_param(c, p + "Wo", {C, C});
            if (k.moe_experts > 0) {
                const int E = k.moe_experts, Hd = 4 * C;
                b.gate = idx(); add_param(c, p + "gate", {C, E});
                b.W1e = idx(); add_param(c, p + "W1e", {E, C, Hd});
                b.W2e = idx(); add_param(c, p + "W2e", {E, Hd, C});
            } else {
                const int F = c->F;
                b.W1 = idx(); add_param(c, p + "W1", {C, F});
                b.W2 = idx(); add_param(c, p + "W2", {F, C});
                if (k.ffn_swiglu) { b.W3 = idx(); add_param(c, p + "W3", {C, F}); }
                b.b1 = idx(); add_param(c, p + "b1", {F});
                b.b2 = idx(); add_param(c, p + "b2", {C});
            }
            b.ln1g = idx(); add_param(c, p + "ln1_gamma", {C});
            b.ln1b = idx(); add_param(c, p + "ln1_beta", {C});
            b.ln2g = idx(); add_param(c, p + "ln2_gamma", {C});
            b.ln2b = idx(); add_param(c, p + "ln2_beta", {C});
        }
        c->blocks.push_back(b);
    }
}

// Host-side initialisation exactly like the reference constructors: every randn tensor
// draws from a fresh std::mt19937(42) (src/tensor.cpp:147-156), gains 1, biases 0.
void reference_init(Ctx* c, std::vector<float>& host) {
    host.assign((size_t)c->n_floats, 0.0f);
    auto randn = [&](int i, float stdv) {
        std::mt19937 rng(42);
        std::normal_distribution<float> dist(0.0f, stdv);
        float* d = host.data() + c->params[i].offset;
        for (int64_t j = 0; j < c->params[i].numel; ++j) d[j] = dist(rng);
    };
    auto fill = [&](int i, float v) {
        float* d = host.data() + c->params[i].offset;
        for (int64_t j = 0; j < c->params[i].numel; ++j) d[j] = v;
    };
    const auto& k = c->cfg;
    randn(c->i_wte, 0.02f);
    randn(c->i_wpe, 0.02f);
    if (k.pos_encoding == LLMGPU_POS_SINUSOIDAL) {
        // wpe[pos][i] = sin / cos(pos / 10000^(2*(i/2)/C)) for even / odd i (src/model.cpp:34-41)
        float* d = host.data() + c->params[c->i_wpe].offset;
        const int C = k.n_embd;
        for (int pos = 0; pos < k.block_size; ++pos)
            for (int i = 0; i < C; ++i) {
                const float angle = (float)pos / std::pow(10000.0f, (float)(2 * (i / 2)) / (float)C);
                d[(size_t)pos * C + i] = (i % 2 == 0) ? std::sin(angle) : std::cos(angle);
            }
    }
    fill(c->i_lnfg, 1.0f);
    if (c->i_lm >= 0) randn(c->i_lm, 0.02f);
    for (auto& b : c->blocks) {
        if (k.use_mamba) {
            const int C = k.n_embd;
            const int D = (int)c->params[b.in_proj].shape[0] / 2;
            const int K = k.conv_kernel;
            fill(b.norm_w, 1.0f);
            randn(b.in_proj, 1.0f / std::sqrt((float)C));
            randn(b.conv_w, 1.0f / std::sqrt((float)(D * K)));
            randn(b.x_proj, 1.0f / std::sqrt((float)D));
            randn(b.dt_proj, 0.001f);
            fill(b.a_log, -1.0f);
            fill(b.dskip, 1.0f);
            // out_proj_weight_ is not randn'd by the reference constructor (src/mamba.cpp:26-34)
        } else {
            randn(b.Wq, 0.02f);
            randn(b.Wk, 0.02f);
            randn(b.Wv, 0.02f);
            randn(b.Wo, 0.02f);
            if (b.gate >= 0) {
                randn(b.gate, 0.02f);
                // experts: each W1/W2 is its own randn(0,0.02) from seed 42 (src/moe.cpp:8-22)
                const int E = k.moe_experts;
                const int64_t per1 = c->params[b.W1e].numel / E, per2 = c->params[b.W2e].numel / E;
                for (int e = 0; e < E; ++e) {
                    std::mt19937 r1(42), r2(42);
                    std::normal_distribution<float> d1(0.0f, 0.02f), d2(0.0f, 0.02f);
                    float* w1 = host.data() + c->params[b.W1e].offset + e * per1;
                    float* w2 = host.data() + c->params[b.W2e].offset + e * per2;
                    for (int64_t j = 0; j < per1; ++j) w1[j] = d1(r1);
                    for (int64_t j = 0; j < per2; ++j) w2[j] = d2(r2);
                }
            } else {
                randn(b.W1, 0.02f);
                randn(b.W2, 0.02f);
                if (b.W3 >= 0) randn(b.W3, 0.02f);
            }
            fill(b.ln1g, 1.0f);
            fill(b.ln2g, 1.0f);
        }
    }
}

// Split-K factor of a weight-gradient GEMM (K = tokens) on 256x256 CTA-pair tiles. Cost in
// units of one 64-deep k-block of a tile (about 0.4 us): the waves of (tile, split) work
// units over the resident pairs, each with ~6 units of tile overhead, plus the split-K
// reduction's memory traffic ((s + 1) fp32 planes of M x N at ~6 TB/s).
int choose_splits(Ctx* c, int M, int N, int K) {
    const int slots = gemm_pair_slots(c->num_sms);
    const double tiles = (double)((M + 255) / 256) * ((N + 255) / 256);
    const int kb = (K + 63) / 64;
    int best_s = 1;
    double best = 1e30;
    const int cand[6] = {1, 2, 3, 4, 6, 8};
    for (int i = 0; i < 6; ++i) {
        const int s = cand[i];
        if (s > 1 && kb / s < 8) break;
        const double waves = std::ceil(tiles * s / slots);
        const double reduce_us = s > 1 ? (double)(s + 1) * M * N * 4.0 / 6.0e6 : 0.0;
        const double cost = waves * ((double)kb / s + 6.0) + reduce_us / 0.41;
        if (cost < best - 1e-9) {
            best = cost;
            best_s = s;
        }
    }
    return best_s;
}

// One product at a call site: operands, shape, epilogue and split-K factor; the plan index,
// final output and stride are filled in by gemm_prepare.
struct GemmCall {
    const void* A;
    long long lda;
    int amn;
    const void* B;
    long long ldb;
    int bmn;
    int M, N, K;
    GemmArgs a;
    int splits;
    size_t plan;
    void* final_out;
    long long final_ldo;
};

// Resolves the split-K factor (partials in c->splitws) and the call site's cached plan.
int gemm_prepare(Ctx* c, GemmCall& g) {
    GemmArgs& a = g.a;
    a.err = c->d_err;
    a.splits = 1;
    g.final_out = a.out;
    g.final_ldo = a.ldo;
    if (g.splits > 1) {
        if ((size_t)g.splits * g.M * g.N > c->splitws_floats)
            g.splits = (int)(c->splitws_floats / ((size_t)g.M * g.N));
        if (g.splits < 2) g.splits = 1;
    }
    if (g.splits > 1) {
        a.epi = kEpiSplitPartial;
        a.out = c->splitws;
        a.ldo = g.N;
        a.splits = g.splits;
    }
    struct Key {
        const void *A, *B;
        long long lda, ldb;
        int amn, bmn, M, N, K;
        GemmArgs args;
    } key;
    std::memset(&key, 0, sizeof(key));
    key.A = g.A;
    key.B = g.B;
    key.lda = g.lda;
    key.ldb = g.ldb;
    key.amn = g.amn;
    key.bmn = g.bmn;
    key.M = g.M;
    key.N = g.N;
    key.K = g.K;
    key.args = a;
    std::vector<uint8_t> kb(sizeof(Key));
    std::memcpy(kb.data(), &key, sizeof(Key));
    const size_t i = c->plan_cursor++;
    if (i >= c->plan_cache.size()) {
        c->plan_cache.resize(i + 1);
        c->plan_keys.resize(i + 1);
    }
    if (c->plan_keys[i] != kb) {
        int rc = gemm_make_plan(&c->plan_cache[i], g.A, g.lda, g.amn, g.B, g.ldb, g.bmn, g.M, g.N,
                                g.K, a, 0, c->num_sms);
        if (rc) {
            c->err = "gemm_make_plan failed (" + std::to_string(rc) + ") M=" +
                     std::to_string(g.M) + " N=" + std::to_string(g.N) +
                     " K=" + std::to_string(g.K);
            c->plan_keys[i].clear();
            return LLMGPU_E_ARG;
        }
        c->plan_keys[i] = kb;
    }
    g.plan = i;
    return 0;
}

void prof_begin(Ctx* c, const GemmCall& g0, const GemmCall* g1 = nullptr) {
    if (!c->profile) return;
    if (c->prof_ev.size() < 2 * (c->prof_n + 1)) {
        cudaEvent_t e0, e1;
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        c->prof_ev.push_back(e0);
        c->prof_ev.push_back(e1);
        c->prof_flops.push_back(0);
        c->prof_shape.resize(c->prof_shape.size() + 6, 0);
    }
    double flops = 2.0 * g0.M * g0.N * (double)g0.K;
    int* sh = &c->prof_shape[6 * c->prof_n];
    sh[0] = g0.M, sh[1] = g0.N, sh[2] = g0.K, sh[3] = sh[4] = sh[5] = 0;
    if (g1) {
        flops += 2.0 * g1->M * g1->N * (double)g1->K;
        sh[3] = g1->M, sh[4] = g1->N, sh[5] = g1->K;
    }
    c->prof_flops[c->prof_n] = flops;
    cudaEventRecord(c->prof_ev[2 * c->prof_n], c->stream);
}
void prof_end(Ctx* c) {
    if (!c->profile) return;
    cudaEventRecord(c->prof_ev[2 * c->prof_n + 1], c->stream);
    c->prof_n++;
}

int gemm_finish(Ctx* c, const GemmCall& g) {
    if (g.splits > 1)
        KC(gemm_splitk_reduce(c->splitws, g.splits, g.M, g.N,
                              reinterpret_cast<float*>(g.final_out), g.final_ldo,
                              g.a.col_group > 0 ? g.a.col_group : g.N, g.a.group_stride,
                              g.a.accumulate, c->stream));
    return 0;
}

// GEMM through the per-call-site plan cache.
int gemm(Ctx* c, const void* A, long long lda, int amn, const void* B, long long ldb, int bmn,
         int M, int N, int K, GemmArgs a, int splits = 1) {
    GemmCall g{A, lda, amn, B, ldb, bmn, M, N, K, a, splits, 0, nullptr, 0};
    int rc = gemm_prepare(c, g);
    if (rc) return rc;
    prof_begin(c, g);
    KC(gemm_run(c->plan_cache[g.plan], c->stream));
    prof_end(c);
    return gemm_finish(c, g);
}

// The data- and weight-gradient products of one layer (independent: both read the upstream
// gradient) in one launch of the pair kernel, their tiles balanced over all pairs. Falls back
// to two launches when either plan is not on pair tiles. At most one of them may split K.
int gemm_dual(Ctx* c, GemmCall g0, GemmCall g1) {
    int rc;
    if ((rc = gemm_prepare(c, g0)) || (rc = gemm_prepare(c, g1))) return rc;
    if (g0.splits > 1 && g1.splits > 1) return LLMGPU_E_ARG;  // one split-K workspace
    const size_t i = c->plan2_cursor++;
    if (i >= c->plan2_cache.size()) {
        c->plan2_cache.resize(i + 1);
        c->plan2_keys.resize(i + 1);
        c->plan2_ok.resize(i + 1, 0);
    }
    std::vector<uint8_t> key = c->plan_keys[g0.plan];
    key.insert(key.end(), c->plan_keys[g1.plan].begin(), c->plan_keys[g1.plan].end());
    if (c->plan2_keys[i] != key) {
        gemm_free_plan2(&c->plan2_cache[i]);
        c->plan2_ok[i] = gemm_make_plan2(&c->plan2_cache[i], c->plan_cache[g0.plan],
                                         c->plan_cache[g1.plan], c->num_sms) == 0;
        c->plan2_keys[i] = key;
    }
    prof_begin(c, g0, &g1);
    if (c->plan2_ok[i]) {
        // run-time tile queue with data parallelism: the all-reduce kernels hold SMs during
        // the backward's launches (2 x B200: 11.67 against 11.83 ms per step; alone the
        // host's lists are 0.08 ms faster)
        KC(gemm_run2(c->plan2_cache[i], c->stream, c->world > 1));
    } else {
        KC(gemm_run(c->plan_cache[g0.plan], c->stream));
        KC(gemm_run(c->plan_cache[g1.plan], c->stream));
    }
    prof_end(c);
    if ((rc = gemm_finish(c, g0)) || (rc = gemm_finish(c, g1))) return rc;
    return 0;
}

GemmArgs epi_args(int epi, void* out, long long ldo) {
    GemmArgs a{};
    a.epi = epi;
    a.out = out;
    a.ldo = ldo;
    a.splits = 1;
    return a;
}

template <typename T>
int dalloc(Ctx* c, T** p, size_t n) {
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T) + 256);
    if (e != cudaSuccess) {
        c->err = std::string("cudaMalloc: ") + cudaGetErrorString(e);
        return LLMGPU_E_CUDA;
    }
    // ordered on the context stream (a legacy-stream memset would not be ordered with it)
    cudaMemsetAsync(*p, 0, n * sizeof(T), c->stream);
    return 0;
}

}  // namespace

// Host<->device copies ordered on the context stream and completed before returning.
// (A plain cudaMemcpy runs on the legacy stream, which the context's non-blocking streams
// do not wait for, and from pageable memory it may return before the DMA has landed.)
int copy_sync(Ctx* c, void* dst, const void* src, size_t bytes, cudaMemcpyKind kind) {
    if (bytes == 0) return 0;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, kind, c->stream);
    if (e != cudaSuccess) {
        c->err = std::string("copy: ") + cudaGetErrorString(e);
        return LLMGPU_E_CUDA;
    }
    return wait_stream(c, c->stream);
}

// ---------------------------------------------------------------------------- shadows
void refresh_shadows(Ctx* c) {
    write_shadows(c->d_aparams, c->d_chunks, c->nchunks, c->p, c->stream);
}

// ---------------------------------------------------------------------------- create
Ctx* ctx_create(const llmgpu_config& cfg, int max_batch, int max_seq, int rank, int world,
                const void* uid, std::string* errout) {
    auto fail = [&](Ctx* c, const std::string& m) -> Ctx* {
        *errout = m.empty() ? c->err : m;
        ctx_destroy(c);
        return nullptr;
    };
    Ctx* c = new Ctx();
    c->cfg = cfg;
    c->rank = rank;
    c->world = world;
    if (const char* e = std::getenv("LLMGPU_GRAPH")) c->use_graph = std::atoi(e) != 0;
    if (cfg.vocab_size <= 0 || cfg.n_layers <= 0 || cfg.n_embd <= 0 || cfg.block_size <= 0 ||
        max_batch <= 0 || max_seq <= 0 || max_seq > cfg.block_size)
        return fail(c, "invalid configuration");
    if (cfg.pos_encoding < LLMGPU_POS_LEARNED || cfg.pos_encoding > LLMGPU_POS_ROPE)
        return fail(c, "pos_encoding must be 0 (learned), 1 (sinusoidal) or 2 (RoPE)");
    if (!cfg.use_mamba && (cfg.n_heads <= 0 || cfg.n_embd % cfg.n_heads != 0))
        return fail(c, "n_heads must divide n_embd");  // src/config.cpp:39-68
    c->C = cfg.n_embd;
    c->V = cfg.vocab_size;
    c->Vp = (int)align_up(c->V, 128);
    c->L = cfg.n_layers;
    c->H = cfg.use_mamba ? 1 : cfg.n_heads;
    c->hd = c->C / c->H;
    c->F = cfg.ffn_hidden > 0 ? cfg.ffn_hidden : 4 * c->C;
    c->max_b = max_batch;
    c->max_t = max_seq;
    c->max_bt = max_batch * max_seq;
    c->moe = cfg.moe_experts > 0 && !cfg.use_mamba;
    if (c->moe) {
        // MoEFFN (src/moe.cpp:8-22): experts of hidden 4 * n_embd, GELU, top-k routing
        c->moe_E = cfg.moe_experts;
        c->moe_k = cfg.moe_top_k > 0 ? cfg.moe_top_k : 2;
        c->moe_He = 4 * cfg.n_embd;
        c->moe_coef = cfg.moe_aux_coef;
        if (c->moe_E > kMoeMaxExperts || c->moe_k > kMoeMaxTopK || c->moe_k > c->moe_E ||
            cfg.ffn_swiglu || cfg.n_embd % 64 != 0)
            return fail(c, "unsupported MoE configuration (at most 16 experts, top-k <= 4, "
                           "n_embd a multiple of 64, GELU experts)");
        c->moe_cap = moe_capacity(max_batch * max_seq, c->moe_E, c->moe_k);
    }
    c->mamba = cfg.use_mamba != 0;
    c->swiglu = cfg.ffn_swiglu != 0;
    const int FH = c->swiglu ? 2 * c->F : c->F;  // width of the FFN up-projection output
    if (c->mamba) {
        // MambaBlock dims (src/model.cpp:44-47): d_inner 0 -> 2*n_embd, dt_rank 0 -> ceil(n_embd/16)
        c->mD = cfg.d_inner ? cfg.d_inner : 2 * c->C;
        c->mN = cfg.d_state;
        c->mR = cfg.dt_rank ? cfg.dt_rank : (c->C + 15) / 16;
        c->mK = cfg.conv_kernel;
        c->mRP = c->mR + 2 * c->mN;
        c->mRPp = (int)align_up(c->mRP, 8);
        c->mRp = (int)align_up(c->mR, 8);
        if (c->C % 8 != 0 || c->mD % 8 != 0 || c->mN < 1 || c->mN > 16 || c->mK < 1 ||
            c->mK > 8 || c->mR < 1 || c->mR > 64)
            return fail(c, "unsupported Mamba dimensions (n_embd, d_inner multiples of 8; "
                           "d_state <= 16; conv_kernel <= 8)");
    } else {
        if (c->hd != 32 && c->hd != 64) return fail(c, "head_dim must be 32 or 64");
        if (c->C % 32 != 0 || c->F % 32 != 0)
            return fail(c, "n_embd and ffn hidden must be multiples of 32");
    }
    if (c->max_bt > 16384) return fail(c, "at most 16384 tokens per micro-batch");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(c, "no CUDA device");
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return fail(c, "no CUDA device");
    if (prop.major != 10) return fail(c, "requires an sm_100 (B200) device");
    c->device = dev;
    c->num_sms = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) != cudaSuccess)
        return fail(c, "stream creation failed");
    cudaEventCreateWithFlags(&c->ev_keys, cudaEventDisableTiming);
    for (auto& e : c->ev) cudaEventCreate(&e);

    build_params(c);
    const int C = c->C, F = c->F, BT = c->max_bt, L = c->L;
    if (dalloc(c, &c->p, c->n_floats) || dalloc(c, &c->g, c->n_floats) ||
        dalloc(c, &c->m, c->n_floats) || dalloc(c, &c->v, c->n_floats))
        return fail(c, "");

    // bf16 shadows laid out for the GEMMs
    size_t sh = (size_t)c->Vp * C;                            // wte16 [Vp, C]
    if (!cfg.weight_tying) sh += (size_t)C * c->Vp;           // lm16 [C, Vp]
    if (c->mamba)
        sh += (size_t)L * (2 * (size_t)c->mD * C + (size_t)c->mRP * c->mD +
                           (size_t)c->mD * c->mRp + (size_t)C * c->mD + 64 * 4);
    else if (c->moe)
        sh += (size_t)L * ((size_t)C * 3 * C + (size_t)C * C +
                           2 * (size_t)c->moe_E * C * c->moe_He + 64 * 4);
    else
        sh += (size_t)L * ((size_t)C * 3 * C + (size_t)C * C + (size_t)C * FH + (size_t)C * F +
                           64 * 4);
    c->shadow_elems = sh;
    if (dalloc(c, &c->shadow_arena, sh)) return fail(c, "");
    {
        bf16* q = c->shadow_arena;
        auto take = [&](size_t n) {
            bf16* r = q;
            q += align_up((int64_t)n, 64);
            return r;
        };
        c->wte16 = take((size_t)c->Vp * C);
        c->params[c->i_wte].shadow = c->wte16;
        c->params[c->i_wte].shadow_ld = C;
        if (!cfg.weight_tying) {
            c->lm16 = take((size_t)C * c->Vp);
            c->params[c->i_lm].shadow = c->lm16;
            c->params[c->i_lm].shadow_ld = c->Vp;
        }
        for (int l = 0; l < L && c->mamba; ++l) {
            auto& b = c->blocks[l];
            const int D = c->mD;
            bf16* in = take((size_t)2 * D * C);           // in_proj  [2D, E]
            bf16* xw = take((size_t)c->mRP * D);          // x_proj   [R+2N, D]
            bf16* dw = take((size_t)D * c->mRp);          // dt_proj  [D, R] (row stride Rp)
            bf16* ow = take((size_t)C * D);               // out_proj [E, D]
            c->in16.push_back(in);
            c->xproj16.push_back(xw);
            c->dtp16.push_back(dw);
            c->out16.push_back(ow);
            c->params[b.in_proj].shadow = in;
            c->params[b.in_proj].shadow_ld = C;
            c->params[b.x_proj].shadow = xw;
            c->params[b.x_proj].shadow_ld = D;
            c->params[b.dt_proj].shadow = dw;
            c->params[b.dt_proj].shadow_ld = c->mRp;
            c->params[b.out_proj].shadow = ow;
            c->params[b.out_proj].shadow_ld = D;
        }
        for (int l = 0; l < L && !c->mamba; ++l) {
            auto& b = c->blocks[l];
            bf16* wqkv = take((size_t)C * 3 * C);
            bf16* wo = take((size_t)C * C);
            c->wqkv16.push_back(wqkv);
            c->wo16.push_back(wo);
            c->params[b.Wq].shadow = wqkv;
            c->params[b.Wk].shadow = wqkv + C;
            c->params[b.Wv].shadow = wqkv + 2 * C;
            c->params[b.Wq].shadow_ld = c->params[b.Wk].shadow_ld = c->params[b.Wv].shadow_ld = 3 * C;
            c->params[b.Wo].shadow = wo;
            c->params[b.Wo].shadow_ld = C;
            if (c->moe) {
                // expert stacks, row-major like the parameters: W1e [E*C, He], W2e [E*He, C]
                const size_t ne = (size_t)c->moe_E * C * c->moe_He;
                bf16* w1e = take(ne);
                bf16* w2e = take(ne);
                c->w1e16.push_back(w1e);
                c->w2e16.push_back(w2e);
                c->params[b.W1e].shadow = w1e;
                c->params[b.W1e].shadow_ld = c->moe_He;
                c->params[b.W2e].shadow = w2e;
                c->params[b.W2e].shadow_ld = C;
                continue;
            }
            bf16* w1 = take((size_t)C * FH);  // [C, F] or, for SwiGLU, [W1 | W3] as [C, 2F]
            bf16* w2 = take((size_t)F * C);
            c->w1_16.push_back(w1);
            c->w2_16.push_back(w2);
            c->params[b.W1].shadow = w1;
            c->params[b.W1].shadow_ld = FH;
            if (b.W3 >= 0) {
                c->params[b.W3].shadow = w1 + F;
                c->params[b.W3].shadow_ld = FH;
            }
            c->params[b.W2].shadow = w2;
            c->params[b.W2].shadow_ld = C;
        }
    }
    // RoPE (cos, sin) table [max_t][hd/2] for the rotation fused into the attention loads
    if (cfg.rope_qk) {
        const int P = c->hd / 2;
        std::vector<float> tab((size_t)max_seq * P * 2);
        for (int pos = 0; pos < max_seq; ++pos)
            for (int j = 0; j < P; ++j) {
                const double freq = std::pow((double)cfg.rope_theta, -2.0 * j / (double)c->hd);
                const double ang = pos * freq;
                tab[((size_t)pos * P + j) * 2] = (float)std::cos(ang);
                tab[((size_t)pos * P + j) * 2 + 1] = (float)std::sin(ang);
            }
        if (dalloc(c, &c->rope, tab.size() / 2) ||
            copy_sync(c, c->rope, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice))
            return fail(c, "");
    }

    // Config::pos_encoding == RoPE: rope_cfg (src/model.cpp:71-104) evaluated once per position
    // and column pair with the reference's own float expressions (NTK base * scaling, or the
    // YaRN ramp with its attention scale), applied by the embedding gather
    if (cfg.pos_encoding == LLMGPU_POS_ROPE) {
        const float scaling = cfg.rope_scaling < 1.0f ? 1.0f : cfg.rope_scaling;
        const float base = cfg.rope_theta * (cfg.rope_mode == 0 ? scaling : 1.0f);
        const bool yarn = cfg.rope_mode == 1 && scaling > 1.0f;
        c->emb_rope_scale = yarn ? std::sqrt(1.0f + 0.1f * std::log(scaling)) : 1.0f;
        auto ramp = [&](int dim) {  // yarn_ramp (src/model.cpp:71-78)
            const float d = (float)dim / (float)C * cfg.yarn_beta;
            const float low = cfg.yarn_beta / 2.0f, high = cfg.yarn_beta;
            if (d < low) return 0.0f;
            if (d > high) return 1.0f;
            return (d - low) / (high - low);
        };
        const int P = C / 2;
        std::vector<float> tab((size_t)max_seq * P * 2);
        for (int pos = 0; pos < max_seq; ++pos)
            for (int j = 0; j < P; ++j) {
                const int i = 2 * j;
                float freq = std::pow(base, -(float)i / (float)C);
                if (yarn) {
                    const float m = ramp(i);
                    freq = ((1.0f - m) / scaling + m) * std::pow(cfg.rope_theta, -(float)i / (float)C);
                }
                const float angle = (float)pos * freq * cfg.yarn_alpha;
                tab[((size_t)pos * P + j) * 2] = std::cos(angle);
                tab[((size_t)pos * P + j) * 2 + 1] = std::sin(angle);
            }
        if (dalloc(c, &c->emb_rope, tab.size() / 2) ||
            copy_sync(c, c->emb_rope, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice))
            return fail(c, "");
    }

    // activations
    c->act.resize(L);
    const int nparts = norm_backward_grid(BT);
    if (c->mamba) {
        const size_t D = c->mD;
        const int nch = (max_seq + kScanChunk - 1) / kScanChunk;
        c->mact.resize(L);
        for (int l = 0; l < L; ++l) {
            auto& a = c->act[l];
            auto& m = c->mact[l];
            if (dalloc(c, &a.x, (size_t)BT * C) || dalloc(c, &a.ln1, (size_t)BT * C) ||
                dalloc(c, &a.mean1, BT) || dalloc(c, &a.rstd1, BT) ||
                dalloc(c, &m.proj, (size_t)BT * 2 * D) || dalloc(c, &m.u32, (size_t)BT * D) ||
                dalloc(c, &m.u16, (size_t)BT * D) || dalloc(c, &m.xp, (size_t)BT * c->mRPp) ||
                dalloc(c, &m.xp16, (size_t)BT * c->mRPp) || dalloc(c, &m.raw, (size_t)BT * D) ||
                dalloc(c, &m.y, (size_t)BT * D) || dalloc(c, &m.gated, (size_t)BT * D) ||
                dalloc(c, &m.hchk, (size_t)max_batch * nch * D * c->mN))
                return fail(c, "");
        }
        const int groups = mamba_scan_groups(c->mD, c->mN);
        if (dalloc(c, &c->m_dgated, (size_t)BT * D) || dalloc(c, &c->m_du, (size_t)BT * D) ||
            dalloc(c, &c->m_duxp, (size_t)BT * D) ||
            dalloc(c, &c->m_dpre, (size_t)BT * D) ||
            dalloc(c, &c->m_dbc, (size_t)groups * 2 * BT * c->mN) ||
            dalloc(c, &c->m_da,
                   (size_t)mamba_scan_parts_max(max_batch, max_seq, D, c->mN) * D * c->mN) ||
            dalloc(c, &c->m_dd, (size_t)mamba_scan_parts_max(max_batch, max_seq, D, c->mN) * D) ||
            dalloc(c, &c->m_convpart, (size_t)mamba_conv_blocks(BT) * D * (c->mK + 1)) ||
            dalloc(c, &c->m_dproj, (size_t)BT * 2 * D) ||
            dalloc(c, &c->m_dxp, (size_t)BT * c->mRPp) ||
            dalloc(c, &c->m_sgpart,
                   std::max((size_t)kSgSplitRows * BT, (size_t)kSgSplitCols * D) * c->mR) ||
            dalloc(c, &c->m_segwork, mamba_scan_seg_floats(max_batch, max_seq, D, c->mN)))
            return fail(c, "");
    }
    for (int l = 0; l < L && !c->mamba; ++l) {
        auto& a = c->act[l];
        if (dalloc(c, &a.x, (size_t)BT * C) || dalloc(c, &a.y, (size_t)BT * C) ||
            dalloc(c, &a.ln1, (size_t)BT * C) || dalloc(c, &a.mean1, BT) ||
            dalloc(c, &a.rstd1, BT) || dalloc(c, &a.qkv, (size_t)BT * 3 * C) ||
            dalloc(c, &a.att, (size_t)BT * C) || dalloc(c, &a.lse, (size_t)BT * c->H) ||
            dalloc(c, &a.ln2, (size_t)BT * C) || dalloc(c, &a.mean2, BT) ||
            dalloc(c, &a.rstd2, BT))
            return fail(c, "");
        if (!c->moe && (dalloc(c, &a.h, (size_t)BT * FH) || dalloc(c, &a.act, (size_t)BT * F)))
            return fail(c, "");
    }
    if (c->moe) {
        const size_t E = c->moe_E, k = c->moe_k, He = c->moe_He, cap = c->moe_cap;
        c->moeact.resize(L);
        for (int l = 0; l < L; ++l) {
            auto& e = c->moeact[l];
            if (dalloc(c, &e.probs, (size_t)BT * E) || dalloc(c, &e.idx, (size_t)BT * k) ||
                dalloc(c, &e.wts, (size_t)BT * k) || dalloc(c, &e.ssum, BT) ||
                dalloc(c, &e.grp, 2 * E + 1) || dalloc(c, &e.row_of, (size_t)BT * k) ||
                dalloc(c, &e.tok_of, cap) || dalloc(c, &e.xg, cap * C) ||
                dalloc(c, &e.pre, cap * He) || dalloc(c, &e.act, cap * He) ||
                dalloc(c, &e.yg, cap * C))
                return fail(c, "");
        }
        if (dalloc(c, &c->moe_load, (size_t)L * max_batch * E) ||
            dalloc(c, &c->moe_aux, (size_t)L * max_batch) || dalloc(c, &c->e_dyg, cap * C) ||
            dalloc(c, &c->e_dpre, cap * He) || dalloc(c, &c->e_dxg, cap * C) ||
            dalloc(c, &c->e_dscores, (size_t)BT * E) ||
            dalloc(c, &c->e_gpart, (size_t)moe_gate_grad_parts(BT) * C * E))
            return fail(c, "");
    }
    if (dalloc(c, &c->xL, (size_t)BT * C) || dalloc(c, &c->lnf, (size_t)BT * C) ||
        dalloc(c, &c->meanf, BT) || dalloc(c, &c->rstdf, BT) ||
        dalloc(c, &c->logits, (size_t)BT * c->Vp) || dalloc(c, &c->dres, (size_t)BT * C) ||
        dalloc(c, &c->dy, (size_t)BT * C) || dalloc(c, &c->dln, (size_t)BT * C) ||
        dalloc(c, &c->dres16, (size_t)BT * C) || dalloc(c, &c->dy16, (size_t)BT * C) ||
        dalloc(c, &c->datt, (size_t)BT * C) || dalloc(c, &c->dqkv, (size_t)BT * 3 * C) ||
        dalloc(c, &c->dh, (size_t)BT * FH) || dalloc(c, &c->dvec, (size_t)BT * c->H) ||
        (!c->mamba &&
         dalloc(c, &c->attn_ds,
                attention_work_bytes(max_batch, max_seq, c->H, c->hd) / sizeof(bf16))) ||
        (c->swiglu && dalloc(c, &c->dact, (size_t)BT * F)) ||
        dalloc(c, &c->partial, (size_t)nparts * 3 * C) ||
        dalloc(c, &c->colwork, colsum_work_floats(F > C ? F : C)))
        return fail(c, "");
    c->splitws_floats = (size_t)8 * C * (FH > 3 * C ? FH : 3 * C);
    if (c->mamba) {  // largest Mamba weight gradient: in_proj [2D, E]
        const size_t mx = std::max<size_t>((size_t)2 * c->mD * C, (size_t)c->mRP * c->mD);
        c->splitws_floats = std::max(c->splitws_floats, (size_t)8 * mx);
    }
    if (dalloc(c, &c->splitws, c->splitws_floats)) return fail(c, "");
    if (dalloc(c, &c->d_tokens, BT) || dalloc(c, &c->d_keys, BT) ||
        dalloc(c, &c->d_row_loss, BT) || dalloc(c, &c->d_out, 8) || dalloc(c, &c->d_hp, 16) ||
        dalloc(c, &c->d_normpart, grad_norm_blocks()) || dalloc(c, &c->d_nonfinite, 1) ||
        dalloc(c, &c->d_err, 1) || dalloc(c, &c->d_kscale, 1))
        return fail(c, "");
    if (cudaMallocHost(&c->h_tokens, sizeof(int32_t) * BT) != cudaSuccess ||
        cudaMallocHost(&c->h_out, sizeof(float) * 8) != cudaSuccess ||
        cudaMallocHost(&c->h_hp, sizeof(float) * 16) != cudaSuccess ||
        cudaMallocHost(&c->h_err, sizeof(int)) != cudaSuccess)
        return fail(c, "cudaMallocHost failed");

    // optimizer tables
    {
        std::vector<AdamParam> ap;
        std::vector<AdamChunk> ch;
        const int64_t CH = 16384;
        for (size_t i = 0; i < c->params.size(); ++i) {
            const auto& p = c->params[i];
            AdamParam a{};
            a.offset = p.offset;
            a.numel = p.numel;
            a.cols = p.cols;
            a.decay = p.decay;
            a.shadow = p.shadow;
            a.shadow_ld = p.shadow ? p.shadow_ld : p.cols;
            ap.push_back(a);
            for (int64_t s = 0; s < p.numel; s += CH) {
                AdamChunk k{};
                k.param = (int)i;
                k.start = s;
                k.len = (int)std::min<int64_t>(CH, p.numel - s);
                ch.push_back(k);
            }
        }
        c->nchunks = (int)ch.size();
        if (dalloc(c, &c->d_aparams, ap.size()) || dalloc(c, &c->d_chunks, ch.size()))
            return fail(c, "");
        if (copy_sync(c, c->d_aparams, ap.data(), ap.size() * sizeof(AdamParam), cudaMemcpyHostToDevice) ||
            copy_sync(c, c->d_chunks, ch.data(), ch.size() * sizeof(AdamChunk), cudaMemcpyHostToDevice))
            return fail(c, "");
    }

    // parameters initialised like the reference constructors
    {
        std::vector<float> host;
        reference_init(c, host);
        if (copy_sync(c, c->p, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice))
            return fail(c, "");
        refresh_shadows(c);
    }

    // gradient buckets: block l's contiguous parameter range, then the rest (embeddings, ln_f,
    // untied head) as bucket L
    {
        std::vector<int64_t> start(c->L + 1, c->n_floats);
        for (size_t i = 0; i < c->params.size(); ++i) {
            const std::string& n = c->params[i].name;
            if (n.compare(0, 3, "blk") == 0) {
                const int l = std::atoi(n.c_str() + 3);
                start[l] = std::min(start[l], c->params[i].offset);
            }
        }
        c->buckets.resize(c->L + 1);
        for (int l = 0; l < c->L; ++l) c->buckets[l] = {start[l], l + 1 < c->L ? start[l + 1] : c->n_floats};
        c->buckets[c->L] = {0, start[0]};
    }
    if (world > 1) {
        if (cudaStreamCreateWithFlags(&c->comm, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ev_grad, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ev_comm, cudaEventDisableTiming) != cudaSuccess)
            return fail(c, "stream creation failed");
        ncclUniqueId id;
        std::memcpy(&id, uid, sizeof(id));
        ncclComm_t comm = nullptr;
        // NCCL's own CTA count by default; LLMGPU_NCCL_MAX_CTAS caps it (fewer CTAs leave more
        // SMs to the backward the buckets overlap, but slow the last, unoverlapped bucket).
        // Non-blocking, so that no host call waits on a peer without a bound.
        ncclConfig_t ncfg = NCCL_CONFIG_INITIALIZER;
        ncfg.blocking = 0;
        if (const char* e = std::getenv("LLMGPU_NCCL_MAX_CTAS")) ncfg.maxCTAs = std::atoi(e);
        if (const char* e = std::getenv("LLMGPU_COMM_TIMEOUT_S")) c->comm_timeout_s = std::atof(e);
        ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &ncfg);
        c->nccl = comm;
        if (!comm && r != ncclSuccess)
            return fail(c, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
        if (nccl_settle(c, r, "ncclCommInitRankConfig", c->comm_timeout_s)) return fail(c, "");
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return fail(c, "device error during setup");
    return c;
}

void ctx_destroy(Ctx* c) {
    if (!c) return;
    // a collective that never completes (a peer gone) would block the device sync below
    if (c->nccl && c->stream && wait_stream(c, c->stream) == 0 && c->comm)
        wait_stream(c, c->comm);
    cudaDeviceSynchronize();
    decode_free(c);
    if (c->graph) cudaGraphExecDestroy(c->graph);
    if (c->nccl) {
        ncclComm_t comm = reinterpret_cast<ncclComm_t>(c->nccl);
        if (nccl_settle(c, ncclCommFinalize(comm), "ncclCommFinalize", c->comm_timeout_s) == 0)
            ncclCommDestroy(comm);
        c->nccl = nullptr;
    }
    auto F = [](void* p) {
        if (p) cudaFree(p);
    };
    F(c->p); F(c->g); F(c->m); F(c->v); F(c->shadow_arena);
    for (auto& a : c->act) {
        F(a.x); F(a.y); F(a.ln1); F(a.mean1); F(a.rstd1); F(a.qkv); F(a.att); F(a.lse);
        F(a.ln2); F(a.mean2); F(a.rstd2); F(a.h); F(a.act);
    }
    F(c->xL); F(c->lnf); F(c->meanf); F(c->rstdf); F(c->logits); F(c->dres); F(c->dy);
    F(c->dln); F(c->dres16); F(c->dy16); F(c->datt); F(c->dqkv); F(c->dh); F(c->dvec);
    F(c->attn_ds);
    for (auto& p2 : c->plan2_cache) gemm_free_plan2(&p2);
    F(c->partial); F(c->colwork); F(c->splitws); F(c->d_tokens); F(c->d_keys);
    F(c->dact); F(c->rope); F(c->emb_rope);
    for (auto& m : c->mact) {
        F(m.proj); F(m.u32); F(m.u16); F(m.xp); F(m.xp16); F(m.raw); F(m.y); F(m.gated);
        F(m.hchk);
    }
    F(c->m_dgated); F(c->m_du); F(c->m_duxp); F(c->m_dpre); F(c->m_dbc);
    F(c->m_da); F(c->m_dd); F(c->m_convpart); F(c->m_segwork); F(c->m_dproj); F(c->m_dxp);
    F(c->m_sgpart);
    for (auto& e : c->moeact) {
        F(e.probs); F(e.idx); F(e.wts); F(e.ssum); F(e.grp); F(e.row_of); F(e.tok_of);
        F(e.xg); F(e.pre); F(e.act); F(e.yg);
    }
    F(c->moe_load); F(c->moe_aux); F(c->e_dyg); F(c->e_dpre); F(c->e_dxg); F(c->e_dscores);
    F(c->e_gpart);
    F(c->d_row_loss); F(c->d_out); F(c->d_hp); F(c->d_normpart); F(c->d_nonfinite); F(c->d_err);
    F(c->d_aparams); F(c->d_chunks); F(c->d_kscale);
    if (c->h_tokens) cudaFreeHost(c->h_tokens);
    if (c->h_out) cudaFreeHost(c->h_out);
    if (c->h_hp) cudaFreeHost(c->h_hp);
    if (c->h_err) cudaFreeHost(c->h_err);
    if (c->ev_keys) cudaEventDestroy(c->ev_keys);
    for (auto& e : c->ev)
        if (e) cudaEventDestroy(e);
    if (c->stream) cudaStreamDestroy(c->stream);
    if (c->side) cudaStreamDestroy(c->side);
    if (c->comm) cudaStreamDestroy(c->comm);
    if (c->ev_grad) cudaEventDestroy(c->ev_grad);
    if (c->ev_comm) cudaEventDestroy(c->ev_comm);
    delete c;
}

// ---------------------------------------------------------------------------- step
namespace {
// Phase timing events. While the step is being captured they are recorded as external
// events so that they also fire at every replay (the external flag is only valid during
// capture).
void mark(Ctx* c, int i) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(c->stream, &st);
    if (st == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(c->ev[i], c->stream, cudaEventRecordExternal);
    else
        cudaEventRecord(c->ev[i], c->stream);
}
}  // namespace

namespace {

MambaDims mamba_dims(const Ctx* c, int B, int T) {
    MambaDims m;
    m.B = B;
    m.T = T;
    m.D = c->mD;
    m.N = c->mN;
    m.R = c->mR;
    m.K = c->mK;
    m.ldp = 2LL * c->mD;
    m.ldx = c->mRPp;
    return m;
}

// MambaBlock::forward (src/mamba.cpp:60-166): norm -> in_proj -> conv+SiLU -> x_proj -> dt ->
// selective scan -> SiLU(z) gate -> out_proj + residual.
int mamba_forward_layer(Ctx* c, int l, int B, int T, float* xnext) {
    const int C = c->C, D = c->mD, BT = B * T;
    const int rms = c->cfg.use_rmsnorm;
    cudaStream_t s = c->stream;
    auto& a = c->act[l];
    auto& m = c->mact[l];
    auto& b = c->blocks[l];
    auto pp = [&](int i) { return c->p + c->params[i].offset; };
    const MambaDims md = mamba_dims(c, B, T);
    int rc;
    // the block's norm has no bias (src/mamba.cpp:67)
    KC(norm_forward(a.x, pp(b.norm_w), nullptr, a.ln1, a.mean1, a.rstd1, BT, C, rms, s));
    if ((rc = gemm(c, a.ln1, C, 0, c->in16[l], C, 0, BT, 2 * D, C,
                   epi_args(kEpiStoreBF16, m.proj, 2 * D))))
        return rc;
    KC(mamba_conv_forward(md, m.proj, pp(b.conv_w), pp(b.conv_b), m.u32, m.u16, s));
    // x_proj: the dt_rank columns feed softplus + a hard clamp whose mask gates the dt
    // gradient (src/mamba.cpp:318-328); a bf16 operand moves dt_raw enough to flip that mask
    // near its edges, so those columns are computed in fp32. B and C use the tensor cores.
    KC(small_gemm_f32(m.u32, D, 1, pp(b.x_proj), 1, D, BT, c->mR, D, kSgSplitRows, c->m_sgpart,
                      m.xp, nullptr, c->mRPp, 0, s));
    if ((rc = gemm(c, m.u16, D, 0, c->xproj16[l] + (size_t)c->mR * D, D, 0, BT, 2 * c->mN, D,
                   epi_args(kEpiStoreF32, m.xp + c->mR, c->mRPp))))
        return rc;
    KC(mamba_dt_forward(md, m.xp, pp(b.dt_proj), m.raw, s));
    KC(mamba_scan_forward(md, m.raw, m.u32, m.xp, pp(b.a_log), pp(b.dskip), m.proj, m.y, m.gated,
                          m.hchk, c->m_segwork, s));
    GemmArgs r = epi_args(kEpiResidF32, xnext, C);
    r.resid = a.x;
    r.ldr = C;
    return gemm(c, m.gated, D, 0, c->out16[l], D, 0, BT, C, D, r);
}

// MambaBlock::backward (src/mamba.cpp:179-413). On entry c->dres/c->dres16 hold the gradient
// of the block output; on exit c->dres holds the gradient of the block input.
int mamba_backward_layer(Ctx* c, int l, int B, int T, int acc) {
    const int C = c->C, D = c->mD, BT = B * T, R = c->mR;
    const int rms = c->cfg.use_rmsnorm;
    cudaStream_t s = c->stream;
    auto& a = c->act[l];
    auto& m = c->mact[l];
    auto& b = c->blocks[l];
    auto pp = [&](int i) { return c->p + c->params[i].offset; };
    auto gp = [&](int i) { return c->g + c->params[i].offset; };
    const MambaDims md = mamba_dims(c, B, T);
    int rc;
    // out = x + gated out_proj^T: dgated = dY out_proj, dout_proj = dY^T gated
    GemmArgs wo = epi_args(kEpiStoreF32, gp(b.out_proj), D);
    wo.accumulate = acc;
    if ((rc = gemm_dual(c,
                        GemmCall{c->dres16, C, 0, c->out16[l], D, 1, BT, D, C,
                                 epi_args(kEpiStoreF32, c->m_dgated, D), 1},
                        GemmCall{c->dres16, C, 1, m.gated, D, 1, C, D, BT, wo,
                                 choose_splits(c, C, D, BT)})))
        return rc;
    // gate + scan backward (dx_z goes straight into dproj[:, 0:D]); the dt gradient comes out
    // through the clamp mask and softplus (src/mamba.cpp:310-329) as draw, fp32
    float* draw = c->m_dpre;
    KC(mamba_scan_backward(md, m.raw, m.u32, m.xp, pp(b.a_log), pp(b.dskip), m.proj, m.y,
                           c->m_dgated, m.hchk, c->m_du, draw, c->m_dproj, c->m_dbc, c->m_da,
                           c->m_dd, c->m_segwork, s));
    const int parts = B * mamba_scan_segments(B, T, D, c->mN);
    KC(mamba_batch_reduce(c->m_da, parts, (long long)D * c->mN, gp(b.a_log), acc, s));
    KC(mamba_batch_reduce(c->m_dd, parts, D, gp(b.dskip), acc, s));
    KC(mamba_reduce_dbc(md, c->m_dbc, c->m_dxp, s));  // dB, dC -> dxp[:, R:R+2N]
    // draw through dt_proj. These two dt_rank-wide contractions are sums with heavy
    // cancellation, so they stay in fp32 (a bf16 operand costs ~5% on the dt_proj gradient).
    // dxp[:, :R] = draw dt_proj  ([BT, D] x [D, R]) -> bf16 columns [0, R) of dxp
    KC(small_gemm_f32(draw, D, 1, pp(b.dt_proj), R, 1, BT, R, D, kSgSplitRows, c->m_sgpart,
                      nullptr, c->m_dxp, c->mRPp, 0, s));
    // ddt_proj = draw^T xp[:, :R]  ([D, BT] x [BT, R], K split)
    KC(small_gemm_f32(draw, 1, D, m.xp, c->mRPp, 1, D, R, BT, kSgSplitCols, c->m_sgpart,
                      gp(b.dt_proj), nullptr, R, acc, s));
    // x_proj (src/mamba.cpp:330-347)
    GemmArgs wx = epi_args(kEpiStoreF32, gp(b.x_proj), D);
    wx.accumulate = acc;
    if ((rc = gemm_dual(c,
                        GemmCall{c->m_dxp, c->mRPp, 0, c->xproj16[l], D, 1, BT, D, c->mRP,
                                 epi_args(kEpiStoreF32, c->m_duxp, D), 1},
                        GemmCall{c->m_dxp, c->mRPp, 1, m.u16, D, 1, c->mRP, D, BT, wx,
                                 choose_splits(c, c->mRP, D, BT)})))
        return rc;
    // SiLU + causal conv backward; dx_ssm into dproj[:, D:2D] (src/mamba.cpp:348-371)
    KC(mamba_conv_backward(md, m.proj, pp(b.conv_w), pp(b.conv_b), c->m_du, c->m_duxp,
                           c->m_convpart, c->m_dproj, gp(b.conv_w), gp(b.conv_b), acc, s));
    // in_proj (src/mamba.cpp:379-396)
    GemmArgs wi = epi_args(kEpiStoreF32, gp(b.in_proj), C);
    wi.accumulate = acc;
    if ((rc = gemm_dual(c,
                        GemmCall{c->m_dproj, 2 * D, 0, c->in16[l], C, 1, BT, C, 2 * D,
                                 epi_args(kEpiStoreF32, c->dln, C), 1},
                        GemmCall{c->m_dproj, 2 * D, 1, a.ln1, C, 1, 2 * D, C, BT, wi,
                                 choose_splits(c, 2 * D, C, BT)})))
        return rc;
    // norm backward + residual (src/mamba.cpp:397-412); updates c->dres in place
    int nparts = 0;
    KC(norm_backward(c->dln, a.x, pp(b.norm_w), a.mean1, a.rstd1, c->dres, c->dres, c->dres16,
                     c->partial, BT, C, rms, &nparts, s, c->d_err));
    KC(reduce_partials(c->partial, nparts, C, gp(b.norm_w), nullptr, nullptr, acc, s));
    return 0;
}

MoeDims moe_dims(const Ctx* c, int B, int T) {
    MoeDims m;
    m.B = B;
    m.T = T;
    m.C = c->C;
    m.E = c->moe_E;
    m.k = c->moe_k;
    m.cap = c->moe_cap;
    return m;
}

// Grouped-GEMM arguments over the expert row blocks of table `grp`.
GemmArgs grouped(GemmArgs a, const int* grp, int E, int mode, long long b_grp_rows,
                 long long out_grp_stride) {
    a.grp = grp;
    a.groups = E;
    a.grp_mode = mode;
    a.b_grp_rows = b_grp_rows;
    a.out_grp_stride = out_grp_stride;
    return a;
}

// MoEFFN::forward (src/moe.cpp:23-62) and aux_loss (:64-75) on the norm output of block l:
// route, dispatch into expert row blocks, expert GEMMs (GELU fused), weighted combine
// + residual into xnext.
int moe_forward_ffn(Ctx* c, int l, int B, int T, float* xnext) {
    const int C = c->C, E = c->moe_E, He = c->moe_He, cap = c->moe_cap;
    const int rms = c->cfg.use_rmsnorm;
    cudaStream_t s = c->stream;
    auto pp = [&](int i) { return c->p + c->params[i].offset; };
    auto& a = c->act[l];
    auto& b = c->blocks[l];
    auto& e = c->moeact[l];
    const MoeDims md = moe_dims(c, B, T);
    KC(moe_router_forward(md, a.y, a.mean2, a.rstd2, pp(b.ln2g), pp(b.ln2b), rms, pp(b.gate),
                          e.probs, e.idx, e.wts, e.ssum, s));
    KC(moe_aux_forward(md, e.probs, c->moe_coef, c->moe_load + (size_t)l * B * E,
                       c->moe_aux + (size_t)l * B, s));
    KC(moe_dispatch(md, e.idx, e.grp, e.row_of, e.tok_of, s));
    KC(moe_gather(md, a.ln2, e.tok_of, e.grp, e.xg, s));
    int rc;
    // h = GELU(xg W1e[g]): W1e[g] is [C, He] (MN-major B), group g from row g*C of the stack
    GemmArgs g1 = grouped(epi_args(kEpiGeluBF16, e.act, He), e.grp, E, kGroupRows, C, 0);
    g1.aux = e.pre;
    g1.ld_aux = He;
    if ((rc = gemm(c, e.xg, C, 0, c->w1e16[l], He, 1, cap, He, C, g1))) return rc;
    // y = h W2e[g]: W2e[g] is [He, C], group g from row g*He
    GemmArgs g2 = grouped(epi_args(kEpiStoreF32, e.yg, C), e.grp, E, kGroupRows, He, 0);
    if ((rc = gemm(c, e.act, He, 0, c->w2e16[l], C, 1, cap, C, He, g2))) return rc;
    KC(moe_combine(md, a.y, e.yg, e.row_of, e.wts, xnext, s));
    return 0;
}

// Backward of moe_forward_ffn: c->dres is the gradient of the block output; writes the
// gradient of the norm output into c->dln and the expert / gate parameter gradients.
int moe_backward_ffn(Ctx* c, int l, int B, int T, int acc) {
    const int C = c->C, E = c->moe_E, He = c->moe_He, cap = c->moe_cap;
    const int rms = c->cfg.use_rmsnorm;
    cudaStream_t s = c->stream;
    auto pp = [&](int i) { return c->p + c->params[i].offset; };
    auto gp = [&](int i) { return c->g + c->params[i].offset; };
    auto& a = c->act[l];
    auto& b = c->blocks[l];
    auto& e = c->moeact[l];
    const MoeDims md = moe_dims(c, B, T);
    // each sequence's loss weighs 1/B in the micro-batch mean (src/trainer.cpp:148-150)
    KC(moe_combine_backward(md, c->dres, e.yg, e.row_of, e.idx, e.wts, e.ssum, e.probs,
                            c->moe_load + (size_t)l * B * E, c->moe_coef, 1.0f / (float)B,
                            c->e_dyg, c->e_dscores, s));
    KC(moe_zero_pad_rows(md, e.grp, c->e_dyg, C, s));
    int rc;
    // dW2e[g] = h_g^T dy_g over the rows of expert g
    GemmArgs w2 = grouped(epi_args(kEpiStoreF32, gp(b.W2e), C), e.grp, E, kGroupK, 0,
                          (long long)He * C);
    w2.accumulate = acc;
    if ((rc = gemm(c, e.act, He, 1, c->e_dyg, C, 1, He, C, cap, w2))) return rc;
    // dpre = (dy W2e[g]^T) * GELU'(pre): W2e[g] read as [N=He, K=C]
    GemmArgs dg = grouped(epi_args(kEpiDGeluBF16, c->e_dpre, He), e.grp, E, kGroupRows, He, 0);
    dg.aux = e.pre;
    dg.ld_aux = He;
    if ((rc = gemm(c, c->e_dyg, C, 0, c->w2e16[l], C, 0, cap, He, C, dg))) return rc;
    // dW1e[g] = xg_g^T dpre_g
    GemmArgs w1 = grouped(epi_args(kEpiStoreF32, gp(b.W1e), He), e.grp, E, kGroupK, 0,
                          (long long)C * He);
    w1.accumulate = acc;
    if ((rc = gemm(c, e.xg, C, 1, c->e_dpre, He, 1, C, He, cap, w1))) return rc;
    // dxg = dpre W1e[g]^T: W1e[g] read as [N=C, K=He]
    GemmArgs dx = grouped(epi_args(kEpiStoreF32, c->e_dxg, C), e.grp, E, kGroupRows, C, 0);
    if ((rc = gemm(c, c->e_dpre, He, 0, c->w1e16[l], He, 0, cap, C, He, dx))) return rc;
    KC(moe_scatter_sum(md, c->e_dxg, e.row_of, c->e_dscores, pp(b.gate), c->dln, s));
    KC(moe_gate_grad(md, a.y, a.mean2, a.rstd2, pp(b.ln2g), pp(b.ln2b), rms, c->e_dscores,
                     c->e_gpart, gp(b.gate), acc, s));
    return 0;
}

}  // namespace

// All-reduce (average over ranks) of gradient floats [begin, end) on the comm stream, after
// everything enqueued so far on the main stream.
int allreduce_bucket(Ctx* c, int64_t begin, int64_t end) {
    if (end <= begin) return 0;
    CK(cudaEventRecord(c->ev_grad, c->stream));
    CK(cudaStreamWaitEvent(c->comm, c->ev_grad, 0));
    if (!c->nccl) {
        c->err = "the communicator was aborted after an earlier failure";
        return LLMGPU_E_NCCL;
    }
    ncclResult_t r = ncclAllReduce(c->g + begin, c->g + begin, (size_t)(end - begin), ncclFloat,
                                   ncclAvg, reinterpret_cast<ncclComm_t>(c->nccl), c->comm);
    if (int rc = nccl_settle(c, r, "ncclAllReduce", c->comm_timeout_s)) return rc;
    c->launches++;
    return 0;
}

int run_fwd_bwd(Ctx* c, int B, int T, int accumulate, bool backward, bool reduce) {
    const int C = c->C, F = c->F, H = c->H, hd = c->hd, L = c->L, V = c->V, Vp = c->Vp;
    const int BT = B * T;
    const int rms = c->cfg.use_rmsnorm;
    const bool tied = c->cfg.weight_tying != 0;
    cudaStream_t s = c->stream;
    float* G = c->g;
    auto gp = [&](int i) { return G + c->params[i].offset; };
    auto pp = [&](int i) { return c->p + c->params[i].offset; };

    mark(c, 0);
    // deterministic token sort for the embedding backward, overlapped on the side stream
    if (backward) {
        CK(cudaEventRecord(c->ev_keys, s));
        CK(cudaStreamWaitEvent(c->side, c->ev_keys, 0));
        const int rc = embed_sort_keys(c->d_tokens, BT, V, c->d_keys, c->side);
        if (rc) {
            c->err = "embed_sort_keys failed with status " + std::to_string(rc);
            if (rc <= -1000)
                c->err += std::string(" (") + cudaGetErrorName((cudaError_t)(-rc - 1000)) + ")";
            return LLMGPU_E_CUDA;
        }
        c->launches++;
        CK(cudaEventRecord(c->ev_keys, c->side));
    }
    // ------------------------------------------------------------------ forward
    KC(embed_forward(c->d_tokens, pp(c->i_wte), pp(c->i_wpe), c->act[0].x, B, T, C, V, s,
                     reinterpret_cast<const float*>(c->emb_rope), c->emb_rope_scale));
    for (int l = 0; l < L; ++l) {
        auto& a = c->act[l];
        auto& b = c->blocks[l];
        float* xnext = (l + 1 < L) ? c->act[l + 1].x : c->xL;
        if (c->mamba) {
            const int rc = mamba_forward_layer(c, l, B, T, xnext);
            if (rc) return rc;
            continue;
        }
        KC(norm_forward(a.x, pp(b.ln1g), pp(b.ln1b), a.ln1, a.mean1, a.rstd1, BT, C, rms, s));
        // RoPE on Q/K at head_dim 64: rotated in the QKV projection's epilogue (before the bf16
        // rounding), so the tcgen05 attention takes q and k as they are
        GemmArgs qa = epi_args(kEpiStoreBF16, a.qkv, 3 * C);
        if (c->rope && hd == 64) {
            qa.rope = c->rope;
            qa.rope_T = T;
            qa.rope_hd = hd;
            qa.rope_cols = 2 * C;
        }
        int rc = gemm(c, a.ln1, C, 0, c->wqkv16[l], 3 * C, 1, BT, 3 * C, C, qa);
        if (rc) return rc;
        if (c->rope && hd == 64) {
            KC(attention_forward(a.qkv, a.att, a.lse, B, T, H, hd, nullptr, s, c->d_err,
                                 c->attn_ds));
        } else {
            KC(attention_forward(a.qkv, a.att, a.lse, B, T, H, hd, c->rope, s, c->d_err,
                                 c->attn_ds));
        }
        GemmArgs r = epi_args(kEpiResidF32, a.y, C);
        r.resid = a.x;
        r.ldr = C;
        if ((rc = gemm(c, a.att, C, 0, c->wo16[l], C, 1, BT, C, C, r))) return rc;
        KC(norm_forward(a.y, pp(b.ln2g), pp(b.ln2b), a.ln2, a.mean2, a.rstd2, BT, C, rms, s));
        if (c->moe) {
            if ((rc = moe_forward_ffn(c, l, B, T, xnext))) return rc;
            continue;
        }
        if (c->swiglu) {  // h13 = ln2 [W1 | W3]; act = silu(h1) * h3 (src/transformer.cpp:22-30)
            if ((rc = gemm(c, a.ln2, C, 0, c->w1_16[l], 2 * F, 1, BT, 2 * F, C,
                           epi_args(kEpiStoreBF16, a.h, 2 * F))))
                return rc;
            KC(swiglu_forward(a.h, a.act, BT, F, s));
        } else {
            GemmArgs ge = epi_args(kEpiGeluBF16, a.act, F);
            ge.aux = a.h;
            ge.ld_aux = F;
            if ((rc = gemm(c, a.ln2, C, 0, c->w1_16[l], F, 1, BT, F, C, ge))) return rc;
        }
        GemmArgs r2 = epi_args(kEpiResidF32, xnext, C);
        r2.resid = a.y;
        r2.ldr = C;
        if ((rc = gemm(c, a.act, F, 0, c->w2_16[l], C, 1, BT, C, F, r2))) return rc;
    }
    KC(norm_forward(c->xL, pp(c->i_lnfg), pp(c->i_lnfb), c->lnf, c->meanf, c->rstdf, BT, C, rms, s));
    {
        int rc;
        if (tied)
            rc = gemm(c, c->lnf, C, 0, c->wte16, C, 0, BT, Vp, C,
                      epi_args(kEpiStoreBF16, c->logits, Vp));
        else
            rc = gemm(c, c->lnf, C, 0, c->lm16, Vp, 1, BT, Vp, C,
                      epi_args(kEpiStoreBF16, c->logits, Vp));
        if (rc) return rc;
    }
    mark(c, 1);
    if (c->logits_only) return 0;  // llmgpu_forward_logits reads them
    // ------------------------------------------------------------------ loss
    KC(cross_entropy_fwd_bwd(c->logits, BT, V, Vp, c->d_tokens, c->d_row_loss,
                             c->loss_scale / (float)BT,
                             c->smoothing, s, c->d_err));
    KC(mean_reduce(c->d_row_loss, BT, c->d_out, s));
    if (c->moe) KC(moe_add_aux(c->moe_aux, L, B, c->d_out, s));
    mark(c, 2);
    if (!backward) return 0;
    // ------------------------------------------------------------------ backward
    int rc;
    const int acc = accumulate;
    // lm head: weight gradient (into wte when tied) and dHidden  (src/model.cpp:248-270)
    if (tied) {
        GemmArgs w = epi_args(kEpiStoreF32, gp(c->i_wte), C);
        w.accumulate = acc;
        if ((rc = gemm_dual(c,
                            GemmCall{c->logits, Vp, 1, c->lnf, C, 1, V, C, BT, w,
                                     choose_splits(c, V, C, BT)},
                            GemmCall{c->logits, Vp, 0, c->wte16, C, 1, BT, C, Vp,
                                     epi_args(kEpiStoreF32, c->dln, C), 1})))
            return rc;
    } else {
        GemmArgs w = epi_args(kEpiStoreF32, gp(c->i_lm), V);
        w.accumulate = acc;
        if ((rc = gemm_dual(c,
                            GemmCall{c->lnf, C, 1, c->logits, Vp, 1, C, V, BT, w,
                                     choose_splits(c, C, V, BT)},
                            GemmCall{c->logits, Vp, 0, c->lm16, Vp, 0, BT, C, Vp,
                                     epi_args(kEpiStoreF32, c->dln, C), 1})))
            return rc;
        if (!acc) CK(cudaMemsetAsync(gp(c->i_wte), 0, sizeof(float) * c->params[c->i_wte].numel, s));
    }
    int nparts = 0;
    KC(norm_backward(c->dln, c->xL, pp(c->i_lnfg), c->meanf, c->rstdf, nullptr, c->dres,
                     c->dres16, c->partial, BT, C, rms, &nparts, s, c->d_err));
    KC(reduce_partials(c->partial, nparts, C, gp(c->i_lnfg), rms ? nullptr : gp(c->i_lnfb),
                       c->blocks[L - 1].b2 >= 0 ? gp(c->blocks[L - 1].b2) : nullptr, acc, s));
    for (int l = L - 1; l >= 0; --l) {
        auto& a = c->act[l];
        auto& b = c->blocks[l];
        if (c->mamba) {
            if ((rc = mamba_backward_layer(c, l, B, T, acc))) return rc;
            if (reduce && (rc = allreduce_bucket(c, c->buckets[l].first, c->buckets[l].second)))
                return rc;
            continue;
        }
        // ---- FFN  (src/transformer.cpp:120-183)
        // Each layer's weight-gradient product runs in one launch with its data-gradient
        // product (both read the same upstream gradient).
        auto dw2 = [&]() {
            GemmArgs w2 = epi_args(kEpiStoreF32, gp(b.W2), C);
            w2.accumulate = acc;
            return GemmCall{a.act, F, 1, c->dres16, C, 1, F, C, BT, w2, choose_splits(c, F, C, BT)};
        };
        if (c->moe) {
            if ((rc = moe_backward_ffn(c, l, B, T, acc))) return rc;
        } else if (c->swiglu) {  // src/transformer.cpp:41-119
            // dgated = dY W2^T, then dh13 = [dh1 | dh3]
            if ((rc = gemm_dual(c, dw2(),
                                GemmCall{c->dres16, C, 0, c->w2_16[l], C, 0, BT, F, C,
                                         epi_args(kEpiStoreBF16, c->dact, F), 1})))
                return rc;
            KC(swiglu_backward(c->dact, a.h, c->dh, BT, F, s));
            // dW1 | dW3 from one GEMM, written into the two parameter gradients
            GemmArgs w13 = epi_args(kEpiStoreF32, gp(b.W1), F);
            w13.accumulate = acc;
            w13.col_group = F;
            w13.group_stride = c->params[b.W3].offset - c->params[b.W1].offset;
            if ((rc = gemm_dual(c,
                                GemmCall{a.ln2, C, 1, c->dh, 2 * F, 1, C, 2 * F, BT, w13,
                                         choose_splits(c, C, 2 * F, BT)},
                                GemmCall{c->dh, 2 * F, 0, c->w1_16[l], 2 * F, 0, BT, C, 2 * F,
                                         epi_args(kEpiStoreF32, c->dln, C), 1})))
                return rc;
            KC(colsum_bf16(c->dh, 2 * F, BT, F, gp(b.b1), acc, c->colwork, s));  // db1 = sum dh1
        } else {
            GemmArgs dg = epi_args(kEpiDGeluBF16, c->dh, F);
            dg.aux = a.h;
            dg.ld_aux = F;
            if ((rc = gemm_dual(c, dw2(),
                                GemmCall{c->dres16, C, 0, c->w2_16[l], C, 0, BT, F, C, dg, 1})))
                return rc;
            GemmArgs w1 = epi_args(kEpiStoreF32, gp(b.W1), F);
            w1.accumulate = acc;
            if ((rc = gemm_dual(c,
                                GemmCall{a.ln2, C, 1, c->dh, F, 1, C, F, BT, w1,
                                         choose_splits(c, C, F, BT)},
                                GemmCall{c->dh, F, 0, c->w1_16[l], F, 0, BT, C, F,
                                         epi_args(kEpiStoreF32, c->dln, C), 1})))
                return rc;
            KC(colsum_bf16(c->dh, F, BT, F, gp(b.b1), acc, c->colwork, s));
        }
        KC(norm_backward(c->dln, a.y, pp(b.ln2g), a.mean2, a.rstd2, c->dres, c->dy, c->dy16,
                         c->partial, BT, C, rms, &nparts, s, c->d_err));
        KC(reduce_partials(c->partial, nparts, C, gp(b.ln2g), rms ? nullptr : gp(b.ln2b), nullptr,
                           acc, s));
        // ---- attention  (src/attention.cpp:183-363)
        GemmArgs wo = epi_args(kEpiStoreF32, gp(b.Wo), C);
        wo.accumulate = acc;
        if ((rc = gemm_dual(c,
                            GemmCall{a.att, C, 1, c->dy16, C, 1, C, C, BT, wo,
                                     choose_splits(c, C, C, BT)},
                            GemmCall{c->dy16, C, 0, c->wo16[l], C, 0, BT, C, C,
                                     epi_args(kEpiStoreBF16, c->datt, C), 1})))
            return rc;
        if (c->rope && hd == 64) {  // q, k were rotated by the projection: dq, dk rotate back
            KC(attention_backward(a.qkv, a.att, c->datt, a.lse, c->dvec, c->dqkv, B, T, H, hd,
                                  nullptr, s, c->d_err, c->attn_ds, c->rope));
        } else {
            KC(attention_backward(a.qkv, a.att, c->datt, a.lse, c->dvec, c->dqkv, B, T, H, hd,
                                  c->rope, s, c->d_err, c->attn_ds));
        }
        GemmArgs wq = epi_args(kEpiStoreF32, gp(b.Wq), C);
        wq.accumulate = acc;
        wq.col_group = C;
        wq.group_stride = c->params[b.Wk].offset - c->params[b.Wq].offset;
        if ((rc = gemm_dual(c,
                            GemmCall{a.ln1, C, 1, c->dqkv, 3 * C, 1, C, 3 * C, BT, wq,
                                     choose_splits(c, C, 3 * C, BT)},
                            GemmCall{c->dqkv, 3 * C, 0, c->wqkv16[l], 3 * C, 0, BT, C, 3 * C,
                                     epi_args(kEpiStoreF32, c->dln, C), 1})))
            return rc;
        KC(norm_backward(c->dln, a.x, pp(b.ln1g), a.mean1, a.rstd1, c->dy, c->dres, c->dres16,
                         c->partial, BT, C, rms, &nparts, s, c->d_err));
        KC(reduce_partials(c->partial, nparts, C, gp(b.ln1g), rms ? nullptr : gp(b.ln1b),
                           (l > 0 && c->blocks[l - 1].b2 >= 0) ? gp(c->blocks[l - 1].b2) : nullptr,
                           acc, s));
        // every gradient of block l is final now (its b2 was reduced in block l+1's pass)
        if (reduce && (rc = allreduce_bucket(c, c->buckets[l].first, c->buckets[l].second)))
            return rc;
    }
    // embedding scatter (src/model.cpp:314-322)
    CK(cudaStreamWaitEvent(s, c->ev_keys, 0));
    // c->dy is free once the last block's backward is done: piece partials go there
    KC(embed_backward(c->d_keys, c->dres, gp(c->i_wte), gp(c->i_wpe), B, T, C, acc, c->dy, s));
    mark(c, 3);
    if (reduce) {
        // the embeddings / ln_f / head range, then hand the comm stream back to the step
        if ((rc = allreduce_bucket(c, c->buckets[L].first, c->buckets[L].second))) return rc;
        CK(cudaEventRecord(c->ev_comm, c->comm));
    }
    return 0;
}

int run_optimizer(Ctx* c, int K) {
    cudaStream_t s = c->stream;
    // Per-step scalars come from pinned host memory (c->h_hp, filled by
    // prepare_step_scalars before the step is launched), so that a captured step graph
    // reads the current values at every replay.
    CK(cudaMemcpyAsync(c->d_hp, c->h_hp, sizeof(float) * 16, cudaMemcpyHostToDevice, s));
    // data parallel: the gradient buckets were all-reduced (averaged) on the comm stream
    // during the last micro-batch's backward
    if (c->world > 1) CK(cudaStreamWaitEvent(s, c->ev_comm, 0));
    if (K > 1 || c->loss_scale != 1.0f) {
        // train_step_accum averages the accumulated gradients (src/trainer.cpp:148-150); a
        // loss scale is divided out before the non-finite check and the clip (:103-105)
        KC(scale_inplace(c->g, c->n_floats, c->d_hp + 8, s));
    }
    mark(c, 4);
    KC(grad_norm_partials(c->g, c->n_floats, c->d_normpart, c->d_nonfinite, grad_norm_blocks(), s));
    KC(grad_norm_finalize(c->d_normpart, grad_norm_blocks(), c->d_nonfinite, c->clip, c->d_out + 1, s));
    KC(adamw_update(c->d_aparams, c->d_chunks, c->nchunks, c->p, c->g, c->m, c->v, c->d_out + 1,
                    c->d_hp, s));
    mark(c, 5);
    return 0;
}

// Host-side scalars of the next optimizer step. The Adam step counter advances only for
// steps that are not skipped: the bias corrections are prepared for t+1 and the caller
// rolls t back if the device reports a skip.
void prepare_step_scalars(Ctx* c, int K) {
    c->adam_t += 1;
    c->h_hp[0] = c->lr;
    c->h_hp[1] = c->b1;
    c->h_hp[2] = c->b2;
    c->h_hp[3] = c->eps;
    c->h_hp[4] = c->wd;
    c->h_hp[5] = (float)(1.0 - std::pow((double)c->b1, (double)c->adam_t));
    c->h_hp[6] = (float)(1.0 - std::pow((double)c->b2, (double)c->adam_t));
    c->h_hp[7] = 1.0f;
    c->h_hp[8] = 1.0f / ((float)(K > 0 ? K : 1) * c->loss_scale);
}

int wait_stream(Ctx* c, cudaStream_t s) {
    if (!c->nccl) {
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e == cudaSuccess) return 0;
        c->err = std::string("stream: ") + cudaGetErrorString(e);
        return LLMGPU_E_CUDA;
    }
    ncclComm_t comm = reinterpret_cast<ncclComm_t>(c->nccl);
    const double deadline = now_s() + c->comm_timeout_s;
    for (;;) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return 0;
        if (e != cudaErrorNotReady) {
            c->err = std::string("stream: ") + cudaGetErrorString(e);
            return LLMGPU_E_CUDA;
        }
        ncclResult_t ar = ncclSuccess;
        ncclCommGetAsyncError(comm, &ar);
        const bool late = now_s() > deadline;
        if ((ar != ncclSuccess && ar != ncclInProgress) || late) {
            c->err = late ? "a collective did not complete within " +
                                std::to_string(c->comm_timeout_s) +
                                " s (a peer rank stopped taking part); communicator aborted"
                          : std::string("collective failed: ") + ncclGetErrorString(ar) +
                                "; communicator aborted";
            abort_comm(c);
            // the aborted communicator's kernels return; wait for the stream a bounded time
            const double drain = now_s() + 30.0;
            while (cudaStreamQuery(s) == cudaErrorNotReady && now_s() < drain)
                std::this_thread::sleep_for(std::chrono::microseconds(200));
            return LLMGPU_E_NCCL;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

int ctx_sync_check(Ctx* c) {
    CK(cudaMemcpyAsync(c->h_err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    if (int rc = wait_stream(c, c->stream)) return rc;
    if (*c->h_err != 0) {
        c->err = "device-side wait timed out (code " + std::to_string(*c->h_err) + ")";
        return LLMGPU_E_DEVICE;
    }
    return 0;
}

// ---------------------------------------------------------------------------- checkpoints
namespace {
bool read_exact(std::ifstream& in, void* p, size_t n) {
    in.read(reinterpret_cast<char*>(p), (std::streamsize)n);
    return (size_t)in.gcount() == n;
}
}  // namespace

// Binary checkpoint v3/v4 (src/model.cpp:568-635), written atomically (tmp + fsync + rename,
// src/model.cpp:558-567).
int save_binary(Ctx* c, const char* path) {
    std::vector<float> host((size_t)c->n_floats);
    if (copy_sync(c, host.data(), c->p, host.size() * sizeof(float), cudaMemcpyDeviceToHost))
        return LLMGPU_E_CUDA;
    const std::string tmp = std::string(path) + ".tmp";
    {
        std::ofstream out(tmp, std::ios::binary);
        if (!out) {
            c->err = "cannot open " + tmp;
            return LLMGPU_E_IO;
        }
        auto& k = c->cfg;
        const uint32_t magic = 0x4C4C4D00u, version = k.use_mamba ? 4 : 3;
        out.write((const char*)&magic, 4);
        out.write((const char*)&version, 4);
        const uint64_t hdr[5] = {(uint64_t)k.vocab_size, (uint64_t)k.n_layers, (uint64_t)k.n_heads,
                                 (uint64_t)k.n_embd, (uint64_t)k.block_size};
        out.write((const char*)hdr, sizeof(hdr));
        auto wt = [&](const std::vector<int64_t>& shape, const float* d, int64_t n) {
            uint64_t nd = shape.size();
            out.write((const char*)&nd, 8);
            for (auto s : shape) {
                uint64_t v = (uint64_t)s;
                out.write((const char*)&v, 8);
            }
            uint64_t nn = (uint64_t)n;
            out.write((const char*)&nn, 8);
            out.write((const char*)d, n * sizeof(float));
        };
        auto wparam = [&](int i) {
            const auto& p = c->params[i];
            wt(p.shape, host.data() + p.offset, p.numel);
        };
        wparam(c->i_wte);
        wparam(c->i_wpe);
        wparam(c->i_lnfg);
        wparam(c->i_lnfb);
        if (c->i_lm >= 0) {
            wparam(c->i_lm);
        } else {  // tied: the reference's lm_head_ holds wte^T (tie_weights, src/model.cpp:931-939)
            const int V = c->V, C = c->C;
            std::vector<float> lm((size_t)C * V);
            const float* w = host.data() + c->params[c->i_wte].offset;
            for (int v = 0; v < V; ++v)
                for (int j = 0; j < C; ++j) lm[(size_t)j * V + v] = w[(size_t)v * C + j];
            wt({C, V}, lm.data(), (int64_t)lm.size());
        }
        if (k.use_mamba) {
            const auto& b = c->blocks[0];
            const uint64_t mh[4] = {(uint64_t)c->params[b.in_proj].shape[0] / 2,
                                    (uint64_t)c->params[b.a_log].shape[1],
                                    (uint64_t)c->params[b.dt_proj].shape[1],
                                    (uint64_t)c->params[b.conv_w].shape[2]};
            out.write((const char*)mh, sizeof(mh));
        }
        const uint64_t nb = (uint64_t)c->L;
        out.write((const char*)&nb, 8);
        const int first_block = c->i_lm >= 0 ? c->i_lm + 1 : c->i_lnfb + 1;
        const int per = (int)((c->params.size() - first_block) / c->L);
        for (int l = 0; l < c->L; ++l) {
            const uint64_t np = (uint64_t)per;
            out.write((const char*)&np, 8);
            for (int j = 0; j < per; ++j) wparam(first_block + l * per + j);
        }
        if (!out) {
            c->err = "write failed: " + tmp;
            return LLMGPU_E_IO;
        }
    }
    int fd = ::open(tmp.c_str(), O_RDONLY);
    if (fd >= 0) {
        ::fsync(fd);
        ::close(fd);
    }
    if (std::rename(tmp.c_str(), path) != 0) {
        c->err = std::string("rename failed: ") + path;
        return LLMGPU_E_IO;
    }
    return 0;
}

// load_binary (src/model.cpp:636-811): header must match the configuration; unlike the
// reference (which prints and keeps random init) a mismatch is reported as an error.
int load_binary(Ctx* c, const char* path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) {
        c->err = std::string("cannot open ") + path;
        return LLMGPU_E_IO;
    }
    uint32_t magic = 0, version = 0;
    uint64_t hdr[5];
    if (!read_exact(in, &magic, 4) || !read_exact(in, &version, 4) || magic != 0x4C4C4D00u ||
        !read_exact(in, hdr, sizeof(hdr))) {
        c->err = "bad checkpoint header";
        return LLMGPU_E_IO;
    }
    auto& k = c->cfg;
    if (hdr[0] != (uint64_t)k.vocab_size || hdr[1] != (uint64_t)k.n_layers ||
        hdr[2] != (uint64_t)k.n_heads || hdr[3] != (uint64_t)k.n_embd ||
        hdr[4] != (uint64_t)k.block_size) {
        c->err = "checkpoint config mismatch";
        return LLMGPU_E_ARG;
    }
    std::vector<float> host((size_t)c->n_floats, 0.0f);
    if (copy_sync(c, host.data(), c->p, host.size() * sizeof(float), cudaMemcpyDeviceToHost))
        return LLMGPU_E_CUDA;
    auto rt = [&](std::vector<int64_t>* shape_out, std::vector<float>* data) -> bool {
        uint64_t nd = 0;
        if (!read_exact(in, &nd, 8) || nd > 8) return false;
        shape_out->resize(nd);
        for (uint64_t i = 0; i < nd; ++i) {
            uint64_t v;
            if (!read_exact(in, &v, 8)) return false;
            (*shape_out)[i] = (int64_t)v;
        }
        uint64_t n = 0;
        if (!read_exact(in, &n, 8)) return false;
        data->resize(n);
        return read_exact(in, data->data(), n * sizeof(float));
    };
    auto into = [&](int i, const std::vector<int64_t>& shape, const std::vector<float>& d) -> bool {
        const auto& p = c->params[i];
        if ((int64_t)d.size() != p.numel) return false;
        (void)shape;
        std::memcpy(host.data() + p.offset, d.data(), d.size() * sizeof(float));
        return true;
    };
    std::vector<int64_t> shp;
    std::vector<float> dat;
    const int top[4] = {c->i_wte, c->i_wpe, c->i_lnfg, c->i_lnfb};
    for (int t = 0; t < 4; ++t)
        if (!rt(&shp, &dat) || !into(top[t], shp, dat)) {
            c->err = "bad tensor in checkpoint";
            return LLMGPU_E_IO;
        }
    if (!rt(&shp, &dat)) {
        c->err = "bad lm_head";
        return LLMGPU_E_IO;
    }
    if (c->i_lm >= 0 && !into(c->i_lm, shp, dat)) {
        c->err = "lm_head size mismatch";
        return LLMGPU_E_IO;
    }
    if (version >= 4) {
        uint64_t mh[4];
        if (!read_exact(in, mh, sizeof(mh))) {
            c->err = "bad v4 header";
            return LLMGPU_E_IO;
        }
    }
    uint64_t nb = 0;
    if (!read_exact(in, &nb, 8) || nb != (uint64_t)c->L) {
        c->err = "block count mismatch";
        return LLMGPU_E_ARG;
    }
    const int first_block = c->i_lm >= 0 ? c->i_lm + 1 : c->i_lnfb + 1;
    const int per = (int)((c->params.size() - first_block) / c->L);
    for (int l = 0; l < c->L; ++l) {
        uint64_t np = 0;
        if (!read_exact(in, &np, 8) || np != (uint64_t)per) {
            c->err = "param count mismatch";
            return LLMGPU_E_ARG;
        }
        for (int j = 0; j < per; ++j)
            if (!rt(&shp, &dat) || !into(first_block + l * per + j, shp, dat)) {
                c->err = "bad block tensor";
                return LLMGPU_E_IO;
            }
    }
    if (copy_sync(c, c->p, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice))
        return LLMGPU_E_CUDA;
    refresh_shadows(c);
    return wait_stream(c, c->stream);
}

// Adam state persistence (src/optimizer.cpp:129-173): magic "ADAM", lr, b1, b2, eps, t,
// then m[] and v[] as shape-prefixed tensors in parameters() order.
int save_adam(Ctx* c, const char* path) {
    std::ofstream os(path, std::ios::binary);
    if (!os) {
        c->err = std::string("cannot open ") + path;
        return LLMGPU_E_IO;
    }
    std::vector<float> m((size_t)c->n_floats), v((size_t)c->n_floats);
    if (copy_sync(c, m.data(), c->m, m.size() * 4, cudaMemcpyDeviceToHost) ||
        copy_sync(c, v.data(), c->v, v.size() * 4, cudaMemcpyDeviceToHost))
        return LLMGPU_E_CUDA;
    const uint32_t magic = 0x4144414Du;
    os.write((const char*)&magic, 4);
    os.write((const char*)&c->lr, 4);
    os.write((const char*)&c->b1, 4);
    os.write((const char*)&c->b2, 4);
    os.write((const char*)&c->eps, 4);
    const int t = c->adam_t;
    os.write((const char*)&t, 4);
    for (int which = 0; which < 2; ++which) {
        const uint64_t n = c->adam_t > 0 ? c->params.size() : 0;  // empty before the first step
        os.write((const char*)&n, 8);
        if (!n) continue;
        const float* src = which == 0 ? m.data() : v.data();
        for (const auto& p : c->params) {
            uint64_t nd = p.shape.size();
            os.write((const char*)&nd, 8);
            for (auto s : p.shape) {
                uint64_t d = (uint64_t)s;
                os.write((const char*)&d, 8);
            }
            uint64_t nn = (uint64_t)p.numel;
            os.write((const char*)&nn, 8);
            os.write((const char*)(src + p.offset), p.numel * 4);
        }
    }
    return os ? 0 : LLMGPU_E_IO;
}

int load_adam(Ctx* c, const char* path) {
    std::ifstream is(path, std::ios::binary);
    if (!is) {
        c->err = std::string("cannot open ") + path;
        return LLMGPU_E_IO;
    }
    uint32_t magic = 0;
    if (!read_exact(is, &magic, 4) || magic != 0x4144414Du) {
        c->err = "bad adam state magic";
        return LLMGPU_E_IO;
    }
    int t = 0;
    if (!read_exact(is, &c->lr, 4) || !read_exact(is, &c->b1, 4) || !read_exact(is, &c->b2, 4) ||
        !read_exact(is, &c->eps, 4) || !read_exact(is, &t, 4)) {
        c->err = "truncated adam state";
        return LLMGPU_E_IO;
    }
    c->adam_t = t;
    std::vector<float> m((size_t)c->n_floats, 0.f), v((size_t)c->n_floats, 0.f);
    for (int which = 0; which < 2; ++which) {
        uint64_t n = 0;
        if (!read_exact(is, &n, 8)) {
            c->err = "truncated adam state";
            return LLMGPU_E_IO;
        }
        if (n != 0 && n != c->params.size()) {
            c->err = "adam state tensor count mismatch";
            return LLMGPU_E_ARG;
        }
        float* dst = which == 0 ? m.data() : v.data();
        for (uint64_t i = 0; i < n; ++i) {
            uint64_t nd = 0;
            if (!read_exact(is, &nd, 8) || nd > 8) return LLMGPU_E_IO;
            for (uint64_t d = 0; d < nd; ++d) {
                uint64_t x;
                if (!read_exact(is, &x, 8)) return LLMGPU_E_IO;
            }
            uint64_t nn = 0;
            if (!read_exact(is, &nn, 8) || (int64_t)nn != c->params[i].numel) return LLMGPU_E_IO;
            if (!read_exact(is, dst + c->params[i].offset, nn * 4)) return LLMGPU_E_IO;
        }
    }
    if (copy_sync(c, c->m, m.data(), m.size() * 4, cudaMemcpyHostToDevice) ||
        copy_sync(c, c->v, v.data(), v.size() * 4, cudaMemcpyHostToDevice))
        return LLMGPU_E_CUDA;
    return 0;
}

}  // namespace llmgpu
