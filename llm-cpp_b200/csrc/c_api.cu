// extern "C" boundary of libllmgpu.so (include/llmgpu.h), in the style of the
// reference's C ABI (src/c_api.cpp:10-72): opaque handle, status codes, no exceptions.
#include <nccl.h>

#include <cstring>
#include <fstream>
#include <new>
#include <sstream>
#include <string>

#include "llmgpu.h"
#include "model.h"

using namespace llmgpu;

struct llmgpu_ctx {
    Ctx* c;
};

namespace {
thread_local std::string g_create_error;

int check_ctx(const llmgpu_ctx* h) { return (h && h->c) ? 0 : LLMGPU_E_ARG; }

int stage_tokens(Ctx* c, const int32_t* tokens, int B, int T) {
    const size_t n = (size_t)B * T;
    std::memcpy(c->h_tokens, tokens, n * sizeof(int32_t));
    if (cudaMemcpyAsync(c->d_tokens, c->h_tokens, n * sizeof(int32_t), cudaMemcpyHostToDevice,
                        c->stream) != cudaSuccess) {
        c->err = "token upload failed";
        return LLMGPU_E_CUDA;
    }
    return 0;
}

// Forgets the captured step, so that the next step is captured again with the current
// kernel arguments.
void drop_graph(Ctx* c) {
    if (c->graph) {
        cudaGraphExecDestroy(c->graph);
        c->graph = nullptr;
    }
    c->graph_B = -1;
}

int validate_bt(Ctx* c, int B, int T) {
    if (B <= 0 || T <= 0 || B > c->max_b || T > c->max_t || (long long)B * T > c->max_bt) {
        c->err = "B x T outside the context's capacity";
        return LLMGPU_E_ARG;
    }
    if (T != c->last_T) {
        // rows >= T of the position-embedding gradient are never written by a step of
        // length T; clear them when T changes so no stale gradient survives
        const auto& p = c->params[c->i_wpe];
        cudaMemsetAsync(c->g + p.offset, 0, sizeof(float) * p.numel, c->stream);
        c->last_T = T;
    }
    c->last_B = B;
    return 0;
}

int enqueue_step(Ctx* c, int B, int T, int accumulate, bool do_step, int K) {
    if (c->comm_failed) {
        c->err = "the communicator was aborted (a collective failed or a peer is gone)";
        return LLMGPU_E_NCCL;
    }
    c->plan_cursor = 0;
    c->plan2_cursor = 0;
    c->prof_n = 0;
    int rc = run_fwd_bwd(c, B, T, accumulate, true, do_step && c->world > 1);
    if (rc) return rc;
    if (do_step) rc = run_optimizer(c, K);
    return rc;
}

// Captures the step for (B, T, accumulate, do_step, K) as a CUDA graph. The graph reads
// the tokens from c->d_tokens and its per-step scalars from pinned host memory, so a
// replay needs no host work besides the launch. On any capture problem the context falls
// back to eager execution for good.
void capture_step(Ctx* c, int B, int T, int accumulate, bool do_step, int K) {
    if (c->graph) {
        cudaGraphExecDestroy(c->graph);
        c->graph = nullptr;
    }
    const int saved = c->launches;
    c->launches = 0;
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        c->use_graph = false;
        c->launches = saved;
        return;
    }
    const int rc = enqueue_step(c, B, T, accumulate, do_step, K);
    const cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (rc != 0 || e != cudaSuccess || !g ||
        cudaGraphInstantiate(&c->graph, g, 0) != cudaSuccess) {
        c->graph = nullptr;
        c->use_graph = false;
        cudaGetLastError();
    } else {
        c->graph_B = B;
        c->graph_T = T;
        c->graph_acc = accumulate;
        c->graph_mode = do_step ? 1 : 0;
        c->graph_K = K;
        c->graph_launches = c->launches;
    }
    if (g) cudaGraphDestroy(g);
    c->launches = saved;
}

// Runs one micro-batch (+ optimizer when `do_step`), eagerly or through the step graph.
int run_step(Ctx* c, int B, int T, int accumulate, bool do_step, int K) {
    if (c->comm_failed) {  // a captured step would replay collectives of the aborted communicator
        c->err = "the communicator was aborted (a collective failed or a peer is gone)";
        return LLMGPU_E_NCCL;
    }
    cudaMemsetAsync(c->d_out + 1, 0, sizeof(float) * 4, c->stream);
    if (do_step) prepare_step_scalars(c, K);
    const bool graphable = c->use_graph && !c->profile;
    const bool hit = graphable && c->graph && c->graph_B == B && c->graph_T == T &&
                     c->graph_acc == accumulate && c->graph_mode == (do_step ? 1 : 0) &&
                     c->graph_K == K;
    int rc = 0;
    if (hit) {
        if (cudaGraphLaunch(c->graph, c->stream) != cudaSuccess) {
            c->err = "cudaGraphLaunch failed";
            return LLMGPU_E_CUDA;
        }
        c->launches = c->graph_launches;
    } else {
        c->launches = 0;
        rc = enqueue_step(c, B, T, accumulate, do_step, K);
        if (rc) return rc;
        if (graphable) capture_step(c, B, T, accumulate, do_step, K);
    }
    if (cudaMemcpyAsync(c->h_out, c->d_out, sizeof(float) * 8, cudaMemcpyDeviceToHost,
                        c->stream) != cudaSuccess)
        return LLMGPU_E_CUDA;
    rc = ctx_sync_check(c);
    if (rc) return rc;
    cudaEventElapsedTime(&c->timings[0], c->ev[0], c->ev[1]);
    cudaEventElapsedTime(&c->timings[1], c->ev[1], c->ev[2]);
    cudaEventElapsedTime(&c->timings[2], c->ev[2], c->ev[3]);
    if (do_step) {
        cudaEventElapsedTime(&c->timings[3], c->ev[3], c->ev[4]);
        cudaEventElapsedTime(&c->timings[4], c->ev[4], c->ev[5]);
        cudaEventElapsedTime(&c->timings[5], c->ev[0], c->ev[5]);
    } else {
        c->timings[3] = c->timings[4] = 0.f;
        cudaEventElapsedTime(&c->timings[5], c->ev[0], c->ev[3]);
    }
    if (c->profile) {
        c->prof_last_ms.assign(c->prof_n, 0.f);
        for (size_t i = 0; i < c->prof_n; ++i) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, c->prof_ev[2 * i], c->prof_ev[2 * i + 1]);
            c->prof_last_ms[i] = ms;
            c->prof_total_ms += ms;
            c->prof_total_flops += c->prof_flops[i];
        }
        c->prof_launches += (int)c->prof_n;
    }
    c->last_loss = c->h_out[0];
    if (do_step) {
        if (c->h_out[4] != 0.0f) {  // non-finite gradient: step skipped (src/trainer.cpp:151-156)
            c->adam_t -= 1;
            c->skipped += 1;
            return LLMGPU_SKIPPED;
        }
        c->last_gnorm = c->h_out[3];
        // the bf16 shadows were rewritten by the AdamW pass
    }
    return 0;
}
}  // namespace

extern "C" {

void llmgpu_config_default(llmgpu_config* cfg) {
    if (!cfg) return;
    std::memset(cfg, 0, sizeof(*cfg));
    cfg->vocab_size = 50257;  // include/llm/model.h:18-22
    cfg->n_layers = 12;
    cfg->n_heads = 12;
    cfg->n_embd = 768;
    cfg->block_size = 1024;
    cfg->weight_tying = 1;
    cfg->d_state = 16;
    cfg->conv_kernel = 4;
    cfg->rope_theta = 10000.0f;
    cfg->moe_top_k = 2;
    cfg->moe_aux_coef = 0.01f;
    cfg->pos_encoding = LLMGPU_POS_LEARNED;
    cfg->rope_scaling = 1.0f;
    cfg->rope_mode = 0;
    cfg->yarn_alpha = 1.0f;
    cfg->yarn_beta = 32.0f;
}

int llmgpu_get_unique_id(void* uid128) {
    if (!uid128) return LLMGPU_E_ARG;
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return LLMGPU_E_NCCL;
    std::memcpy(uid128, &id, sizeof(id));
    return 0;
}

llmgpu_ctx* llmgpu_create(const llmgpu_config* cfg, int max_batch, int max_seq, int rank,
                          int world, const void* uid128) {
    if (!cfg || world < 1 || rank < 0 || rank >= world || (world > 1 && !uid128)) {
        g_create_error = "invalid arguments";
        return nullptr;
    }
    std::string err;
    Ctx* c = ctx_create(*cfg, max_batch, max_seq, rank, world, uid128, &err);
    if (!c) {
        g_create_error = err;
        return nullptr;
    }
    auto* h = new (std::nothrow) llmgpu_ctx{c};
    if (!h) {
        ctx_destroy(c);
        g_create_error = "out of host memory";
    }
    return h;
}

int llmgpu_destroy(llmgpu_ctx* h) {
    if (!h) return LLMGPU_E_ARG;
    ctx_destroy(h->c);
    delete h;
    return 0;
}

const char* llmgpu_last_error(const llmgpu_ctx* h) {
    if (!h || !h->c) return g_create_error.c_str();
    return h->c->err.c_str();
}

int llmgpu_set_adamw(llmgpu_ctx* h, float lr, float b1, float b2, float eps, float wd) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    c->lr = lr;
    c->b1 = b1;
    c->b2 = b2;
    c->eps = eps;
    c->wd = wd;
    return 0;
}

int llmgpu_set_lr(llmgpu_ctx* h, float lr) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    h->c->lr = lr;
    return 0;
}

int llmgpu_set_train(llmgpu_ctx* h, float grad_clip, int grad_accum_steps, float label_smoothing) {
    if (check_ctx(h) || grad_accum_steps < 1) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    // the clip and the smoothing are arguments of kernels inside the captured step
    if (grad_clip != c->clip || label_smoothing != c->smoothing) drop_graph(c);
    c->clip = grad_clip;
    c->accum_k = grad_accum_steps;
    c->accum_count = 0;
    c->smoothing = label_smoothing;
    return 0;
}

int llmgpu_set_loss_scale(llmgpu_ctx* h, float scale) {
    if (check_ctx(h) || !(scale > 0.0f)) return LLMGPU_E_ARG;
    if (scale != h->c->loss_scale) drop_graph(h->c);
    h->c->loss_scale = scale;
    return 0;
}

int llmgpu_train_step(llmgpu_ctx* h, const int32_t* tokens, int B, int T, float* loss_out,
                      float* grad_norm_out) {
    if (check_ctx(h) || !tokens) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    int rc = validate_bt(c, B, T);
    if (rc) return rc;
    if ((rc = stage_tokens(c, tokens, B, T))) return rc;
    rc = run_step(c, B, T, 0, true, 1);
    if (rc < 0) return rc;
    if (loss_out) *loss_out = c->last_loss;
    if (grad_norm_out) *grad_norm_out = c->last_gnorm;
    return rc;
}

int llmgpu_train_step_device(llmgpu_ctx* h, const int32_t* d_tokens, int B, int T,
                             float* loss_out, float* grad_norm_out) {
    if (check_ctx(h) || !d_tokens) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    int rc = validate_bt(c, B, T);
    if (rc) return rc;
    if (cudaMemcpyAsync(c->d_tokens, d_tokens, sizeof(int32_t) * B * T, cudaMemcpyDeviceToDevice,
                        c->stream) != cudaSuccess)
        return LLMGPU_E_CUDA;
    rc = run_step(c, B, T, 0, true, 1);
    if (rc < 0) return rc;
    if (loss_out) *loss_out = c->last_loss;
    if (grad_norm_out) *grad_norm_out = c->last_gnorm;
    return rc;
}

int llmgpu_train_step_accum(llmgpu_ctx* h, const int32_t* tokens, int B, int T, float* loss_out,
                            int* stepped_out) {
    if (check_ctx(h) || !tokens) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    int rc = validate_bt(c, B, T);
    if (rc) return rc;
    if ((rc = stage_tokens(c, tokens, B, T))) return rc;
    const bool step = (c->accum_count + 1 >= c->accum_k);
    rc = run_step(c, B, T, c->accum_count > 0 ? 1 : 0, step, c->accum_k);
    c->accum_count = step ? 0 : c->accum_count + 1;
    if (rc < 0) return rc;
    if (loss_out) *loss_out = c->last_loss;
    if (stepped_out) *stepped_out = (step && rc == 0) ? 1 : 0;
    return rc;
}

int llmgpu_eval_loss(llmgpu_ctx* h, const int32_t* tokens, int B, int T, float* loss_out) {
    if (check_ctx(h) || !tokens) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    if (B <= 0 || T <= 0 || (long long)B * T > c->max_bt || T > c->max_t) return LLMGPU_E_ARG;
    int rc = stage_tokens(c, tokens, B, T);
    if (rc) return rc;
    c->plan_cursor = 0;
    c->plan2_cursor = 0;
    c->launches = 0;
    if ((rc = run_fwd_bwd(c, B, T, 0, false))) return rc;
    if (cudaMemcpyAsync(c->h_out, c->d_out, sizeof(float), cudaMemcpyDeviceToHost, c->stream) !=
        cudaSuccess)
        return LLMGPU_E_CUDA;
    if ((rc = ctx_sync_check(c))) return rc;
    if (loss_out) *loss_out = c->h_out[0];
    return 0;
}

// Forward up to the lm head, then rows of the bf16 logits to host floats: the last position
// of each sequence (all_rows false) or every position.
static int64_t forward_rows(llmgpu_ctx* h, const int32_t* tokens, int B, int T, float* logits,
                            int64_t cap, bool all_rows) {
    if (check_ctx(h) || !tokens || !logits) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    if (B <= 0 || T <= 0 || (long long)B * T > c->max_bt || T > c->max_t) return LLMGPU_E_ARG;
    const int64_t nrows = all_rows ? (int64_t)B * T : B;
    if (cap < nrows * c->V) return LLMGPU_E_ARG;
    int rc = stage_tokens(c, tokens, B, T);
    if (rc) return rc;
    c->plan_cursor = 0;
    c->plan2_cursor = 0;
    c->launches = 0;
    c->logits_only = true;  // stop after the lm head: the fused loss would overwrite the logits
    rc = run_fwd_bwd(c, B, T, 0, false);
    c->logits_only = false;
    if (rc) return rc;
    // row T-1 of each sequence (B rows T * Vp apart), or all B*T rows (Vp apart)
    std::vector<uint16_t> rows((size_t)nrows * c->V);
    const bf16* src = all_rows ? c->logits : c->logits + (size_t)(T - 1) * c->Vp;
    const size_t pitch = (all_rows ? (size_t)1 : (size_t)T) * c->Vp * 2;
    if (cudaMemcpy2DAsync(rows.data(), (size_t)c->V * 2, src, pitch, (size_t)c->V * 2,
                          (size_t)nrows, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return LLMGPU_E_CUDA;
    if ((rc = ctx_sync_check(c))) return rc;
    for (size_t i = 0; i < rows.size(); ++i) {
        const uint32_t bits = (uint32_t)rows[i] << 16;
        std::memcpy(&logits[i], &bits, sizeof(float));
    }
    return nrows * c->V;
}

int64_t llmgpu_forward_logits(llmgpu_ctx* h, const int32_t* tokens, int B, int T, float* logits,
                              int64_t cap) {
    return forward_rows(h, tokens, B, T, logits, cap, false);
}

int64_t llmgpu_forward_logits_all(llmgpu_ctx* h, const int32_t* tokens, int B, int T,
                                  float* logits, int64_t cap) {
    return forward_rows(h, tokens, B, T, logits, cap, true);
}

static int decode_check(llmgpu_ctx* h, int B) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    std::string why;
    if (int rc = decode_supported(c, &why)) {
        c->err = why;
        return rc;
    }
    if (B < 1 || B > c->max_b || B > 8) {
        c->err = "decode: B must be in [1, min(max_batch, 8)]";
        return LLMGPU_E_ARG;
    }
    return decode_alloc(c);
}

int llmgpu_decode_reset(llmgpu_ctx* h, int B) {
    if (int rc = decode_check(h, B)) return rc;
    h->c->dec.B = B;
    h->c->dec.pos = 0;
    return 0;
}

int64_t llmgpu_decode_prefill(llmgpu_ctx* h, const int32_t* tokens, int B, int T, float* logits,
                              int64_t cap) {
    if (int rc = decode_check(h, B)) return rc;
    Ctx* c = h->c;
    const int64_t n = forward_rows(h, tokens, B, T, logits, cap, false);
    if (n < 0) return n;
    if (int rc = decode_fill(c, B, T)) return rc;
    if (int rc = ctx_sync_check(c)) return rc;
    return n;
}

int64_t llmgpu_decode_step(llmgpu_ctx* h, const int32_t* tokens, int B, float* logits,
                           int64_t cap) {
    if (check_ctx(h) || !tokens || !logits) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    if (!c->dec.ready || B != c->dec.B) {
        c->err = "decode: call llmgpu_decode_prefill or llmgpu_decode_reset with this B first";
        return LLMGPU_E_ARG;
    }
    if (cap < (int64_t)B * c->V) return LLMGPU_E_ARG;
    std::memcpy(c->h_tokens, tokens, sizeof(int32_t) * B);
    if (cudaMemcpyAsync(c->dec.tokens, c->h_tokens, sizeof(int32_t) * B, cudaMemcpyHostToDevice,
                        c->stream) != cudaSuccess)
        return LLMGPU_E_CUDA;
    if (int rc = decode_step(c, B)) return rc;
    if (cudaMemcpy2DAsync(logits, (size_t)c->V * 4, c->dec.logits, (size_t)c->Vp * 4,
                          (size_t)c->V * 4, (size_t)B, cudaMemcpyDeviceToHost, c->stream) !=
        cudaSuccess)
        return LLMGPU_E_CUDA;
    if (int rc = ctx_sync_check(c)) return rc;
    return (int64_t)B * c->V;
}

int llmgpu_decode_position(const llmgpu_ctx* h) {
    return check_ctx(h) ? LLMGPU_E_ARG : (h->c->dec.ready ? h->c->dec.pos : 0);
}

int llmgpu_num_params(const llmgpu_ctx* h) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    return (int)h->c->params.size();
}

size_t llmgpu_num_parameters(const llmgpu_ctx* h) {
    if (check_ctx(h)) return 0;
    size_t n = 0;
    for (const auto& p : h->c->params) n += (size_t)p.numel;
    return n;
}

int llmgpu_param_info(const llmgpu_ctx* h, int idx, char* name, int name_cap, int64_t* shape) {
    if (check_ctx(h) || idx < 0 || idx >= (int)h->c->params.size()) return LLMGPU_E_ARG;
    const auto& p = h->c->params[idx];
    if (name && name_cap > 0) {
        std::strncpy(name, p.name.c_str(), (size_t)name_cap - 1);
        name[name_cap - 1] = 0;
    }
    if (shape)
        for (size_t i = 0; i < p.shape.size() && i < 4; ++i) shape[i] = p.shape[i];
    return (int)p.shape.size();
}

static int64_t copy_out(llmgpu_ctx* h, int idx, const float* base, float* out, int64_t cap) {
    if (check_ctx(h) || idx < 0 || idx >= (int)h->c->params.size()) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    const auto& p = c->params[idx];
    if (!out || cap <= 0) return p.numel;
    const int64_t n = cap < p.numel ? cap : p.numel;
    if (copy_sync(c, out, base + p.offset, n * sizeof(float), cudaMemcpyDeviceToHost))
        return LLMGPU_E_CUDA;
    return n;
}

int64_t llmgpu_get_param(llmgpu_ctx* h, int idx, float* out, int64_t cap) {
    return check_ctx(h) ? LLMGPU_E_ARG : copy_out(h, idx, h->c->p, out, cap);
}

int64_t llmgpu_get_grad(llmgpu_ctx* h, int idx, float* out, int64_t cap) {
    return check_ctx(h) ? LLMGPU_E_ARG : copy_out(h, idx, h->c->g, out, cap);
}

int64_t llmgpu_get_adam_state(llmgpu_ctx* h, int idx, float* m_out, float* v_out, int64_t cap) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    int64_t r = copy_out(h, idx, h->c->m, m_out, cap);
    if (r < 0) return r;
    return copy_out(h, idx, h->c->v, v_out, cap);
}

int llmgpu_set_param(llmgpu_ctx* h, int idx, const float* data, int64_t n) {
    if (check_ctx(h) || !data || idx < 0 || idx >= (int)h->c->params.size()) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    const auto& p = c->params[idx];
    if (n != p.numel) return LLMGPU_E_ARG;
    if (copy_sync(c, c->p + p.offset, data, n * sizeof(float), cudaMemcpyHostToDevice))
        return LLMGPU_E_CUDA;
    refresh_shadows(c);
    return wait_stream(c, c->stream);
}

int llmgpu_save_binary(llmgpu_ctx* h, const char* path) {
    if (check_ctx(h) || !path) return LLMGPU_E_ARG;
    return save_binary(h->c, path);
}

int llmgpu_load_binary(llmgpu_ctx* h, const char* path) {
    if (check_ctx(h) || !path) return LLMGPU_E_ARG;
    return load_binary(h->c, path);
}

// Trainer::save_train_state / load_train_state (src/trainer.cpp:194-227)
int llmgpu_save_train_state(llmgpu_ctx* h, const char* prefix) {
    if (check_ctx(h) || !prefix) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    const std::string pre(prefix);
    int rc = save_binary(c, (pre + ".model.bin").c_str());
    if (rc) return rc;
    if ((rc = save_adam(c, (pre + ".opt.bin").c_str()))) return rc;
    std::ofstream js(pre + ".json");
    js << "{\"step\":" << c->step_count << ",\"skipped\":" << c->skipped << ",\"seed\":" << 42
       << "}\n";
    return js ? 0 : LLMGPU_E_IO;
}

int llmgpu_load_train_state(llmgpu_ctx* h, const char* prefix) {
    if (check_ctx(h) || !prefix) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    const std::string pre(prefix);
    int rc = load_binary(c, (pre + ".model.bin").c_str());
    if (rc) return rc;
    {
        std::ifstream probe(pre + ".opt.bin", std::ios::binary);
        if (probe && (rc = load_adam(c, (pre + ".opt.bin").c_str()))) return rc;
    }
    std::ifstream js(pre + ".json");
    if (js) {
        std::stringstream ss;
        ss << js.rdbuf();
        const std::string s = ss.str();
        auto num = [&](const char* k) {
            auto p = s.find(k);
            if (p == std::string::npos) return 0;
            return std::atoi(s.substr(s.find(':', p) + 1).c_str());
        };
        c->step_count = num("\"step\"");
        c->skipped = num("\"skipped\"");
    }
    return 0;
}

int llmgpu_step(const llmgpu_ctx* h) { return check_ctx(h) ? LLMGPU_E_ARG : h->c->step_count; }
int llmgpu_set_step(llmgpu_ctx* h, int step) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    h->c->step_count = step;
    return 0;
}
int llmgpu_skipped_steps(const llmgpu_ctx* h) { return check_ctx(h) ? LLMGPU_E_ARG : h->c->skipped; }
float llmgpu_last_loss(const llmgpu_ctx* h) { return check_ctx(h) ? 0.f : h->c->last_loss; }
float llmgpu_last_grad_norm(const llmgpu_ctx* h) { return check_ctx(h) ? 0.f : h->c->last_gnorm; }

int llmgpu_last_timings(const llmgpu_ctx* h, float* ms6) {
    if (check_ctx(h) || !ms6) return LLMGPU_E_ARG;
    std::memcpy(ms6, h->c->timings, sizeof(float) * 6);
    return 0;
}

int llmgpu_last_launches(const llmgpu_ctx* h) { return check_ctx(h) ? LLMGPU_E_ARG : h->c->launches; }

int llmgpu_set_comm_timeout(llmgpu_ctx* h, double seconds) {
    if (check_ctx(h) || !(seconds > 0.0)) return LLMGPU_E_ARG;
    h->c->comm_timeout_s = seconds;
    return 0;
}

int llmgpu_abort_comm(llmgpu_ctx* h) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    if (!c->nccl) return 0;
    int rc = wait_stream(c, c->stream);  // aborts by itself if the wait runs out
    if (rc == 0 && c->comm) rc = wait_stream(c, c->comm);
    if (c->nccl) {
        // Nothing of this rank is in flight, so no kernel needs the communicator's abort to
        // return; its teardown would talk to the peer that is gone (on 2 x B200 the abort did
        // not return within minutes). The context lets go of it; the process's exit frees it.
        c->nccl = nullptr;
        c->comm_failed = true;
        c->err = "communicator released on request (a peer rank is gone)";
    }
    return rc ? LLMGPU_E_NCCL : 0;
}

int llmgpu_set_graph(llmgpu_ctx* h, int enable) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    h->c->use_graph = enable != 0;
    return 0;
}

void* llmgpu_stream(const llmgpu_ctx* h) { return check_ctx(h) ? nullptr : (void*)h->c->stream; }

int llmgpu_set_profile(llmgpu_ctx* h, int enable) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    h->c->profile = enable != 0;
    return 0;
}

int llmgpu_gemm_stats(llmgpu_ctx* h, double* flops, double* ms, int* launches, int reset) {
    if (check_ctx(h)) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    if (flops) *flops = c->prof_total_flops;
    if (ms) *ms = c->prof_total_ms;
    if (launches) *launches = c->prof_launches;
    if (reset) {
        c->prof_total_flops = c->prof_total_ms = 0;
        c->prof_launches = 0;
    }
    return 0;
}

int llmgpu_gemm_last_step(llmgpu_ctx* h, int32_t* shapes, float* ms, int cap) {
    if (check_ctx(h) || cap < 0) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    const int n = (int)c->prof_last_ms.size();
    for (int i = 0; i < n && i < cap; ++i) {
        if (shapes)
            for (int j = 0; j < 6; ++j) shapes[6 * i + j] = c->prof_shape[6 * i + j];
        if (ms) ms[i] = c->prof_last_ms[i];
    }
    return n;
}

int64_t llmgpu_moe_routing(llmgpu_ctx* h, int layer, int32_t* idx, int64_t n) {
    if (check_ctx(h) || !idx) return LLMGPU_E_ARG;
    Ctx* c = h->c;
    if (!c->moe) return LLMGPU_E_UNSUPPORTED;
    if (layer < 0 || layer >= c->L || c->last_B <= 0) return LLMGPU_E_ARG;
    const int64_t total = (int64_t)c->last_B * c->last_T * c->moe_k;
    if (n < total) return LLMGPU_E_ARG;
    if (copy_sync(c, idx, c->moeact[layer].idx, sizeof(int32_t) * total, cudaMemcpyDeviceToHost))
        return LLMGPU_E_CUDA;
    return total;
}

}  // extern "C"
