// Device-resident GPT training context behind the C ABI (include/llmgpu.h).
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"
#include "llmgpu.h"

namespace llmgpu {

struct Param {
    std::string name;
    std::vector<int64_t> shape;
    int64_t offset = 0;  // floats, into the arena
    int64_t numel = 0;
    int decay = 0;
    bf16* shadow = nullptr;
    int64_t shadow_ld = 0;
    int cols = 1;
};

// Indices into Ctx::params of one transformer / Mamba block.
struct BlockIdx {
    int Wq = -1, Wk = -1, Wv = -1, Wo = -1, W1 = -1, W2 = -1, W3 = -1, b1 = -1, b2 = -1;
    int ln1g = -1, ln1b = -1, ln2g = -1, ln2b = -1;
    int gate = -1, W1e = -1, W2e = -1;  // MoE
    // Mamba
    int norm_w = -1, in_proj = -1, conv_w = -1, conv_b = -1, x_proj = -1, dt_proj = -1,
        a_log = -1, dskip = -1, out_proj = -1;
};

// Activations kept from the forward for the backward, per block.
struct BlockAct {
    float* x = nullptr;      // block input, fp32 [BT, C]
    float* y = nullptr;      // after attention residual, fp32 [BT, C]
    bf16* ln1 = nullptr;     // [BT, C]
    float* mean1 = nullptr;
    float* rstd1 = nullptr;
    bf16* qkv = nullptr;     // [BT, 3C]
    bf16* att = nullptr;     // [BT, C]
    float* lse = nullptr;    // [B, H, T]
    bf16* ln2 = nullptr;
    float* mean2 = nullptr;
    float* rstd2 = nullptr;
    bf16* h = nullptr;       // FFN pre-activation [BT, F] (GELU) or [BT, 2F] (h1|h3, SwiGLU)
    bf16* act = nullptr;     // FFN activation [BT, F]
};

// Mamba block activations kept for the backward (mamba.cuh has the layouts).
struct MambaAct {
    bf16* proj = nullptr;    // [BT, 2D]  x_z | x_ssm
    float* u32 = nullptr;    // [BT, D]
    bf16* u16 = nullptr;     // [BT, D]
    float* xp = nullptr;     // [BT, RPp] dt_in | B | C (fp32)
    bf16* xp16 = nullptr;    // [BT, RPp]
    float* raw = nullptr;    // [BT, D]   dt before softplus/clamp
    float* y = nullptr;      // [BT, D]
    bf16* gated = nullptr;   // [BT, D]
    float* hchk = nullptr;   // saved scan states
};

// MoE FFN activations kept for the backward, per block (moe.cuh has the layouts).
struct MoeAct {
    float* probs = nullptr;  // [BT, E]
    int* idx = nullptr;      // [BT, k]
    float* wts = nullptr;    // [BT, k]
    float* ssum = nullptr;   // [BT]
    int* grp = nullptr;      // [2E+1] expert row offsets and counts
    int* row_of = nullptr;   // [BT, k]
    int* tok_of = nullptr;   // [cap]
    bf16* xg = nullptr;      // [cap, C]  gathered norm output
    bf16* pre = nullptr;     // [cap, He] expert pre-activation
    bf16* act = nullptr;     // [cap, He] GELU(pre)
    float* yg = nullptr;     // [cap, C]  expert outputs
};

// KV-cached decoding (decode.cu): per layer K and V caches [max_b][max_t][C] bf16 and the
// one-row activations of a decode step, allocated at the first decode call.
struct DecodeState {
    bool ready = false;
    int max_b = 0, B = 0, pos = 0;
    std::vector<bf16*> kc, vc;
    float *x = nullptr, *y = nullptr, *stat = nullptr, *logits = nullptr;
    bf16 *ln = nullptr, *qkv = nullptr, *att = nullptr, *act = nullptr;
    int32_t* tokens = nullptr;
};

struct Ctx {
    llmgpu_config cfg{};
    int rank = 0, world = 1;
    int device = 0, num_sms = 148;
    int max_bt = 0, max_b = 0, max_t = 0;
    int C = 0, V = 0, Vp = 0, H = 0, hd = 0, F = 0, L = 0;
    cudaStream_t stream = nullptr, side = nullptr;
    cudaEvent_t ev_keys = nullptr;
    // data parallel: gradient buckets (one per block, then the embeddings/head range) are
    // all-reduced on `comm` as soon as the backward has finished them
    cudaStream_t comm = nullptr;
    cudaEvent_t ev_grad = nullptr, ev_comm = nullptr;
    std::vector<std::pair<int64_t, int64_t>> buckets;  // [begin, end) floats; index l = block l
    cudaEvent_t ev[6] = {};
    void* nccl = nullptr;  // ncclComm_t, created non-blocking
    // host-side bound on any wait for a collective (a peer that stopped, a lost link): past
    // it the communicator is aborted and the call returns LLMGPU_E_NCCL; the context is then
    // unusable for steps (comm_failed)
    double comm_timeout_s = 600.0;
    bool comm_failed = false;

    std::vector<Param> params;
    std::vector<BlockIdx> blocks;
    int i_wte = -1, i_wpe = -1, i_lnfg = -1, i_lnfb = -1, i_lm = -1;
    int64_t n_floats = 0;
    float *p = nullptr, *g = nullptr, *m = nullptr, *v = nullptr;
    bf16* shadow_arena = nullptr;
    size_t shadow_elems = 0;
    bf16* wte16 = nullptr;   // [Vp, C]   tied head / embedding shadow
    bf16* lm16 = nullptr;    // [C, Vp]   untied head shadow
    std::vector<bf16*> wqkv16, wo16, w1_16, w2_16;
    bool swiglu = false;
    float2* rope = nullptr;  // [max_t][hd/2] (cos, sin) when rope_qk
    // Config::pos_encoding == RoPE: rope_cfg's (cos, sin) per position and column pair of the
    // embedding sum, [max_t][C/2], and its attention scale
    float2* emb_rope = nullptr;
    float emb_rope_scale = 1.0f;
    // Mamba
    bool mamba = false;
    int mD = 0, mN = 0, mR = 0, mK = 0, mRP = 0, mRPp = 0, mRp = 0;
    std::vector<bf16*> in16, xproj16, dtp16, out16;
    std::vector<MambaAct> mact;
    float *m_dgated = nullptr, *m_du = nullptr, *m_duxp = nullptr,
          *m_dpre = nullptr, *m_dbc = nullptr, *m_da = nullptr, *m_dd = nullptr,
          *m_convpart = nullptr, *m_sgpart = nullptr, *m_segwork = nullptr;
    bf16 *m_dproj = nullptr, *m_dxp = nullptr;
    // MoE FFN: E experts of hidden He = 4C, top-k, expert row capacity cap
    bool moe = false;
    int moe_E = 0, moe_k = 0, moe_He = 0, moe_cap = 0;
    float moe_coef = 0.f;
    std::vector<bf16*> w1e16, w2e16;  // [E*C, He], [E*He, C]
    std::vector<MoeAct> moeact;
    float *moe_load = nullptr, *moe_aux = nullptr;  // [L][B][E], [L][B]
    bf16 *e_dyg = nullptr, *e_dpre = nullptr;       // [cap, C], [cap, He]
    float *e_dxg = nullptr, *e_dscores = nullptr, *e_gpart = nullptr;

    // activations
    std::vector<BlockAct> act;
    float* xL = nullptr;
    bf16* lnf = nullptr;
    float *meanf = nullptr, *rstdf = nullptr;
    bf16* logits = nullptr;
    // backward scratch
    float *dres = nullptr, *dy = nullptr, *dln = nullptr;
    bf16* attn_ds = nullptr;  // dS tiles of the attention backward (attention_ds_bytes)
    bf16 *dres16 = nullptr, *dy16 = nullptr, *datt = nullptr, *dqkv = nullptr, *dh = nullptr,
         *dact = nullptr;
    float* dvec = nullptr;
    float* partial = nullptr;
    float* colwork = nullptr;
    float* splitws = nullptr;
    size_t splitws_floats = 0;

    // per-step device scalars / buffers
    int32_t* d_tokens = nullptr;
    uint64_t* d_keys = nullptr;
    float* d_row_loss = nullptr;
    float* d_out = nullptr;        // [0] loss [1] pre-clip norm [2] clip scale [3] post norm [4] skip
    float* d_hp = nullptr;         // [0..7] AdamW scalars, [8] 1/K
    double* d_normpart = nullptr;
    int* d_nonfinite = nullptr;
    int* d_err = nullptr;
    AdamParam* d_aparams = nullptr;
    AdamChunk* d_chunks = nullptr;
    int nchunks = 0;
    float* d_kscale = nullptr;

    // pinned host staging
    int32_t* h_tokens = nullptr;
    float* h_out = nullptr;  // 8 floats
    float* h_hp = nullptr;   // 16 floats, mirrored into d_hp by every step
    int* h_err = nullptr;

    // optimizer / trainer state
    float lr = 3e-4f, b1 = 0.9f, b2 = 0.95f, eps = 1e-8f, wd = 0.1f;
    int adam_t = 0;
    bool adam_init = false;
    float clip = 1.0f, smoothing = 0.0f;
    float loss_scale = 1.0f;  // TrainConfig::loss_scale
    bool logits_only = false;  // forward stops after the lm head (llmgpu_forward_logits)
    int accum_k = 1, accum_count = 0;
    int step_count = 0, skipped = 0;
    float last_loss = 0.f, last_gnorm = 0.f;
    int last_T = -1;
    int last_B = 0;  // micro-batch of the last forward
    float timings[6] = {};
    int launches = 0;

    // gemm plan cache (deterministic call order)
    std::vector<GemmPlan> plan_cache;
    std::vector<std::vector<uint8_t>> plan_keys;
    size_t plan_cursor = 0;
    std::vector<GemmPlan2> plan2_cache;  // co-scheduled data/weight-gradient products
    std::vector<std::vector<uint8_t>> plan2_keys;
    std::vector<char> plan2_ok;
    size_t plan2_cursor = 0;

    // GEMM profiling (events around each GEMM launch)
    bool profile = false;
    std::vector<cudaEvent_t> prof_ev;
    std::vector<double> prof_flops;
    std::vector<int> prof_shape;     // per launch: M, N, K of each product (zeros: none)
    std::vector<float> prof_last_ms; // per launch of the last profiled step
    size_t prof_n = 0;
    double prof_total_flops = 0, prof_total_ms = 0;
    int prof_launches = 0;

    // CUDA graph of the whole step
    bool use_graph = true;
    cudaGraphExec_t graph = nullptr;
    int graph_B = -1, graph_T = -1, graph_acc = -1, graph_mode = -1, graph_K = -1;
    int graph_launches = 0;
    int graph_seen = 0;  // consecutive eager runs with the current key (capture on the 2nd)

    DecodeState dec;

    std::string err;
};

// lifecycle
Ctx* ctx_create(const llmgpu_config& cfg, int max_batch, int max_seq, int rank, int world,
                const void* uid, std::string* err);
void ctx_destroy(Ctx* c);
// one micro-batch forward+backward on device tokens (ctx->d_tokens) with accumulate flag;
// `reduce` (data parallel, last micro-batch) all-reduces each gradient bucket on the comm
// stream as soon as the backward has finished it
int run_fwd_bwd(Ctx* c, int B, int T, int accumulate, bool backward, bool reduce = false);
// optimizer: (wait for the bucket all-reduces) -> scale by 1/K -> norm/clip -> AdamW
int run_optimizer(Ctx* c, int K);
int ctx_sync_check(Ctx* c);
// Waits for stream `s` to drain. With a communicator it polls the communicator's
// asynchronous error state and aborts it at the first error or past comm_timeout_s.
int wait_stream(Ctx* c, cudaStream_t s);
void abort_comm(Ctx* c);
void prepare_step_scalars(Ctx* c, int K);
int save_binary(Ctx* c, const char* path);
int load_binary(Ctx* c, const char* path);
int save_adam(Ctx* c, const char* path);
int load_adam(Ctx* c, const char* path);
void refresh_shadows(Ctx* c);
int copy_sync(Ctx* c, void* dst, const void* src, size_t bytes, cudaMemcpyKind kind);
// KV-cached decoding (decode.cu)
int decode_supported(const Ctx* c, std::string* why);
int decode_alloc(Ctx* c);
void decode_free(Ctx* c);
int decode_fill(Ctx* c, int B, int T);
int decode_step(Ctx* c, int B);

}  // namespace llmgpu
