/* libllmgpu.so — B200-native (sm_100a) training step of llm-cpp behind a C ABI.
 *
 * Drop-in boundary for the reference's training hot path `Trainer::train_step`
 * (src/trainer.cpp:37-124) and `Trainer::train_step_accum` (src/trainer.cpp:127-169):
 * GPT::forward_with_hidden -> cross-entropy -> GPT::backward -> clip -> AdamW::step.
 * Written in the style of the reference's C ABI (src/c_api.cpp:10-72): an opaque
 * handle, `extern "C"`, no exceptions across the boundary, plain pointers and sizes,
 * caller-owned output buffers with a capacity argument.
 *
 * Status codes: 0 success; negative on error (see LLMGPU_E_*). A step whose gradients
 * are not finite is skipped like the reference does (src/trainer.cpp:151-156) and
 * reported by LLMGPU_SKIPPED (> 0), not as an error. There is no CPU fallback: without
 * a usable sm_100 device llmgpu_create returns NULL and llmgpu_last_error(NULL) says why.
 *
 * Threading: one context per GPU rank, used by one host thread at a time (the
 * reference's Trainer and GPT are likewise not thread-safe).
 */
#ifndef LLMGPU_H
#define LLMGPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LLMGPU_OK 0
#define LLMGPU_SKIPPED 1          /* non-finite gradient: optimizer step skipped */
#define LLMGPU_E_ARG (-1)         /* invalid argument / shape */
#define LLMGPU_E_CUDA (-2)        /* CUDA runtime error */
#define LLMGPU_E_DEVICE (-3)      /* a kernel reported a device-side timeout/error */
#define LLMGPU_E_NCCL (-4)        /* collective error or timeout */
#define LLMGPU_E_IO (-5)          /* checkpoint file error */
#define LLMGPU_E_UNSUPPORTED (-6) /* configuration not supported by the kernels */

typedef struct llmgpu_ctx llmgpu_ctx;

/* Model configuration: the fields of llm::Config (include/llm/model.h:17-46) used by
 * the training step, plus the switches of the extension configurations that have no
 * reference GPT path (SwiGLU FFN + RoPE on Q/K; MoE FFN). */
typedef struct llmgpu_config {
    int vocab_size;     /* Config::vocab_size */
    int n_layers;       /* Config::n_layers */
    int n_heads;        /* Config::n_heads */
    int n_embd;         /* Config::n_embd */
    int block_size;     /* Config::block_size */
    int weight_tying;   /* Config::weight_tying */
    int use_rmsnorm;    /* Config::use_rmsnorm */
    int use_mamba;      /* Config::use_mamba */
    int d_inner;        /* Config::d_inner (0 = 2*n_embd) */
    int d_state;        /* Config::d_state */
    int dt_rank;        /* Config::dt_rank (0 = ceil(n_embd/16)) */
    int conv_kernel;    /* Config::conv_kernel */
    /* extensions */
    int ffn_swiglu;     /* 1: SILU-gated FeedForward (src/transformer.cpp:22-30) */
    int ffn_hidden;     /* 0 = 4*n_embd */
    int rope_qk;        /* 1: RoPE applied per head to Q and K */
    float rope_theta;
    int moe_experts;    /* >0: MoEFFN (src/moe.cpp) replaces the FFN */
    int moe_top_k;
    float moe_aux_coef;
    /* Config::pos_encoding and its RoPE options (include/llm/model.h:15-33):
     * LLMGPU_POS_LEARNED, LLMGPU_POS_SINUSOIDAL (wpe initialised with sin/cos,
     * src/model.cpp:34-41) or LLMGPU_POS_ROPE (rope_cfg rotates the embedding sum,
     * src/model.cpp:81-104,158; the backward scatters the gradient of the rotated sum into
     * wte/wpe unrotated, as src/model.cpp:314-322 does). rope_theta above is Config::rope_theta. */
    int pos_encoding;
    float rope_scaling; /* Config::rope_scaling (values below 1 act as 1, as rope_cfg clamps) */
    int rope_mode;      /* Config::rope_mode: 0 NTK (base * scaling), 1 YaRN ramp */
    float yarn_alpha;   /* Config::yarn_alpha (multiplies every angle) */
    float yarn_beta;    /* Config::yarn_beta (ramp between beta/2 and beta) */
} llmgpu_config;

#define LLMGPU_POS_LEARNED 0
#define LLMGPU_POS_SINUSOIDAL 1
#define LLMGPU_POS_ROPE 2

/* Fills `cfg` with the reference defaults (Config{} of include/llm/model.h). */
void llmgpu_config_default(llmgpu_config* cfg);

/* NCCL unique id (128 bytes) for data-parallel contexts; rank 0 creates it and shares
 * it with the other ranks (any channel). Returns 0 or a negative status. */
int llmgpu_get_unique_id(void* uid128);

/* Creates a context on the current CUDA device. world > 1 enables data parallelism over
 * NCCL with `uid128` (ignored when world == 1). max_batch x max_seq bounds the tokens of
 * one micro-batch (activation buffers are sized for it). Parameters are initialised like
 * the reference's constructors; load a checkpoint or set parameters to override. */
llmgpu_ctx* llmgpu_create(const llmgpu_config* cfg, int max_batch, int max_seq, int rank,
                          int world, const void* uid128);
int llmgpu_destroy(llmgpu_ctx* ctx);
/* Last error message of `ctx` (or of the last failed llmgpu_create when ctx is NULL). */
const char* llmgpu_last_error(const llmgpu_ctx* ctx);

/* Hyper-parameters: AdamW(lr, b1, b2, eps, wd) (src/optimizer.cpp:72) and
 * TrainConfig::grad_clip / grad_accum_steps / label_smoothing (include/llm/trainer.h:10-22). */
int llmgpu_set_adamw(llmgpu_ctx* ctx, float lr, float b1, float b2, float eps, float wd);
int llmgpu_set_lr(llmgpu_ctx* ctx, float lr); /* Optimizer::set_lr */
int llmgpu_set_train(llmgpu_ctx* ctx, float grad_clip, int grad_accum_steps,
                     float label_smoothing);
/* TrainConfig::loss_scale (src/trainer.cpp:91,103-105): the loss gradient is multiplied by
 * `scale` and the parameter gradients are divided by it before the non-finite check and the
 * clip. 1 (the default) leaves the step unchanged; a power of two gives the same result bit
 * for bit (the scale is exact in fp32 and bf16). Returns 0 or LLMGPU_E_ARG (scale <= 0). */
int llmgpu_set_loss_scale(llmgpu_ctx* ctx, float scale);

/* One optimizer step over B sequences of T tokens (targets = inputs, src/trainer.cpp:39),
 * equal to the reference's train_step_accum with K = B micro-batches of one sequence
 * each (and, with world > 1, K = world * B). `tokens` is a host pointer to B*T int32.
 * loss_out (nullable) receives the mean loss over the B sequences; grad_norm_out
 * (nullable) the post-clip global gradient norm (Trainer::last_grad_norm).
 * Returns 0, LLMGPU_SKIPPED or a negative status. */
int llmgpu_train_step(llmgpu_ctx* ctx, const int32_t* tokens, int B, int T, float* loss_out,
                      float* grad_norm_out);
/* Trainer::train_step_accum (src/trainer.cpp:127-169): accumulates the gradients of B
 * sequences; every grad_accum_steps calls it averages, clips and steps. *stepped_out
 * (nullable) is set to 1 when this call ran the optimizer. */
int llmgpu_train_step_accum(llmgpu_ctx* ctx, const int32_t* tokens, int B, int T,
                            float* loss_out, int* stepped_out);
/* Same as llmgpu_train_step with `tokens` already in device memory (B*T int32). */
int llmgpu_train_step_device(llmgpu_ctx* ctx, const int32_t* d_tokens, int B, int T,
                             float* loss_out, float* grad_norm_out);
/* Forward + loss only (no gradient, no step): mean loss over B sequences. */
int llmgpu_eval_loss(llmgpu_ctx* ctx, const int32_t* tokens, int B, int T, float* loss_out);
/* Forward without the loss: the logits of each sequence's last position (GPT::forward,
 * src/model.cpp:144-170, row T-1; what GPT::generate samples from). Writes B*V floats to
 * `logits` (capacity `cap` floats; the device holds bf16 logits) and returns B*V, or a
 * negative status. */
int64_t llmgpu_forward_logits(llmgpu_ctx* ctx, const int32_t* tokens, int B, int T,
                              float* logits, int64_t cap);
/* The same forward, returning the logits of every position (GPT::forward, src/model.cpp:140-171):
 * B*T*V floats in sequence-major order, capacity `cap` floats. Returns B*T*V or a negative
 * status. */
int64_t llmgpu_forward_logits_all(llmgpu_ctx* ctx, const int32_t* tokens, int B, int T,
                                  float* logits, int64_t cap);

/* KV-cached decoding on the device, as GPT::generate runs the transformer incrementally
 * (src/model.cpp:393-474: MultiHeadAttention::forward_incremental src/attention.cpp:104-181
 * with the KVCache of src/kv_cache.cpp). llmgpu_decode_prefill runs B prompts of T tokens
 * through the forward, keeps every layer's keys and values, and returns each prompt's
 * last-position logits (B*V floats); llmgpu_decode_step appends one token per sequence at the
 * next position and returns that position's logits. All B sequences (B <= 8 and <= the
 * context's max_batch) share one position, which stops at max_seq. llmgpu_decode_reset
 * starts B empty sequences (the reference's empty prompt: its first logits are zeros).
 * The caches hold the weights of the prefill: prefill again after a training step.
 * Covered: the reference's transformer GPT (GELU FFN, LayerNorm or RMSNorm, tied or untied
 * head, learned, sinusoidal or RoPE positions); other configurations return
 * LLMGPU_E_UNSUPPORTED (the reference itself re-runs the whole sequence for Mamba). */
int llmgpu_decode_reset(llmgpu_ctx* ctx, int B);
int64_t llmgpu_decode_prefill(llmgpu_ctx* ctx, const int32_t* tokens, int B, int T,
                              float* logits, int64_t cap);
int64_t llmgpu_decode_step(llmgpu_ctx* ctx, const int32_t* tokens, int B, float* logits,
                           int64_t cap);
int llmgpu_decode_position(const llmgpu_ctx* ctx);

/* Parameters in GPT::parameters() order (src/model.cpp:889-909). */
int llmgpu_num_params(const llmgpu_ctx* ctx);           /* number of parameter tensors */
size_t llmgpu_num_parameters(const llmgpu_ctx* ctx);     /* GPT::num_parameters() */
/* Name and shape of tensor `idx`; returns ndim (<= 4) and fills shape[0..ndim). */
int llmgpu_param_info(const llmgpu_ctx* ctx, int idx, char* name, int name_cap,
                      int64_t* shape);
/* Copies the fp32 master value / raw (pre-clip, averaged) gradient / Adam moments of
 * tensor idx into `out` (cap floats). Returns the element count (or the needed count
 * when out == NULL), negative on error. */
int64_t llmgpu_get_param(llmgpu_ctx* ctx, int idx, float* out, int64_t cap);
int64_t llmgpu_get_grad(llmgpu_ctx* ctx, int idx, float* out, int64_t cap);
int64_t llmgpu_get_adam_state(llmgpu_ctx* ctx, int idx, float* m_out, float* v_out,
                              int64_t cap);
int llmgpu_set_param(llmgpu_ctx* ctx, int idx, const float* data, int64_t n);

/* Checkpoints: binary v3/v4 (src/model.cpp:568-811; atomic tmp+fsync+rename like
 * save_binary_atomic :558-567) and the train state <prefix>.model.bin / .opt.bin / .json
 * (src/trainer.cpp:194-227, Adam state src/optimizer.cpp:129-173). */
int llmgpu_save_binary(llmgpu_ctx* ctx, const char* path);
int llmgpu_load_binary(llmgpu_ctx* ctx, const char* path);
int llmgpu_save_train_state(llmgpu_ctx* ctx, const char* prefix);
int llmgpu_load_train_state(llmgpu_ctx* ctx, const char* prefix);

/* Trainer counters (include/llm/trainer.h:41-59). */
int llmgpu_step(const llmgpu_ctx* ctx);
int llmgpu_set_step(llmgpu_ctx* ctx, int step);
int llmgpu_skipped_steps(const llmgpu_ctx* ctx);
float llmgpu_last_loss(const llmgpu_ctx* ctx);
float llmgpu_last_grad_norm(const llmgpu_ctx* ctx);

/* Timing/profiling of the last step (device time in ms per phase, CUDA events):
 * [0] forward, [1] loss, [2] backward, [3] allreduce, [4] optimizer, [5] total. */
int llmgpu_last_timings(const llmgpu_ctx* ctx, float* ms6);
/* Kernel launches issued by the last training step (library kernels counted). */
int llmgpu_last_launches(const llmgpu_ctx* ctx);

/* Data parallel: the longest a host call waits for a collective to complete before it
 * aborts the communicator and returns LLMGPU_E_NCCL (a peer rank that stopped, a lost
 * link), in seconds; default 600, or LLMGPU_COMM_TIMEOUT_S from the environment at
 * llmgpu_create (which bounds the communicator's set-up the same way). After an abort the
 * context's steps return LLMGPU_E_NCCL; parameters and checkpoints stay readable. The
 * reference has no collectives (its data parallelism is mean_reduce_grads in one process,
 * src/trainer.cpp:171-182); this bound replaces the wait a blocking collective would do. */
int llmgpu_set_comm_timeout(llmgpu_ctx* ctx, double seconds);

/* Data parallel: ends the use of the communicator between steps, after a rank has learned on
 * the host that a peer is gone (PeerWatch in the Python binding). Waits (bounded by the
 * collective timeout) for this rank's work in flight, then lets go of the communicator
 * without a teardown that would wait on the missing peer (its resources are freed when the
 * process exits); later steps return LLMGPU_E_NCCL at once, without launching; parameters
 * and checkpoints stay readable and llmgpu_destroy returns. Returns 0, or LLMGPU_E_NCCL if
 * the work in flight did not finish (the communicator is then aborted). No-op on a
 * single-process context. */
int llmgpu_abort_comm(llmgpu_ctx* ctx);

/* Executes steps as a captured CUDA graph when enable != 0 (default 1). */
int llmgpu_set_graph(llmgpu_ctx* ctx, int enable);

/* The cudaStream_t (as void*) all work of the context is issued on, so that a caller can
 * order its own work and timing events with it. */
void* llmgpu_stream(const llmgpu_ctx* ctx);
/* GEMM profiling: when on, every tensor-core GEMM launch of a step is bracketed by CUDA
 * events; llmgpu_gemm_stats returns the accumulated algorithmic FLOPs (2*M*N*K), device
 * milliseconds and launch count since the last reset (reset != 0 clears them). */
int llmgpu_set_profile(llmgpu_ctx* ctx, int enable);
int llmgpu_gemm_stats(llmgpu_ctx* ctx, double* flops, double* ms, int* launches, int reset);
/* Per GEMM launch of the last profiled step, in launch order: shapes[6*i..6*i+5] = M, N, K of
 * the launch's first product and of its second (zeros for a single product), ms[i] its
 * device time. Fills at most cap entries (either pointer may be null); returns the count. */
int llmgpu_gemm_last_step(llmgpu_ctx* ctx, int32_t* shapes, float* ms, int cap);
/* MoE routing of the last forward pass (introspection; the reference's MoEFFN keeps its
 * choices internal, src/moe.cpp:36-45): the top-k expert indices [B*T, k] chosen by block
 * `layer`'s router, in descending router probability (ties: lower index first). Copies at
 * most n entries into idx and returns B*T*k, or a negative status (not an MoE model, layer
 * out of range, n too small). Waits for the context stream. */
int64_t llmgpu_moe_routing(llmgpu_ctx* ctx, int layer, int32_t* idx, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
