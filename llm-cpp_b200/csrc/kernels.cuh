// Launchers of the memory-bound and attention kernels of the training step.
// All launchers are asynchronous on `stream` and return 0 or a negative status.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace llmgpu {

using bf16 = __nv_bfloat16;

// ----------------------------------------------------------------- embedding
// x[b*T+t, :] = wte[tok mod V, :] + wpe[t, :]   (src/model.cpp:149-157), then, when `rope`
// is given ([T][C/2] (cos, sin) pairs), rotated pairwise and scaled by rope_scale like
// rope_cfg (src/model.cpp:81-104,158).
int embed_forward(const int32_t* tokens, const float* wte, const float* wpe, float* x, int B,
                  int T, int C, int V, cudaStream_t s, const float* rope = nullptr,
                  float rope_scale = 1.0f);
// Sorts (token mod V, row) pairs of the batch once per step so that the wte
// gradient can be formed deterministically (each token's rows summed in row order).
// `keys` holds n uint64 entries. n <= 16384.
int embed_sort_keys(const int32_t* tokens, int n, int V, uint64_t* keys, cudaStream_t s);
// wte_grad[tok, :] += dx[row, :] for every (tok,row) in sorted `keys`, and
// wpe_grad[t, :] (+)= sum_b dx[b*T+t, :]   (src/model.cpp:314-322). `scratch` holds
// B*T*C floats of piece partial sums.
int embed_backward(const uint64_t* keys, const float* dx, float* wte_grad, float* wpe_grad,
                   int B, int T, int C, int accumulate_wpe, float* scratch, cudaStream_t s);

// ----------------------------------------------------------------- norms
// LayerNorm (rms=0, src/tensor.cpp:388-413) or RMSNorm (rms=1, :604-623) of fp32 rows into
// bf16, saving mean (0 for RMSNorm) and rstd per row. beta may be null.
int norm_forward(const float* x, const float* gamma, const float* beta, bf16* y, float* mean,
                 float* rstd, int rows, int C, int rms, cudaStream_t s);
// dx = resid_in + norm_backward(dy) (src/tensor.cpp:556-602 / :625-655), written as fp32
// (dx_f32) and bf16 (dx_bf16, may be null). Per-CTA partial column sums are written to
// `partial` [gridDim][3][C]: dgamma, dbeta, and the column sum of dx (used for the FFN
// output-bias gradient of the block below). Returns the number of partial rows via *nparts.
// A copy wait that gave up sets *err (when given) to kDevTimeoutFull.
int norm_backward(const float* dy, const float* x, const float* gamma, const float* mean,
                  const float* rstd, const float* resid_in, float* dx_f32, bf16* dx_bf16,
                  float* partial, int rows, int C, int rms, int* nparts, cudaStream_t s,
                  int* err = nullptr);
int norm_backward_grid(int rows);
// out[j*C + c] (+)= sum_p partial[p][j][c] for the selected planes j (mask bit j set), out
// pointers per plane (null = skip).
int reduce_partials(const float* partial, int nparts, int C, float* out0, float* out1,
                    float* out2, int accumulate, cudaStream_t s);
// Column sums of a [rows, C] bf16 matrix into out (fp32, accumulate flag). Uses `work`
// (>= colsum_work_floats(C) floats) for deterministic two-stage reduction.
int colsum_bf16(const bf16* a, long long lda, int rows, int C, float* out, int accumulate,
                float* work, cudaStream_t s);
size_t colsum_work_floats(int C);

// ----------------------------------------------------------------- cross-entropy
// Per row of bf16 logits [rows, Vp] (first V columns valid): loss[row] = lse - logit[tgt],
// and logits overwritten in place by dlogits = (softmax - y) * scale (0 in padded columns),
// with y = 1 - smoothing at tgt and smoothing/(V-1) elsewhere (src/loss.cpp:6-40).
// Targets are tokens mod V (the inputs themselves, src/trainer.cpp:39). Vp * 4 bytes (two
// rows) must fit in shared memory; `err` receives a code if a row's copy times out.
int cross_entropy_fwd_bwd(bf16* logits, int rows, int V, int Vp, const int32_t* tokens,
                          float* row_loss, float scale, float smoothing, cudaStream_t s,
                          int* err = nullptr);
// out[0] = mean of v[0..n) (fixed summation order).
int mean_reduce(const float* v, int n, float* out, cudaStream_t s);

// ----------------------------------------------------------------- attention
// Causal multi-head attention over qkv [B*T, 3C] bf16 (q | k | v, heads contiguous):
// out [B*T, C] bf16, lse [B, H, T] fp32 (natural-log softmax normaliser of scaled scores).
// src/attention.cpp:35-102 / src/flash_attention.cpp:88-123.
// rope (nullable): [T][hd/2] (cos, sin) table; when given, Q and K are rotated per head as
// they are loaded and dQ/dK are rotated back before they are stored.
// head_dim 64 without a fused rope runs on the tcgen05 kernel (attention_tc.cu); so does a
// head_dim below 64 (a multiple of 8) when `work` is given (attention_work_bytes): the heads
// are zero-padded to 64 (rope, if any, applied while padding), which leaves scores and
// outputs unchanged. err (nullable) receives the device error code of a timed-out wait.
int attention_forward(const bf16* qkv, bf16* out, float* lse, int B, int T, int H, int hd,
                      const float2* rope, cudaStream_t s, int* err = nullptr,
                      void* work = nullptr);
// tcgen05 forward (head_dim 64) on a tensor map made by attention_qkv_tmap
int attention_qkv_tmap(CUtensorMap* tm, const bf16* qkv, int B, int T, int C);
int attention_forward_tc(const CUtensorMap& tm, bf16* out, float* lse, int B, int T, int H, int hd,
                         float scale, int* err, cudaStream_t s);
// In-place RoPE of the q and k parts of qkv [B*T, 3C] (pairs 2j, 2j+1 of every head, table
// [T][hd/2] of (cos, sin)); inverse != 0 applies the transposed rotation, which maps
// gradients with respect to rotated q / k back to the unrotated ones.
int rope_qk_inplace(bf16* qkv, int B, int T, int H, int hd, const float2* rope, int inverse,
                    cudaStream_t s);
// Backward: dqkv [B*T, 3C] bf16 from dout [B*T, C]; dvec [B, H, T] fp32 scratch.
// src/attention.cpp:183-363.
// head_dim 64 without a fused rope and T % 4 == 0 runs on the tcgen05 kernels, which need
// ds_work: attention_ds_bytes(B, T, H) bytes of scratch for the dS tiles; a head_dim below 64
// (a multiple of 8) with T % 4 == 0 runs there too, zero-padded, when ds_work holds
// attention_work_bytes(B, T, H, hd).
// rope_back (nullable): q and k in qkv were already rotated by this table ([T][hd/2] (cos, sin));
// dq and dk are rotated back before they are written.
int attention_backward(const bf16* qkv, const bf16* out, const bf16* dout, const float* lse,
                       float* dvec, bf16* dqkv, int B, int T, int H, int hd, const float2* rope,
                       cudaStream_t s, int* err = nullptr, void* ds_work = nullptr,
                       const float2* rope_back = nullptr);
size_t attention_ds_bytes(int B, int T, int H);
// dS tiles plus, for head_dim below 64, the zero-padded q|k|v, dout and dq|dk|dv
size_t attention_work_bytes(int B, int T, int H, int hd);
int attention_backward_tc(const bf16* qkv, const bf16* dout, const float* lse, const float* dvec,
                          bf16* dqkv, int B, int T, int H, int hd, float scale, void* ds_work,
                          int* err, cudaStream_t s, const float2* rope_back = nullptr);

// ----------------------------------------------------------------- SwiGLU FFN
// gated[r, j] = silu(h13[r, j]) * h13[r, F + j]   (src/transformer.cpp:22-30)
int swiglu_forward(const bf16* h13, bf16* gated, int rows, int F, cudaStream_t s);
// dh13 = [dgated * h3 * silu'(h1) | dgated * silu(h1)]   (src/transformer.cpp:76-89)
int swiglu_backward(const bf16* dgated, const bf16* h13, bf16* dh13, int rows, int F,
                    cudaStream_t s);

// ----------------------------------------------------------------- optimizer
struct AdamParam {
    long long offset;    // into the flat fp32 buffers
    long long numel;
    int cols;            // row length of the parameter (for the bf16 shadow)
    int decay;           // AdamW::default_decay (ndim > 1)
    bf16* shadow;        // bf16 copy read by the GEMMs (null = none)
    long long shadow_ld; // shadow row stride
};
struct AdamChunk {
    int param;
    int len;
    long long start;     // element offset within the parameter
};
// Sum of squares (fp64 per block) and non-finite detection over n floats.
int grad_norm_partials(const float* g, long long n, double* partial, int* nonfinite,
                       int nblocks, cudaStream_t s);
// Finalises: scal[0] = pre-clip norm, scal[1] = clip scale, scal[2] = post-clip norm,
// scal[3] = 1 if the step must be skipped (non-finite). src/optimizer.cpp:90-101,
// src/trainer.cpp:148-161.
int grad_norm_finalize(const double* partial, int nblocks, const int* nonfinite, float clip,
                       float* scal, cudaStream_t s);
int grad_norm_blocks();
// AdamW over all parameters (src/optimizer.cpp:54-89), skipped when scal[3] != 0.
// hp: {lr, b1, b2, eps, wd, 1-b1^t, 1-b2^t, grad_mul}
int adamw_update(const AdamParam* params, const AdamChunk* chunks, int nchunks, float* p,
                 const float* g, float* m, float* v, const float* scal, const float* hp,
                 cudaStream_t s);
// Writes the bf16 shadows of all parameters from the fp32 master copy.
int write_shadows(const AdamParam* params, const AdamChunk* chunks, int nchunks, const float* p,
                  cudaStream_t s);
// Multiplies n floats by a device scalar in place.
int scale_inplace(float* x, long long n, const float* scale, cudaStream_t s);

}  // namespace llmgpu
