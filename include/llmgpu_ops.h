/* Kernel-level C ABI of libllmgpu.so.
 *
 * These entry points run one hand-written sm_100a kernel on caller-owned device
 * buffers (plain pointers, element strides, no framework types). They exist so
 * that each kernel of the training step can be checked in isolation against the
 * CPU oracle; the training step itself is driven through llmgpu.h.
 *
 * Conventions (shared with llmgpu.h): return 0 on success, a negative status on
 * error; `stream` is a cudaStream_t passed as void* (NULL = legacy default
 * stream); every call is asynchronous on that stream.
 */
#ifndef LLMGPU_OPS_H
#define LLMGPU_OPS_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* D[M,N] = A[M,K] * B[N,K]^T with bf16 operands and fp32 accumulation on the
 * 5th-generation tensor cores. Replaces the fp32 contractions of
 * Tensor::matmul (src/tensor.cpp:229-321) and the hand-written gradient loops
 * (src/attention.cpp:234-241,322-334; src/transformer.cpp:129-181;
 * src/model.cpp:249-270).
 *   a_mn_major = 0: A is row-major [M][lda] (K contiguous); 1: A is [K][lda] (M contiguous)
 *   b_mn_major = 0: B is row-major [N][ldb] (K contiguous); 1: B is [K][ldb] (N contiguous)
 *   epi: 0 bf16 store, 1 f32 store (+= if accumulate), 2 f32 out = resid + acc,
 *        3 gelu (aux = acc in bf16, out = gelu(acc) in bf16),
 *        4 gelu backward (out = acc * gelu'(aux)) in bf16.
 *   splits > 1 (epi 1 only) splits K; `workspace` must hold splits*M*N floats.
 *   col_group/group_stride (epi 1): column n is written to
 *        out + (n / col_group) * group_stride + m * ldo + n % col_group.
 *   bn: tile width 64/128/256, 512 = 256x256 tiles on a CTA pair, 0 = automatic.
 *   err: device int that receives a nonzero code if a device-side wait timed out. */
int llmgpu_op_gemm(const void* A, long long lda, int a_mn_major, const void* B, long long ldb,
                   int b_mn_major, int M, int N, int K, int epi, void* out, long long ldo,
                   int accumulate, const float* resid, long long ldr, void* aux, long long ld_aux,
                   int splits, float* workspace, int col_group, long long group_stride, int bn,
                   int* err, void* stream);

/* Split-K form of llmgpu_op_gemm (f32 output, epi 1) that allocates no device memory.
 * It has no counterpart in the reference.
 * For callers that cannot call cudaMalloc: code that draws every byte from its own
 * pre-reserved pool or custom allocator, or that runs under a fixed memory budget, and so
 * cannot provide the `workspace` that llmgpu_op_gemm needs when splits > 1. Its split-K
 * partial sums live in a fixed 16 MiB device array inside the library (4,194,304 floats),
 * which every GPU that loads the library holds until the process exits.
 *   - Requires splits * M * N <= 4194304; larger sizes return -101 and do nothing.
 *   - The first call on a device looks up that array's device address (once per device);
 *     make that first call before any stream capture.
 *   - All calls share the one array: calls whose kernels overlap on the GPU (different
 *     streams, concurrent threads) race and must be serialised by the caller. Each call
 *     overwrites the part it uses, so no clearing is needed.
 *   - No cudaMalloc, cudaFree or other allocating call is made.
 * Same arguments and result as llmgpu_op_gemm with epi = 1. Returns 0 or a negative status. */
int llmgpu_op_gemm_splitk_noalloc(const void* A, long long lda, int a_mn_major, const void* B,
                                  long long ldb, int b_mn_major, int M, int N, int K, float* out,
                                  long long ldo, int accumulate, int splits, int col_group,
                                  long long group_stride, int* err, void* stream);

/* x[b*T+t,:] = wte[tok mod V,:] + wpe[t,:] in fp32 (src/model.cpp:149-157). */
int llmgpu_op_embed(const int32_t* tokens, const float* wte, const float* wpe, float* x, int B,
                    int T, int C, int V, void* stream);
/* Embedding backward (src/model.cpp:314-322): wte_grad[tok mod V] += dx[row] for every token
 * row (the rows of a repeated id summed in a fixed order, so the result is deterministic) and
 * wpe_grad[t] (+)= sum_b dx[b*T + t] (accumulate_wpe). B*T <= 16384. `work` must hold
 * llmgpu_op_embed_bwd_work(B, T, C) bytes. */
long long llmgpu_op_embed_bwd_work(int B, int T, int C);
int llmgpu_op_embed_bwd(const int32_t* tokens, const float* dx, float* wte_grad, float* wpe_grad,
                        int B, int T, int C, int V, int accumulate_wpe, void* work, void* stream);
/* LayerNorm (rms=0, src/tensor.cpp:388-413) / RMSNorm (rms=1, :604-623): fp32 rows in,
 * bf16 rows out, per-row mean and rstd saved. */
int llmgpu_op_norm_fwd(const float* x, const float* gamma, const float* beta, void* y_bf16,
                       float* mean, float* rstd, int rows, int C, int rms, void* stream);
/* Norm backward (src/tensor.cpp:556-602 / :625-655): dx = resid + d/dx, written fp32 (and
 * bf16 if dx_bf16 != NULL); dgamma, dbeta (nullable) and the column sums of dx (nullable)
 * are written to their outputs. `work` must hold llmgpu_op_norm_bwd_work(rows, C) floats.
 * dx may be resid itself (each row is read before it is written). */
int llmgpu_op_norm_bwd(const float* dy, const float* x, const float* gamma, const float* mean,
                       const float* rstd, const float* resid, float* dx, void* dx_bf16,
                       float* dgamma, float* dbeta, float* dxsum, float* work, int rows, int C,
                       int rms, void* stream);
long long llmgpu_op_norm_bwd_work(int rows, int C);
/* Fused softmax cross-entropy over bf16 logits [rows, Vp] (src/loss.cpp:6-40): per-row loss,
 * logits overwritten by (softmax - y) * scale. */
int llmgpu_op_cross_entropy(void* logits_bf16, int rows, int V, int Vp, const int32_t* tokens,
                            float* row_loss, float scale, float smoothing, void* stream);
/* Causal attention forward/backward over packed bf16 qkv [B*T, 3C]
 * (src/attention.cpp:35-102, :183-363). dvec: B*H*T floats of scratch.
 * rope_cs (nullable): [T][hd/2][2] (cos, sin) of pos * theta^(-2j/hd); when given, Q and K
 * are rotated per head on load (pairs 2j, 2j+1, as rope_cfg pairs them, src/model.cpp:88-100)
 * and dQ/dK are returned for the unrotated inputs. */
int llmgpu_op_attention_fwd(const void* qkv, void* out, float* lse, int B, int T, int H, int hd,
                            const float* rope_cs, void* stream);
/* The same forward with the backward's workspace (llmgpu_op_attention_bwd_work bytes): a
 * head_dim below 64 (a multiple of 8) then also runs on the tcgen05 kernel, its heads
 * zero-padded to 64 in the workspace (and rotated there when rope_cs is given). */
int llmgpu_op_attention_fwd_ws(const void* qkv, void* out, float* lse, int B, int T, int H,
                               int hd, const float* rope_cs, void* work, void* stream);
/* The backward's `work` must hold llmgpu_op_attention_bwd_work(B, T, H, hd) bytes (the dS
 * tiles that the dK/dV kernel stores and the dQ kernel reads, and for a head_dim below 64 the
 * zero-padded heads; 0 bytes when head_dim keeps it off the tcgen05 kernels), 256-byte
 * aligned. */
int llmgpu_op_attention_bwd(const void* qkv, const void* out, const void* dout, const float* lse,
                            float* dvec, void* dqkv, int B, int T, int H, int hd,
                            const float* rope_cs, void* work, void* stream);
long long llmgpu_op_attention_bwd_work(int B, int T, int H, int hd);
/* SILU-gated FFN activation (src/transformer.cpp:22-30, 76-89) over h13 = [h1 | h3]
 * ([rows, 2F] bf16): gated = silu(h1) * h3; backward gives dh13 = [dh1 | dh3]. */
int llmgpu_op_swiglu_fwd(const void* h13, void* gated, int rows, int F, void* stream);
int llmgpu_op_swiglu_bwd(const void* dgated, const void* h13, void* dh13, int rows, int F,
                         void* stream);

/* Grouped (per-expert) GEMM for the MoE FFN experts (the per-token [1,C] matmuls of
 * MoEFFN::forward, src/moe.cpp:46-56, batched by expert). grp is a device table of
 * groups+1 ascending row offsets, each a multiple of 128.
 *   mode 1 (rows): rows [off[g], off[g+1]) of A ([M = row capacity, K], K-major) times group
 *     g of B, whose rows start at g * b_grp_rows of B's outer dimension; K a multiple of 64;
 *     epi 0, 1, 3 or 4 as in llmgpu_op_gemm.
 *   mode 2 (K): out + g * out_grp_stride (+)= A_g^T B_g over rows [off[g], off[g+1]) of
 *     A ([K = row capacity, M]) and B ([K, N]), both MN-major; epi 1; empty groups write
 *     zeros (or leave out as is when accumulating).
 * Returns 0 or a negative status. */
int llmgpu_op_gemm_grouped(const void* A, long long lda, int a_mn_major, const void* B,
                           long long ldb, int b_mn_major, int M, int N, int K, int epi, void* out,
                           long long ldo, int accumulate, void* aux, long long ld_aux,
                           const int* grp, int groups, int mode, long long b_grp_rows,
                           long long out_grp_stride, int* err, void* stream);
/* MoE router (src/moe.cpp:28-45) on B*T rows: the norm output (y - mean) * rstd * gamma
 * (+ beta unless rms) recomputed in fp32, probs = softmax(. gate) with gate [C, E] fp32,
 * top-k experts by descending probability (ties: lower index first) and weights
 * renormalised over the chosen k (sum below 1e-8 -> 1). Outputs probs [BT, E], idx [BT, k],
 * wts [BT, k], ssum [BT]. */
int llmgpu_op_moe_route(const float* y, const float* mean, const float* rstd, const float* gamma,
                        const float* beta, int rms, const float* gate, int B, int T, int C, int E,
                        int k, float* probs, int* idx, float* wts, float* ssum, void* stream);
/* Dispatch of the (token, slot) assignments idx [BT, k] into per-expert row blocks:
 * grp [2E+1] = row offsets off[0..E] (each block padded to a multiple of 128) then the row
 * counts cnt[0..E-1]; row_of [BT, k] = expert row of each assignment, rows of one expert in
 * token order; tok_of [BT*k + 128*E] = token of each expert row, -1 for padding rows. */
int llmgpu_op_moe_dispatch(const int* idx, int B, int T, int E, int k, int* grp, int* row_of,
                           int* tok_of, void* stream);

/* Number of SMs the library sizes persistent grids for (device 0 of the caller). */
int llmgpu_op_num_sms(void);
/* CTA pairs (clusters of two SMs) the 256x256-tile GEMM keeps resident at once. */
int llmgpu_op_gemm_pair_slots(void);

#ifdef __cplusplus
}
#endif
#endif
