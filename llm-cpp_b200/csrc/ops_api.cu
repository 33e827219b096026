// Kernel-level C ABI (include/llmgpu_ops.h): thin wrappers that run one kernel
// on caller-owned device buffers, used by the per-kernel parity tests.
#include <cuda_runtime.h>

#include "gemm.cuh"
#include "kernels.cuh"
#include "llmgpu_ops.h"
#include "moe.cuh"

using namespace llmgpu;

static int device_num_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
    return n > 0 ? n : 148;
}

extern "C" int llmgpu_op_num_sms(void) { return device_num_sms(); }

extern "C" int llmgpu_op_gemm_pair_slots(void) { return gemm_pair_slots(device_num_sms()); }

extern "C" int llmgpu_op_gemm(const void* A, long long lda, int a_mn_major, const void* B,
                              long long ldb, int b_mn_major, int M, int N, int K, int epi,
                              void* out, long long ldo, int accumulate, const float* resid,
                              long long ldr, void* aux, long long ld_aux, int splits,
                              float* workspace, int col_group, long long group_stride, int bn,
                              int* err, void* stream) {
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    GemmArgs g{};
    g.epi = epi;
    g.accumulate = accumulate;
    g.out = out;
    g.ldo = ldo;
    g.col_group = col_group;
    g.group_stride = group_stride;
    g.resid = resid;
    g.ldr = ldr;
    g.aux = aux;
    g.ld_aux = ld_aux;
    g.splits = splits < 1 ? 1 : splits;
    g.err = err;
    if (g.splits > 1) {
        if (epi != kEpiStoreF32 || workspace == nullptr) return -100;
        g.epi = kEpiSplitPartial;
        g.out = workspace;
        g.ldo = N;
    }
    GemmPlan plan;
    int rc = gemm_make_plan(&plan, A, lda, a_mn_major, B, ldb, b_mn_major, M, N, K, g, bn,
                            device_num_sms());
    if (rc) return rc;
    rc = gemm_run(plan, st);
    if (rc) return rc;
    if (g.splits > 1)
        rc = gemm_splitk_reduce(workspace, g.splits, M, N, reinterpret_cast<float*>(out), ldo,
                                col_group <= 0 ? N : col_group, group_stride, accumulate, st);
    return rc;
}

extern "C" int llmgpu_op_embed(const int32_t* tokens, const float* wte, const float* wpe, float* x,
                               int B, int T, int C, int V, void* stream) {
    return embed_forward(tokens, wte, wpe, x, B, T, C, V, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" long long llmgpu_op_embed_bwd_work(int B, int T, int C) {
    const long long n = (long long)B * T;
    return ((n * 8 + 255) / 256) * 256 + n * C * 4;
}

extern "C" int llmgpu_op_embed_bwd(const int32_t* tokens, const float* dx, float* wte_grad,
                                   float* wpe_grad, int B, int T, int C, int V,
                                   int accumulate_wpe, void* work, void* stream) {
    const long long n = (long long)B * T;
    if (B <= 0 || T <= 0 || C <= 0 || V <= 0 || n > 16384 || !work) return -1;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint64_t* keys = reinterpret_cast<uint64_t*>(work);
    float* scratch = reinterpret_cast<float*>(reinterpret_cast<char*>(work) +
                                              ((n * 8 + 255) / 256) * 256);
    const int rc = embed_sort_keys(tokens, (int)n, V, keys, s);
    if (rc) return rc;
    return embed_backward(keys, dx, wte_grad, wpe_grad, B, T, C, accumulate_wpe, scratch, s);
}

extern "C" int llmgpu_op_norm_fwd(const float* x, const float* gamma, const float* beta,
                                  void* y_bf16, float* mean, float* rstd, int rows, int C, int rms,
                                  void* stream) {
    return norm_forward(x, gamma, beta, reinterpret_cast<bf16*>(y_bf16), mean, rstd, rows, C, rms,
                        reinterpret_cast<cudaStream_t>(stream));
}

extern "C" long long llmgpu_op_norm_bwd_work(int rows, int C) {
    return (long long)norm_backward_grid(rows) * 3 * C;
}

extern "C" int llmgpu_op_norm_bwd(const float* dy, const float* x, const float* gamma,
                                  const float* mean, const float* rstd, const float* resid,
                                  float* dx, void* dx_bf16, float* dgamma, float* dbeta,
                                  float* dxsum, float* work, int rows, int C, int rms,
                                  void* stream) {
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int nparts = 0;
    int rc = norm_backward(dy, x, gamma, mean, rstd, resid, dx, reinterpret_cast<bf16*>(dx_bf16),
                           work, rows, C, rms, &nparts, st);
    if (rc) return rc;
    return reduce_partials(work, nparts, C, dgamma, dbeta, dxsum, 0, st);
}

extern "C" int llmgpu_op_cross_entropy(void* logits_bf16, int rows, int V, int Vp,
                                       const int32_t* tokens, float* row_loss, float scale,
                                       float smoothing, void* stream) {
    return cross_entropy_fwd_bwd(reinterpret_cast<bf16*>(logits_bf16), rows, V, Vp, tokens,
                                 row_loss, scale, smoothing, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int llmgpu_op_attention_fwd(const void* qkv, void* out, float* lse, int B, int T,
                                       int H, int hd, const float* rope_cs, void* stream) {
    return attention_forward(reinterpret_cast<const bf16*>(qkv), reinterpret_cast<bf16*>(out), lse,
                             B, T, H, hd, reinterpret_cast<const float2*>(rope_cs),
                             reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int llmgpu_op_attention_fwd_ws(const void* qkv, void* out, float* lse, int B, int T,
                                          int H, int hd, const float* rope_cs, void* work,
                                          void* stream) {
    return attention_forward(reinterpret_cast<const bf16*>(qkv), reinterpret_cast<bf16*>(out), lse,
                             B, T, H, hd, reinterpret_cast<const float2*>(rope_cs),
                             reinterpret_cast<cudaStream_t>(stream), nullptr, work);
}

extern "C" int llmgpu_op_attention_bwd(const void* qkv, const void* out, const void* dout,
                                       const float* lse, float* dvec, void* dqkv, int B, int T,
                                       int H, int hd, const float* rope_cs, void* work,
                                       void* stream) {
    return attention_backward(reinterpret_cast<const bf16*>(qkv), reinterpret_cast<const bf16*>(out),
                              reinterpret_cast<const bf16*>(dout), lse, dvec,
                              reinterpret_cast<bf16*>(dqkv), B, T, H, hd,
                              reinterpret_cast<const float2*>(rope_cs),
                              reinterpret_cast<cudaStream_t>(stream), nullptr, work);
}

extern "C" long long llmgpu_op_attention_bwd_work(int B, int T, int H, int hd) {
    if (B <= 0 || T <= 0 || H <= 0 || hd > 64 || hd < 8 || hd % 8 != 0) return 0;
    return (long long)attention_work_bytes(B, T, H, hd);
}

extern "C" int llmgpu_op_swiglu_fwd(const void* h13, void* gated, int rows, int F, void* stream) {
    return swiglu_forward(reinterpret_cast<const bf16*>(h13), reinterpret_cast<bf16*>(gated), rows,
                          F, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int llmgpu_op_swiglu_bwd(const void* dgated, const void* h13, void* dh13, int rows,
                                    int F, void* stream) {
    return swiglu_backward(reinterpret_cast<const bf16*>(dgated), reinterpret_cast<const bf16*>(h13),
                           reinterpret_cast<bf16*>(dh13), rows, F,
                           reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int llmgpu_op_gemm_grouped(const void* A, long long lda, int a_mn_major, const void* B,
                                      long long ldb, int b_mn_major, int M, int N, int K, int epi,
                                      void* out, long long ldo, int accumulate, void* aux,
                                      long long ld_aux, const int* grp, int groups, int mode,
                                      long long b_grp_rows, long long out_grp_stride, int* err,
                                      void* stream) {
    if (mode != kGroupRows && mode != kGroupK) return -100;
    GemmArgs g{};
    g.epi = epi;
    g.accumulate = accumulate;
    g.out = out;
    g.ldo = ldo;
    g.aux = aux;
    g.ld_aux = ld_aux;
    g.splits = 1;
    g.err = err;
    g.grp = grp;
    g.groups = groups;
    g.grp_mode = mode;
    g.b_grp_rows = b_grp_rows;
    g.out_grp_stride = out_grp_stride;
    GemmPlan plan;
    int rc = gemm_make_plan(&plan, A, lda, a_mn_major, B, ldb, b_mn_major, M, N, K, g, 0,
                            device_num_sms());
    if (rc) return rc;
    return gemm_run(plan, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int llmgpu_op_moe_route(const float* y, const float* mean, const float* rstd,
                                   const float* gamma, const float* beta, int rms,
                                   const float* gate, int B, int T, int C, int E, int k,
                                   float* probs, int* idx, float* wts, float* ssum,
                                   void* stream) {
    MoeDims m{B, T, C, E, k, moe_capacity(B * T, E, k)};
    return moe_router_forward(m, y, mean, rstd, gamma, beta, rms, gate, probs, idx, wts, ssum,
                              reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int llmgpu_op_moe_dispatch(const int* idx, int B, int T, int E, int k, int* grp,
                                      int* row_of, int* tok_of, void* stream) {
    MoeDims m{B, T, 8 /* C: unused by the dispatch */, E, k, moe_capacity(B * T, E, k)};
    return moe_dispatch(m, idx, grp, row_of, tok_of, reinterpret_cast<cudaStream_t>(stream));
}
