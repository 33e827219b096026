// Launchers of the MoE FFN kernels (moe.cu): router, dispatch into per-expert row blocks,
// combine, load-balancing loss, and their backward.
//
// Layouts, per micro-batch of B sequences of T tokens (BT = B*T rows), E experts, top-k:
//   probs   fp32 [BT][E]    router softmax
//   idx     int  [BT][k]    chosen experts, descending probability (ties: lower index first)
//   wts     fp32 [BT][k]    renormalised weights p_j / s, s = sum of the chosen p (1 if < 1e-8)
//   ssum    fp32 [BT]       s
//   grp     int  [2E+1]     off[0..E] padded row offsets of the expert blocks (multiples of
//                           128), then cnt[0..E-1] rows in use per expert
//   row_of  int  [BT][k]    expert row of assignment (t, j)
//   tok_of  int  [cap]      token of an expert row, -1 for padding rows
//   xg      bf16 [cap][C]   gathered expert inputs (padding rows zero)
// Expert rows keep token order within each expert, so every sum is deterministic.
#pragma once
#include "kernels.cuh"

namespace llmgpu {

constexpr int kMoeMaxExperts = 16;
constexpr int kMoeMaxTopK = 4;
constexpr int kMoeRowAlign = 128;

struct MoeDims {
    int B, T, C, E, k;
    int cap;  // expert row capacity: BT*k + E*128
};

inline int moe_capacity(int bt, int E, int k) { return bt * k + E * kMoeRowAlign; }
int moe_gate_grad_parts(int rows);  // row chunks of the gate-gradient partials

// Router of MoEFFN::forward (src/moe.cpp:28-45): probs = softmax(ln2 gate) in fp32 on the
// norm output recomputed in fp32 from its input y and the saved mean / rstd.
int moe_router_forward(const MoeDims& m, const float* y, const float* mean, const float* rstd,
                       const float* gamma, const float* beta, int rms, const float* gate,
                       float* probs, int* idx, float* wts, float* ssum, cudaStream_t s);
int moe_dispatch(const MoeDims& m, const int* idx, int* grp, int* row_of, int* tok_of,
                 cudaStream_t s);
int moe_gather(const MoeDims& m, const bf16* x, const int* tok_of, const int* grp, bf16* xg,
               cudaStream_t s);
// out[t] = resid[t] + sum_j wts[t,j] * yg[row_of[t,j]]   (src/moe.cpp:46-59)
int moe_combine(const MoeDims& m, const float* resid, const float* yg, const int* row_of,
                const float* wts, float* out, cudaStream_t s);
// per-sequence expert load (mean of probs over T) and aux = coef * CV^2 (src/moe.cpp:64-75)
int moe_aux_forward(const MoeDims& m, const float* probs, float coef, float* load, float* aux,
                    cudaStream_t s);
// loss[0] += sum over layers of mean over sequences of aux  (aux: [layers][B])
int moe_add_aux(const float* aux, int layers, int B, float* loss, cudaStream_t s);

// Backward. dout: fp32 gradient of the FFN output. Writes dyg = w * dout into the expert rows
// (bf16) and dscores = d loss / d router logits, including the aux-loss term scaled by
// aux_scale (the weight of one sequence's loss in the micro-batch loss).
int moe_combine_backward(const MoeDims& m, const float* dout, const float* yg, const int* row_of,
                         const int* idx, const float* wts, const float* ssum, const float* probs,
                         const float* load, float coef, float aux_scale, bf16* dyg,
                         float* dscores, cudaStream_t s);
// zeros the padding rows [off[e] + cnt[e], off[e+1]) of an expert-row buffer
int moe_zero_pad_rows(const MoeDims& m, const int* grp, bf16* buf, int ld, cudaStream_t s);
// dln[t] = sum_j dxg[row_of[t,j]] + dscores[t] gate^T
int moe_scatter_sum(const MoeDims& m, const float* dxg, const int* row_of, const float* dscores,
                    const float* gate, float* dln, cudaStream_t s);
// dgate (+)= ln2^T dscores with ln2 recomputed in fp32; part: moe_gate_grad_parts(BT)*C*E
int moe_gate_grad(const MoeDims& m, const float* y, const float* mean, const float* rstd,
                  const float* gamma, const float* beta, int rms, const float* dscores,
                  float* part, float* dgate, int accumulate, cudaStream_t s);

}  // namespace llmgpu
