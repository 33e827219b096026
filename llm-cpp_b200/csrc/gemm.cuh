// Host-side interface of the tcgen05 GEMM used by every dense contraction of the
// training step (projections, FFN, lm head, and all their gradients).
//
//   D[M,N] = A[M,K] * B[N,K]^T    (bf16 operands, fp32 accumulation in TMEM)
//
// A and B may each be stored K-major (row-major with K contiguous) or MN-major
// (row-major with M/N contiguous), so that forward (x*W), data-gradient (dY*W^T)
// and weight-gradient (X^T*dY) products all read the same bf16 buffers without
// transposed copies.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace llmgpu {

enum GemmEpilogue : int {
    kEpiStoreBF16 = 0,   // out_bf16 = acc
    kEpiStoreF32 = 1,    // out_f32 = acc (+ out_f32 if accumulate)
    kEpiResidF32 = 2,    // out_f32 = resid + acc
    kEpiGeluBF16 = 3,    // aux_bf16 = acc ; out_bf16 = gelu(acc)
    kEpiDGeluBF16 = 4,   // out_bf16 = acc * gelu'(aux_bf16)
    kEpiSplitPartial = 5 // out_f32[split][M][N] = partial acc (reduced by gemm_splitk_reduce)
};

struct GemmArgs {
    int M, N, K;
    int a_mn_major, b_mn_major;
    int epi;
    int accumulate;        // kEpiStoreF32: add into existing output
    void* out;             // bf16 or f32
    long long ldo;         // row stride of out (elements)
    // Column grouping for f32 outputs: column n lands at
    //   out + (n / col_group) * group_stride + m * ldo + (n % col_group)
    // (used to write the gradients of adjacent same-shape parameters, e.g.
    // Wq|Wk|Wv, from one GEMM). col_group == N disables grouping.
    int col_group;
    long long group_stride;
    const float* resid;    // kEpiResidF32
    long long ldr;
    void* aux;             // bf16 pre-activation (written by Gelu, read by DGelu)
    long long ld_aux;
    int splits;            // >=1; kEpiSplitPartial writes `splits` partial planes
    int scalar_store;      // set by the planner when the output is not 16-byte aligned
    int tma_epi;           // set by the planner: outputs (and epilogue inputs) go through TMA
    int* err;              // device error word
    // Grouped (per-expert) products. `grp` is a device table of groups+1 ascending row
    // offsets, each a multiple of 128 (entry `groups` = rows in use), written by an earlier
    // kernel on the same stream, so the grouping needs no host synchronisation.
    //   kGroupRows: A's rows (and out's) are the groups' rows stacked. A tile of rows in
    //               [off[g], off[g+1]) multiplies group g of B, whose rows in B's tensor map
    //               start at g * b_grp_rows. Tiles at or past off[groups] do nothing.
    //   kGroupK:    A and B are both MN-major with the groups' rows stacked along K; group g
    //               contracts rows [off[g], off[g+1]) into out + g * out_grp_stride (an
    //               empty group writes zeros, or leaves `out` as is when accumulating).
    const int* grp;
    int groups;
    int grp_mode;
    long long b_grp_rows;
    long long out_grp_stride;
    // kEpiStoreBF16 through TMA: rotary embedding of the output columns [0, rope_cols) before
    // the bf16 rounding. Pairs (2j, 2j+1) of each rope_hd-wide head of row m rotate by the
    // (cos, sin) rope[(m % rope_T) * rope_hd / 2 + j] (the queries and keys of a QKV
    // projection, RoPE applied per head). rope_hd and rope_cols are multiples of 32.
    const float2* rope;
    int rope_T, rope_hd, rope_cols;
};

enum GemmGroupMode : int { kGroupNone = 0, kGroupRows = 1, kGroupK = 2 };
constexpr int kMaxGemmGroups = 64;
constexpr int kGemmRowAlign = 128;  // group offsets are multiples of the tile height
constexpr int kGemmPairTile = 512;  // plan tile code: 256x256 tiles on a cluster of two CTAs

// Precomputed launch: tensor maps + args + tile config. Encoding tensor maps
// costs host time, so the model builds one GemmPlan per call site at setup.
struct GemmPlan {
    CUtensorMap tmA;
    CUtensorMap tmB;
    CUtensorMap tmO;       // output boxes of 32x32 (3-D: column groups, splits or groups)
    CUtensorMap tmX;       // epilogue input / second output (residual or pre-activation)
    GemmArgs args;
    int bn;                // 64, 128, 256, or kGemmPairTile (256x256 on a CTA pair)
    int grid;
    size_t smem_bytes;
};

// Builds a plan. A is [M,K] (K-major, lda >= K) or [K,M] (MN-major, lda >= M);
// B is [N,K] (K-major) or [K,N] (MN-major). Returns 0 on success.
// Grouped plans: kGroupRows takes M = row capacity of A/out and K a multiple of 64;
// kGroupK takes M, N of one group's output and K = row capacity of A and B.
int gemm_make_plan(GemmPlan* plan, const void* A, long long lda, int a_mn_major, const void* B,
                   long long ldb, int b_mn_major, int M, int N, int K, const GemmArgs& epi,
                   int bn_hint, int num_sms);
// Launches a plan on a stream.
int gemm_run(const GemmPlan& plan, cudaStream_t stream);
// CTA pairs of the pair-tile kernel that can be resident at once.
int gemm_pair_slots(int num_sms);

// Two independent products in one launch of the pair-tile kernel (both plans bn =
// kGemmPairTile, ungrouped; split-K partials allowed): the data- and weight-gradient products
// of a layer, whose tiles alone leave pairs idle in their last wave. The tiles of both,
// longest first, are spread over the resident pairs by a host-built table (device memory
// owned by the plan: gemm_free_plan2).
struct GemmPlan2 {
    GemmPlan p[2];
    int grid;
    int* sched;
    int sched_stride;
    int* queue;       // two device counters for the run-time unit queue (in the sched block)
    int q_first;      // the product whose units are longest (handed out first)
    int q_total[2];   // units of each product
};
int gemm_make_plan2(GemmPlan2* plan, const GemmPlan& p0, const GemmPlan& p1, int num_sms);
// queue: hand the units out at run time (see PairParams) instead of the host's per-pair
// lists. It pays where another kernel holds SMs during the launch (a data-parallel step's
// all-reduce); LLMGPU_GEMM_QUEUE=0 or 1 overrides the caller's choice.
int gemm_run2(const GemmPlan2& plan, cudaStream_t stream, bool queue);
void gemm_free_plan2(GemmPlan2* plan);

// Reduces split-K partials [splits][M][N] (fp32) into the final output with the
// same epilogue options as kEpiStoreF32 (accumulate, column grouping).
int gemm_splitk_reduce(const float* partial, int splits, int M, int N, float* out, long long ldo,
                       int col_group, long long group_stride, int accumulate,
                       cudaStream_t stream);

}  // namespace llmgpu
