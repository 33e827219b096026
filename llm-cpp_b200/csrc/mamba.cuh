// Launchers of the Mamba block kernels (mamba.cu). Layouts, per micro-batch of B sequences
// of T tokens (rows = B*T):
//   proj  bf16 [rows][ldp]   in_proj output: x_z in columns [0, D), x_ssm in [D, 2D)
//   u     fp32/bf16 [rows][D] SiLU(conv(x_ssm))
//   xp    fp32 [rows][ldx]   x_proj output: dt_in [0, R), B [R, R+N), C [R+N, R+2N)
//   raw   fp32 [rows][D]     dt before softplus/clamp
//   y     fp32 [rows][D]     scan output; gated = y * SiLU(x_z) as bf16
#pragma once
#include "kernels.cuh"

namespace llmgpu {

constexpr int kScanChunk = 16;  // steps between saved scan states

struct MambaDims {
    int B, T, D, N, R, K;
    long long ldp;  // row stride of proj / dproj (2D)
    long long ldx;  // row stride of xp / dxp
};

int mamba_scan_groups(int D, int N);       // channel groups of the scan grid (partial count)
int mamba_conv_blocks(long long rows);     // row blocks of the conv backward (partial count)

int mamba_conv_forward(const MambaDims& m, const bf16* proj, const float* w, const float* bias,
                       float* u32, bf16* u16, cudaStream_t s);
int mamba_dt_forward(const MambaDims& m, const float* xp, const float* dt_proj, float* raw,
                     cudaStream_t s);
// hchk: B * ceil(T/kScanChunk) * D * N floats. Each sequence is scanned in
// mamba_scan_segments(B, T, D, N) segments side by side (one unless the grid would leave SMs
// idle); seg_work: mamba_scan_seg_floats(max batch, max length, D, N) floats, and
// mamba_scan_parts_max(...) bounds B x segments over batches up to max batch.
int mamba_scan_segments(int B, int T, int D, int N);
int mamba_scan_parts_max(int max_batch, int max_seq, int D, int N);
size_t mamba_scan_seg_floats(int max_batch, int max_seq, int D, int N);
int mamba_scan_forward(const MambaDims& m, const float* raw, const float* u, const float* xp,
                       const float* alog, const float* dskip, const bf16* proj, float* y32,
                       bf16* gated, float* hchk, float* seg_work, cudaStream_t s);
// dgated: fp32 gradient of the gated output. Writes du (scan + skip part), draw (the
// gradient of dt_raw: through the clamp mask and softplus), the x_z gradient into
// dproj[:, 0:D], and partials: dbc_part [groups][2][rows][N], da_part [B * nseg][D][N],
// dd_part [B * nseg][D] with nseg = mamba_scan_segments(B, T, D, N); seg_work as for the forward.
int mamba_scan_backward(const MambaDims& m, const float* raw, const float* u, const float* xp,
                        const float* alog, const float* dskip, const bf16* proj, const float* y32,
                        const float* dgated, const float* hchk, float* du, float* draw, bf16* dproj,
                        float* dbc_part, float* da_part, float* dd_part, float* seg_work,
                        cudaStream_t s);
int mamba_reduce_dbc(const MambaDims& m, const float* dbc_part, bf16* dxp, cudaStream_t s);
int mamba_batch_reduce(const float* part, int B, long long n, float* out, int accumulate,
                       cudaStream_t s);
// part: mamba_conv_blocks(rows) * D * (K+1) floats; writes dx_ssm into dproj[:, D:2D]
int mamba_conv_backward(const MambaDims& m, const bf16* proj, const float* w, const float* bias,
                        const float* du_scan, const float* du_xp, float* part, bf16* dproj,
                        float* gw, float* gb, int accumulate, cudaStream_t s);

// out = A B in fp32 on the CUDA cores (the dt path's contractions), K split `ksplit` ways
// through `part` (ksplit * M * N floats, unused when ksplit is 1) and reduced in order;
// writes fp32 `out` (+= if accumulate) or bf16 `out16` when given.
// A(m,k) = A[m*sam + k*sak], B(k,n) = B[k*sbk + n*sbn].
constexpr int kSgSplitRows = 8;   // K split of the rows x dt_rank products (K = d_inner)
constexpr int kSgSplitCols = 64;  // K split of the d_inner x dt_rank product (K = rows)
int small_gemm_f32(const float* A, long long sam, long long sak, const float* B, long long sbk,
                   long long sbn, int M, int N, int K, int ksplit, float* part, float* out,
                   bf16* out16, long long ldo, int accumulate, cudaStream_t s);
// dst[r, c] = bf16(src[r, c]) for c < cols
int convert_f32_bf16(const float* src, long long lds, bf16* dst, long long ldd, long long rows,
                     int cols, cudaStream_t s);

}  // namespace llmgpu
