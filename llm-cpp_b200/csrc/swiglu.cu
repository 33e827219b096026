// SILU-gated feed-forward activation and its backward (FeedForward with Activation::SILU,
// src/transformer.cpp:22-30 forward, :41-119 backward), over h13 = [h1 | h3] produced by one
// GEMM against the concatenated [W1 | W3] bf16 shadow. 128-bit loads, 8 columns per thread.
#include "common.cuh"
#include "kernels.cuh"

namespace llmgpu {

namespace {

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }
__device__ __forceinline__ float silu_grad_f(float v) {
    const float s = 1.0f / (1.0f + __expf(-v));
    return s * (1.0f + v * (1.0f - s));
}

__global__ void swiglu_fwd_kernel(const bf16* __restrict__ h13, bf16* __restrict__ gated, int rows,
                                  int F) {
    const int f8 = F >> 3;
    const long long n = (long long)rows * f8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / f8;
        const int j = (int)(i - r * f8) * 8;
        const uint4 a = *reinterpret_cast<const uint4*>(h13 + r * 2 * F + j);
        const uint4 b = *reinterpret_cast<const uint4*>(h13 + r * 2 * F + F + j);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            o[k] = pack_bf16x2(silu_f(bf16_lo(aw[k])) * bf16_lo(bw[k]),
                               silu_f(bf16_hi(aw[k])) * bf16_hi(bw[k]));
        *reinterpret_cast<uint4*>(gated + r * F + j) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

__global__ void swiglu_bwd_kernel(const bf16* __restrict__ dg, const bf16* __restrict__ h13,
                                  bf16* __restrict__ dh13, int rows, int F) {
    const int f8 = F >> 3;
    const long long n = (long long)rows * f8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / f8;
        const int j = (int)(i - r * f8) * 8;
        const uint4 d = *reinterpret_cast<const uint4*>(dg + r * F + j);
        const uint4 a = *reinterpret_cast<const uint4*>(h13 + r * 2 * F + j);
        const uint4 b = *reinterpret_cast<const uint4*>(h13 + r * 2 * F + F + j);
        const uint32_t dw[4] = {d.x, d.y, d.z, d.w}, aw[4] = {a.x, a.y, a.z, a.w},
                       bw[4] = {b.x, b.y, b.z, b.w};
        uint32_t o1[4], o3[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float d0 = bf16_lo(dw[k]), d1 = bf16_hi(dw[k]);
            const float h10 = bf16_lo(aw[k]), h11 = bf16_hi(aw[k]);
            const float h30 = bf16_lo(bw[k]), h31 = bf16_hi(bw[k]);
            o1[k] = pack_bf16x2(d0 * h30 * silu_grad_f(h10), d1 * h31 * silu_grad_f(h11));
            o3[k] = pack_bf16x2(d0 * silu_f(h10), d1 * silu_f(h11));
        }
        *reinterpret_cast<uint4*>(dh13 + r * 2 * F + j) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
        *reinterpret_cast<uint4*>(dh13 + r * 2 * F + F + j) =
            make_uint4(o3[0], o3[1], o3[2], o3[3]);
    }
}

}  // namespace

int swiglu_forward(const bf16* h13, bf16* gated, int rows, int F, cudaStream_t s) {
    if ((F & 7) != 0) return -1;
    swiglu_fwd_kernel<<<148 * 8, 256, 0, s>>>(h13, gated, rows, F);
    return launch_status();
}

int swiglu_backward(const bf16* dgated, const bf16* h13, bf16* dh13, int rows, int F,
                    cudaStream_t s) {
    if ((F & 7) != 0) return -1;
    swiglu_bwd_kernel<<<148 * 8, 256, 0, s>>>(dgated, h13, dh13, rows, F);
    return launch_status();
}

}  // namespace llmgpu
