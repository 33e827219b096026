// Global-norm clipping + non-finite guard + multi-tensor AdamW over one flat fp32
// parameter arena, writing the bf16 shadow weights read by the GEMMs in the same pass.
#include <cmath>

#include "common.cuh"
#include "kernels.cuh"

namespace llmgpu {

namespace {

constexpr int kNormBlocks = 592;  // 4 x 148 SMs
constexpr int kNormThreads = 512;

__global__ void __launch_bounds__(kNormThreads) grad_norm_kernel(const float* __restrict__ g,
                                                                 long long n,
                                                                 double* __restrict__ partial,
                                                                 int* __restrict__ nonfinite) {
    pdl_enter();
    __shared__ double red[kNormThreads / 32];
    float acc = 0.f;
    int bad = 0;
    const long long n4 = n >> 2;
    const float4* g4 = reinterpret_cast<const float4*>(g);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
         i += (long long)gridDim.x * blockDim.x) {
        float4 v = g4[i];
        acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
    }
    for (long long i = (n4 << 2) + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float v = g[i];
        acc += v * v;
        bad |= !isfinite(v);
    }
    double d = acc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    if (bad) atomicOr(nonfinite, 1);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = d;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0;
        for (int w = 0; w < kNormThreads / 32; ++w) s += red[w];
        partial[blockIdx.x] = s;
    }
}

__global__ void grad_norm_final_kernel(const double* __restrict__ partial, int nblocks,
                                       const int* __restrict__ nonfinite, float clip,
                                       float* __restrict__ scal) {
    pdl_enter();
    __shared__ double red[32];
    double s = 0;
    for (int i = threadIdx.x; i < nblocks; i += blockDim.x) s += partial[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
        const double norm = sqrt(tot);
        float sc = 1.0f;
        if (norm > (double)clip && norm > 0) sc = clip / (float)norm;
        scal[0] = (float)norm;
        scal[1] = sc;
        scal[2] = (float)(norm * (double)sc);
        scal[3] = *nonfinite ? 1.0f : 0.0f;
    }
}

struct AdamHp {
    float lr, b1, b2, eps, c1, c2, gmul, decay;
};
// One element of AdamW (src/optimizer.cpp:54-89): decoupled decay, then the Adam step.
__device__ __forceinline__ void adam_elem(const AdamHp& h, float& pv, float gv, float& mv,
                                          float& vv) {
    gv *= h.gmul;
    pv -= h.decay * pv;
    mv = h.b1 * mv + (1.0f - h.b1) * gv;
    vv = h.b2 * vv + (1.0f - h.b2) * gv * gv;
    const float mhat = mv / h.c1, vhat = vv / h.c2;
    pv -= h.lr * mhat / (sqrtf(vhat) + h.eps);
}
__device__ __forceinline__ long long shadow_off(const AdamParam& pr, long long k) {
    if (pr.shadow_ld == pr.cols) return k;
    const long long r = k / pr.cols;
    return r * pr.shadow_ld + (k - r * pr.cols);
}

// A chunk of one parameter per block: 16-byte loads and stores of p, g, m and v (parameter
// offsets are multiples of 64 floats, chunk starts of 16384), four in flight per thread, and
// the bf16 shadow written 4 values at a time when its rows keep 4-element groups aligned.
__global__ void __launch_bounds__(256) adamw_kernel(const AdamParam* __restrict__ params,
                                                    const AdamChunk* __restrict__ chunks,
                                                    float* __restrict__ p,
                                                    const float* __restrict__ g,
                                                    float* __restrict__ m, float* __restrict__ v,
                                                    const float* __restrict__ scal,
                                                    const float* __restrict__ hp) {
    pdl_enter();
    if (scal[3] != 0.0f) return;  // non-finite gradient: the step is skipped
    const AdamChunk ch = chunks[blockIdx.x];
    const AdamParam pr = params[ch.param];
    AdamHp h;
    h.lr = hp[0];
    h.b1 = hp[1];
    h.b2 = hp[2];
    h.eps = hp[3];
    h.c1 = hp[5];
    h.c2 = hp[6];
    h.gmul = hp[7] * scal[1];
    h.decay = pr.decay ? hp[0] * hp[4] : 0.0f;
    const long long base = pr.offset + ch.start;
    const int n4 = ch.len >> 2;
    const bool vec_shadow = pr.shadow && (pr.cols & 3) == 0 && (pr.shadow_ld & 3) == 0;
    float4* p4 = reinterpret_cast<float4*>(p + base);
    const float4* g4 = reinterpret_cast<const float4*>(g + base);
    float4* m4 = reinterpret_cast<float4*>(m + base);
    float4* v4 = reinterpret_cast<float4*>(v + base);
#pragma unroll 4
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 pv = p4[i];
        const float4 gv = g4[i];
        float4 mv = m4[i], vv = v4[i];
        adam_elem(h, pv.x, gv.x, mv.x, vv.x);
        adam_elem(h, pv.y, gv.y, mv.y, vv.y);
        adam_elem(h, pv.z, gv.z, mv.z, vv.z);
        adam_elem(h, pv.w, gv.w, mv.w, vv.w);
        p4[i] = pv;
        m4[i] = mv;
        v4[i] = vv;
        if (pr.shadow) {
            const long long k = ch.start + 4LL * i;
            if (vec_shadow) {
                uint2 w;
                w.x = pack_bf16x2(pv.x, pv.y);
                w.y = pack_bf16x2(pv.z, pv.w);
                *reinterpret_cast<uint2*>(pr.shadow + shadow_off(pr, k)) = w;
            } else {
                pr.shadow[shadow_off(pr, k)] = __float2bfloat16_rn(pv.x);
                pr.shadow[shadow_off(pr, k + 1)] = __float2bfloat16_rn(pv.y);
                pr.shadow[shadow_off(pr, k + 2)] = __float2bfloat16_rn(pv.z);
                pr.shadow[shadow_off(pr, k + 3)] = __float2bfloat16_rn(pv.w);
            }
        }
    }
    for (int i = 4 * n4 + threadIdx.x; i < ch.len; i += blockDim.x) {
        const long long e = base + i;
        float pv = p[e], mv = m[e], vv = v[e];
        adam_elem(h, pv, g[e], mv, vv);
        p[e] = pv;
        m[e] = mv;
        v[e] = vv;
        if (pr.shadow) pr.shadow[shadow_off(pr, ch.start + i)] = __float2bfloat16_rn(pv);
    }
}

__global__ void __launch_bounds__(256) shadow_kernel(const AdamParam* __restrict__ params,
                                                     const AdamChunk* __restrict__ chunks,
                                                     const float* __restrict__ p) {
    pdl_enter();
    const AdamChunk ch = chunks[blockIdx.x];
    const AdamParam pr = params[ch.param];
    if (!pr.shadow) return;
    const long long base = pr.offset + ch.start;
    for (int i = threadIdx.x; i < ch.len; i += blockDim.x) {
        const long long k = ch.start + i;
        long long off = k;
        if (pr.shadow_ld != pr.cols) {
            const long long r = k / pr.cols;
            off = r * pr.shadow_ld + (k - r * pr.cols);
        }
        pr.shadow[off] = __float2bfloat16_rn(p[base + i]);
    }
}

__global__ void scale_kernel(float* x, long long n, const float* scale) {
    pdl_enter();
    const float s = *scale;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        x[i] *= s;
}

}  // namespace

int grad_norm_blocks() { return kNormBlocks; }

int grad_norm_partials(const float* g, long long n, double* partial, int* nonfinite, int nblocks,
                       cudaStream_t s) {
    if (nblocks != kNormBlocks) return -1;
    cudaMemsetAsync(nonfinite, 0, sizeof(int), s);
    launch_kernel(grad_norm_kernel, kNormBlocks, kNormThreads, 0, s, g, n, partial, nonfinite);
    return launch_status();
}

int grad_norm_finalize(const double* partial, int nblocks, const int* nonfinite, float clip,
                       float* scal, cudaStream_t s) {
    launch_kernel(grad_norm_final_kernel, 1, 1024, 0, s, partial, nblocks, nonfinite, clip, scal);
    return launch_status();
}

int adamw_update(const AdamParam* params, const AdamChunk* chunks, int nchunks, float* p,
                 const float* g, float* m, float* v, const float* scal, const float* hp,
                 cudaStream_t s) {
    launch_kernel(adamw_kernel, nchunks, 256, 0, s, params, chunks, p, g, m, v, scal, hp);
    return launch_status();
}

int write_shadows(const AdamParam* params, const AdamChunk* chunks, int nchunks, const float* p,
                  cudaStream_t s) {
    launch_kernel(shadow_kernel, nchunks, 256, 0, s, params, chunks, p);
    return launch_status();
}

int scale_inplace(float* x, long long n, const float* scale, cudaStream_t s) {
    launch_kernel(scale_kernel, 592, 256, 0, s, x, n, scale);
    return launch_status();
}

}  // namespace llmgpu
