// Fused softmax cross-entropy forward + backward over bf16 logits, one CTA per row:
// the row is read from HBM once into shared memory, the loss is emitted and the
// row is overwritten in place by dlogits (src/loss.cpp:6-40).
#include <cfloat>

#include "common.cuh"
#include "kernels.cuh"

namespace llmgpu {

namespace {

constexpr int kCeThreads = 512;

__device__ __forceinline__ float block_reduce(float v, float* sh, bool is_max) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? fmaxf(v, w) : v + w;
    }
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? sh[lane] : (is_max ? -FLT_MAX : 0.f);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float w = __shfl_xor_sync(0xffffffffu, v, o);
            v = is_max ? fmaxf(v, w) : v + w;
        }
        if (lane == 0) sh[32] = v;
    }
    __syncthreads();
    return sh[32];
}

__global__ void __launch_bounds__(kCeThreads) ce_kernel(bf16* __restrict__ logits, int V, int Vp,
                                                         const int32_t* __restrict__ tokens,
                                                         float* __restrict__ row_loss, float scale,
                                                         float smoothing) {
    extern __shared__ uint4 srow[];  // Vp bf16 (Vp % 8 == 0)
    __shared__ float red[33];
    const int row = blockIdx.x;
    uint4* g = reinterpret_cast<uint4*>(logits + (long long)row * Vp);
    const int n8 = Vp >> 3;
    float mx = -FLT_MAX;
    for (int i = threadIdx.x; i < n8; i += blockDim.x) {
        uint4 u = g[i];
        srow[i] = u;
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int c = i * 8 + 2 * k;
            if (c < V) mx = fmaxf(mx, bf16_lo(w[k]));
            if (c + 1 < V) mx = fmaxf(mx, bf16_hi(w[k]));
        }
    }
    mx = block_reduce(mx, red, true);
    float se = 0.f;
    for (int i = threadIdx.x; i < n8; i += blockDim.x) {
        uint4 u = srow[i];
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int c = i * 8 + 2 * k;
            if (c < V) se += __expf(bf16_lo(w[k]) - mx);
            if (c + 1 < V) se += __expf(bf16_hi(w[k]) - mx);
        }
    }
    se = block_reduce(se, red, false);
    const float lse = mx + logf(se);
    int tgt = tokens[row] % V;
    if (tgt < 0) tgt += V;
    const float off = (smoothing > 0.f && V > 1) ? smoothing / (float)(V - 1) : 0.f;
    const float on = 1.0f - smoothing;
    if (threadIdx.x == 0) {
        const bf16* sb = reinterpret_cast<const bf16*>(srow);
        row_loss[row] = lse - __bfloat162float(sb[tgt]);
    }
    for (int i = threadIdx.x; i < n8; i += blockDim.x) {
        uint4 u = srow[i];
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int c = i * 8 + 2 * k;
            float a = 0.f, b = 0.f;
            if (c < V) a = (__expf(bf16_lo(w[k]) - lse) - (c == tgt ? on : off)) * scale;
            if (c + 1 < V) b = (__expf(bf16_hi(w[k]) - lse) - (c + 1 == tgt ? on : off)) * scale;
            o[k] = pack_bf16x2(a, b);
        }
        g[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

__global__ void mean_kernel(const float* __restrict__ v, int n, float* out) {
    __shared__ float red[33];
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
    s = block_reduce(s, red, false);
    if (threadIdx.x == 0) out[0] = s / (float)n;
}

}  // namespace

int cross_entropy_fwd_bwd(bf16* logits, int rows, int V, int Vp, const int32_t* tokens,
                          float* row_loss, float scale, float smoothing, cudaStream_t s) {
    if ((Vp & 7) != 0 || V > Vp) return -1;
    const size_t smem = (size_t)Vp * sizeof(bf16);
    if (smem > 200 * 1024) return -2;
    static bool set = false;
    if (!set) {
        cudaFuncSetAttribute(ce_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        set = true;
    }
    ce_kernel<<<rows, kCeThreads, smem, s>>>(logits, V, Vp, tokens, row_loss, scale, smoothing);
    return launch_status();
}

int mean_reduce(const float* v, int n, float* out, cudaStream_t s) {
    mean_kernel<<<1, 1024, 0, s>>>(v, n, out);
    return launch_status();
}

}  // namespace llmgpu
