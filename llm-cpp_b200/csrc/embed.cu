// Token/position embedding gather and its deterministic scatter-add backward.
#include "common.cuh"
#include "kernels.cuh"

namespace llmgpu {

namespace {

__device__ __forceinline__ int wrap_token(int tok, int V) {
    // ((tok % V) + V) % V, as src/model.cpp:152-153 clamps out-of-vocabulary ids
    int r = tok % V;
    return r < 0 ? r + V : r;
}

__global__ void embed_fwd_kernel(const int32_t* __restrict__ tokens, const float* __restrict__ wte,
                                 const float* __restrict__ wpe, float* __restrict__ x, int B, int T,
                                 int C, int V) {
    const int row = blockIdx.x;  // b*T + t
    const int t = row % T;
    const int tok = wrap_token(tokens[row], V);
    const float4* a = reinterpret_cast<const float4*>(wte + (long long)tok * C);
    const float4* p = reinterpret_cast<const float4*>(wpe + (long long)t * C);
    float4* o = reinterpret_cast<float4*>(x + (long long)row * C);
    for (int i = threadIdx.x; i < (C >> 2); i += blockDim.x) {
        float4 u = a[i], w = p[i];
        o[i] = make_float4(u.x + w.x, u.y + w.y, u.z + w.z, u.w + w.w);
    }
}

// Single-CTA bitonic sort of n <= 16384 keys (token << 32 | row) in shared memory.
__global__ void __launch_bounds__(1024) sort_keys_kernel(const int32_t* __restrict__ tokens, int n,
                                                         int V, uint64_t* __restrict__ keys) {
    extern __shared__ uint64_t sk[];
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = threadIdx.x; i < np2; i += blockDim.x) {
        sk[i] = i < n ? (((uint64_t)wrap_token(tokens[i], V) << 32) | (uint32_t)i) : ~0ull;
    }
    __syncthreads();
    for (int size = 2; size <= np2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < np2; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    uint64_t a = sk[i], b = sk[j];
                    if ((a > b) == up) {
                        sk[i] = b;
                        sk[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) keys[i] = sk[i];
}

// One warp per sorted position; the warp that starts a run of equal tokens sums the
// run's rows in row order and adds the sum to that token's gradient row.
__global__ void wte_grad_kernel(const uint64_t* __restrict__ keys, int n,
                                const float* __restrict__ dx, float* __restrict__ wte_grad, int C) {
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= n) return;
    const uint32_t tok = (uint32_t)(keys[w] >> 32);
    if (w > 0 && (uint32_t)(keys[w - 1] >> 32) == tok) return;
    int end = w + 1;
    while (end < n && (uint32_t)(keys[end] >> 32) == tok) ++end;
    float* g = wte_grad + (long long)tok * C;
    for (int c = lane * 4; c < C; c += 128) {
        float4 acc = reinterpret_cast<float4*>(g + c)[0];
        for (int k = w; k < end; ++k) {
            const int row = (int)(keys[k] & 0xffffffffu);
            float4 v = *reinterpret_cast<const float4*>(dx + (long long)row * C + c);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        reinterpret_cast<float4*>(g + c)[0] = acc;
    }
}

__global__ void wpe_grad_kernel(const float* __restrict__ dx, float* __restrict__ wpe_grad, int B,
                                int T, int C, int accumulate) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;  // over T*C/4
    if (i >= (long long)T * C / 4) return;
    const int t = (int)(i / (C / 4));
    const int c4 = (int)(i - (long long)t * (C / 4));
    float4 acc = accumulate ? reinterpret_cast<float4*>(wpe_grad + (long long)t * C)[c4]
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int b = 0; b < B; ++b) {
        float4 v = reinterpret_cast<const float4*>(dx + ((long long)b * T + t) * C)[c4];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    reinterpret_cast<float4*>(wpe_grad + (long long)t * C)[c4] = acc;
}

}  // namespace

int embed_forward(const int32_t* tokens, const float* wte, const float* wpe, float* x, int B,
                  int T, int C, int V, cudaStream_t s) {
    if ((C & 3) != 0) return -1;
    embed_fwd_kernel<<<B * T, 128, 0, s>>>(tokens, wte, wpe, x, B, T, C, V);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int embed_sort_keys(const int32_t* tokens, int n, int V, uint64_t* keys, cudaStream_t s) {
    if (n > 16384 || n <= 0) return -1;
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    const size_t smem = (size_t)np2 * sizeof(uint64_t);
    static bool set = false;
    if (!set) {
        cudaFuncSetAttribute(sort_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             16384 * 8);
        set = true;
    }
    sort_keys_kernel<<<1, 1024, smem, s>>>(tokens, n, V, keys);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int embed_backward(const uint64_t* keys, const float* dx, float* wte_grad, float* wpe_grad, int B,
                   int T, int C, int accumulate_wpe, cudaStream_t s) {
    if ((C & 3) != 0) return -1;
    const int n = B * T;
    wte_grad_kernel<<<(n * 32 + 255) / 256, 256, 0, s>>>(keys, n, dx, wte_grad, C);
    const long long m = (long long)T * C / 4;
    wpe_grad_kernel<<<(int)((m + 255) / 256), 256, 0, s>>>(dx, wpe_grad, B, T, C, accumulate_wpe);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace llmgpu
