// Fused softmax cross-entropy forward + backward over bf16 logits: each row is read from
// HBM once into shared memory, the loss is emitted and the row is overwritten in place by
// dlogits (src/loss.cpp:6-40).
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

// Combines two (max, sum of 2^((x - max) log2e)) pairs of the same row.
__device__ __forceinline__ float2 lse_combine(float2 a, float2 b) {
    constexpr float kLog2e = 1.4426950408889634f;
    const float m = fmaxf(a.x, b.x);
    const float sa = a.y == 0.f ? 0.f : a.y * ex2_approx((a.x - m) * kLog2e);
    const float sb = b.y == 0.f ? 0.f : b.y * ex2_approx((b.x - m) * kLog2e);
    return make_float2(m, sa + sb);
}

// Persistent over rows, two CTAs per SM: CTA b takes rows b, b + grid, ... A row (Vp bf16)
// sits in the CTA's shared buffer in two halves, each with its own bulk copy in and out: a
// half is refilled with the next row as soon as its gradient store has read it, so the copies
// overlap the arithmetic of the other half, and while one CTA of an SM waits the other
// computes. Each row takes two passes over shared memory: an online max / sum of
// exponentials (a thread rescales its running sum when its maximum grows; the per-thread
// pairs meet in one block reduction), then the gradient, written in place.
__global__ void __launch_bounds__(kCeThreads, 2) ce_kernel(bf16* __restrict__ logits, int rows,
                                                            int V, int Vp,
                                                            const int32_t* __restrict__ tokens,
                                                            float* __restrict__ row_loss,
                                                            float scale, float smoothing, int* err) {
    pdl_enter();
    extern __shared__ __align__(128) uint8_t ce_smem[];  // Vp bf16 (Vp % 8 == 0)
    __shared__ float2 red[kCeThreads / 32 + 1];
    __shared__ float s_tgt;
    __shared__ __align__(8) uint64_t bar[2];
    const int n8 = Vp >> 3;
    const int h8 = n8 >> 1;  // uint4 groups in the first half
    const uint32_t bytes0 = (uint32_t)h8 * 16u, bytes1 = (uint32_t)(n8 - h8) * 16u;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    int row = blockIdx.x;
    if (row >= rows) return;
    uint4* srow = reinterpret_cast<uint4*>(ce_smem);
    const float off = (smoothing > 0.f && V > 1) ? smoothing / (float)(V - 1) : 0.f;
    const float on = 1.0f - smoothing;
    constexpr float kLog2e = 1.4426950408889634f;
    // groups of 8 columns: [0, nfull) all valid, then at most one partly valid group, then
    // padding up to Vp
    const int nfull = V >> 3, nval = (V + 7) >> 3;
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar[0], bytes0);
        bulk_load_g2s(ce_smem, logits + (long long)row * Vp, bytes0, &bar[0]);
    }
    for (int it = 0; row < rows; ++it, row += gridDim.x) {
        if (threadIdx.x == 0) {
            // the second half is refilled once the previous row's second-half store has read it
            if (it > 0) bulk_wait_group_read<0>();
            mbar_arrive_expect_tx(&bar[1], bytes1);
            bulk_load_g2s(ce_smem + bytes0, logits + (long long)row * Vp + 8 * h8, bytes1, &bar[1]);
        }
        int tgt = tokens[row] % V;
        if (tgt < 0) tgt += V;
        float2 ms = make_float2(-FLT_MAX, 0.f);  // running (max, sum of 2^((x - max) log2e))
        auto pass1 = [&](int i0, int i1) {
            for (int i = i0 + (int)threadIdx.x; i < i1; i += blockDim.x) {
                const uint4 u = srow[i];
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
                const float m8 =
                    fmaxf(fmaxf(fmaxf(bf16_lo(u.x), bf16_hi(u.x)), fmaxf(bf16_lo(u.y), bf16_hi(u.y))),
                          fmaxf(fmaxf(bf16_lo(u.z), bf16_hi(u.z)), fmaxf(bf16_lo(u.w), bf16_hi(u.w))));
                if (m8 > ms.x) {
                    ms.y = ms.y == 0.f ? 0.f : ms.y * ex2_approx((ms.x - m8) * kLog2e);
                    ms.x = m8;
                }
                const float ml = ms.x * kLog2e;
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    acc += ex2_approx(fmaf(bf16_lo(w[k]), kLog2e, -ml)) +
                           ex2_approx(fmaf(bf16_hi(w[k]), kLog2e, -ml));
                ms.y += acc;
            }
        };
        mbar_wait_bounded(&bar[0], (uint32_t)(it & 1), err, kDevTimeoutFull);
        pass1(0, min(h8, nfull));
        mbar_wait_bounded(&bar[1], (uint32_t)(it & 1), err, kDevTimeoutFull);
        pass1(min(h8, nfull), nfull);
        if (threadIdx.x == 0) {
            if (nval > nfull) {
                const bf16* t = reinterpret_cast<const bf16*>(srow + nfull);
                for (int c = nfull * 8; c < V; ++c)
                    ms = lse_combine(ms, make_float2(__bfloat162float(t[c - nfull * 8]), 1.f));
            }
            s_tgt = __bfloat162float(reinterpret_cast<const bf16*>(srow)[tgt]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            ms = lse_combine(ms, make_float2(__shfl_xor_sync(0xffffffffu, ms.x, o),
                                             __shfl_xor_sync(0xffffffffu, ms.y, o)));
        if (lane == 0) red[warp] = ms;
        __syncthreads();
        if (warp == 0) {
            ms = lane < (int)(blockDim.x >> 5) ? red[lane] : make_float2(-FLT_MAX, 0.f);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                ms = lse_combine(ms, make_float2(__shfl_xor_sync(0xffffffffu, ms.x, o),
                                                 __shfl_xor_sync(0xffffffffu, ms.y, o)));
            if (lane == 0) red[kCeThreads / 32] = ms;
        }
        __syncthreads();
        ms = red[kCeThreads / 32];
        const float lse = ms.x + logf(ms.y);
        const float lsel = lse * kLog2e;
        if (threadIdx.x == 0) row_loss[row] = lse - s_tgt;
        // dlogits = (softmax - y) * scale; y = off everywhere but `on` at the target, and the
        // padding columns get 0
        const float offs = off * scale;
        auto pass2 = [&](int i0, int i1) {
            for (int i = i0 + (int)threadIdx.x; i < i1; i += blockDim.x) {
                const uint4 u = srow[i];
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
                uint32_t o[4];
                if (i < nfull) {
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        o[k] = pack_bf16x2(ex2_approx(fmaf(bf16_lo(w[k]), kLog2e, -lsel)) * scale - offs,
                                           ex2_approx(fmaf(bf16_hi(w[k]), kLog2e, -lsel)) * scale - offs);
                } else {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int c = i * 8 + 2 * k;
                        const float a =
                            c < V ? ex2_approx(fmaf(bf16_lo(w[k]), kLog2e, -lsel)) * scale - offs : 0.f;
                        const float bb =
                            c + 1 < V ? ex2_approx(fmaf(bf16_hi(w[k]), kLog2e, -lsel)) * scale - offs
                                      : 0.f;
                        o[k] = pack_bf16x2(a, bb);
                    }
                }
                if (i == (tgt >> 3)) {  // the target column takes `on` instead of `off`
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        if (k != ((tgt & 7) >> 1)) continue;
                        const float x = (tgt & 1) ? bf16_hi(w[k]) : bf16_lo(w[k]);
                        const float gt = (ex2_approx(fmaf(x, kLog2e, -lsel)) - on) * scale;
                        const float lo = (tgt & 1) ? bf16_lo(o[k]) : gt;
                        const float hi = (tgt & 1) ? gt : bf16_hi(o[k]);
                        o[k] = pack_bf16x2(lo, hi);
                    }
                }
                srow[i] = make_uint4(o[0], o[1], o[2], o[3]);
            }
        };
        pass2(0, h8);
        fence_proxy_async_smem();  // this thread's gradient writes before the bulk store
        __syncthreads();
        if (threadIdx.x == 0) {
            bulk_store_s2g(logits + (long long)row * Vp, srow, bytes0);
            bulk_commit_group();
        }
        pass2(h8, n8);
        fence_proxy_async_smem();
        __syncthreads();
        if (threadIdx.x == 0) {
            bulk_store_s2g(logits + (long long)row * Vp + 8 * h8, ce_smem + bytes0, bytes1);
            bulk_commit_group();
            // the first half is refilled with the next row once its store has read it
            const int next = row + gridDim.x;
            if (next < rows) {
                bulk_wait_group_read<1>();
                mbar_arrive_expect_tx(&bar[0], bytes0);
                bulk_load_g2s(ce_smem, logits + (long long)next * Vp, bytes0, &bar[0]);
            }
        }
    }
    if (threadIdx.x == 0) bulk_wait_group_all();
}

__global__ void mean_kernel(const float* __restrict__ v, int n, float* out) {
    pdl_enter();
    __shared__ float red[33];
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
    s = block_reduce(s, red, false);
    if (threadIdx.x == 0) out[0] = s / (float)n;
}

}  // namespace

int cross_entropy_fwd_bwd(bf16* logits, int rows, int V, int Vp, const int32_t* tokens,
                          float* row_loss, float scale, float smoothing, cudaStream_t s,
                          int* err) {
    if ((Vp & 7) != 0 || V > Vp || rows <= 0) return -1;
    if ((reinterpret_cast<uintptr_t>(logits) & 15) != 0) return -3;
    // one row per CTA in shared memory: two CTAs per SM for rows up to 110 KB (vocabularies
    // up to 56,320), one for rows up to 220 KB
    constexpr size_t kMaxSmem = 220 * 1024;
    const size_t smem = (size_t)Vp * sizeof(bf16);
    if (smem > kMaxSmem) return -2;
    static bool set = false;
    if (!set) {
        cudaFuncSetAttribute(ce_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
        set = true;
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int per_sm = smem <= kMaxSmem / 2 ? 2 : 1;
    const int grid = rows < per_sm * sms ? rows : per_sm * sms;
    launch_kernel(ce_kernel, grid, kCeThreads, smem, s, logits, rows, V, Vp, tokens, row_loss, scale,
                                             smoothing, err);
    return launch_status();
}

int mean_reduce(const float* v, int n, float* out, cudaStream_t s) {
    launch_kernel(mean_kernel, 1, 1024, 0, s, v, n, out);
    return launch_status();
}

}  // namespace llmgpu
