// MoE FFN (src/moe.cpp:23-75) on device: fp32 router with deterministic top-k, dispatch of
// the (token, slot) assignments into per-expert row blocks padded to the GEMM tile height,
// gather, weighted combine, load-balancing loss, and the backward of all of them. The expert
// products themselves are grouped tcgen05 GEMMs (gemm.cu, kGroupRows / kGroupK).
//
// Every reduction runs in a fixed order (warp butterflies, ordered partial planes, token
// order inside each expert block), so a step is bit-reproducible.
#include <cmath>

#include "common.cuh"
#include "moe.cuh"

namespace llmgpu {

namespace {

constexpr int kGateChunk = 64;  // rows per gate-gradient partial

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// gate [C][E] -> sgT [E][C] in shared memory (conflict-free float4 reads along C)
__device__ __forceinline__ void load_gate_t(const float* gate, int C, int E, float* sgT) {
    for (int i = threadIdx.x; i < C * E; i += blockDim.x) {
        const int c = i / E, e = i - c * E;
        sgT[e * C + c] = gate[i];
    }
}

template <int MAXE>
__global__ void __launch_bounds__(256)
    moe_router_kernel(const float* __restrict__ y, const float* __restrict__ mean,
                      const float* __restrict__ rstd, const float* __restrict__ gamma,
                      const float* __restrict__ beta, int rms, const float* __restrict__ gate,
                      int rows, int C, int E, int k, float* __restrict__ probs,
                      int* __restrict__ idx, float* __restrict__ wts, float* __restrict__ ssum) {
    extern __shared__ float sgT[];
    load_gate_t(gate, C, E, sgT);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nv = C >> 2;
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    const float4* b4 = reinterpret_cast<const float4*>(beta);
    const bool use_b = beta && !rms;
    for (int row = blockIdx.x * 8 + warp; row < rows; row += gridDim.x * 8) {
        const float mu = mean[row], r = rstd[row];
        const float4* yr = reinterpret_cast<const float4*>(y + (long long)row * C);
        float acc[MAXE];
#pragma unroll
        for (int e = 0; e < MAXE; ++e) acc[e] = 0.f;
        for (int i = lane; i < nv; i += 32) {
            const float4 v = yr[i], g = g4[i];
            const float4 b = use_b ? b4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            // the norm output exactly as the norm kernel computes it, before bf16 rounding
            const float l0 = (v.x - mu) * r * g.x + b.x;
            const float l1 = (v.y - mu) * r * g.y + b.y;
            const float l2 = (v.z - mu) * r * g.z + b.z;
            const float l3 = (v.w - mu) * r * g.w + b.w;
#pragma unroll
            for (int e = 0; e < MAXE; ++e) {
                if (e < E) {
                    const float4 w = reinterpret_cast<const float4*>(sgT + e * C)[i];
                    acc[e] += l0 * w.x + l1 * w.y + l2 * w.z + l3 * w.w;
                }
            }
        }
        // butterfly sums leave the same bits in every lane, so all lanes agree on the routing
        float mx = -INFINITY;
#pragma unroll
        for (int e = 0; e < MAXE; ++e) {
            if (e < E) {
                acc[e] = wsum(acc[e]);
                mx = fmaxf(mx, acc[e]);
            }
        }
        float sum = 0.f;
#pragma unroll
        for (int e = 0; e < MAXE; ++e) {
            if (e < E) {
                acc[e] = expf(acc[e] - mx);
                sum += acc[e];
            }
        }
#pragma unroll
        for (int e = 0; e < MAXE; ++e)
            if (e < E) acc[e] = acc[e] / sum;
        if (lane < E) {
            float pv = 0.f;
#pragma unroll
            for (int e = 0; e < MAXE; ++e)
                if (e == lane) pv = acc[e];
            probs[(long long)row * E + lane] = pv;
        }
        if (lane == 0) {
            // top-k by descending probability; among equal probabilities the lower index wins
            unsigned taken = 0u;
            int sel[kMoeMaxTopK];
            float sp[kMoeMaxTopK];
            float s = 0.f;
            for (int j = 0; j < k; ++j) {
                int best = -1;
                float bp = 0.f;
#pragma unroll
                for (int e = 0; e < MAXE; ++e) {
                    if (e < E && !((taken >> e) & 1u) && (best < 0 || acc[e] > bp)) {
                        best = e;
                        bp = acc[e];
                    }
                }
                taken |= 1u << best;
                sel[j] = best;
                sp[j] = bp;
                s += bp;
            }
            if (s < 1e-8f) s = 1.0f;
            for (int j = 0; j < k; ++j) {
                idx[(long long)row * k + j] = sel[j];
                wts[(long long)row * k + j] = sp[j] / s;
            }
            ssum[row] = s;
        }
    }
}

// One CTA assigns every (token, slot) pair its row in the expert blocks: expert by expert, a
// block-wide exclusive scan over per-thread counts of contiguous assignment ranges keeps the
// token order inside each expert.
__global__ void __launch_bounds__(1024)
    moe_dispatch_kernel(const int* __restrict__ idx, int A, int k, int E, int* __restrict__ grp,
                        int* __restrict__ row_of, int* __restrict__ tok_of) {
    __shared__ int s_warp[32];
    __shared__ int s_total;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = (A + blockDim.x - 1) / blockDim.x;
    const int a0 = min(tid * per, A), a1 = min(a0 + per, A);
    const int nwarps = blockDim.x >> 5;
    int off = 0;
    for (int e = 0; e < E; ++e) {
        int cnt = 0;
        for (int a = a0; a < a1; ++a) cnt += (idx[a] == e) ? 1 : 0;
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) s_warp[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const int w = lane < nwarps ? s_warp[lane] : 0;
            int wi = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += v;
            }
            if (lane < nwarps) s_warp[lane] = wi - w;
            if (lane == 31) s_total = wi;
        }
        __syncthreads();
        const int total = s_total;
        int r = off + s_warp[warp] + incl - cnt;
        for (int a = a0; a < a1; ++a) {
            if (idx[a] == e) {
                row_of[a] = r;
                tok_of[r] = a / k;
                ++r;
            }
        }
        const int end = off + ((total + kMoeRowAlign - 1) / kMoeRowAlign) * kMoeRowAlign;
        for (int rr = off + total + tid; rr < end; rr += blockDim.x) tok_of[rr] = -1;
        if (tid == 0) {
            grp[e] = off;
            grp[E + 1 + e] = total;
        }
        off = end;
        __syncthreads();  // s_warp / s_total are reused by the next expert
    }
    if (tid == 0) grp[E] = off;
}

__global__ void moe_gather_kernel(const bf16* __restrict__ x, const int* __restrict__ tok_of,
                                  const int* __restrict__ grp, int E, int C,
                                  bf16* __restrict__ xg) {
    const int rows = grp[E];
    const int nv = C >> 3;
    const int lane = threadIdx.x & 31;
    for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows;
         row += (gridDim.x * blockDim.x) >> 5) {
        const int t = tok_of[row];
        uint4* o = reinterpret_cast<uint4*>(xg + (long long)row * C);
        if (t < 0) {
            for (int i = lane; i < nv; i += 32) o[i] = make_uint4(0u, 0u, 0u, 0u);
        } else {
            const uint4* src = reinterpret_cast<const uint4*>(x + (long long)t * C);
            for (int i = lane; i < nv; i += 32) o[i] = src[i];
        }
    }
}

__global__ void moe_combine_kernel(const float* __restrict__ resid, const float* __restrict__ yg,
                                   const int* __restrict__ row_of, const float* __restrict__ wts,
                                   int rows, int C, int k, float* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int nv = C >> 2;
    for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < rows;
         t += (gridDim.x * blockDim.x) >> 5) {
        int r[kMoeMaxTopK];
        float w[kMoeMaxTopK];
        for (int j = 0; j < k; ++j) {
            r[j] = row_of[(long long)t * k + j];
            w[j] = wts[(long long)t * k + j];
        }
        const float4* x4 = reinterpret_cast<const float4*>(resid + (long long)t * C);
        float4* o4 = reinterpret_cast<float4*>(out + (long long)t * C);
        for (int i = lane; i < nv; i += 32) {
            float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int j = 0; j < k; ++j) {
                const float4 v = reinterpret_cast<const float4*>(yg + (long long)r[j] * C)[i];
                f.x += w[j] * v.x;
                f.y += w[j] * v.y;
                f.z += w[j] * v.z;
                f.w += w[j] * v.w;
            }
            const float4 x = x4[i];
            o4[i] = make_float4(x.x + f.x, x.y + f.y, x.z + f.z, x.w + f.w);
        }
    }
}

template <int MAXE>
__global__ void __launch_bounds__(256)
    moe_aux_kernel(const float* __restrict__ probs, int T, int E, float coef,
                   float* __restrict__ load, float* __restrict__ aux) {
    __shared__ float red[256][MAXE];
    const int b = blockIdx.x;
    float acc[MAXE];
#pragma unroll
    for (int e = 0; e < MAXE; ++e) acc[e] = 0.f;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const float* p = probs + ((long long)b * T + t) * E;
#pragma unroll
        for (int e = 0; e < MAXE; ++e)
            if (e < E) acc[e] += p[e];
    }
#pragma unroll
    for (int e = 0; e < MAXE; ++e) red[threadIdx.x][e] = acc[e];
    __syncthreads();
    for (int st = blockDim.x / 2; st > 0; st >>= 1) {
        if ((int)threadIdx.x < st) {
#pragma unroll
            for (int e = 0; e < MAXE; ++e) red[threadIdx.x][e] += red[threadIdx.x + st][e];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const float mean = 1.0f / (float)E;
        float cv2 = 0.f;
        for (int e = 0; e < E; ++e) {
            const float l = red[0][e] / (float)T;
            load[b * E + e] = l;
            cv2 += (l - mean) * (l - mean);
        }
        cv2 /= mean * mean * (float)E;
        aux[b] = coef * cv2;
    }
}

__global__ void moe_add_aux_kernel(const float* __restrict__ aux, int layers, int B,
                                   float* __restrict__ loss) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    float s = 0.f;
    for (int l = 0; l < layers; ++l) {
        float sl = 0.f;
        for (int b = 0; b < B; ++b) sl += aux[l * B + b];
        s += sl / (float)B;
    }
    loss[0] += s;
}

// Warp per token. dw_j = dout . y_j; the expert-row gradient is w_j dout; then the
// renormalisation, aux-loss and softmax backward give the router-logit gradient (lane e
// handles expert e).
__global__ void moe_combine_bwd_kernel(const float* __restrict__ dout, const float* __restrict__ yg,
                                       const int* __restrict__ row_of, const int* __restrict__ idx,
                                       const float* __restrict__ wts,
                                       const float* __restrict__ ssum,
                                       const float* __restrict__ probs,
                                       const float* __restrict__ load, int rows, int T, int C,
                                       int E, int k, float coef, float aux_scale,
                                       bf16* __restrict__ dyg, float* __restrict__ dscores) {
    const int lane = threadIdx.x & 31;
    const int nv = C >> 2;
    for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < rows;
         t += (gridDim.x * blockDim.x) >> 5) {
        const float4* d4 = reinterpret_cast<const float4*>(dout + (long long)t * C);
        float dw[kMoeMaxTopK];
        int sel[kMoeMaxTopK];
        for (int j = 0; j < k; ++j) {
            const int r = row_of[(long long)t * k + j];
            const float w = wts[(long long)t * k + j];
            sel[j] = idx[(long long)t * k + j];
            const float4* y4 = reinterpret_cast<const float4*>(yg + (long long)r * C);
            uint2* o = reinterpret_cast<uint2*>(dyg + (long long)r * C);
            float dot = 0.f;
            for (int i = lane; i < nv; i += 32) {
                const float4 d = d4[i], v = y4[i];
                dot += d.x * v.x + d.y * v.y + d.z * v.z + d.w * v.w;
                o[i] = make_uint2(pack_bf16x2(w * d.x, w * d.y), pack_bf16x2(w * d.z, w * d.w));
            }
            dw[j] = wsum(dot);
        }
        const float s = ssum[t];
        float st = 0.f;
        for (int j = 0; j < k; ++j) st += dw[j] * probs[(long long)t * E + sel[j]];
        const float mean = 1.0f / (float)E;
        const int b = t / T;
        float p = 0.f, dp = 0.f;
        if (lane < E) {
            p = probs[(long long)t * E + lane];
            dp = aux_scale * coef * 2.0f * (load[b * E + lane] - mean) / (mean * mean * (float)E) /
                 (float)T;
            for (int j = 0; j < k; ++j)
                if (sel[j] == lane) dp += dw[j] / s - st / (s * s);
        }
        const float pd = wsum(lane < E ? dp * p : 0.f);
        if (lane < E) dscores[(long long)t * E + lane] = p * (dp - pd);
    }
}

__global__ void moe_zero_pad_kernel(const int* __restrict__ grp, int E, int C, int ld,
                                    bf16* __restrict__ buf) {
    const int e = blockIdx.y;
    const int row = grp[e] + grp[E + 1 + e] + blockIdx.x;
    if (row >= grp[e + 1]) return;
    uint4* o = reinterpret_cast<uint4*>(buf + (long long)row * ld);
    for (int i = threadIdx.x; i < (C >> 3); i += blockDim.x) o[i] = make_uint4(0u, 0u, 0u, 0u);
}

__global__ void __launch_bounds__(256)
    moe_scatter_sum_kernel(const float* __restrict__ dxg, const int* __restrict__ row_of,
                           const float* __restrict__ dscores, const float* __restrict__ gate,
                           int rows, int C, int E, int k, float* __restrict__ dln) {
    extern __shared__ float sgT[];
    load_gate_t(gate, C, E, sgT);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int nv = C >> 2;
    for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < rows;
         t += (gridDim.x * blockDim.x) >> 5) {
        int r[kMoeMaxTopK];
        for (int j = 0; j < k; ++j) r[j] = row_of[(long long)t * k + j];
        const float* ds = dscores + (long long)t * E;
        float4* o4 = reinterpret_cast<float4*>(dln + (long long)t * C);
        for (int i = lane; i < nv; i += 32) {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int j = 0; j < k; ++j) {
                const float4 v = reinterpret_cast<const float4*>(dxg + (long long)r[j] * C)[i];
                a.x += v.x;
                a.y += v.y;
                a.z += v.z;
                a.w += v.w;
            }
            for (int e = 0; e < E; ++e) {
                const float d = ds[e];
                const float4 w = reinterpret_cast<const float4*>(sgT + e * C)[i];
                a.x += d * w.x;
                a.y += d * w.y;
                a.z += d * w.z;
                a.w += d * w.w;
            }
            o4[i] = a;
        }
    }
}

template <int MAXE>
__global__ void __launch_bounds__(256)
    moe_gate_grad_kernel(const float* __restrict__ y, const float* __restrict__ mean,
                         const float* __restrict__ rstd, const float* __restrict__ gamma,
                         const float* __restrict__ beta, int rms,
                         const float* __restrict__ dscores, int rows, int C, int E,
                         float* __restrict__ part) {
    __shared__ float sd[kGateChunk][MAXE];
    __shared__ float smu[kGateChunk], sr[kGateChunk];
    const int r0 = blockIdx.x * kGateChunk;
    const int nr = min(kGateChunk, rows - r0);
    for (int i = threadIdx.x; i < nr * E; i += blockDim.x) {
        const int rr = i / E, e = i - rr * E;
        sd[rr][e] = dscores[(long long)(r0 + rr) * E + e];
    }
    for (int i = threadIdx.x; i < nr; i += blockDim.x) {
        smu[i] = mean[r0 + i];
        sr[i] = rstd[r0 + i];
    }
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float acc[MAXE];
#pragma unroll
        for (int e = 0; e < MAXE; ++e) acc[e] = 0.f;
        const float g = gamma[c];
        const float bb = (beta && !rms) ? beta[c] : 0.f;
        for (int i = 0; i < nr; ++i) {
            const float l = (y[(long long)(r0 + i) * C + c] - smu[i]) * sr[i] * g + bb;
#pragma unroll
            for (int e = 0; e < MAXE; ++e)
                if (e < E) acc[e] += l * sd[i][e];
        }
        float* o = part + ((long long)blockIdx.x * C + c) * E;
#pragma unroll
        for (int e = 0; e < MAXE; ++e)
            if (e < E) o[e] = acc[e];
    }
}

__global__ void moe_gate_reduce_kernel(const float* __restrict__ part, int nparts, int n,
                                       float* __restrict__ out, int accumulate) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float s = 0.f;
    for (int p = 0; p < nparts; ++p) s += part[(long long)p * n + i];
    out[i] = accumulate ? out[i] + s : s;
}

int grid_for_warps(long long warps) {
    long long b = (warps + 7) / 8;
    if (b > 148 * 16) b = 148 * 16;
    return (int)(b < 1 ? 1 : b);
}

bool dims_ok(const MoeDims& m) {
    return m.E >= 1 && m.E <= kMoeMaxExperts && m.k >= 1 && m.k <= kMoeMaxTopK && m.k <= m.E &&
           m.C > 0 && (m.C % 8) == 0 && m.B > 0 && m.T > 0;
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return 0;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) ==
                   cudaSuccess
               ? 0
               : -3;
}

}  // namespace

int moe_gate_grad_parts(int rows) { return (rows + kGateChunk - 1) / kGateChunk; }

int moe_router_forward(const MoeDims& m, const float* y, const float* mean, const float* rstd,
                       const float* gamma, const float* beta, int rms, const float* gate,
                       float* probs, int* idx, float* wts, float* ssum, cudaStream_t s) {
    if (!dims_ok(m)) return -1;
    const int rows = m.B * m.T;
    const size_t smem = (size_t)m.C * m.E * sizeof(float);
    if (smem > 200 * 1024) return -2;
    const int grid = (int)std::min<long long>((rows + 7) / 8, 148 * 8);
    if (m.E <= 8) {
        if (set_smem(moe_router_kernel<8>, smem)) return -3;
        moe_router_kernel<8><<<grid, 256, smem, s>>>(y, mean, rstd, gamma, beta, rms, gate, rows,
                                                      m.C, m.E, m.k, probs, idx, wts, ssum);
    } else {
        if (set_smem(moe_router_kernel<16>, smem)) return -3;
        moe_router_kernel<16><<<grid, 256, smem, s>>>(y, mean, rstd, gamma, beta, rms, gate,
                                                       rows, m.C, m.E, m.k, probs, idx, wts, ssum);
    }
    return launch_status();
}

int moe_dispatch(const MoeDims& m, const int* idx, int* grp, int* row_of, int* tok_of,
                 cudaStream_t s) {
    if (!dims_ok(m)) return -1;
    const int A = m.B * m.T * m.k;
    if (m.cap < moe_capacity(m.B * m.T, m.E, m.k)) return -2;
    moe_dispatch_kernel<<<1, 1024, 0, s>>>(idx, A, m.k, m.E, grp, row_of, tok_of);
    return launch_status();
}

int moe_gather(const MoeDims& m, const bf16* x, const int* tok_of, const int* grp, bf16* xg,
               cudaStream_t s) {
    if (!dims_ok(m)) return -1;
    moe_gather_kernel<<<grid_for_warps(m.cap), 256, 0, s>>>(x, tok_of, grp, m.E, m.C, xg);
    return launch_status();
}

int moe_combine(const MoeDims& m, const float* resid, const float* yg, const int* row_of,
                const float* wts, float* out, cudaStream_t s) {
    if (!dims_ok(m)) return -1;
    const int rows = m.B * m.T;
    moe_combine_kernel<<<grid_for_warps(rows), 256, 0, s>>>(resid, yg, row_of, wts, rows, m.C,
                                                             m.k, out);
    return launch_status();
}

int moe_aux_forward(const MoeDims& m, const float* probs, float coef, float* load, float* aux,
                    cudaStream_t s) {
    if (!dims_ok(m)) return -1;
    if (m.E <= 8)
        moe_aux_kernel<8><<<m.B, 256, 0, s>>>(probs, m.T, m.E, coef, load, aux);
    else
        moe_aux_kernel<16><<<m.B, 256, 0, s>>>(probs, m.T, m.E, coef, load, aux);
    return launch_status();
}

int moe_add_aux(const float* aux, int layers, int B, float* loss, cudaStream_t s) {
    moe_add_aux_kernel<<<1, 32, 0, s>>>(aux, layers, B, loss);
    return launch_status();
}

int moe_combine_backward(const MoeDims& m, const float* dout, const float* yg, const int* row_of,
                         const int* idx, const float* wts, const float* ssum, const float* probs,
                         const float* load, float coef, float aux_scale, bf16* dyg,
                         float* dscores, cudaStream_t s) {
    if (!dims_ok(m)) return -1;
    const int rows = m.B * m.T;
    moe_combine_bwd_kernel<<<grid_for_warps(rows), 256, 0, s>>>(
        dout, yg, row_of, idx, wts, ssum, probs, load, rows, m.T, m.C, m.E, m.k, coef, aux_scale,
        dyg, dscores);
    return launch_status();
}

int moe_zero_pad_rows(const MoeDims& m, const int* grp, bf16* buf, int ld, cudaStream_t s) {
    if (!dims_ok(m) || (ld % 8) != 0) return -1;
    dim3 grid(kMoeRowAlign, m.E);
    moe_zero_pad_kernel<<<grid, 128, 0, s>>>(grp, m.E, ld, ld, buf);
    return launch_status();
}

int moe_scatter_sum(const MoeDims& m, const float* dxg, const int* row_of, const float* dscores,
                    const float* gate, float* dln, cudaStream_t s) {
    if (!dims_ok(m)) return -1;
    const int rows = m.B * m.T;
    const size_t smem = (size_t)m.C * m.E * sizeof(float);
    if (smem > 200 * 1024) return -2;
    if (set_smem(moe_scatter_sum_kernel, smem)) return -3;
    const int grid = (int)std::min<long long>((rows + 7) / 8, 148 * 8);
    moe_scatter_sum_kernel<<<grid, 256, smem, s>>>(dxg, row_of, dscores, gate, rows, m.C, m.E,
                                                    m.k, dln);
    return launch_status();
}

int moe_gate_grad(const MoeDims& m, const float* y, const float* mean, const float* rstd,
                  const float* gamma, const float* beta, int rms, const float* dscores,
                  float* part, float* dgate, int accumulate, cudaStream_t s) {
    if (!dims_ok(m)) return -1;
    const int rows = m.B * m.T;
    const int np = moe_gate_grad_parts(rows);
    if (m.E <= 8)
        moe_gate_grad_kernel<8><<<np, 256, 0, s>>>(y, mean, rstd, gamma, beta, rms, dscores, rows,
                                                   m.C, m.E, part);
    else
        moe_gate_grad_kernel<16><<<np, 256, 0, s>>>(y, mean, rstd, gamma, beta, rms, dscores,
                                                    rows, m.C, m.E, part);
    int rc = launch_status();
    if (rc) return rc;
    const int n = m.C * m.E;
    moe_gate_reduce_kernel<<<(n + 255) / 256, 256, 0, s>>>(part, np, n, dgate, accumulate);
    return launch_status();
}

}  // namespace llmgpu
