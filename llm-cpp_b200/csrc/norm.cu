// LayerNorm / RMSNorm forward (warp per row, 128-bit loads) and backward (rows streamed
// through a shared-memory ring by bulk copies up to 1024 columns, warp per row above),
// deterministic two-stage column reductions for the norm-parameter and bias gradients.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace llmgpu {

namespace {

constexpr float kNormEps = 1e-5f;  // include/llm/tensor.h:68-69

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <int MAXV>
__global__ void __launch_bounds__(256) norm_fwd_kernel(const float* __restrict__ x,
                                                       const float* __restrict__ gamma,
                                                       const float* __restrict__ beta,
                                                       bf16* __restrict__ y, float* __restrict__ mean,
                                                       float* __restrict__ rstd, int rows, int C,
                                                       int rms) {
    pdl_enter();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int nv = C >> 2;
    const float4* xr = reinterpret_cast<const float4*>(x + (long long)row * C);
    float4 v[MAXV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + i * 32;
        if (idx < nv) {
            v[i] = xr[idx];
            s += v[i].x + v[i].y + v[i].z + v[i].w;
        } else {
            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    s = warp_sum(s);
    const float mu = rms ? 0.f : s / (float)C;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + i * 32;
        if (idx < nv) {
            float a = v[i].x - mu, b = v[i].y - mu, c = v[i].z - mu, d = v[i].w - mu;
            ss += a * a + b * b + c * c + d * d;
        }
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)C + kNormEps);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    const float4* b4 = reinterpret_cast<const float4*>(beta);
    uint2* yr = reinterpret_cast<uint2*>(y + (long long)row * C);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + i * 32;
        if (idx < nv) {
            float4 g = g4[idx];
            float4 b = (beta && !rms) ? b4[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
            float o0 = (v[i].x - mu) * r * g.x + b.x;
            float o1 = (v[i].y - mu) * r * g.y + b.y;
            float o2 = (v[i].z - mu) * r * g.z + b.z;
            float o3 = (v[i].w - mu) * r * g.w + b.w;
            yr[idx] = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
        }
    }
    if (lane == 0) {
        mean[row] = mu;
        rstd[row] = r;
    }
}

__device__ __forceinline__ void add4(float4* p, float a, float b, float c, float d) {
    float4 v = *p;
    v.x += a;
    v.y += b;
    v.z += c;
    v.w += d;
    *p = v;
}

// Column partial sums (dgamma, dbeta, colsum of dx) accumulate per warp in shared memory
// ([8 warps][3][C] floats), which keeps registers low enough for several CTAs per SM.
template <int MAXV>
__global__ void __launch_bounds__(256) norm_bwd_kernel(
    const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ gamma,
    const float* __restrict__ mean, const float* __restrict__ rstd,
    const float* __restrict__ resid_in, float* __restrict__ dx_f32, bf16* __restrict__ dx_bf16,
    float* __restrict__ partial, int rows, int C, int rms) {
    pdl_enter();
    extern __shared__ float red[];  // [8][3][C]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps_total = gridDim.x * 8;
    const int nv = C >> 2;
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    for (int i = threadIdx.x; i < 8 * 3 * C; i += blockDim.x) red[i] = 0.f;
    __syncthreads();
    float4* sg = reinterpret_cast<float4*>(red + (warp * 3 + 0) * C);
    float4* sb = reinterpret_cast<float4*>(red + (warp * 3 + 1) * C);
    float4* so = reinterpret_cast<float4*>(red + (warp * 3 + 2) * C);
    const float invC = 1.0f / (float)C;
    for (int row = blockIdx.x * 8 + warp; row < rows; row += nwarps_total) {
        const float4* dyr = reinterpret_cast<const float4*>(dy + (long long)row * C);
        const float4* xr = reinterpret_cast<const float4*>(x + (long long)row * C);
        const float mu = mean[row], r = rstd[row];
        float s1 = 0.f, s2 = 0.f;
        float4 d[MAXV], xv[MAXV], rv[MAXV];
        const float4* rin = reinterpret_cast<const float4*>(resid_in + (long long)row * C);
        // every load of the row is issued before the reductions need the first of them
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int idx = lane + i * 32;
            if (idx < nv) {
                d[i] = dyr[idx];
                xv[i] = xr[idx];
                rv[i] = resid_in ? rin[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int idx = lane + i * 32;
            if (idx < nv) {
                float4 g = g4[idx];
                if (!rms) {
                    float gx = d[i].x * g.x, gy = d[i].y * g.y, gz = d[i].z * g.z,
                          gw = d[i].w * g.w;
                    s1 += gx + gy + gz + gw;
                    s2 += gx * (xv[i].x - mu) * r + gy * (xv[i].y - mu) * r +
                          gz * (xv[i].z - mu) * r + gw * (xv[i].w - mu) * r;
                } else {
                    s2 += d[i].x * g.x * xv[i].x + d[i].y * g.y * xv[i].y +
                          d[i].z * g.z * xv[i].z + d[i].w * g.w * xv[i].w;
                }
            }
        }
        s1 = warp_sum(s1);
        s2 = warp_sum(s2);
        const float m1 = s1 * invC, m2 = s2 * invC;
        const float coef = rms ? s2 * r * r * r * invC : 0.f;
        float4* o32 = reinterpret_cast<float4*>(dx_f32 + (long long)row * C);
        uint2* o16 = dx_bf16 ? reinterpret_cast<uint2*>(dx_bf16 + (long long)row * C) : nullptr;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int idx = lane + i * 32;
            if (idx < nv) {
                float4 g = g4[idx];
                float dd[4] = {d[i].x, d[i].y, d[i].z, d[i].w};
                float xx[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
                float gg[4] = {g.x, g.y, g.z, g.w};
                float o[4], xh[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    xh[k] = (xx[k] - mu) * r;
                    if (!rms)
                        o[k] = r * (dd[k] * gg[k] - m1 - xh[k] * m2);
                    else
                        o[k] = dd[k] * gg[k] * r - xx[k] * coef;
                }
                o[0] += rv[i].x;
                o[1] += rv[i].y;
                o[2] += rv[i].z;
                o[3] += rv[i].w;
                o32[idx] = make_float4(o[0], o[1], o[2], o[3]);
                if (o16) o16[idx] = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
                add4(sg + idx, dd[0] * xh[0], dd[1] * xh[1], dd[2] * xh[2], dd[3] * xh[3]);
                add4(sb + idx, dd[0], dd[1], dd[2], dd[3]);
                add4(so + idx, o[0], o[1], o[2], o[3]);
            }
        }
    }
    // CTA-level reduction of the three partial planes (fixed order: warp 0..7)
    __syncthreads();
    for (int i = threadIdx.x; i < 3 * C; i += blockDim.x) {
        const int plane = i / C, c = i - plane * C;
        float acc = 0.f;
        for (int w = 0; w < 8; ++w) acc += red[(w * 3 + plane) * C + c];
        partial[((long long)blockIdx.x * 3 + plane) * C + c] = acc;
    }
}

// The same backward with its inputs streamed through a ring of shared-memory stages by bulk
// copies: one CTA per SM, a stage holds a group of 8 consecutive rows of dy, x and the
// incoming residual gradient (three contiguous copies), and up to kNbStages - 1 groups are
// in flight while the 8 warps work on the current one (a warp per row). The per-row work
// alone kept too few bytes in flight to cover DRAM latency. Column partial sums stay in
// registers across the CTA's rows (a lane owns fixed 4-column groups) and meet once, in
// warp order, at the end: partial[blockIdx.x][3][C], the layout of norm_bwd_kernel.
// dx may alias resid_in: a row is read (copied) before it is written, by the same CTA.
constexpr int kNbStages = 4;
constexpr int kNbRows = 8;  // rows per group = warps per CTA

template <int MAXV>
__global__ void __launch_bounds__(256, 1) norm_bwd_ring_kernel(
    const float* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ gamma,
    const float* __restrict__ mean, const float* __restrict__ rstd, const float* resid_in,
    float* dx_f32, bf16* __restrict__ dx_bf16, float* __restrict__ partial, int rows, int C,
    int rms, int nstages, int* err) {
    pdl_enter();
    extern __shared__ __align__(128) uint8_t nb_smem[];  // nstages x [3][8][C] floats
    __shared__ __align__(8) uint64_t bar[kNbStages];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nv = C >> 2;
    const int ngroups = (rows + kNbRows - 1) / kNbRows;
    const size_t plane = (size_t)kNbRows * C;  // floats of one tensor in a stage
    float* stages = reinterpret_cast<float*>(nb_smem);
    const bool has_resid = resid_in != nullptr;
    auto issue = [&](int g, int st) {  // thread 0: copy group g into stage st
        const int r0 = g * kNbRows;
        const int nr = min(kNbRows, rows - r0);
        const uint32_t bytes = (uint32_t)nr * (uint32_t)C * 4u;
        float* dst = stages + (size_t)st * 3 * plane;
        mbar_arrive_expect_tx(&bar[st], bytes * (has_resid ? 3u : 2u));
        bulk_load_g2s(dst, dy + (size_t)r0 * C, bytes, &bar[st]);
        bulk_load_g2s(dst + plane, x + (size_t)r0 * C, bytes, &bar[st]);
        if (has_resid) bulk_load_g2s(dst + 2 * plane, resid_in + (size_t)r0 * C, bytes, &bar[st]);
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < nstages; ++s) mbar_init(&bar[s], 1);
        fence_barrier_init();
        for (int j = 0, g = blockIdx.x; j < nstages && g < ngroups; ++j, g += gridDim.x)
            issue(g, j);
    }
    float4 gv[MAXV], pg[MAXV], pb[MAXV], po[MAXV];
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + i * 32;
        gv[i] = idx < nv ? g4[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
        pg[i] = pb[i] = po[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    const float invC = 1.0f / (float)C;
    int st = 0;
    uint32_t phase = 0;
    for (int g = blockIdx.x; g < ngroups; g += gridDim.x) {
        const int row = g * kNbRows + warp;
        float mu = 0.f, r = 0.f;
        if (row < rows) {
            mu = mean[row];
            r = rstd[row];
        }
        mbar_wait_bounded(&bar[st], phase, err, kDevTimeoutFull);
        if (row < rows) {
            const float* base = stages + (size_t)st * 3 * plane + (size_t)warp * C;
            const float4* sd = reinterpret_cast<const float4*>(base);
            const float4* sx = reinterpret_cast<const float4*>(base + plane);
            const float4* sr = reinterpret_cast<const float4*>(base + 2 * plane);
            float s1 = 0.f, s2 = 0.f;
#pragma unroll
            for (int i = 0; i < MAXV; ++i) {
                const int idx = lane + i * 32;
                if (idx < nv) {
                    const float4 d = sd[idx], xv = sx[idx], g = gv[i];
                    const float gx = d.x * g.x, gy = d.y * g.y, gz = d.z * g.z, gw = d.w * g.w;
                    if (!rms) {
                        s1 += gx + gy + gz + gw;
                        s2 += gx * (xv.x - mu) * r + gy * (xv.y - mu) * r +
                              gz * (xv.z - mu) * r + gw * (xv.w - mu) * r;
                    } else {
                        s2 += gx * xv.x + gy * xv.y + gz * xv.z + gw * xv.w;
                    }
                }
            }
            s1 = warp_sum(s1);
            s2 = warp_sum(s2);
            const float m1 = s1 * invC, m2 = s2 * invC;
            const float coef = rms ? s2 * r * r * r * invC : 0.f;
            float4* o32 = reinterpret_cast<float4*>(dx_f32 + (size_t)row * C);
            uint2* o16 = dx_bf16 ? reinterpret_cast<uint2*>(dx_bf16 + (size_t)row * C) : nullptr;
#pragma unroll
            for (int i = 0; i < MAXV; ++i) {
                const int idx = lane + i * 32;
                if (idx < nv) {
                    const float4 d4 = sd[idx], x4 = sx[idx], g4v = gv[i];
                    const float4 r4 = has_resid ? sr[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
                    const float dd[4] = {d4.x, d4.y, d4.z, d4.w};
                    const float xx[4] = {x4.x, x4.y, x4.z, x4.w};
                    const float gg[4] = {g4v.x, g4v.y, g4v.z, g4v.w};
                    const float rr[4] = {r4.x, r4.y, r4.z, r4.w};
                    float o[4], xh[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        xh[k] = (xx[k] - mu) * r;
                        if (!rms)
                            o[k] = r * (dd[k] * gg[k] - m1 - xh[k] * m2);
                        else
                            o[k] = dd[k] * gg[k] * r - xx[k] * coef;
                        o[k] += rr[k];
                    }
                    o32[idx] = make_float4(o[0], o[1], o[2], o[3]);
                    if (o16) o16[idx] = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
                    pg[i].x += dd[0] * xh[0];
                    pg[i].y += dd[1] * xh[1];
                    pg[i].z += dd[2] * xh[2];
                    pg[i].w += dd[3] * xh[3];
                    pb[i].x += dd[0];
                    pb[i].y += dd[1];
                    pb[i].z += dd[2];
                    pb[i].w += dd[3];
                    po[i].x += o[0];
                    po[i].y += o[1];
                    po[i].z += o[2];
                    po[i].w += o[3];
                }
            }
        }
        __syncthreads();  // every warp is done with this stage
        if (threadIdx.x == 0) {
            const int gn = g + nstages * gridDim.x;
            if (gn < ngroups) issue(gn, st);
        }
        if (++st == nstages) {
            st = 0;
            phase ^= 1u;
        }
    }
    // Every copy issued was waited for: the stages are free for the CTA reduction,
    // [8 warps][3][C] floats (one stage's size).
    float4* red = reinterpret_cast<float4*>(stages);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int idx = lane + i * 32;
        if (idx < nv) {
            red[(warp * 3 + 0) * nv + idx] = pg[i];
            red[(warp * 3 + 1) * nv + idx] = pb[i];
            red[(warp * 3 + 2) * nv + idx] = po[i];
        }
    }
    __syncthreads();
    float4* out = reinterpret_cast<float4*>(partial + (size_t)blockIdx.x * 3 * C);
    for (int i = threadIdx.x; i < 3 * nv; i += blockDim.x) {
        const int p = i / nv, c = i - p * nv;
        float4 acc = red[p * nv + c];
        for (int w = 1; w < kNbRows; ++w) {
            const float4 v = red[(w * 3 + p) * nv + c];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        out[i] = acc;  // i = p * nv + c: plane p, columns 4c..4c+3
    }
}

// Sums nparts partial rows of C floats: out_y[c] = sum_p part[p * pstride + y * plane_off + c]
// for planes y = blockIdx.y (a null output skips its plane). A block is 32 columns x 32 part
// groups; group g adds parts g, g + 32, ... in order with four loads in flight, then the 32
// group sums are added in group order: a fixed order, so the result is deterministic.
__global__ void __launch_bounds__(1024) sum_parts_kernel(const float* __restrict__ part,
                                                         int nparts, long long pstride,
                                                         long long plane_off, int C, float* out0,
                                                         float* out1, float* out2,
                                                         int accumulate) {
    pdl_enter();
    __shared__ float red[32][33];
    const int plane = blockIdx.y;
    float* out = plane == 0 ? out0 : (plane == 1 ? out1 : out2);
    if (!out) return;  // uniform across the block
    const int cc = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + cc;
    float acc = 0.f;
    if (c < C) {
        const float* base = part + plane * plane_off + c;
        int p = grp;
        for (; p + 96 < nparts; p += 128) {
            const float v0 = base[(long long)p * pstride];
            const float v1 = base[(long long)(p + 32) * pstride];
            const float v2 = base[(long long)(p + 64) * pstride];
            const float v3 = base[(long long)(p + 96) * pstride];
            acc += v0;
            acc += v1;
            acc += v2;
            acc += v3;
        }
        for (; p < nparts; p += 32) acc += base[(long long)p * pstride];
    }
    red[grp][cc] = acc;
    __syncthreads();
    if (grp == 0 && c < C) {
        float t = 0.f;
        for (int g = 0; g < 32; ++g) t += red[g][cc];
        out[c] = accumulate ? out[c] + t : t;
    }
}

constexpr int kColsumGroups = 256;

__global__ void colsum_stage1(const bf16* __restrict__ a, long long lda, int rows, int C,
                              float* __restrict__ work) {
    pdl_enter();
    // blockIdx.x: 2048-column tile (256 threads x 8 columns); blockIdx.y: row group
    const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (c0 >= C) return;
    const int rg = blockIdx.y;
    const int r0 = (int)((long long)rg * rows / kColsumGroups);
    const int r1 = (int)((long long)(rg + 1) * rows / kColsumGroups);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const bool vec = (c0 + 8 <= C) && ((lda & 7) == 0);
    if (vec) {
        // rows in batches of 8 with all 8 loads in flight, summed in row order
        int r = r0;
        for (; r + 8 <= r1; r += 8) {
            uint4 u[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                u[j] = *reinterpret_cast<const uint4*>(a + (long long)(r + j) * lda + c0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t w[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    acc[2 * k] += bf16_lo(w[k]);
                    acc[2 * k + 1] += bf16_hi(w[k]);
                }
            }
        }
        for (; r < r1; ++r) {
            const uint4 u = *reinterpret_cast<const uint4*>(a + (long long)r * lda + c0);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                acc[2 * k] += bf16_lo(w[k]);
                acc[2 * k + 1] += bf16_hi(w[k]);
            }
        }
    } else {
        for (int r = r0; r < r1; ++r) {
            const bf16* p = a + (long long)r * lda + c0;
            for (int k = 0; k < 8 && c0 + k < C; ++k) acc[k] += __bfloat162float(p[k]);
        }
    }
    for (int k = 0; k < 8 && c0 + k < C; ++k) work[(long long)rg * C + c0 + k] = acc[k];
}

}  // namespace

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
int sm_count() {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}
}  // namespace

int norm_forward(const float* x, const float* gamma, const float* beta, bf16* y, float* mean,
                 float* rstd, int rows, int C, int rms, cudaStream_t s) {
    if ((C & 3) != 0 || rows <= 0) return -1;
    const int blocks = (rows + 7) / 8;
    if (C <= 512)
        launch_kernel(norm_fwd_kernel<4>, blocks, 256, 0, s, x, gamma, beta, y, mean, rstd, rows, C, rms);
    else if (C <= 1024)
        launch_kernel(norm_fwd_kernel<8>, blocks, 256, 0, s, x, gamma, beta, y, mean, rstd, rows, C, rms);
    else if (C <= 2048)
        launch_kernel(norm_fwd_kernel<16>, blocks, 256, 0, s, x, gamma, beta, y, mean, rstd, rows, C, rms);
    else
        return -2;
    return launch_status();
}

int norm_backward_grid(int rows) {
    int g = (rows + 7) / 8;
    return g < 296 ? g : 296;
}

int norm_backward(const float* dy, const float* x, const float* gamma, const float* mean,
                  const float* rstd, const float* resid_in, float* dx_f32, bf16* dx_bf16,
                  float* partial, int rows, int C, int rms, int* nparts, cudaStream_t s,
                  int* err) {
    if ((C & 3) != 0 || rows <= 0 || C > 2048) return -1;
    // The ring kernel, where at least two stages of 8 rows fit in shared memory and every
    // bulk-copy source is 16-byte aligned (rows start at multiples of 16 bytes as C % 4 == 0).
    constexpr size_t kRingSmem = 226 * 1024;
    const size_t stage_bytes = 3 * (size_t)kNbRows * C * sizeof(float);
    const int nstages = (int)std::min<size_t>(kNbStages, kRingSmem / stage_bytes);
    if (C <= 1024 && nstages >= 2 && aligned16(dy) && aligned16(x) &&
        (!resid_in || aligned16(resid_in)) && aligned16(dx_f32) && aligned16(gamma)) {
        static bool ring_set = false;
        if (!ring_set) {
            const int mx = (int)kRingSmem;
            cudaFuncSetAttribute(norm_bwd_ring_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
            cudaFuncSetAttribute(norm_bwd_ring_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
            cudaFuncSetAttribute(norm_bwd_ring_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
            cudaFuncSetAttribute(norm_bwd_ring_kernel<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
            cudaFuncSetAttribute(norm_bwd_ring_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
            ring_set = true;
        }
        const int ngroups = (rows + kNbRows - 1) / kNbRows;
        const int grid = std::min(sm_count(), ngroups);  // never above norm_backward_grid(rows)
        // groups per CTA bound the stages; one stage still holds the final [8][3][C] sums
        const int nst = std::min(nstages, (ngroups + grid - 1) / grid);
        const size_t smem = (size_t)nst * stage_bytes;
        if (nparts) *nparts = grid;
#define NR_LAUNCH(MV)                                                                          \
    launch_kernel(norm_bwd_ring_kernel<MV>, grid, 256, smem, s, dy, x, gamma, mean, rstd,      \
                  resid_in, dx_f32, dx_bf16, partial, rows, C, rms, nst, err)
        if (C <= 128)
            NR_LAUNCH(1);
        else if (C <= 256)
            NR_LAUNCH(2);
        else if (C <= 512)
            NR_LAUNCH(4);
        else if (C <= 768)
            NR_LAUNCH(6);
        else
            NR_LAUNCH(8);
#undef NR_LAUNCH
        return launch_status();
    }
    const int grid = norm_backward_grid(rows);
    const size_t smem = 8 * 3 * (size_t)C * sizeof(float);
    if (nparts) *nparts = grid;
    static bool set = false;
    if (!set) {
        const int mx = 8 * 3 * 2048 * 4;
        cudaFuncSetAttribute(norm_bwd_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
        cudaFuncSetAttribute(norm_bwd_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
        cudaFuncSetAttribute(norm_bwd_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
        cudaFuncSetAttribute(norm_bwd_kernel<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
        cudaFuncSetAttribute(norm_bwd_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
        cudaFuncSetAttribute(norm_bwd_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
        set = true;
    }
#define NB_LAUNCH(MV)                                                                   \
    launch_kernel(norm_bwd_kernel<MV>, grid, 256, smem, s, dy, x, gamma, mean, rstd, resid_in, \
                  dx_f32, dx_bf16, partial, rows, C, rms)
    if (C <= 128)
        NB_LAUNCH(1);
    else if (C <= 256)
        NB_LAUNCH(2);
    else if (C <= 512)
        NB_LAUNCH(4);
    else if (C <= 768)
        NB_LAUNCH(6);
    else if (C <= 1024)
        NB_LAUNCH(8);
    else
        NB_LAUNCH(16);
#undef NB_LAUNCH
    return launch_status();
}

int reduce_partials(const float* partial, int nparts, int C, float* out0, float* out1,
                    float* out2, int accumulate, cudaStream_t s) {
    dim3 grid((C + 31) / 32, 3);  // partials are [part][3][C]
    launch_kernel(sum_parts_kernel, grid, 1024, 0, s, partial, nparts, 3LL * C, C, C, out0, out1, out2,
                                           accumulate);
    return launch_status();
}

size_t colsum_work_floats(int C) { return (size_t)kColsumGroups * C; }

int colsum_bf16(const bf16* a, long long lda, int rows, int C, float* out, int accumulate,
                float* work, cudaStream_t s) {
    dim3 g1((C + 2047) / 2048, kColsumGroups);
    launch_kernel(colsum_stage1, g1, 256, 0, s, a, lda, rows, C, work);
    launch_kernel(sum_parts_kernel, dim3((C + 31) / 32, 1), 1024, 0, s, work, kColsumGroups, C, 0, C, out,
                                                             nullptr, nullptr, accumulate);
    return launch_status();
}

}  // namespace llmgpu
