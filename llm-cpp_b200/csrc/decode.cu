// KV-cached decoding: one new token per sequence against the keys and values of all earlier
// positions, as GPT::generate runs the transformer incrementally (src/model.cpp:393-474,
// MultiHeadAttention::forward_incremental src/attention.cpp:104-181, KVCache
// src/kv_cache.cpp). Decode-shaped kernels: with one row per sequence the projections are
// matrix-vector products that stream each bf16 weight once (HBM-bound), and the attention of
// one query row runs a key per lane with an online softmax.
//
// Same arithmetic as the training forward: bf16 operands, fp32 accumulation, fp32 residual
// stream, bf16 keys and values (the prefill copies them from the forward's qkv activations).
#include <cfloat>

#include "common.cuh"
#include "kernels.cuh"
#include "model.h"

namespace llmgpu {

namespace {

constexpr int kDecMaxB = 8;         // sequences per decode step
constexpr int kGemvCols = 64;       // output columns per CTA (2 per lane)
constexpr int kGemvWarps = 4;       // warps splitting K

enum { kDecBF16 = 0, kDecResid = 1, kDecGelu = 2, kDecF32 = 3 };

// y[b, n] = epi(sum_k x[b, k] W[k, n]) for b < B; W [K, N] bf16 row-major (ldw elements).
// x (bf16 [B, K], ldx) is staged in shared memory as fp32; warp w sums rows k = w (mod 4)
// for 64 columns; the four partial sums meet in shared memory.
template <int EPI>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(
    const bf16* __restrict__ x, int ldx, const bf16* __restrict__ W, long long ldw, int K, int N,
    int B, void* __restrict__ out, long long ldo, const float* __restrict__ resid, long long ldr) {
    extern __shared__ float gsm[];  // [B][K] x, then [kGemvWarps][B][kGemvCols] partials
    float* xs = gsm;
    float* part = gsm + (size_t)B * K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kGemvCols;
    for (int i = threadIdx.x; i < B * K; i += blockDim.x) {
        const int b = i / K, k = i - b * K;
        xs[i] = __bfloat162float(x[(long long)b * ldx + k]);
    }
    __syncthreads();
    const int n = n0 + 2 * lane;
    float acc[kDecMaxB][2];
#pragma unroll
    for (int b = 0; b < kDecMaxB; ++b) acc[b][0] = acc[b][1] = 0.f;
    if (n < N) {
        const bf16* w = W + n;
        int k = warp;
        for (; k + 3 * kGemvWarps < K; k += 4 * kGemvWarps) {
            uint32_t wv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                wv[u] = *reinterpret_cast<const uint32_t*>(w + (long long)(k + u * kGemvWarps) * ldw);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float w0 = bf16_lo(wv[u]), w1 = bf16_hi(wv[u]);
#pragma unroll
                for (int b = 0; b < kDecMaxB; ++b)
                    if (b < B) {
                        const float xv = xs[b * K + k + u * kGemvWarps];
                        acc[b][0] = fmaf(xv, w0, acc[b][0]);
                        acc[b][1] = fmaf(xv, w1, acc[b][1]);
                    }
            }
        }
        for (; k < K; k += kGemvWarps) {
            const uint32_t wv = *reinterpret_cast<const uint32_t*>(w + (long long)k * ldw);
            const float w0 = bf16_lo(wv), w1 = bf16_hi(wv);
#pragma unroll
            for (int b = 0; b < kDecMaxB; ++b)
                if (b < B) {
                    acc[b][0] = fmaf(xs[b * K + k], w0, acc[b][0]);
                    acc[b][1] = fmaf(xs[b * K + k], w1, acc[b][1]);
                }
        }
    }
#pragma unroll
    for (int b = 0; b < kDecMaxB; ++b)
        if (b < B) {
            part[(warp * B + b) * kGemvCols + 2 * lane] = acc[b][0];
            part[(warp * B + b) * kGemvCols + 2 * lane + 1] = acc[b][1];
        }
    __syncthreads();
    for (int i = threadIdx.x; i < B * kGemvCols; i += blockDim.x) {
        const int b = i / kGemvCols, c = i - b * kGemvCols, nn = n0 + c;
        if (nn >= N) continue;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) v += part[(w * B + b) * kGemvCols + c];
        if constexpr (EPI == kDecBF16) {
            reinterpret_cast<bf16*>(out)[(long long)b * ldo + nn] = __float2bfloat16_rn(v);
        } else if constexpr (EPI == kDecGelu) {
            reinterpret_cast<bf16*>(out)[(long long)b * ldo + nn] = __float2bfloat16_rn(gelu_tanh(v));
        } else if constexpr (EPI == kDecResid) {
            reinterpret_cast<float*>(out)[(long long)b * ldo + nn] = resid[(long long)b * ldr + nn] + v;
        } else {
            reinterpret_cast<float*>(out)[(long long)b * ldo + nn] = v;
        }
    }
}

// y[b, n] = sum_k x[b, k] W[n, k] (the tied head: W = wte [N, K] bf16); a warp per output
// row n reads the row once, 8 elements per lane at a time.
__global__ void __launch_bounds__(256) gemv_t_kernel(const bf16* __restrict__ x, int ldx,
                                                     const bf16* __restrict__ W, long long ldw,
                                                     int K, int N, int B,
                                                     float* __restrict__ out, long long ldo) {
    extern __shared__ float gsm[];  // [B][K]
    for (int i = threadIdx.x; i < B * K; i += blockDim.x) {
        const int b = i / K, k = i - b * K;
        gsm[i] = __bfloat162float(x[(long long)b * ldx + k]);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + warp;
    if (n >= N) return;
    const bf16* w = W + (long long)n * ldw;
    float acc[kDecMaxB];
#pragma unroll
    for (int b = 0; b < kDecMaxB; ++b) acc[b] = 0.f;
    for (int k = 8 * lane; k < K; k += 256) {
        const uint4 u = *reinterpret_cast<const uint4*>(w + k);
        const float wv[8] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y),
                             bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w)};
#pragma unroll
        for (int b = 0; b < kDecMaxB; ++b)
            if (b < B) {
                const float* xb = gsm + b * K + k;
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[b] = fmaf(xb[j], wv[j], acc[b]);
            }
    }
#pragma unroll
    for (int b = 0; b < kDecMaxB; ++b) {
        float v = acc[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && b < B) out[(long long)b * ldo + n] = v;
    }
}

// x[b] = wte[tok_b mod V] + wpe[pos], rotated by rope_cfg's (cos, sin) of position `pos` when
// given (src/model.cpp:149-158; apply_rope_incremental :119-139 is the same rotation).
__global__ void embed_decode_kernel(const int32_t* __restrict__ tokens, const float* __restrict__ wte,
                                    const float* __restrict__ wpe, float* __restrict__ x, int C,
                                    int V, int pos, const float2* __restrict__ rope,
                                    float rope_scale) {
    const int b = blockIdx.x;
    int tok = tokens[b] % V;
    if (tok < 0) tok += V;
    for (int j = 2 * threadIdx.x; j < C; j += 2 * blockDim.x) {
        float v0 = wte[(long long)tok * C + j] + wpe[(long long)pos * C + j];
        float v1 = wte[(long long)tok * C + j + 1] + wpe[(long long)pos * C + j + 1];
        if (rope) {
            const float2 cs = rope[(long long)pos * (C / 2) + j / 2];
            const float r0 = (v0 * cs.x - v1 * cs.y) * rope_scale;
            const float r1 = (v0 * cs.y + v1 * cs.x) * rope_scale;
            v0 = r0;
            v1 = r1;
        }
        x[(long long)b * C + j] = v0;
        x[(long long)b * C + j + 1] = v1;
    }
}

// Keys and values of B prompts of T tokens (the forward's qkv rows) into the caches
// [max_t][C] per sequence.
__global__ void kv_fill_kernel(const bf16* __restrict__ qkv, bf16* __restrict__ kc,
                               bf16* __restrict__ vc, int B, int T, int C, int max_t) {
    const long long n = (long long)B * T * (C / 8);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / (C / 8);
        const int c8 = (int)(i - row * (C / 8)) * 8;
        const int b = (int)(row / T), t = (int)(row - (long long)b * T);
        const bf16* src = qkv + row * 3 * C + c8;
        const long long dst = ((long long)b * max_t + t) * C + c8;
        *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(src + C);
        *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(src + 2 * C);
    }
}

// One query row per (head, sequence) against cached keys 0..pos (the new token's key and value
// are appended at pos first). Lane-parallel over keys: each lane scores its own keys with an
// online softmax and accumulates its p V; lanes, then warps, merge (max, sum, output).
template <int HD>
__global__ void __launch_bounds__(256) attn_decode_kernel(const bf16* __restrict__ qkv,
                                                          bf16* __restrict__ kc,
                                                          bf16* __restrict__ vc,
                                                          bf16* __restrict__ out, int H,
                                                          int max_t, int pos, float scale_log2) {
    const int h = blockIdx.x, b = blockIdx.y, C = H * HD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kW = 8;
    __shared__ float q[HD];
    __shared__ float wm[kW], wl[kW];
    __shared__ float wo[kW][HD];
    const bf16* row = qkv + (long long)b * 3 * C + h * HD;
    bf16* kb = kc + (long long)b * max_t * C + h * HD;
    bf16* vb = vc + (long long)b * max_t * C + h * HD;
    if (threadIdx.x < HD) {
        q[threadIdx.x] = __bfloat162float(row[threadIdx.x]) * scale_log2;
        kb[(long long)pos * C + threadIdx.x] = row[C + threadIdx.x];
        vb[(long long)pos * C + threadIdx.x] = row[2 * C + threadIdx.x];
    }
    __syncthreads();
    float m = -FLT_MAX, l = 0.f, o[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) o[d] = 0.f;
    for (int j = warp * 32 + lane; j <= pos; j += kW * 32) {
        const uint4* kr = reinterpret_cast<const uint4*>(kb + (long long)j * C);
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) {
            const uint4 u = kr[c];
            s = fmaf(q[8 * c], bf16_lo(u.x), s);
            s = fmaf(q[8 * c + 1], bf16_hi(u.x), s);
            s = fmaf(q[8 * c + 2], bf16_lo(u.y), s);
            s = fmaf(q[8 * c + 3], bf16_hi(u.y), s);
            s = fmaf(q[8 * c + 4], bf16_lo(u.z), s);
            s = fmaf(q[8 * c + 5], bf16_hi(u.z), s);
            s = fmaf(q[8 * c + 6], bf16_lo(u.w), s);
            s = fmaf(q[8 * c + 7], bf16_hi(u.w), s);
        }
        // s is the score in base 2 (q carries scale * log2 e)
        if (s > m) {
            const float a = ex2_approx(m - s);
            l *= a;
#pragma unroll
            for (int d = 0; d < HD; ++d) o[d] *= a;
            m = s;
        }
        const float p = ex2_approx(s - m);
        l += p;
        const uint4* vr = reinterpret_cast<const uint4*>(vb + (long long)j * C);
#pragma unroll
        for (int c = 0; c < HD / 8; ++c) {
            const uint4 u = vr[c];
            o[8 * c] = fmaf(p, bf16_lo(u.x), o[8 * c]);
            o[8 * c + 1] = fmaf(p, bf16_hi(u.x), o[8 * c + 1]);
            o[8 * c + 2] = fmaf(p, bf16_lo(u.y), o[8 * c + 2]);
            o[8 * c + 3] = fmaf(p, bf16_hi(u.y), o[8 * c + 3]);
            o[8 * c + 4] = fmaf(p, bf16_lo(u.z), o[8 * c + 4]);
            o[8 * c + 5] = fmaf(p, bf16_hi(u.z), o[8 * c + 5]);
            o[8 * c + 6] = fmaf(p, bf16_lo(u.w), o[8 * c + 6]);
            o[8 * c + 7] = fmaf(p, bf16_hi(u.w), o[8 * c + 7]);
        }
    }
    // merge the lanes of the warp
    float mw = m;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, off));
    const float a = l > 0.f ? ex2_approx(m - mw) : 0.f;
    l *= a;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
#pragma unroll
    for (int d = 0; d < HD; ++d) {
        float v = o[d] * a;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        o[d] = v;
    }
    if (lane == 0) {
        wm[warp] = mw;
        wl[warp] = l;
#pragma unroll
        for (int d = 0; d < HD; ++d) wo[warp][d] = o[d];
    }
    __syncthreads();
    if (threadIdx.x < HD) {
        float M = -FLT_MAX;
#pragma unroll
        for (int w = 0; w < kW; ++w)
            if (wl[w] > 0.f) M = fmaxf(M, wm[w]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kW; ++w)
            if (wl[w] > 0.f) {
                const float f = ex2_approx(wm[w] - M);
                L += wl[w] * f;
                O += wo[w][threadIdx.x] * f;
            }
        out[(long long)b * C + h * HD + threadIdx.x] = __float2bfloat16_rn(O / L);
    }
}

template <int EPI>
int gemv(const bf16* x, int ldx, const bf16* W, long long ldw, int K, int N, int B, void* out,
         long long ldo, const float* resid, long long ldr, cudaStream_t s) {
    const size_t smem = sizeof(float) * ((size_t)B * K + (size_t)kGemvWarps * B * kGemvCols);
    if (B < 1 || B > kDecMaxB || (N & 1) || (ldw & 1) || smem > 200 * 1024) return -1;
    static bool set = false;
    if (!set) {
        cudaFuncSetAttribute(gemv_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024);
        set = true;
    }
    gemv_kernel<EPI><<<(N + kGemvCols - 1) / kGemvCols, kGemvWarps * 32, smem, s>>>(
        x, ldx, W, ldw, K, N, B, out, ldo, resid, ldr);
    return launch_status();
}

int gemv_t(const bf16* x, int ldx, const bf16* W, long long ldw, int K, int N, int B, float* out,
           long long ldo, cudaStream_t s) {
    const size_t smem = sizeof(float) * (size_t)B * K;
    if (B < 1 || B > kDecMaxB || (K & 7) || (ldw & 7) || smem > 200 * 1024) return -1;
    static bool set = false;
    if (!set) {
        cudaFuncSetAttribute(gemv_t_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024);
        set = true;
    }
    gemv_t_kernel<<<(N + 7) / 8, 256, smem, s>>>(x, ldx, W, ldw, K, N, B, out, ldo);
    return launch_status();
}

#define DK(call)                                                                        \
    do {                                                                                \
        const int _rc = (call);                                                         \
        if (_rc) {                                                                      \
            c->err = std::string("decode kernel launch failed: ") + #call + " -> " +   \
                     std::to_string(_rc);                                               \
            return LLMGPU_E_CUDA;                                                       \
        }                                                                               \
    } while (0)

}  // namespace

int decode_supported(const Ctx* c, std::string* why) {
    const auto& k = c->cfg;
    if (k.use_mamba || c->moe || c->swiglu || k.rope_qk) {
        *why = "KV-cached decoding covers the reference's transformer GPT (GELU FFN, attention "
               "without RoPE on Q/K); this configuration decodes by re-running the forward";
        return LLMGPU_E_UNSUPPORTED;
    }
    return 0;
}

// Caches and one-row buffers, allocated at the first decode call.
int decode_alloc(Ctx* c) {
    if (c->dec.ready) return 0;
    const size_t C = c->C, L = c->L, Bm = std::min(c->max_b, kDecMaxB), Tm = c->max_t;
    auto& d = c->dec;
    d.kc.assign(L, nullptr);
    d.vc.assign(L, nullptr);
    for (size_t l = 0; l < L; ++l) {
        if (cudaMalloc((void**)&d.kc[l], Bm * Tm * C * sizeof(bf16)) != cudaSuccess ||
            cudaMalloc((void**)&d.vc[l], Bm * Tm * C * sizeof(bf16)) != cudaSuccess) {
            c->err = "decode: KV cache allocation failed";
            return LLMGPU_E_CUDA;
        }
    }
    const size_t F = c->F;
    if (cudaMalloc((void**)&d.x, Bm * C * 4) != cudaSuccess ||
        cudaMalloc((void**)&d.y, Bm * C * 4) != cudaSuccess ||
        cudaMalloc((void**)&d.ln, Bm * C * 2) != cudaSuccess ||
        cudaMalloc((void**)&d.qkv, Bm * 3 * C * 2) != cudaSuccess ||
        cudaMalloc((void**)&d.att, Bm * C * 2) != cudaSuccess ||
        cudaMalloc((void**)&d.act, Bm * F * 2) != cudaSuccess ||
        cudaMalloc((void**)&d.stat, Bm * 2 * 4) != cudaSuccess ||
        cudaMalloc((void**)&d.logits, Bm * (size_t)c->Vp * 4) != cudaSuccess ||
        cudaMalloc((void**)&d.tokens, Bm * 4) != cudaSuccess) {
        c->err = "decode: buffer allocation failed";
        return LLMGPU_E_CUDA;
    }
    d.max_b = (int)Bm;
    d.ready = true;
    return 0;
}

void decode_free(Ctx* c) {
    auto& d = c->dec;
    for (void* p : d.kc) cudaFree(p);
    for (void* p : d.vc) cudaFree(p);
    d.kc.clear();
    d.vc.clear();
    for (void* p : {(void*)d.x, (void*)d.y, (void*)d.ln, (void*)d.qkv, (void*)d.att,
                    (void*)d.act, (void*)d.stat, (void*)d.logits, (void*)d.tokens})
        if (p) cudaFree(p);
    d = DecodeState{};
}

// Keys and values of the forward just run (B prompts of T tokens) into the caches.
int decode_fill(Ctx* c, int B, int T) {
    auto& d = c->dec;
    for (int l = 0; l < c->L; ++l) {
        const long long n = (long long)B * T * (c->C / 8);
        const int grid = (int)std::min<long long>((n + 255) / 256, 4 * 148);
        kv_fill_kernel<<<grid, 256, 0, c->stream>>>(c->act[l].qkv, d.kc[l], d.vc[l], B, T, c->C,
                                                     c->max_t);
        DK(launch_status());
    }
    d.B = B;
    d.pos = T;
    return 0;
}

// One token per sequence at position d.pos; logits (fp32 [B, Vp]) in d.logits.
int decode_step(Ctx* c, int B) {
    auto& d = c->dec;
    const int C = c->C, F = c->F, H = c->H, hd = c->hd, V = c->V, Vp = c->Vp;
    const int rms = c->cfg.use_rmsnorm;
    cudaStream_t s = c->stream;
    auto pp = [&](int i) { return c->p + c->params[i].offset; };
    const int pos = d.pos;
    if (pos >= c->max_t) {
        c->err = "decode: the cache is full (max_seq positions)";
        return LLMGPU_E_ARG;
    }
    embed_decode_kernel<<<B, 128, 0, s>>>(d.tokens, pp(c->i_wte), pp(c->i_wpe), d.x, C, V, pos,
                                          c->emb_rope, c->emb_rope_scale);
    DK(launch_status());
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)hd);
    float* mean = d.stat;
    float* rstd = d.stat + d.max_b;
    for (int l = 0; l < c->L; ++l) {
        const auto& b = c->blocks[l];
        DK(norm_forward(d.x, pp(b.ln1g), pp(b.ln1b), d.ln, mean, rstd, B, C, rms, s));
        DK(gemv<kDecBF16>(d.ln, C, c->wqkv16[l], 3 * C, C, 3 * C, B, d.qkv, 3 * C, nullptr, 0, s));
        if (hd == 64)
            attn_decode_kernel<64><<<dim3(H, B), 256, 0, s>>>(d.qkv, d.kc[l], d.vc[l], d.att, H,
                                                              c->max_t, pos, scale_log2);
        else
            attn_decode_kernel<32><<<dim3(H, B), 256, 0, s>>>(d.qkv, d.kc[l], d.vc[l], d.att, H,
                                                              c->max_t, pos, scale_log2);
        DK(launch_status());
        DK(gemv<kDecResid>(d.att, C, c->wo16[l], C, C, C, B, d.y, C, d.x, C, s));
        DK(norm_forward(d.y, pp(b.ln2g), pp(b.ln2b), d.ln, mean, rstd, B, C, rms, s));
        DK(gemv<kDecGelu>(d.ln, C, c->w1_16[l], F, C, F, B, d.act, F, nullptr, 0, s));
        DK(gemv<kDecResid>(d.act, F, c->w2_16[l], C, F, C, B, d.x, C, d.y, C, s));
    }
    DK(norm_forward(d.x, pp(c->i_lnfg), pp(c->i_lnfb), d.ln, mean, rstd, B, C, rms, s));
    if (c->cfg.weight_tying)
        DK(gemv_t(d.ln, C, c->wte16, C, C, V, B, d.logits, Vp, s));
    else
        DK(gemv<kDecF32>(d.ln, C, c->lm16, Vp, C, Vp, B, d.logits, Vp, nullptr, 0, s));
    d.pos = pos + 1;
    return 0;
}

}  // namespace llmgpu
