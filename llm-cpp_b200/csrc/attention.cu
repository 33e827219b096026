// Causal flash attention forward and backward over a packed qkv buffer [B*T, 3C] (bf16).
//
// Forward: one CTA per (64-query block, head, sequence); 4 warps x 16 query rows; K/V tiles
// double-buffered in shared memory with cp.async; online softmax in base 2; saves the
// natural-log normaliser (lse) per row for the backward.
// Backward is deterministic (no atomics): one kernel accumulates dK/dV per 64-key block
// over the query blocks that see it, a second accumulates dQ per 64-query block.
//
// Semantics follow MultiHeadAttention (src/attention.cpp:35-102, :183-363): scores scaled by
// 1/sqrt(head_dim), causal mask, softmax over keys, no bias, no dropout.
#include <cfloat>

#include "common.cuh"
#include "kernels.cuh"

namespace llmgpu {

namespace {

constexpr int BLK = 64;       // queries and keys per tile
constexpr int ATT_THREADS = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const uint32_t s = smem_u32(smem);
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// D(16x8 f32) += A(16x16 bf16) * B(16x8 bf16)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `ch` of tile row `r` (row = HD bf16), XOR-swizzled so that
// ldmatrix over 8 consecutive rows at a fixed chunk touches 8 distinct bank groups.
template <int HD>
__device__ __forceinline__ uint32_t swz(int r, int ch) {
    if constexpr (HD == 64) {
        return (uint32_t)(r * 128 + ((ch ^ (r & 7)) << 4));
    } else {
        return (uint32_t)(r * 64 + ((ch ^ ((r >> 1) & 3)) << 4));
    }
}

// Loads a 64 x HD tile whose row r is at gmem + (row0 + r) * ld (elements); rows >= nrows
// are zero-filled.
template <int HD>
__device__ __forceinline__ void load_tile(uint8_t* smem, const bf16* gmem, long long ld, int row0,
                                          int nrows) {
    constexpr int CH = HD / 8;
    for (int i = threadIdx.x; i < BLK * CH; i += ATT_THREADS) {
        const int r = i / CH, ch = i % CH;
        const bool ok = (row0 + r) < nrows;
        const bf16* src = gmem + (long long)(ok ? row0 + r : 0) * ld + ch * 8;
        cp_async16(smem + swz<HD>(r, ch), src, ok);
    }
}

// A fragments (16 rows x HD) of tile rows [r0, r0+16) -> HD/16 k-steps x 4 regs
template <int HD>
__device__ __forceinline__ void load_a_frags(const uint8_t* tile, int r0, uint32_t (&a)[HD / 16][4]) {
    const int lane = threadIdx.x & 31;
    const uint32_t base = smem_u32(tile);
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
        const int r = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = kk * 2 + (lane >> 4);
        ldsm_x4(base + swz<HD>(r, ch), a[kk][0], a[kk][1], a[kk][2], a[kk][3]);
    }
}

// S(16 x 64) = A(16 x HD) * T^T where T is a 64 x HD tile (rows = the n dimension).
template <int HD>
__device__ __forceinline__ void mma_abt(float (&s)[8][4], const uint32_t (&a)[HD / 16][4],
                                        const uint8_t* tile) {
    const int lane = threadIdx.x & 31;
    const uint32_t base = smem_u32(tile);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int k = 0; k < 4; ++k) s[n][k] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // pairs of n8 blocks
            const int r = np * 16 + (lane & 7) + (lane >> 4) * 8;
            const int ch = kk * 2 + ((lane >> 3) & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(base + swz<HD>(r, ch), b0, b1, b2, b3);
            mma16816(s[2 * np], a[kk], b0, b1);
            mma16816(s[2 * np + 1], a[kk], b2, b3);
        }
    }
}

// acc(16 x HD) += P(16 x 64) * T where T is a 64 x HD tile (rows = the k dimension).
template <int HD>
__device__ __forceinline__ void mma_pt(float (&acc)[HD / 8][4], const float (&p)[8][4],
                                       const uint8_t* tile) {
    const int lane = threadIdx.x & 31;
    const uint32_t base = smem_u32(tile);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per k-step
        uint32_t a[4];
        a[0] = pack_bf16x2(p[2 * kk][0], p[2 * kk][1]);
        a[1] = pack_bf16x2(p[2 * kk][2], p[2 * kk][3]);
        a[2] = pack_bf16x2(p[2 * kk + 1][0], p[2 * kk + 1][1]);
        a[3] = pack_bf16x2(p[2 * kk + 1][2], p[2 * kk + 1][3]);
#pragma unroll
        for (int dp = 0; dp < HD / 16; ++dp) {  // pairs of n8 blocks along HD
            const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            const int ch = dp * 2 + (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(base + swz<HD>(r, ch), b0, b1, b2, b3);
            mma16816(acc[2 * dp], a, b0, b1);
            mma16816(acc[2 * dp + 1], a, b2, b3);
        }
    }
}

// RoPE on a 64 x HD tile in shared memory: row r holds sequence position pos0 + r; pairs
// (2j, 2j+1) of every head vector are rotated by angle pos * theta^(-2j/HD), whose
// (cos, sin) come from `tab` [T][HD/2] (the pairing and frequencies of rope_cfg,
// src/model.cpp:88-100, with dim = head_dim).
template <int HD>
__device__ __forceinline__ void rope_tile(uint8_t* tile, int pos0, int T, const float2* tab) {
    constexpr int P = HD / 2;
    for (int i = threadIdx.x; i < BLK * P; i += ATT_THREADS) {
        const int r = i / P, j = i - r * P;
        const int pos = pos0 + r;
        if (pos >= T) continue;
        __nv_bfloat162* w =
            reinterpret_cast<__nv_bfloat162*>(tile + swz<HD>(r, j >> 2) + ((j & 3) << 2));
        const float2 v = __bfloat1622float2(*w);
        const float2 cs = tab[(long long)pos * P + j];
        *w = __floats2bfloat162_rn(v.x * cs.x - v.y * cs.y, v.x * cs.y + v.y * cs.x);
    }
}

// Inverse RoPE of an accumulator fragment (16 rows x HD, rows row0 and row0 + 8 of this
// thread): the pair (2j, 2j+1) of n8 block i at columns 2c, 2c+1 is held by one thread.
template <int HD>
__device__ __forceinline__ void rope_unrotate_acc(float (&acc)[HD / 8][4], int row0, int T,
                                                  const float2* tab) {
    const int c = threadIdx.x & 3;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int pos = row0 + r * 8;
        if (pos >= T) continue;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
            const int j = i * 4 + c;
            const float2 cs = tab[(long long)pos * (HD / 2) + j];
            const float y0 = acc[i][2 * r], y1 = acc[i][2 * r + 1];
            acc[i][2 * r] = y0 * cs.x + y1 * cs.y;
            acc[i][2 * r + 1] = -y0 * cs.y + y1 * cs.x;
        }
    }
}

// ---------------------------------------------------------------- forward
template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_fwd_kernel(const bf16* __restrict__ qkv,
                                                               bf16* __restrict__ out,
                                                               float* __restrict__ lse, int T,
                                                               int H, float scale_log2,
                                                               const float2* __restrict__ rope) {
    extern __shared__ __align__(128) uint8_t sm[];
    constexpr int TILE = BLK * HD * 2;
    uint8_t* sQ = sm;
    uint8_t* sK[2] = {sm + TILE, sm + 3 * TILE};
    uint8_t* sV[2] = {sm + 2 * TILE, sm + 4 * TILE};
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int C = H * HD;
    const long long ld = 3LL * C;
    const bf16* base = qkv + (long long)b * T * ld;
    const bf16* Qg = base + h * HD;
    const bf16* Kg = base + C + h * HD;
    const bf16* Vg = base + 2 * C + h * HD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = qb * BLK;
    const int nkb = min(qb + 1, (T + BLK - 1) / BLK);

    load_tile<HD>(sQ, Qg, ld, q0, T);
    load_tile<HD>(sK[0], Kg, ld, 0, T);
    load_tile<HD>(sV[0], Vg, ld, 0, T);
    cp_async_commit();

    uint32_t qa[HD / 16][4];
    float o[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) o[i][k] = 0.f;
    float mrow[2] = {-FLT_MAX, -FLT_MAX}, lrow[2] = {0.f, 0.f};
    const int g = lane >> 2, c = lane & 3;
    const int qrow0 = q0 + warp * 16 + g;  // this thread's rows: qrow0, qrow0 + 8

    for (int kb = 0; kb < nkb; ++kb) {
        const int cur = kb & 1;
        if (kb + 1 < nkb) {
            load_tile<HD>(sK[cur ^ 1], Kg, ld, (kb + 1) * BLK, T);
            load_tile<HD>(sV[cur ^ 1], Vg, ld, (kb + 1) * BLK, T);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (rope) {  // RoPE fused into the Q/K tile loads
            if (kb == 0) rope_tile<HD>(sQ, q0, T, rope);
            rope_tile<HD>(sK[cur], kb * BLK, T, rope);
            __syncthreads();
        }
        if (kb == 0) load_a_frags<HD>(sQ, warp * 16, qa);
        float s[8][4];
        mma_abt<HD>(s, qa, sK[cur]);
        const int k0 = kb * BLK;
        float mnew[2] = {mrow[0], mrow[1]};
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int key = k0 + n * 8 + 2 * c + (k & 1);
                const int q = qrow0 + (k >> 1) * 8;
                float v = s[n][k] * scale_log2;
                if (key > q || key >= T) v = -FLT_MAX;
                s[n][k] = v;
                mnew[k >> 1] = fmaxf(mnew[k >> 1], v);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 1));
            mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 2));
        }
        float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
        for (int r = 0; r < 2; ++r) alpha[r] = exp2f(mrow[r] - mnew[r]);
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float p = (s[n][k] == -FLT_MAX) ? 0.f : exp2f(s[n][k] - mnew[k >> 1]);
                s[n][k] = p;
                rs[k >> 1] += p;
            }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            lrow[r] = lrow[r] * alpha[r] + rs[r];
            mrow[r] = mnew[r];
        }
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
            o[i][0] *= alpha[0];
            o[i][1] *= alpha[0];
            o[i][2] *= alpha[1];
            o[i][3] *= alpha[1];
        }
        mma_pt<HD>(o, s, sV[cur]);
        __syncthreads();
    }
    // row sums across the 4 threads sharing a row
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int q = qrow0 + r * 8;
        if (q >= T) continue;
        const float inv = 1.0f / lrow[r];
        bf16* orow = out + ((long long)b * T + q) * C + h * HD;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
            *reinterpret_cast<uint32_t*>(orow + i * 8 + 2 * c) =
                pack_bf16x2(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
        }
        if (c == 0) lse[((long long)b * H + h) * T + q] = (mrow[r] + log2f(lrow[r])) * kLn2;
    }
}

// ---------------------------------------------------------------- backward helpers
// dvec[b,h,t] = sum_d dout[t, h*HD+d] * out[t, h*HD+d]
__global__ void attn_dvec_kernel(const bf16* __restrict__ out, const bf16* __restrict__ dout,
                                 float* __restrict__ dvec, int B, int T, int H, int HD) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)B * T * H) return;
    const int h = (int)(i % H);
    const long long row = i / H;  // b*T + t
    const int C = H * HD;
    const uint4* o4 = reinterpret_cast<const uint4*>(out + row * C + h * HD);
    const uint4* d4 = reinterpret_cast<const uint4*>(dout + row * C + h * HD);
    float acc = 0.f;
    for (int j = 0; j < HD / 8; ++j) {
        uint4 a = o4[j], d = d4[j];
        uint32_t aw[4] = {a.x, a.y, a.z, a.w}, dw[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
            acc += bf16_lo(aw[k]) * bf16_lo(dw[k]) + bf16_hi(aw[k]) * bf16_hi(dw[k]);
    }
    const int b = (int)(row / T), t = (int)(row % T);
    dvec[((long long)b * H + h) * T + t] = acc;
}

// The same by token rows: a warp per row, lanes reading consecutive 16-byte pieces (all ITER
// loads of a lane in flight at once), and the LPH = HD/8 lanes of a head adding their parts
// with shuffles. Needs LPH to divide 32 and H * LPH <= 32 * ITER.
template <int LPH, int ITER>
__global__ void __launch_bounds__(256) attn_dvec_rows_kernel(const bf16* __restrict__ out,
                                                             const bf16* __restrict__ dout,
                                                             float* __restrict__ dvec, int B,
                                                             int T, int H) {
    pdl_enter();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long row = blockIdx.x * 8LL + warp;  // b*T + t
    if (row >= (long long)B * T) return;
    const int C8 = H * LPH;  // 16-byte pieces per row
    const uint4* o4 = reinterpret_cast<const uint4*>(out) + row * C8;
    const uint4* d4 = reinterpret_cast<const uint4*>(dout) + row * C8;
    uint4 a[ITER], d[ITER];
#pragma unroll
    for (int k = 0; k < ITER; ++k) {
        const int u = lane + 32 * k;
        if (u < C8) {
            a[k] = o4[u];
            d[k] = d4[u];
        } else {
            a[k] = d[k] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    const int b = (int)(row / T), t = (int)(row % T);
#pragma unroll
    for (int k = 0; k < ITER; ++k) {
        const uint32_t aw[4] = {a[k].x, a[k].y, a[k].z, a[k].w};
        const uint32_t dw[4] = {d[k].x, d[k].y, d[k].z, d[k].w};
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            acc += bf16_lo(aw[j]) * bf16_lo(dw[j]) + bf16_hi(aw[j]) * bf16_hi(dw[j]);
#pragma unroll
        for (int off = LPH / 2; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        const int u = lane + 32 * k;
        if (u < C8 && (lane % LPH) == 0) dvec[((long long)b * H + u / LPH) * T + t] = acc;
    }
}

// dK, dV for one 64-key block; warps own 16 keys each and loop over query blocks.
template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_bwd_dkdv_kernel(
    const bf16* __restrict__ qkv, const bf16* __restrict__ dout, const float* __restrict__ lse,
    const float* __restrict__ dvec, bf16* __restrict__ dqkv, int T, int H, float scale,
    const float2* __restrict__ rope) {
    extern __shared__ __align__(128) uint8_t sm[];
    constexpr int TILE = BLK * HD * 2;
    uint8_t* sK = sm;
    uint8_t* sV = sm + TILE;
    uint8_t* sQ[2] = {sm + 2 * TILE, sm + 4 * TILE};
    uint8_t* sO[2] = {sm + 3 * TILE, sm + 5 * TILE};
    float* sL[2] = {reinterpret_cast<float*>(sm + 6 * TILE),
                    reinterpret_cast<float*>(sm + 6 * TILE) + 2 * BLK};
    float* sD[2] = {sL[0] + BLK, sL[1] + BLK};

    const int kb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int C = H * HD;
    const long long ld = 3LL * C;
    const bf16* base = qkv + (long long)b * T * ld;
    const bf16* Qg = base + h * HD;
    const bf16* Kg = base + C + h * HD;
    const bf16* Vg = base + 2 * C + h * HD;
    const bf16* dOg = dout + (long long)b * T * C + h * HD;
    const float* Lg = lse + ((long long)b * H + h) * T;
    const float* Dg = dvec + ((long long)b * H + h) * T;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int k0 = kb * BLK;
    const int nqb = (T + BLK - 1) / BLK;
    const float scale_log2 = scale * kLog2e;

    auto load_q = [&](int qb, int buf) {
        load_tile<HD>(sQ[buf], Qg, ld, qb * BLK, T);
        load_tile<HD>(sO[buf], dOg, C, qb * BLK, T);
        for (int i = threadIdx.x; i < BLK; i += ATT_THREADS) {
            const int q = qb * BLK + i;
            sL[buf][i] = q < T ? Lg[q] * kLog2e : 0.f;
            sD[buf][i] = q < T ? Dg[q] : 0.f;
        }
    };
    load_tile<HD>(sK, Kg, ld, k0, T);
    load_tile<HD>(sV, Vg, ld, k0, T);
    load_q(kb, 0);
    cp_async_commit();

    uint32_t ka[HD / 16][4], va[HD / 16][4];
    float dk[HD / 8][4], dv[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) dk[i][k] = dv[i][k] = 0.f;
    const int key0 = k0 + warp * 16 + g;  // this thread's keys: key0, key0 + 8

    for (int qb = kb; qb < nqb; ++qb) {
        const int cur = (qb - kb) & 1;
        if (qb + 1 < nqb) {
            load_q(qb + 1, cur ^ 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (rope) {
            if (qb == kb) rope_tile<HD>(sK, k0, T, rope);
            rope_tile<HD>(sQ[cur], qb * BLK, T, rope);
            __syncthreads();
        }
        if (qb == kb) {
            load_a_frags<HD>(sK, warp * 16, ka);
            load_a_frags<HD>(sV, warp * 16, va);
        }
        const int qbase = qb * BLK;
        // P^T (16 keys x 64 queries)
        float p[8][4];
        mma_abt<HD>(p, ka, sQ[cur]);
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int ql = n * 8 + 2 * c + (k & 1);
                const int q = qbase + ql;
                const int key = key0 + (k >> 1) * 8;
                const float v = p[n][k] * scale_log2 - sL[cur][ql];
                p[n][k] = (key > q || q >= T || key >= T) ? 0.f : exp2f(v);
            }
        // dV += P^T dO
        mma_pt<HD>(dv, p, sO[cur]);
        // dP^T = V dO^T
        float dp[8][4];
        mma_abt<HD>(dp, va, sO[cur]);
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int ql = n * 8 + 2 * c + (k & 1);
                dp[n][k] = p[n][k] * (dp[n][k] - sD[cur][ql]);
            }
        // dK += dS^T Q
        mma_pt<HD>(dk, dp, sQ[cur]);
        __syncthreads();
    }
    if (rope) rope_unrotate_acc<HD>(dk, key0, T, rope);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int key = key0 + r * 8;
        if (key >= T) continue;
        bf16* krow = dqkv + ((long long)b * T + key) * ld + C + h * HD;
        bf16* vrow = krow + C;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
            *reinterpret_cast<uint32_t*>(krow + i * 8 + 2 * c) =
                pack_bf16x2(dk[i][2 * r] * scale, dk[i][2 * r + 1] * scale);
            *reinterpret_cast<uint32_t*>(vrow + i * 8 + 2 * c) =
                pack_bf16x2(dv[i][2 * r], dv[i][2 * r + 1]);
        }
    }
}

// dQ for one 64-query block; warps own 16 queries and loop over key blocks.
template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_bwd_dq_kernel(
    const bf16* __restrict__ qkv, const bf16* __restrict__ dout, const float* __restrict__ lse,
    const float* __restrict__ dvec, bf16* __restrict__ dqkv, int T, int H, float scale,
    const float2* __restrict__ rope) {
    extern __shared__ __align__(128) uint8_t sm[];
    constexpr int TILE = BLK * HD * 2;
    uint8_t* sQ = sm;
    uint8_t* sO = sm + TILE;
    uint8_t* sK[2] = {sm + 2 * TILE, sm + 4 * TILE};
    uint8_t* sV[2] = {sm + 3 * TILE, sm + 5 * TILE};
    const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int C = H * HD;
    const long long ld = 3LL * C;
    const bf16* base = qkv + (long long)b * T * ld;
    const bf16* Qg = base + h * HD;
    const bf16* Kg = base + C + h * HD;
    const bf16* Vg = base + 2 * C + h * HD;
    const bf16* dOg = dout + (long long)b * T * C + h * HD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int q0 = qb * BLK;
    const int nkb = min(qb + 1, (T + BLK - 1) / BLK);
    const float scale_log2 = scale * kLog2e;
    const int qrow0 = q0 + warp * 16 + g;
    float lrow[2], drow[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int q = qrow0 + r * 8;
        lrow[r] = q < T ? lse[((long long)b * H + h) * T + q] * kLog2e : 0.f;
        drow[r] = q < T ? dvec[((long long)b * H + h) * T + q] : 0.f;
    }
    load_tile<HD>(sQ, Qg, ld, q0, T);
    load_tile<HD>(sO, dOg, C, q0, T);
    load_tile<HD>(sK[0], Kg, ld, 0, T);
    load_tile<HD>(sV[0], Vg, ld, 0, T);
    cp_async_commit();
    uint32_t qa[HD / 16][4], oa[HD / 16][4];
    float dq[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) dq[i][k] = 0.f;

    for (int kb = 0; kb < nkb; ++kb) {
        const int cur = kb & 1;
        if (kb + 1 < nkb) {
            load_tile<HD>(sK[cur ^ 1], Kg, ld, (kb + 1) * BLK, T);
            load_tile<HD>(sV[cur ^ 1], Vg, ld, (kb + 1) * BLK, T);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (rope) {
            if (kb == 0) rope_tile<HD>(sQ, q0, T, rope);
            rope_tile<HD>(sK[cur], kb * BLK, T, rope);
            __syncthreads();
        }
        if (kb == 0) {
            load_a_frags<HD>(sQ, warp * 16, qa);
            load_a_frags<HD>(sO, warp * 16, oa);
        }
        const int k0 = kb * BLK;
        float p[8][4], dp[8][4];
        mma_abt<HD>(p, qa, sK[cur]);
        mma_abt<HD>(dp, oa, sV[cur]);
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int key = k0 + n * 8 + 2 * c + (k & 1);
                const int q = qrow0 + (k >> 1) * 8;
                const float pv = (key > q || key >= T || q >= T)
                                     ? 0.f
                                     : exp2f(p[n][k] * scale_log2 - lrow[k >> 1]);
                dp[n][k] = pv * (dp[n][k] - drow[k >> 1]);
            }
        mma_pt<HD>(dq, dp, sK[cur]);
        __syncthreads();
    }
    if (rope) rope_unrotate_acc<HD>(dq, qrow0, T, rope);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int q = qrow0 + r * 8;
        if (q >= T) continue;
        bf16* qrow = dqkv + ((long long)b * T + q) * ld + h * HD;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i)
            *reinterpret_cast<uint32_t*>(qrow + i * 8 + 2 * c) =
                pack_bf16x2(dq[i][2 * r] * scale, dq[i][2 * r + 1] * scale);
    }
}

template <typename K>
void set_smem(K kernel, int bytes) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace

namespace {
// Heads of width hd < 64 as 64-wide heads for the tcgen05 kernels (attention_tc.cu): rows of
// `parts` x H heads, [B*T][parts*H*hd] <-> [B*T][parts*H*64], zeros in dims hd..63. A thread
// moves 8 consecutive dims (16 bytes) of one head. With `rope` ([T][hd/2] (cos, sin)), the
// q and k parts (0 and 1) are rotated per pair (2j, 2j+1) on the way: forward when padding,
// the transposed rotation when unpadding (gradients with respect to rotated q / k).
constexpr int kPadHD = 64;

__device__ __forceinline__ void rope8(float (&v)[8], const float2* tab, int t, int hd, int j0,
                                      bool inverse) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 cs = tab[(long long)t * (hd / 2) + j0 + k];
        const float sn = inverse ? -cs.y : cs.y;
        const float x = v[2 * k], y = v[2 * k + 1];
        v[2 * k] = x * cs.x - y * sn;
        v[2 * k + 1] = x * sn + y * cs.x;
    }
}

__global__ void pad_heads_kernel(const bf16* __restrict__ src, bf16* __restrict__ dst,
                                 long long rows, int parts, int H, int hd, int T,
                                 const float2* __restrict__ rope) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const int per_row = parts * H * (kPadHD / 8);
    if (i >= rows * per_row) return;
    const long long row = i / per_row;
    const int r = (int)(i - row * per_row);
    const int c8 = r % (kPadHD / 8), head = r / (kPadHD / 8);  // head over parts * H
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (c8 * 8 < hd) {
        w = *reinterpret_cast<const uint4*>(src + row * parts * H * hd + (long long)head * hd +
                                            c8 * 8);
        if (rope && head < 2 * H) {
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
            float v[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[2 * k] = bf16_lo(u[k]);
                v[2 * k + 1] = bf16_hi(u[k]);
            }
            rope8(v, rope, (int)(row % T), hd, c8 * 4, false);
            w = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                           pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
        }
    }
    *reinterpret_cast<uint4*>(dst + row * parts * H * kPadHD + (long long)head * kPadHD +
                              c8 * 8) = w;
}

__global__ void unpad_heads_kernel(const bf16* __restrict__ src, bf16* __restrict__ dst,
                                   long long rows, int parts, int H, int hd, int T,
                                   const float2* __restrict__ rope) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const int per_row = parts * H * (hd / 8);
    if (i >= rows * per_row) return;
    const long long row = i / per_row;
    const int r = (int)(i - row * per_row);
    const int c8 = r % (hd / 8), head = r / (hd / 8);
    uint4 w = *reinterpret_cast<const uint4*>(src + row * parts * H * kPadHD +
                                              (long long)head * kPadHD + c8 * 8);
    if (rope && head < 2 * H) {
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
        float v[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[2 * k] = bf16_lo(u[k]);
            v[2 * k + 1] = bf16_hi(u[k]);
        }
        rope8(v, rope, (int)(row % T), hd, c8 * 4, true);
        w = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                       pack_bf16x2(v[6], v[7]));
    }
    *reinterpret_cast<uint4*>(dst + row * parts * H * hd + (long long)head * hd + c8 * 8) = w;
}

bool pad_path(int hd) { return hd < kPadHD && hd >= 8 && hd % 8 == 0; }

size_t pad_unit_bytes(int B, int T, int H) {  // one [B*T][H*64] bf16 plane, 256-byte multiple
    return ((size_t)B * T * H * kPadHD * sizeof(bf16) + 255) / 256 * 256;
}

int pad_heads(const bf16* src, bf16* dst, int B, int T, int parts, int H, int hd,
              const float2* rope, cudaStream_t s) {
    const long long n = (long long)B * T * parts * H * (kPadHD / 8);
    return launch_kernel(pad_heads_kernel, (unsigned)((n + 255) / 256), 256, 0, s, src, dst,
                         (long long)B * T, parts, H, hd, T, rope);
}

int unpad_heads(const bf16* src, bf16* dst, int B, int T, int parts, int H, int hd,
                const float2* rope, cudaStream_t s) {
    const long long n = (long long)B * T * parts * H * (hd / 8);
    return launch_kernel(unpad_heads_kernel, (unsigned)((n + 255) / 256), 256, 0, s, src, dst,
                         (long long)B * T, parts, H, hd, T, rope);
}
}  // namespace

size_t attention_work_bytes(int B, int T, int H, int hd) {
    const size_t ds = (attention_ds_bytes(B, T, H) + 255) / 256 * 256;
    return pad_path(hd) ? ds + 7 * pad_unit_bytes(B, T, H) : ds;
}

int attention_forward(const bf16* qkv, bf16* out, float* lse, int B, int T, int H, int hd,
                      const float2* rope, cudaStream_t s, int* err, void* work) {
    const float scale = 1.0f / sqrtf((float)hd);
    dim3 grid((T + BLK - 1) / BLK, H, B);
    if (hd == 64 && !rope) {
        CUtensorMap tm;
        if (attention_qkv_tmap(&tm, qkv, B, T, H * hd)) return -2;
        return attention_forward_tc(tm, out, lse, B, T, H, hd, scale, err, s);
    }
    if (pad_path(hd) && work) {
        // [q|k|v] and the output as 64-wide heads, after the dS region of the workspace
        const size_t unit = pad_unit_bytes(B, T, H);
        char* base = static_cast<char*>(work) + (attention_ds_bytes(B, T, H) + 255) / 256 * 256;
        bf16* qkv64 = reinterpret_cast<bf16*>(base);
        bf16* out64 = reinterpret_cast<bf16*>(base + 3 * unit);
        int rc = pad_heads(qkv, qkv64, B, T, 3, H, hd, rope, s);
        if (rc) return rc;
        CUtensorMap tm;
        if (attention_qkv_tmap(&tm, qkv64, B, T, H * kPadHD)) return -2;
        if ((rc = attention_forward_tc(tm, out64, lse, B, T, H, kPadHD, scale, err, s))) return rc;
        return unpad_heads(out64, out, B, T, 1, H, hd, nullptr, s);
    }
    if (hd == 64) {
        const int smem = 5 * BLK * 64 * 2;
        static bool set = false;
        if (!set) { set_smem(attn_fwd_kernel<64>, smem); set = true; }
        attn_fwd_kernel<64><<<grid, ATT_THREADS, smem, s>>>(qkv, out, lse, T, H, scale * kLog2e, rope);
    } else if (hd == 32) {
        const int smem = 5 * BLK * 32 * 2;
        attn_fwd_kernel<32><<<grid, ATT_THREADS, smem, s>>>(qkv, out, lse, T, H, scale * kLog2e, rope);
    } else {
        return -1;
    }
    return launch_status();
}

namespace {
__global__ void rope_qk_kernel(bf16* __restrict__ qkv, int T, int C, int hd, long long pairs,
                               const float2* __restrict__ tab, int inverse) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= pairs) return;
    const int half = C / 2;
    const long long row = i / half;
    const int pc = (int)(i - row * half);       // pair index within the C columns
    const int t = (int)(row % T);
    const int j = pc % (hd / 2);                // pair within the head
    const float2 cs = tab[(long long)t * (hd / 2) + j];
    const float sn = inverse ? -cs.y : cs.y;
    __nv_bfloat162* base = reinterpret_cast<__nv_bfloat162*>(qkv + row * 3LL * C) + pc;
#pragma unroll
    for (int part = 0; part < 2; ++part) {      // q, then k
        __nv_bfloat162* w = base + part * half;
        const float2 v = __bfloat1622float2(*w);
        *w = __floats2bfloat162_rn(v.x * cs.x - v.y * sn, v.x * sn + v.y * cs.x);
    }
}
}  // namespace

int rope_qk_inplace(bf16* qkv, int B, int T, int H, int hd, const float2* rope, int inverse,
                    cudaStream_t s) {
    if (!rope || (hd & 1)) return -1;
    const int C = H * hd;
    const long long pairs = (long long)B * T * (C / 2);
    rope_qk_kernel<<<(int)((pairs + 255) / 256), 256, 0, s>>>(qkv, T, C, hd, pairs, rope, inverse);
    return launch_status();
}

int attention_backward(const bf16* qkv, const bf16* out, const bf16* dout, const float* lse,
                       float* dvec, bf16* dqkv, int B, int T, int H, int hd, const float2* rope,
                       cudaStream_t s, int* err, void* ds_work, const float2* rope_back) {
    const float scale = 1.0f / sqrtf((float)hd);
    const long long n = (long long)B * T * H;
    const int rows_blocks = (int)(((long long)B * T + 7) / 8);
    if (hd == 64 && H * 8 <= 128) {
        if (H * 8 <= 32)
            launch_kernel(attn_dvec_rows_kernel<8, 1>, rows_blocks, 256, 0, s, out, dout, dvec, B, T, H);
        else if (H * 8 <= 64)
            launch_kernel(attn_dvec_rows_kernel<8, 2>, rows_blocks, 256, 0, s, out, dout, dvec, B, T, H);
        else if (H * 8 <= 96)
            launch_kernel(attn_dvec_rows_kernel<8, 3>, rows_blocks, 256, 0, s, out, dout, dvec, B, T, H);
        else
            launch_kernel(attn_dvec_rows_kernel<8, 4>, rows_blocks, 256, 0, s, out, dout, dvec, B, T, H);
    } else {
        attn_dvec_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(out, dout, dvec, B, T, H, hd);
    }
    if (hd == 64 && !rope && (T % 4) == 0) {
        const int rc = launch_status();
        if (rc) return rc;
        if (!ds_work) return -5;  // the tcgen05 kernels need the dS scratch
        return attention_backward_tc(qkv, dout, lse, dvec, dqkv, B, T, H, hd, scale, ds_work, err,
                                     s, rope_back);
    }
    if (pad_path(hd) && (T % 4) == 0 && ds_work) {
        int rc = launch_status();
        if (rc) return rc;
        const size_t unit = pad_unit_bytes(B, T, H);
        char* base = static_cast<char*>(ds_work) + (attention_ds_bytes(B, T, H) + 255) / 256 * 256;
        bf16* qkv64 = reinterpret_cast<bf16*>(base);
        bf16* dout64 = reinterpret_cast<bf16*>(base + 3 * unit);
        bf16* dqkv64 = reinterpret_cast<bf16*>(base + 4 * unit);
        if ((rc = pad_heads(qkv, qkv64, B, T, 3, H, hd, rope, s)) ||
            (rc = pad_heads(dout, dout64, B, T, 1, H, hd, nullptr, s)) ||
            (rc = attention_backward_tc(qkv64, dout64, lse, dvec, dqkv64, B, T, H, kPadHD, scale,
                                        ds_work, err, s, nullptr)))
            return rc;
        // dq and dk rotate back with the table q and k were rotated by
        return unpad_heads(dqkv64, dqkv, B, T, 3, H, hd, rope ? rope : rope_back, s);
    }
    dim3 grid((T + BLK - 1) / BLK, H, B);
    if (hd == 64) {
        const int smem1 = 6 * BLK * 64 * 2 + 4 * BLK * 4;
        const int smem2 = 6 * BLK * 64 * 2;
        static bool set = false;
        if (!set) {
            set_smem(attn_bwd_dkdv_kernel<64>, smem1);
            set_smem(attn_bwd_dq_kernel<64>, smem2);
            set = true;
        }
        attn_bwd_dkdv_kernel<64><<<grid, ATT_THREADS, smem1, s>>>(qkv, dout, lse, dvec, dqkv, T, H,
                                                                  scale, rope);
        attn_bwd_dq_kernel<64><<<grid, ATT_THREADS, smem2, s>>>(qkv, dout, lse, dvec, dqkv, T, H,
                                                                scale, rope);
    } else if (hd == 32) {
        const int smem1 = 6 * BLK * 32 * 2 + 4 * BLK * 4;
        const int smem2 = 6 * BLK * 32 * 2;
        attn_bwd_dkdv_kernel<32><<<grid, ATT_THREADS, smem1, s>>>(qkv, dout, lse, dvec, dqkv, T, H,
                                                                  scale, rope);
        attn_bwd_dq_kernel<32><<<grid, ATT_THREADS, smem2, s>>>(qkv, dout, lse, dvec, dqkv, T, H,
                                                                scale, rope);
    } else {
        return -1;
    }
    if (rope_back) {
        const int rc = launch_status();
        if (rc) return rc;
        return rope_qk_inplace(dqkv, B, T, H, hd, rope_back, 1, s);
    }
    return launch_status();
}

}  // namespace llmgpu
