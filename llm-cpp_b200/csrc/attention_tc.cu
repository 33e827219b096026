// Causal flash attention forward on the 5th-generation tensor cores (head_dim 64).
//
// One CTA per (128-query tile, head, sequence), two CTAs per SM; 320 threads:
//   warp 0     TMA producer: the Q tile once, then K and V tiles of 128 keys through two
//              independent 2-deep rings (a K slot frees when its QK^T MMA is done, a V slot
//              when its PV MMA is done)
//   warp 1     TMEM allocator + MMA issuer: S_j = Q K_j^T into TMEM, then O += P_{j-1} V_{j-1}
//              with P read straight from TMEM (the A-from-TMEM form of tcgen05.mma)
//   warps 2-9  softmax: a query row per two threads (column half (w - 2) / 4); warp w reads
//              TMEM lanes 32*(w%4).. (the lane quarter a warp may access). Reads S_j, masks, keeps the
//              running max / sum in base 2, writes P_j (bf16 pairs) into TMEM, and rescales O
//              in TMEM only when a row's running max grows by more than 2^8 (otherwise the
//              stale max is kept: the final O / l is exact either way). At the end it writes
//              O / l and the natural-log normaliser lse of each row for the backward.
// TMEM per CTA (256 columns): S [0,128), O [128,192), P [192,256). S_{j+1} = Q K_{j+1}^T runs
// on the tensor cores while the softmax of block j runs, and the two CTAs of an SM
// interleave their softmax warps.
//
// Semantics follow MultiHeadAttention (src/attention.cpp:35-102): scores scaled by
// 1/sqrt(head_dim), causal mask, softmax over keys, no bias, no dropout.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace llmgpu {

namespace {

constexpr int kRows = 128;                    // queries per CTA, keys per tile
constexpr int kHD = 64;
constexpr int kTile = kRows * kHD * 2;        // 16 KB: a Q, K or V tile (128 rows x 128 B)
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColO = 128, kColP = 192;
constexpr int kThreads = 320;
constexpr float kLn2f = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.0f;          // rescale O when the max grows by more than 2^8
constexpr int kPolyEvery = 4;                 // one pair of exponentials in 4 on the FMA pipe

struct Smem {
    static constexpr int Q = 0;
    static constexpr int K = kTile;           // two K slots
    static constexpr int V = K + 2 * kTile;   // two V slots
    static constexpr int XCH = V + 2 * kTile; // row maxima [2][2][128] and sums [2][128]
    static constexpr int BAR = XCH + 6 * kRows * 4;
    static constexpr int TOTAL = BAR + 256;
};
constexpr size_t kSmemBytes = 1024 + Smem::TOTAL;

// The n-th work item of this CTA in a persistent walk over items sorted longest first: rows
// of gridDim.x items, taken left to right in even rows and right to left in odd ones, which
// evens out the CTAs' totals (a plain stride gives the low CTAs the longest item of every row).
__device__ __forceinline__ int snake_item(int n) {
    const int g = (int)gridDim.x, b = (int)blockIdx.x;
    return n * g + ((n & 1) ? g - 1 - b : b);
}

// Bounded wait by every lane of a warp with a warp-uniform result, so that the warp-collective
// TMEM instructions after it are never reached by only part of the warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    const bool ok = mbar_wait_bounded(bar, parity, err, code);
    return __all_sync(0xffffffffu, ok);
}

__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, bf16* __restrict__ out,
                       float* __restrict__ lse, int T, int H, float scale_log2,
                       int* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t* sm = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    uint8_t* sQ = sm + Smem::Q;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + Smem::BAR);
    uint64_t* q_full = bar;
    uint64_t* k_full = bar + 1;      // [2]
    uint64_t* k_empty = k_full + 2;  // [2]
    uint64_t* v_full = k_empty + 2;  // [2]
    uint64_t* v_empty = v_full + 2;  // [2]
    uint64_t* s_full = v_empty + 2;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_free + 1;
    uint64_t* pv_done = p_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 1);

    const int nqb = (T + kRows - 1) / kRows;
    // blocks launch in x-fastest order: all (head, sequence) pairs of the longest query tile
    // (most keys) first, the shortest last, so the last wave holds the shortest tiles
    const int qb = nqb - 1 - (int)blockIdx.y;
    const int h = (int)blockIdx.x % H, b = (int)blockIdx.x / H;
    const int C = H * kHD;
    const int q0 = qb * kRows;
    const int nkv = qb + 1;                      // causal: key tiles 0..qb
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 256);
        mbar_init(p_full, 256);
        mbar_init(pv_done, 1);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    pdl_enter();  // first global-memory access follows
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            bool ok = true;
            mbar_arrive_expect_tx(q_full, kTile);
            tma_load_3d(sQ, &tm, q_full, h * kHD, q0, b);
            for (int j = 0; j < nkv && ok; ++j) {
                const int st = j & 1;
                const uint32_t ph = ((j >> 1) & 1) ^ 1u;
                if (!mbar_wait_bounded(&k_empty[st], ph, err, kDevTimeoutEmpty)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&k_full[st], kTile);
                tma_load_3d(sm + Smem::K + st * kTile, &tm, &k_full[st], C + h * kHD, j * kRows, b);
                if (!mbar_wait_bounded(&v_empty[st], ph, err, kDevTimeoutEmpty)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&v_full[st], kTile);
                tma_load_3d(sm + Smem::V + st * kTile, &tm, &v_full[st], 2 * C + h * kHD, j * kRows,
                            b);
            }
            if (!ok) spin_ns(100000);  // error path: let copies in flight land first
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            const uint32_t idesc_qk = make_idesc_bf16(kRows, kRows, 0, 0);  // Q, K both K-major
            const uint32_t idesc_pv = make_idesc_bf16(kRows, kHD, 0, 1);    // P (TMEM), V MN-major
            const uint32_t q_addr = smem_u32(sQ);
            bool ok = mbar_wait_bounded(q_full, 0, err, kDevTimeoutFull);
            auto issue_pv = [&](int i) -> bool {
                if (!mbar_wait_bounded(p_full, i & 1, err, kDevTimeoutFull) ||
                    !mbar_wait_bounded(&v_full[i & 1], (i >> 1) & 1, err, kDevTimeoutFull))
                    return false;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sm + Smem::V + (i & 1) * kTile);
#pragma unroll
                for (int kk = 0; kk < kRows / 16; ++kk)
                    umma_bf16_ts(tmem + kColO, tmem + kColP + kk * 8,
                                 make_sw128_desc(v_addr + kk * 2048, 8192, 1024), idesc_pv,
                                 (i > 0 || kk > 0) ? 1u : 0u);
                umma_commit(pv_done);
                umma_commit(&v_empty[i & 1]);
                return true;
            };
            for (int j = 0; j < nkv && ok; ++j) {
                const int st = j & 1;
                if (!mbar_wait_bounded(&k_full[st], (j >> 1) & 1, err, kDevTimeoutFull) ||
                    !mbar_wait_bounded(s_free, (j & 1) ^ 1u, err, kDevTimeoutAccFree)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t k_addr = smem_u32(sm + Smem::K + st * kTile);
#pragma unroll
                for (int kk = 0; kk < kHD / 16; ++kk)
                    umma_bf16(tmem + kColS, make_sw128_desc(q_addr + kk * 32, 16, 1024),
                              make_sw128_desc(k_addr + kk * 32, 16, 1024), idesc_qk,
                              kk > 0 ? 1u : 0u);
                umma_commit(s_full);
                umma_commit(&k_empty[st]);
                if (j >= 1 && !issue_pv(j - 1)) ok = false;
            }
            if (ok) issue_pv(nkv - 1);
        }
    } else {
        // ---------------- softmax warps 2-9: warp w reads TMEM lane quarter w % 4 (one query
        // row per thread) and column half hf = (w - 2) / 4 of each 128-key score tile; the two
        // threads of a row exchange their block maxima through shared memory
        const int q = warp & 3, hf = (warp - 2) >> 2;
        const int row = q * 32 + lane;
        const int qrow = q0 + row;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        float* sMax = reinterpret_cast<float*>(sm + Smem::XCH);  // [2][128]
        const int bar_id = 1 + q;   // named barrier of the two warps of lane quarter q
        constexpr int kHalf = kRows / 2;
        float m_run = -INFINITY, l = 0.f;
        // Both warps of a quarter take every block's exchange barrier, also after a timed-out
        // wait (ok false: later waits are skipped and the results are discarded), so neither
        // can be left waiting at a barrier its partner will not reach.
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            if (ok && !warp_wait(s_full, j & 1, err, kDevTimeoutAcc)) ok = false;
            tc_fence_after();
            uint32_t v[kHalf];
#pragma unroll
            for (int c = 0; c < kHalf / 32; ++c)
                tmem_ld_32x32b_x32(tmem + lane_base + kColS + hf * kHalf + c * 32,
                                   *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(s_free);
            const int k0 = j * kRows + hf * kHalf;
            if ((k0 + kHalf - 1 > qrow) || (k0 + kHalf > T)) {  // causal / sequence-end mask
#pragma unroll
                for (int i = 0; i < kHalf; ++i)
                    if (k0 + i > qrow || k0 + i >= T) v[i] = __float_as_uint(-INFINITY);
            }
            // 8 independent partial maxima keep the dependency chains short
            float pm[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) pm[u] = __uint_as_float(v[u]);
#pragma unroll
            for (int i = 8; i < kHalf; ++i) pm[i & 7] = fmaxf(pm[i & 7], __uint_as_float(v[i]));
            float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
            // row maximum over both halves (buffer j & 1: the partner may already be one
            // block ahead when this thread reads)
            sMax[((j & 1) * 2 + hf) * kRows + row] = mx;
            named_barrier_sync(bar_id, 64);
            mx = fmaxf(mx, sMax[((j & 1) * 2 + (hf ^ 1)) * kRows + row]);
            mx *= scale_log2;
            float alpha = 1.f;
            bool rescale = false;
            if (j == 0) {
                m_run = mx;
            } else if (mx > m_run + kRescaleLog2) {
                alpha = ex2_approx(m_run - mx);
                m_run = mx;
                rescale = true;
            }
            // P_j = 2^(s * scale - m_run) as bf16 pairs, packed in place of the scores; one
            // pair in kPolyEvery on the FMA pipe (ex2_poly), the rest on the special-function
            // unit; scale, shift and sum run as packed pairs
            const float2 sc2 = make_float2(scale_log2, scale_log2);
            const float2 nm2 = make_float2(-m_run, -m_run);
            float2 ps[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                            make_float2(0.f, 0.f)};
#pragma unroll
            for (int i = 0; i < kHalf / 2; ++i) {
                const float2 x = ffma2(make_float2(__uint_as_float(v[2 * i]),
                                                   __uint_as_float(v[2 * i + 1])), sc2, nm2);
                float2 pp;
                if (i % kPolyEvery == kPolyEvery - 1)
                    pp = make_float2(ex2_poly(x.x), ex2_poly(x.y));
                else
                    pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                ps[i & 3] = fadd2(ps[i & 3], pp);
                v[i] = pack_bf16x2(pp.x, pp.y);
            }
            const float2 s4 = fadd2(fadd2(ps[0], ps[1]), fadd2(ps[2], ps[3]));
            const float sum = s4.x + s4.y;
            // PV_{j-1} has read the previous P and finished adding into O
            if (ok && j >= 1 && !warp_wait(pv_done, (j - 1) & 1, err, kDevTimeoutAcc)) ok = false;
            tc_fence_after();
            if (__any_sync(0xffffffffu, rescale)) {  // this half's 32 columns of O
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem + lane_base + kColO + hf * 32, r);
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                tmem_st_32x32b_x32(tmem + lane_base + kColO + hf * 32, r);
            }
            tmem_st_32x32b_x32(tmem + lane_base + kColP + hf * 32,
                               *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
            tmem_st_wait();
            l = l * alpha + sum;
            tc_fence_before();
            mbar_arrive(p_full);
        }
        // the row's sum over both halves
        float* sSum = sMax + 4 * kRows;
        sSum[hf * kRows + row] = l;
        named_barrier_sync(bar_id, 64);
        l += sSum[(hf ^ 1) * kRows + row];
        if (ok && warp_wait(pv_done, (nkv - 1) & 1, err, kDevTimeoutAcc)) {
            tc_fence_after();
            const float inv = 1.f / l;
            bf16* o = out + ((long long)b * T + qrow) * C + h * kHD + hf * 32;
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem + lane_base + kColO + hf * 32, r);
            tmem_ld_wait();
            if (qrow < T) {
                uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    o4[i] = make_uint4(
                        pack_bf16x2(__uint_as_float(r[8 * i]) * inv, __uint_as_float(r[8 * i + 1]) * inv),
                        pack_bf16x2(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv),
                        pack_bf16x2(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv),
                        pack_bf16x2(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv));
                if (hf == 0) lse[((long long)b * H + h) * T + qrow] = (m_run + log2f(l)) * kLn2f;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ============================================================================ backward
// Two deterministic kernels (no atomics), head_dim 64. With P = exp(S * scale - lse) (rows:
// queries) and D = rowsum(dO o O):
//   dS = P o (dP - D), dP = dO V^T, dV = P^T dO, dK = scale dS^T Q, dQ = scale dS K.
// dK/dV kernel (320 threads; work item: a 128-key tile of one head, over the query tiles
// that see it):
//   warp 0     TMA producer        warp 1     TMEM allocator + MMA issuer
//   warps 2-9  elementwise: warp w handles TMEM lane quarter w % 4 (one key row per thread)
//              and column half (w - 2) / 4 of every 128-wide score tile, so two warps share
//              each SM sub-partition.
// S^T = K Q^T and dP^T = V dO^T in TMEM; P^T and dS^T (bf16) written back to TMEM feed
// dV += P^T dO and dK += dS^T Q as A-from-TMEM MMAs, and dS^T also goes out to a table of
// dS tiles in global memory. The next tile's S / dP MMAs run while the elementwise warps
// work on the current one; Q, dO, lse and D stream through a 3-stage TMA ring. The kernel is
// persistent: one CTA per SM walks the work items from the longest (most tiles) down, CTA c
// taking items c, c + grid, ...; every role counts tiles across items, the fixed K and V
// tiles of an item are double buffered so that the next item's load overlaps the current
// one, and the next item's first S / dP MMAs run while the current item's accumulators are
// drained. TMEM (512 columns): S [0,128), dP [128,256), dV and dK accumulators [256,384),
// bf16 P and dS operands [384,512).
// dQ kernel (further down): dQ_i = scale * sum_j dS_ij K_j from the stored dS tiles.
constexpr int kBwdThreads = 320;
constexpr int kBwdStages = 3;
constexpr uint32_t kBwdTmem = 512;
constexpr float kLog2ef = 1.4426950408889634f;

struct BwdSmem {
    // two buffers of the two fixed tiles (K, V or Q, dO), then kBwdStages stages of two
    // streamed tiles (+ 512-byte lse and D vectors for the dK/dV kernel)
    static constexpr int FIX = 0;                  // [buffer][tile]
    static constexpr int STAGE0 = 4 * kTile;
    static constexpr int STAGE_BYTES = 2 * kTile + 1024;
    static constexpr int BAR = STAGE0 + kBwdStages * STAGE_BYTES;
    static constexpr int TOTAL = BAR + 256;
};
// The dK/dV kernel also stages each elementwise warp's 32 x 64 block of dS^T (4 KB, 128-byte
// swizzle) for a bulk store to the dS tiles the dQ kernel reads.
constexpr int kDsBoxOff = (BwdSmem::TOTAL + 1023) & ~1023;
constexpr size_t kDkdvSmemBytes = 1024 + kDsBoxOff + 8 * 4096;

// Compact causal tile index of (query tile qi, key tile kj), kj <= qi.
__device__ __forceinline__ int ds_tile(int qi, int kj) { return qi * (qi + 1) / 2 + kj; }

__device__ __forceinline__ void store_row64_bf16(bf16* dst, const uint32_t (&r)[32], float mul) {
    uint4* o4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        o4[i] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * i]) * mul, __uint_as_float(r[8 * i + 1]) * mul),
                           pack_bf16x2(__uint_as_float(r[8 * i + 2]) * mul, __uint_as_float(r[8 * i + 3]) * mul),
                           pack_bf16x2(__uint_as_float(r[8 * i + 4]) * mul, __uint_as_float(r[8 * i + 5]) * mul),
                           pack_bf16x2(__uint_as_float(r[8 * i + 6]) * mul, __uint_as_float(r[8 * i + 7]) * mul));
}

// dQ / dK of a row whose queries / keys were rotated by RoPE before the attention: the
// gradient of the unrotated vector is the inverse rotation, pairs (2j, 2j+1) by the
// (cos, sin) cs[j] of the row's position (r0: columns 0-31, r1: 32-63).
__device__ __forceinline__ void rope_back_row64(uint32_t (&r0)[32], uint32_t (&r1)[32],
                                                const float2* __restrict__ cs) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float2 a = cs[i], b = cs[16 + i];
        const float x0 = __uint_as_float(r0[2 * i]), x1 = __uint_as_float(r0[2 * i + 1]);
        r0[2 * i] = __float_as_uint(x0 * a.x + x1 * a.y);
        r0[2 * i + 1] = __float_as_uint(x1 * a.x - x0 * a.y);
        const float y0 = __uint_as_float(r1[2 * i]), y1 = __uint_as_float(r1[2 * i + 1]);
        r1[2 * i] = __float_as_uint(y0 * b.x + y1 * b.y);
        r1[2 * i + 1] = __float_as_uint(y1 * b.x - y0 * b.y);
    }
}

// Work item `it` of a backward kernel: tile index counted from the longest end (the tile
// with the most partner tiles first), head and sequence.
struct BwdItem {
    int tile, h, b;
};
__device__ __forceinline__ BwdItem bwd_item(int it, int H, int B) {
    const int hb = H * B;
    BwdItem w;
    w.tile = it / hb;
    const int r = it - w.tile * hb;
    w.h = r % H;
    w.b = r / H;
    return w;
}

// Barriers of a persistent backward kernel.
struct BwdBars {
    uint64_t* fix_full;   // [2] fixed tiles of an item loaded
    uint64_t* fix_empty;  // [2] an item's last MMA reading its fixed tiles done
    uint64_t* st_full;    // [kBwdStages]
    uint64_t* st_empty;   // [kBwdStages]
    uint64_t* s_full;     // S / dP of a tile in TMEM
    uint64_t* s_free;     // S / dP read by the elementwise warps
    uint64_t* p_full;     // the tile's bf16 operands written to TMEM
    uint64_t* mm_done;    // the tile's accumulating MMAs done
    uint64_t* acc_free;   // an item's accumulators read out of TMEM
    uint32_t* tmem_slot;
};
__device__ __forceinline__ BwdBars bwd_bars(uint8_t* sm) {
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + BwdSmem::BAR);
    BwdBars r;
    r.fix_full = bar;
    r.fix_empty = bar + 2;
    r.st_full = bar + 4;
    r.st_empty = r.st_full + kBwdStages;
    r.s_full = r.st_empty + kBwdStages;
    r.s_free = r.s_full + 1;
    r.p_full = r.s_free + 1;
    r.mm_done = r.p_full + 1;
    r.acc_free = r.mm_done + 1;
    r.tmem_slot = reinterpret_cast<uint32_t*>(r.acc_free + 1);
    return r;
}
__device__ __forceinline__ void bwd_init(const BwdBars& k, int acc_readers) {
    for (int i = 0; i < 2; ++i) {
        mbar_init(&k.fix_full[i], 1);
        mbar_init(&k.fix_empty[i], 1);
    }
    for (int s = 0; s < kBwdStages; ++s) {
        mbar_init(&k.st_full[s], 1);
        mbar_init(&k.st_empty[s], 1);
    }
    mbar_init(k.s_full, 1);
    mbar_init(k.s_free, 256);
    mbar_init(k.p_full, 256);
    mbar_init(k.mm_done, 1);
    mbar_init(k.acc_free, acc_readers);
    fence_barrier_init();
}

// ---------------------------------------------------------------- dK / dV
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                            const __grid_constant__ CUtensorMap tm_do,
                            const __grid_constant__ CUtensorMap tm_lse,
                            const __grid_constant__ CUtensorMap tm_d,
                            const __grid_constant__ CUtensorMap tm_ds, bf16* __restrict__ dqkv,
                            int B, int T, int H, float scale, const float2* __restrict__ rope,
                            int* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t* sm = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    const BwdBars k = bwd_bars(sm);
    const int nqb = (T + kRows - 1) / kRows;
    const int items = nqb * H * B;
    const int C = H * kHD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float scale_log2 = scale * kLog2ef;
    const int ntiles = nqb * (nqb + 1) / 2;
    constexpr uint32_t kColDV = 256, kColDK = 320, kColP = 384, kColDS = 448;

    if (threadIdx.x == 0) bwd_init(k, 256);
    if (warp == 1) {
        tmem_alloc(k.tmem_slot, kBwdTmem);
        tmem_relinquish();
    }
    pdl_enter();  // first global-memory access follows
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *k.tmem_slot;
    auto stage = [&](int g) { return sm + BwdSmem::STAGE0 + (g % kBwdStages) * BwdSmem::STAGE_BYTES; };
    auto fix = [&](int buf, int t) { return sm + BwdSmem::FIX + (2 * buf + t) * kTile; };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer: K, V of each item, then Q, dO, lse, D per tile
            bool ok = true;
            int g = 0;
            for (int n = 0, it = snake_item(0); it < items && ok; ++n, it = snake_item(n)) {
                const BwdItem w = bwd_item(it, H, B);
                const int kt = w.tile, ns = nqb - kt, fb = n & 1;
                if (!mbar_wait_bounded(&k.fix_empty[fb], ((n >> 1) & 1) ^ 1u, err,
                                       kDevTimeoutEmpty)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&k.fix_full[fb], 2 * kTile);
                tma_load_3d(fix(fb, 0), &tm_qkv, &k.fix_full[fb], C + w.h * kHD, kt * kRows, w.b);
                tma_load_3d(fix(fb, 1), &tm_qkv, &k.fix_full[fb], 2 * C + w.h * kHD, kt * kRows,
                            w.b);
                for (int s = 0; s < ns; ++s, ++g) {
                    const int q0 = (kt + s) * kRows;
                    if (!mbar_wait_bounded(&k.st_empty[g % kBwdStages], ((g / kBwdStages) & 1) ^ 1u,
                                           err, kDevTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = stage(g);
                    uint64_t* f = &k.st_full[g % kBwdStages];
                    mbar_arrive_expect_tx(f, 2 * kTile + 1024);
                    tma_load_3d(st, &tm_qkv, f, w.h * kHD, q0, w.b);                  // Q_i
                    tma_load_3d(st + kTile, &tm_do, f, w.h * kHD, q0, w.b);           // dO_i
                    tma_load_2d(st + 2 * kTile, &tm_lse, f, q0, w.b * H + w.h);       // lse_i
                    tma_load_2d(st + 2 * kTile + 512, &tm_d, f, q0, w.b * H + w.h);   // D_i
                }
            }
            if (!ok) spin_ns(100000);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer; tiles are counted across items (g), so the next
            // tile's S^T / dP^T can be issued before the current tile's dV / dK
            const uint32_t idesc_s = make_idesc_bf16(kRows, kRows, 0, 0);
            const uint32_t idesc_acc = make_idesc_bf16(kRows, kHD, 0, 1);
            bool ok = true;
            // issue S^T = K Q^T and dP^T = V dO^T of tile g (item slot n, tile s of ns)
            auto issue_sdp = [&](int g, int n, int s, int ns) -> bool {
                const int fb = n & 1;
                if (s == 0 && !mbar_wait_bounded(&k.fix_full[fb], (n >> 1) & 1, err, kDevTimeoutFull))
                    return false;
                if (!mbar_wait_bounded(&k.st_full[g % kBwdStages], (g / kBwdStages) & 1, err,
                                       kDevTimeoutFull))
                    return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(fix(fb, 0)), v_addr = smem_u32(fix(fb, 1));
                const uint32_t q_addr = smem_u32(stage(g)), do_addr = q_addr + kTile;
#pragma unroll
                for (int kk = 0; kk < kHD / 16; ++kk)
                    umma_bf16(tmem, make_sw128_desc(k_addr + kk * 32, 16, 1024),
                              make_sw128_desc(q_addr + kk * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
#pragma unroll
                for (int kk = 0; kk < kHD / 16; ++kk)
                    umma_bf16(tmem + 128, make_sw128_desc(v_addr + kk * 32, 16, 1024),
                              make_sw128_desc(do_addr + kk * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
                umma_commit(k.s_full);
                if (s == ns - 1) umma_commit(&k.fix_empty[fb]);  // K, V of the item read
                return true;
            };
            // walk the tiles: (n, s) of tile g, and of tile g + 1
            int it = snake_item(0), n = 0, s = 0;
            int ns = it < items ? nqb - bwd_item(it, H, B).tile : 0;
            if (it < items) ok = issue_sdp(0, 0, 0, ns);
            for (int g = 0; it < items && ok; ++g) {
                int it1 = it, n1 = n, s1 = s + 1, ns1 = ns;
                if (s1 == ns) {
                    n1 = n + 1;
                    it1 = snake_item(n1);
                    s1 = 0;
                    ns1 = it1 < items ? nqb - bwd_item(it1, H, B).tile : 0;
                }
                if (it1 < items) {
                    if (!mbar_wait_bounded(k.s_free, g & 1, err, kDevTimeoutAccFree) ||
                        !issue_sdp(g + 1, n1, s1, ns1)) {
                        ok = false;
                        break;
                    }
                }
                if (!mbar_wait_bounded(k.p_full, g & 1, err, kDevTimeoutFull) ||
                    (s == 0 && n > 0 &&
                     !mbar_wait_bounded(k.acc_free, (n - 1) & 1, err, kDevTimeoutAccFree))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t q_addr = smem_u32(stage(g)), do_addr = q_addr + kTile;
#pragma unroll
                for (int kk = 0; kk < kRows / 16; ++kk) {  // dV += P^T dO ; dK += dS^T Q
                    umma_bf16_ts(tmem + kColDV, tmem + kColP + kk * 8,
                                 make_sw128_desc(do_addr + kk * 2048, 8192, 1024), idesc_acc,
                                 (s > 0 || kk > 0) ? 1u : 0u);
                    umma_bf16_ts(tmem + kColDK, tmem + kColDS + kk * 8,
                                 make_sw128_desc(q_addr + kk * 2048, 8192, 1024), idesc_acc,
                                 (s > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(k.mm_done);
                umma_commit(&k.st_empty[g % kBwdStages]);
                it = it1;
                n = n1;
                s = s1;
                ns = ns1;
            }
        }
    } else {
        // ---------------- elementwise warps: thread = key row, 64 query columns
        const int lq = warp & 3, half = (warp - 2) >> 2;
        const int kr = lq * 32 + lane;
        const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
        bool ok = true;
        int g = 0;
        for (int n = 0, it = snake_item(0); it < items && ok; it = snake_item(++n)) {
            const BwdItem w = bwd_item(it, H, B);
            const int kt = w.tile, ns = nqb - kt;
            const int key = kt * kRows + kr;
            for (int s = 0; s < ns && ok; ++s, ++g) {
                const int q0 = (kt + s) * kRows + half * 64;
                if (!warp_wait(k.s_full, g & 1, err, kDevTimeoutAcc) ||
                    !warp_wait(&k.st_full[g % kBwdStages], (g / kBwdStages) & 1, err,
                               kDevTimeoutAcc)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t sv[64], dp[64];
                tmem_ld_32x32b_x32(tmem + lane_base + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
                tmem_ld_32x32b_x32(tmem + lane_base + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
                tmem_ld_32x32b_x32(tmem + lane_base + 128 + half * 64, *reinterpret_cast<uint32_t(*)[32]>(&dp[0]));
                tmem_ld_32x32b_x32(tmem + lane_base + 128 + half * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&dp[32]));
                tmem_ld_wait();
                tc_fence_before();
                mbar_arrive(k.s_free);
                const float* lse = reinterpret_cast<const float*>(stage(g) + 2 * kTile) + half * 64;
                const float* dv = lse + 128;
#pragma unroll
                for (int c4 = 0; c4 < 16; ++c4) {
                    const float4 l4 = reinterpret_cast<const float4*>(lse)[c4];
                    const float4 d4 = reinterpret_cast<const float4*>(dv)[c4];
                    const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dd[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int c = c4 * 4 + u, q = q0 + c;
                        float p = ex2_approx(fmaf(__uint_as_float(sv[c]), scale_log2, -lv[u] * kLog2ef));
                        if (q < key || q >= T) p = 0.f;
                        sv[c] = __float_as_uint(p);
                        dp[c] = __float_as_uint(p * (__uint_as_float(dp[c]) - dd[u]));
                    }
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    sv[i] = pack_bf16x2(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1]));
                    dp[i] = pack_bf16x2(__uint_as_float(dp[2 * i]), __uint_as_float(dp[2 * i + 1]));
                }
                {
                    // this warp's 32 keys x 64 queries of dS^T also go to the dS tiles
                    uint8_t* box = sm + kDsBoxOff + (warp - 2) * 4096;
                    if (lane == 0) bulk_wait_group_read<0>();  // the box's last store has read it
                    __syncwarp();
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch)
                        *reinterpret_cast<uint4*>(box + lane * 128 + ((ch ^ (lane & 7)) << 4)) =
                            make_uint4(dp[4 * ch], dp[4 * ch + 1], dp[4 * ch + 2], dp[4 * ch + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_3d(&tm_ds, box, half * 64, lq * 32,
                                     (w.b * H + w.h) * ntiles + ds_tile(kt + s, kt));
                        bulk_commit_group();
                    }
                }
                if (g >= 1 && !warp_wait(k.mm_done, (g - 1) & 1, err, kDevTimeoutAcc)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                tmem_st_32x32b_x32(tmem + lane_base + kColP + half * 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
                tmem_st_32x32b_x32(tmem + lane_base + kColDS + half * 32, *reinterpret_cast<uint32_t(*)[32]>(&dp[0]));
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(k.p_full);
            }
            if (!ok || !warp_wait(k.mm_done, (g - 1) & 1, err, kDevTimeoutAcc)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // column half 0 writes dV, half 1 writes scale * dK; the accumulators are free
            // for the next item once read
            const uint32_t col = half == 0 ? kColDV : kColDK;
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(tmem + lane_base + col, r0);
            tmem_ld_32x32b_x32(tmem + lane_base + col + 32, r1);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(k.acc_free);
            if (key < T) {
                if (half == 1 && rope) rope_back_row64(r0, r1, rope + (long long)key * (kHD / 2));
                bf16* dst = dqkv + ((long long)w.b * T + key) * 3LL * C + (half == 0 ? 2 * C : C) +
                            w.h * kHD;
                store_row64_bf16(dst, r0, half == 0 ? 1.f : scale);
                store_row64_bf16(dst + 32, r1, half == 0 ? 1.f : scale);
            }
        }
    }

    if (warp >= 2 && lane == 0) bulk_wait_group_all();  // dS stores done before exit
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kBwdTmem);
}

// ---------------------------------------------------------------- dQ
// dQ_i = scale * sum_j dS_ij K_j over the dS tiles the dK/dV kernel stored (no recompute of S
// and dP). Persistent: one CTA per SM walks the query tiles, longest first. Warp 0 loads per
// key tile the stored dS^T (two 128-key x 64-query boxes: the MN-major A operand) and K_j
// (the MN-major B operand), warp 1 accumulates in TMEM (two 64-column accumulators, so an
// item's MMAs overlap the previous item's read-out), warps 2-5 write dQ. The sum over j runs
// in key-tile order: deterministic.
constexpr int kDqThreads = 192;
constexpr int kDqStages = 4;
constexpr int kDqStageBytes = 3 * kTile;
constexpr int kDqBarOff = kDqStages * kDqStageBytes;
constexpr size_t kDqSmemBytes = 1024 + kDqBarOff + 256;

__global__ void __launch_bounds__(kDqThreads, 1)
    attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                          const __grid_constant__ CUtensorMap tm_ds, bf16* __restrict__ dqkv,
                          int B, int T, int H, float scale, const float2* __restrict__ rope,
                          int* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t* sm = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + kDqBarOff);
    uint64_t* empty = full + kDqStages;
    uint64_t* acc_full = empty + kDqStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    const int nqb = (T + kRows - 1) / kRows;
    const int ntiles = nqb * (nqb + 1) / 2;
    const int items = nqb * H * B;
    const int C = H * kHD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kDqStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * kHD);
        tmem_relinquish();
    }
    pdl_enter();  // first global-memory access follows
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto stage = [&](int g) { return sm + (g % kDqStages) * kDqStageBytes; };

    if (warp == 0) {
        if (lane == 0) {
            bool ok = true;
            int g = 0;
            for (int n = 0, it = snake_item(0); it < items && ok; it = snake_item(++n)) {
                const BwdItem w = bwd_item(it, H, B);
                const int qt = nqb - 1 - w.tile;
                const int z0 = (w.b * H + w.h) * ntiles + ds_tile(qt, 0);
                for (int j = 0; j <= qt; ++j, ++g) {
                    if (!mbar_wait_bounded(&empty[g % kDqStages], ((g / kDqStages) & 1) ^ 1u, err,
                                           kDevTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = stage(g);
                    uint64_t* f = &full[g % kDqStages];
                    mbar_arrive_expect_tx(f, 3 * kTile);
                    tma_load_3d(st, &tm_ds, f, 0, 0, z0 + j);           // dS^T, queries 0-63
                    tma_load_3d(st + kTile, &tm_ds, f, 64, 0, z0 + j);  // queries 64-127
                    tma_load_3d(st + 2 * kTile, &tm_qkv, f, C + w.h * kHD, j * kRows, w.b);  // K_j
                }
            }
            if (!ok) spin_ns(100000);  // error path: let copies in flight land first
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = make_idesc_bf16(kRows, kHD, 1, 1);
            bool ok = true;
            int g = 0;
            for (int n = 0, it = snake_item(0); it < items && ok; ++n, it = snake_item(n)) {
                const int qt = nqb - 1 - bwd_item(it, H, B).tile;
                const int acc = n & 1;
                if (!mbar_wait_bounded(&acc_empty[acc], ((n >> 1) & 1) ^ 1u, err,
                                       kDevTimeoutAccFree)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * kHD);
                for (int j = 0; j <= qt; ++j, ++g) {
                    if (!mbar_wait_bounded(&full[g % kDqStages], (g / kDqStages) & 1, err,
                                           kDevTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(stage(g)), b_addr = a_addr + 2 * kTile;
#pragma unroll
                    for (int kk = 0; kk < kRows / 16; ++kk)  // 16 keys per MMA
                        umma_bf16(d, make_sw128_desc(a_addr + kk * 2048, kTile, 1024),
                                  make_sw128_desc(b_addr + kk * 2048, 8192, 1024), idesc,
                                  (j > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&empty[g % kDqStages]);
                }
                if (!ok) break;
                umma_commit(&acc_full[acc]);
            }
        }
    } else {
        // ---------------- warps 2-5: TMEM lane quarter warp % 4, one query row per thread
        const int lq = warp & 3;
        const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
        for (int n = 0, it = snake_item(0); it < items; ++n, it = snake_item(n)) {
            const BwdItem w = bwd_item(it, H, B);
            const int qt = nqb - 1 - w.tile;
            const int acc = n & 1;
            if (!warp_wait(&acc_full[acc], (n >> 1) & 1, err, kDevTimeoutAcc)) break;
            tc_fence_after();
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(tmem + lane_base + (uint32_t)(acc * kHD), r0);
            tmem_ld_32x32b_x32(tmem + lane_base + (uint32_t)(acc * kHD + 32), r1);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
            const int q = qt * kRows + lq * 32 + lane;
            if (q < T) {
                if (rope) rope_back_row64(r0, r1, rope + (long long)q * (kHD / 2));
                bf16* dst = dqkv + ((long long)w.b * T + q) * 3LL * C + w.h * kHD;
                store_row64_bf16(dst, r0, scale);
                store_row64_bf16(dst + 32, r1, scale);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 2 * kHD);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace

// Tensor map over the packed qkv buffer as [B][T][3C] (rows past T of a sequence read as
// zeros), boxes of 128 rows x 64 columns (one head's q, k or v), 128-byte swizzle.
int attention_qkv_tmap(CUtensorMap* tm, const bf16* qkv, int B, int T, int C) {
    auto enc = encode_fn();
    if (!enc) return -1;
    if ((reinterpret_cast<uintptr_t>(qkv) & 15) != 0 || ((3LL * C * 2) & 15) != 0) return -2;
    cuuint64_t dims[3] = {(cuuint64_t)3 * C, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)3 * C * 2, (cuuint64_t)3 * C * 2 * T};
    cuuint32_t box[3] = {kHD, kRows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<bf16*>(qkv), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -4;
}

int attention_forward_tc(const CUtensorMap& tm, bf16* out, float* lse, int B, int T, int H, int hd,
                         float scale, int* err, cudaStream_t s) {
    if (hd != kHD || B <= 0 || T <= 0 || H <= 0) return -1;
    static int attr = -1;
    static std::once_flag once;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)kSmemBytes) == cudaSuccess
                   ? 0
                   : -3;
    });
    if (attr) return attr;
    const dim3 grid(H * B, (T + kRows - 1) / kRows);
    return launch_kernel(attn_fwd_tc_kernel, grid, kThreads, kSmemBytes, s, tm, out, lse, T, H,
                         scale * kLog2ef, err);
}

namespace {
int encode_map(CUtensorMap* tm, CUtensorMapDataType dt, int rank, const void* ptr,
               const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
               CUtensorMapSwizzle sw) {
    auto enc = encode_fn();
    if (!enc) return -1;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return -2;
    for (int i = 0; i + 1 < rank; ++i)
        if ((strides[i] & 15) != 0) return -2;
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(tm, dt, rank, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -4;
}
}  // namespace

size_t attention_ds_bytes(int B, int T, int H) {
    const long long nqb = (T + kRows - 1) / kRows;
    return (size_t)B * H * (nqb * (nqb + 1) / 2) * kRows * kRows * sizeof(bf16);
}

int attention_backward_tc(const bf16* qkv, const bf16* dout, const float* lse, const float* dvec,
                          bf16* dqkv, int B, int T, int H, int hd, float scale, void* ds_work,
                          int* err, cudaStream_t s, const float2* rope_back) {
    if (hd != kHD || B <= 0 || T <= 0 || H <= 0 || (T % 4) != 0 || !ds_work) return -1;
    const int C = H * hd;
    CUtensorMap tq, tdo, tl, td, tds_st, tds_ld;
    if (attention_qkv_tmap(&tq, qkv, B, T, C)) return -2;
    {
        // dS^T tiles: [B*H*tiles][128 keys][128 queries] bf16
        const int nqb = (T + kRows - 1) / kRows;
        const cuuint64_t dims[3] = {(cuuint64_t)kRows, (cuuint64_t)kRows,
                                    (cuuint64_t)B * H * (nqb * (nqb + 1) / 2)};
        const cuuint64_t strides[2] = {(cuuint64_t)kRows * 2, (cuuint64_t)kRows * kRows * 2};
        const cuuint32_t box_st[3] = {64, 32, 1}, box_ld[3] = {64, kRows, 1};
        if (encode_map(&tds_st, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ds_work, dims, strides,
                       box_st, CU_TENSOR_MAP_SWIZZLE_128B) ||
            encode_map(&tds_ld, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ds_work, dims, strides,
                       box_ld, CU_TENSOR_MAP_SWIZZLE_128B))
            return -2;
    }
    {
        const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)T, (cuuint64_t)B};
        const cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)C * 2 * T};
        const cuuint32_t box[3] = {kHD, kRows, 1};
        if (encode_map(&tdo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dout, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B))
            return -2;
    }
    {
        const cuuint64_t dims[2] = {(cuuint64_t)T, (cuuint64_t)B * H};
        const cuuint64_t strides[1] = {(cuuint64_t)T * 4};
        const cuuint32_t box[2] = {kRows, 1};
        if (encode_map(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, lse, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_NONE) ||
            encode_map(&td, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dvec, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_NONE))
            return -2;
    }
    static int attr = -1;
    static std::once_flag once;
    std::call_once(once, [] {
        attr = (cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kDkdvSmemBytes) == cudaSuccess &&
                cudaFuncSetAttribute(attn_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kDqSmemBytes) == cudaSuccess)
                   ? 0
                   : -3;
    });
    if (attr) return attr;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int items = ((T + kRows - 1) / kRows) * H * B;
    const int grid = items < sms ? items : sms;
    int rc = launch_kernel(attn_bwd_dkdv_tc_kernel, grid, kBwdThreads, kDkdvSmemBytes, s, tq, tdo,
                           tl, td, tds_st, dqkv, B, T, H, scale, rope_back, err);
    if (rc) return rc;
    return launch_kernel(attn_bwd_dq_tc_kernel, grid, kDqThreads, kDqSmemBytes, s, tq, tds_ld, dqkv,
                         B, T, H, scale, rope_back, err);
}

}  // namespace llmgpu
