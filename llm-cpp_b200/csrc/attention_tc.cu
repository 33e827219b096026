// Causal flash attention forward on the 5th-generation tensor cores (head_dim 64).
//
// One CTA per (128-query tile, head, sequence), two CTAs per SM; 192 threads:
//   warp 0     TMA producer: the Q tile once, then K and V tiles of 128 keys through two
//              independent 2-deep rings (a K slot frees when its QK^T MMA is done, a V slot
//              when its PV MMA is done)
//   warp 1     TMEM allocator + MMA issuer: S_j = Q K_j^T into TMEM, then O += P_{j-1} V_{j-1}
//              with P read straight from TMEM (the A-from-TMEM form of tcgen05.mma)
//   warps 2-5  softmax: one query row per thread; warp w reads TMEM lanes 32*(w%4).. (the
//              lane quarter a warp may access). Reads S_j, masks, keeps the
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
constexpr int kThreads = 192;
constexpr float kLn2f = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.0f;          // rescale O when the max grows by more than 2^8

struct Smem {
    static constexpr int Q = 0;
    static constexpr int K = kTile;           // two K slots
    static constexpr int V = K + 2 * kTile;   // two V slots
    static constexpr int BAR = V + 2 * kTile;
    static constexpr int TOTAL = BAR + 256;
};
constexpr size_t kSmemBytes = 1024 + Smem::TOTAL;

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
    const int qb = nqb - 1 - (int)blockIdx.x;    // longest (most keys) tiles first
    const int h = blockIdx.y, b = blockIdx.z;
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
        mbar_init(s_free, 128);
        mbar_init(p_full, 128);
        mbar_init(pv_done, 1);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
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
        // ---------------- softmax warps 2-5: thread = query row
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const int qrow = q0 + row;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        float m_run = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkv && ok; ++j) {
            if (!warp_wait(s_full, j & 1, err, kDevTimeoutAcc)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t v[kRows];
#pragma unroll
            for (int c = 0; c < kRows / 32; ++c)
                tmem_ld_32x32b_x32(tmem + lane_base + kColS + c * 32,
                                   *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(s_free);
            const int k0 = j * kRows;
            if ((k0 + kRows - 1 > qrow) || (k0 + kRows > T)) {  // causal / sequence-end mask
#pragma unroll
                for (int i = 0; i < kRows; ++i)
                    if (k0 + i > qrow || k0 + i >= T) v[i] = __float_as_uint(-INFINITY);
            }
            // 8 independent partial maxima / sums keep the dependency chains short
            float pm[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) pm[u] = __uint_as_float(v[u]);
#pragma unroll
            for (int i = 8; i < kRows; ++i) pm[i & 7] = fmaxf(pm[i & 7], __uint_as_float(v[i]));
            float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
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
            // P_j = 2^(s * scale - m_run) as bf16 pairs, packed in place of the scores
            float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < kRows / 2; ++i) {
                const float p0 = ex2_approx(fmaf(__uint_as_float(v[2 * i]), scale_log2, -m_run));
                const float p1 = ex2_approx(fmaf(__uint_as_float(v[2 * i + 1]), scale_log2, -m_run));
                ps[i & 7] += p0 + p1;
                v[i] = pack_bf16x2(p0, p1);
            }
            const float sum = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
            // PV_{j-1} has read the previous P and finished adding into O
            if (j >= 1 && !warp_wait(pv_done, (j - 1) & 1, err, kDevTimeoutAcc)) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
                for (int c = 0; c < kHD / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(tmem + lane_base + kColO + c * 32, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                    tmem_st_32x32b_x32(tmem + lane_base + kColO + c * 32, r);
                }
            }
            tmem_st_32x32b_x32(tmem + lane_base + kColP, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
            tmem_st_32x32b_x32(tmem + lane_base + kColP + 32,
                               *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
            tmem_st_wait();
            l = l * alpha + sum;
            tc_fence_before();
            mbar_arrive(p_full);
        }
        if (ok && warp_wait(pv_done, (nkv - 1) & 1, err, kDevTimeoutAcc)) {
            tc_fence_after();
            const float inv = 1.f / l;
            bf16* o = out + ((long long)b * T + qrow) * C + h * kHD;
#pragma unroll
            for (int c = 0; c < kHD / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem + lane_base + kColO + c * 32, r);
                tmem_ld_wait();
                if (qrow < T) {
                    uint4* o4 = reinterpret_cast<uint4*>(o + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        o4[i] = make_uint4(
                            pack_bf16x2(__uint_as_float(r[8 * i]) * inv, __uint_as_float(r[8 * i + 1]) * inv),
                            pack_bf16x2(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv),
                            pack_bf16x2(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv),
                            pack_bf16x2(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv));
                }
            }
            if (qrow < T) lse[((long long)b * H + h) * T + qrow] = (m_run + log2f(l)) * kLn2f;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
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
                         int* err, cudaStream_t s) {
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
    const dim3 grid((T + kRows - 1) / kRows, H, B);
    attn_fwd_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(tm, out, lse, T, H,
                                                         1.4426950408889634f / sqrtf((float)hd), err);
    return launch_status();
}

}  // namespace llmgpu
