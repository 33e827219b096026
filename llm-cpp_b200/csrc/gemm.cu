// tcgen05 GEMM for sm_100a: persistent, warp-specialised, TMA-fed, fp32 accumulators in TMEM.
//
// Roles per CTA (256 threads, one CTA per SM):
//   warp 0      : TMA producer (one elected lane) filling a STAGES-deep smem ring
//   warp 1      : TMEM allocator + MMA issuer (one lane issues tcgen05.mma)
//   warps 4..7  : epilogue (tcgen05.ld from TMEM lanes 32*(warp%4).., fused epilogue, global stores)
// Two TMEM accumulators (2*BN columns) let the epilogue of tile i overlap the MMAs of tile i+1.
//
// No TMA multicast is used anywhere: every CTA loads its own tiles.
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"

namespace llmgpu {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kGemmThreads = 256;
constexpr int kGroupM = 16;  // tile raster: groups of 16 m-blocks share B tiles in L2

template <int BN>
struct GemmCfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
};

__device__ __forceinline__ void decode_tile(int t, int num_m, int num_n, int tiles_mn, int& m_blk,
                                            int& n_blk, int& split) {
    split = t / tiles_mn;
    int r = t - split * tiles_mn;
    int per_group = kGroupM * num_n;
    int g = r / per_group;
    int first_m = g * kGroupM;
    int gm = min(kGroupM, num_m - first_m);
    int local = r - g * per_group;
    m_blk = first_m + local % gm;
    n_blk = local / gm;
}

// Resolves tile t into block coordinates, group and k-block range [kb0, kb1). Returns false
// for a tile with no rows in use (row-grouped products, past the last group).
__device__ __forceinline__ bool tile_work(const GemmArgs& a, const int* s_grp, int t, int num_m,
                                          int num_n, int tiles_mn, int kblocks, int& m_blk,
                                          int& n_blk, int& split, int& g, int& kb0, int& kb1) {
    decode_tile(t, num_m, num_n, tiles_mn, m_blk, n_blk, split);
    g = 0;
    if (a.grp_mode == kGroupRows) {
        const int m0 = m_blk * BM;
        if (m0 >= s_grp[a.groups]) return false;
        while (g + 1 < a.groups && s_grp[g + 1] <= m0) ++g;
        kb0 = 0;
        kb1 = kblocks;
    } else if (a.grp_mode == kGroupK) {
        g = split;
        kb0 = min(max(s_grp[g] / BK, 0), kblocks);
        kb1 = min(max(s_grp[g + 1] / BK, kb0), kblocks);
    } else {
        kb0 = (int)((long long)split * kblocks / a.splits);
        kb1 = (int)((long long)(split + 1) * kblocks / a.splits);
    }
    return true;
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* o, const float* v) {
    uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint4 p;
        p.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
        p.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
        p.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
        p.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
        o4[i] = p;
    }
}

// obase: element offset of the output (group g of a K-grouped product; kEpiStoreF32 only)
__device__ __forceinline__ void epi_store(const GemmArgs& a, int row, int col0, int split,
                                          long long obase, float (&v)[32]) {
    const int nvalid = min(32, a.N - col0);
    const bool full = (nvalid == 32) && !a.scalar_store;
    switch (a.epi) {
        case kEpiStoreBF16: {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col0;
            if (full) {
                store_bf16x32(o, v);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < nvalid) o[j] = __float2bfloat16_rn(v[j]);
            }
            break;
        }
        case kEpiStoreF32: {
            int g = col0 / a.col_group;
            int cc = col0 - g * a.col_group;
            float* o = reinterpret_cast<float*>(a.out) + obase + g * a.group_stride +
                       (long long)row * a.ldo + cc;
            if (full) {
                float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float4 w = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    if (a.accumulate) {
                        float4 p = o4[i];
                        w.x += p.x;
                        w.y += p.y;
                        w.z += p.z;
                        w.w += p.w;
                    }
                    o4[i] = w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < nvalid) o[j] = v[j] + (a.accumulate ? o[j] : 0.0f);
            }
            break;
        }
        case kEpiResidF32: {
            float* o = reinterpret_cast<float*>(a.out) + row * a.ldo + col0;
            const float* rr = a.resid + row * a.ldr + col0;
            if (full) {
                float4* o4 = reinterpret_cast<float4*>(o);
                const float4* r4 = reinterpret_cast<const float4*>(rr);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float4 p = r4[i];
                    o4[i] = make_float4(p.x + v[4 * i], p.y + v[4 * i + 1], p.z + v[4 * i + 2],
                                        p.w + v[4 * i + 3]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < nvalid) o[j] = rr[j] + v[j];
            }
            break;
        }
        case kEpiGeluBF16: {
            __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(a.aux) + row * a.ld_aux + col0;
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col0;
            float gv[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) gv[j] = gelu_tanh(v[j]);
            if (full) {
                store_bf16x32(h, v);
                store_bf16x32(o, gv);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (j < nvalid) {
                        h[j] = __float2bfloat16_rn(v[j]);
                        o[j] = __float2bfloat16_rn(gv[j]);
                    }
                }
            }
            break;
        }
        case kEpiDGeluBF16: {
            const __nv_bfloat16* h =
                reinterpret_cast<const __nv_bfloat16*>(a.aux) + row * a.ld_aux + col0;
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col0;
            if (full) {
                const uint4* h4 = reinterpret_cast<const uint4*>(h);
                float dv[32];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint4 p = h4[i];
                    uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        dv[8 * i + 2 * k] = v[8 * i + 2 * k] * gelu_tanh_grad(bf16_lo(w[k]));
                        dv[8 * i + 2 * k + 1] =
                            v[8 * i + 2 * k + 1] * gelu_tanh_grad(bf16_hi(w[k]));
                    }
                }
                store_bf16x32(o, dv);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < nvalid)
                        o[j] = __float2bfloat16_rn(v[j] * gelu_tanh_grad(__bfloat162float(h[j])));
            }
            break;
        }
        case kEpiSplitPartial: {
            float* o = reinterpret_cast<float*>(a.out) + (long long)split * a.M * a.N +
                       (long long)row * a.N + col0;
            if (full && (a.N % 4) == 0) {
                float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < nvalid) o[j] = v[j];
            }
            break;
        }
        default:
            break;
    }
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
    using Cfg = GemmCfg<BN>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int M = args.M, N = args.N, K = args.K;
    const int num_m = (M + BM - 1) / BM;
    const int num_n = (N + BN - 1) / BN;
    const int kblocks = (K + BK - 1) / BK;
    const int splits = args.splits;
    const int tiles_mn = num_m * num_n;
    const int total = tiles_mn * splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
        }
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    __shared__ int s_grp[kMaxGemmGroups + 1];
    if (args.grp_mode != kGroupNone)
        for (int i = threadIdx.x; i <= args.groups; i += blockDim.x) s_grp[i] = args.grp[i];
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer
            int stage = 0;
            uint32_t phase = 0;
            uint32_t last_phase[STAGES];
            bool pending[STAGES];
#pragma unroll
            for (int s = 0; s < STAGES; ++s) {
                last_phase[s] = 0;
                pending[s] = false;
            }
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int m_blk, n_blk, split, g, kb0, kb1;
                if (!tile_work(args, s_grp, t, num_m, num_n, tiles_mn, kblocks, m_blk, n_blk,
                               split, g, kb0, kb1))
                    continue;
                const int m0 = m_blk * BM, n0 = n_blk * BN;
                // row-grouped products read group g of B from row g * b_grp_rows on
                const int bg = (args.grp_mode == kGroupRows) ? (int)(g * args.b_grp_rows) : 0;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, args.err,
                                           kDevTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    const int k0 = kb * BK;
                    uint8_t* a = sA + stage * Cfg::A_BYTES;
                    uint8_t* b = sB + stage * Cfg::B_BYTES;
                    uint32_t bytes = 0;
                    if (!args.a_mn_major) {
                        bytes += Cfg::A_BYTES;
                    } else {
                        bytes += 8192u * ((m0 + 64 < M) ? 2u : 1u);
                    }
                    if (!args.b_mn_major) {
                        bytes += Cfg::B_BYTES;
                    } else {
                        for (int j = 0; j < BN / 64; ++j)
                            if (n0 + 64 * j < N) bytes += 8192u;
                    }
                    mbar_arrive_expect_tx(&full[stage], bytes);
                    if (!args.a_mn_major) {
                        tma_load_2d(a, &tmA, &full[stage], k0, m0);
                    } else {
                        tma_load_2d(a, &tmA, &full[stage], m0, k0);
                        if (m0 + 64 < M) tma_load_2d(a + 8192, &tmA, &full[stage], m0 + 64, k0);
                    }
                    if (!args.b_mn_major) {
                        tma_load_2d(b, &tmB, &full[stage], k0, n0 + bg);
                    } else {
                        for (int j = 0; j < BN / 64; ++j)
                            if (n0 + 64 * j < N)
                                tma_load_2d(b + j * 8192, &tmB, &full[stage], n0 + 64 * j,
                                            k0 + bg);
                    }
                    last_phase[stage] = phase;
                    pending[stage] = true;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                // Error path: let issued copies land before the CTA exits.
#pragma unroll
                for (int s = 0; s < STAGES; ++s)
                    if (pending[s]) mbar_wait_bounded(&full[s], last_phase[s], nullptr, 0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer
            const uint32_t idesc = make_idesc_bf16(BM, BN, args.a_mn_major, args.b_mn_major);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
                int m_blk, n_blk, split, g, kb0, kb1;
                if (!tile_work(args, s_grp, t, num_m, num_n, tiles_mn, kblocks, m_blk, n_blk,
                               split, g, kb0, kb1))
                    continue;
                if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u, args.err,
                                       kDevTimeoutAccFree)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait_bounded(&full[stage], phase, args.err, kDevTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
                    const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t ad =
                            args.a_mn_major ? make_sw128_desc(a_addr + kk * 2048, 8192, 1024)
                                            : make_sw128_desc(a_addr + kk * 32, 16, 1024);
                        const uint64_t bd =
                            args.b_mn_major ? make_sw128_desc(b_addr + kk * 2048, 8192, 1024)
                                            : make_sw128_desc(b_addr + kk * 32, 16, 1024);
                        umma_bf16(d, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                if (kb1 > kb0)
                    umma_commit(&acc_full[acc]);
                else
                    mbar_arrive(&acc_full[acc]);  // empty group: the epilogue writes zeros
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
        }
    } else if (warp >= 4) {
        // ---------------- epilogue warpgroup
        const int q = warp - 4;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int m_blk, n_blk, split, g, kb0, kb1;
            if (!tile_work(args, s_grp, t, num_m, num_n, tiles_mn, kblocks, m_blk, n_blk, split,
                           g, kb0, kb1))
                continue;
            const int m0 = m_blk * BM, n0 = n_blk * BN;
            const bool empty = kb1 <= kb0;
            const long long obase = (args.grp_mode == kGroupK) ? g * args.out_grp_stride : 0;
            if (!mbar_wait_bounded(&acc_full[acc], acc_phase, args.err, kDevTimeoutAcc)) break;
            tc_fence_after();
            const int row = m0 + q * 32 + lane;
            const uint32_t tbase =
                tmem_base + (uint32_t)(acc * BN) + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                if (!empty) {
                    tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), r);
                    tmem_ld_wait();
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) r[j] = 0u;
                }
                const int col0 = n0 + c * 32;
                if (row < M && col0 < N) {
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                    epi_store(args, row, col0, split, obase, v);
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
}

__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int M, int N,
                                     float* __restrict__ out, long long ldo, int col_group,
                                     long long group_stride, int accumulate) {
    const long long total4 = (long long)M * N / 4;
    const long long plane = (long long)M * N;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total4;
         i += (long long)gridDim.x * blockDim.x) {
        const long long e = i * 4;
        const int m = (int)(e / N);
        const int n = (int)(e - (long long)m * N);
        float4 s = reinterpret_cast<const float4*>(part)[i];
        for (int k = 1; k < splits; ++k) {
            float4 p = reinterpret_cast<const float4*>(part + k * plane)[i];
            s.x += p.x;
            s.y += p.y;
            s.z += p.z;
            s.w += p.w;
        }
        const int g = n / col_group;
        float* o = out + g * group_stride + m * ldo + (n - g * col_group);
        if (accumulate) {
            s.x += o[0];
            s.y += o[1];
            s.z += o[2];
            s.w += o[3];
        }
        o[0] = s.x;
        o[1] = s.y;
        o[2] = s.z;
        o[3] = s.w;
    }
}

__global__ void splitk_reduce_scalar_kernel(const float* __restrict__ part, int splits, int M,
                                            int N, float* __restrict__ out, long long ldo,
                                            int col_group, long long group_stride,
                                            int accumulate) {
    const long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long plane = (long long)M * N;
    if (e >= plane) return;
    const int m = (int)(e / N), n = (int)(e - (long long)m * N);
    float s = part[e];
    for (int k = 1; k < splits; ++k) s += part[k * plane + e];
    const int g = n / col_group;
    float* o = out + g * group_stride + m * ldo + (n - g * col_group);
    *o = accumulate ? *o + s : s;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
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

// 2-D bf16 tensor map, 128-byte swizzle: `inner` contiguous elements per row, `outer`
// rows `ld` elements apart; box of box_inner x box_outer elements.
int make_tmap_bf16(CUtensorMap* tm, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
                   uint32_t box_inner, uint32_t box_outer) {
    auto enc = get_encode_fn();
    if (!enc) return -1;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return -2;
    if (((ld * 2) & 15) != 0) return -3;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -4;
}

template <int BN>
int launch_bn(const GemmPlan& p, cudaStream_t stream) {
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(gemm_bf16_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)GemmCfg<BN>::SMEM) != cudaSuccess)
            return -10;
        attr_set = true;
    }
    gemm_bf16_tc_kernel<BN><<<p.grid, kGemmThreads, GemmCfg<BN>::SMEM, stream>>>(p.tmA, p.tmB,
                                                                                p.args);
    return launch_status();
}

}  // namespace

int gemm_make_plan(GemmPlan* plan, const void* A, long long lda, int a_mn_major, const void* B,
                   long long ldb, int b_mn_major, int M, int N, int K, const GemmArgs& epi,
                   int bn_hint, int num_sms) {
    if (M <= 0 || N <= 0 || K <= 0) return -1;
    GemmArgs a = epi;
    a.M = M;
    a.N = N;
    a.K = K;
    a.a_mn_major = a_mn_major;
    a.b_mn_major = b_mn_major;
    if (a.splits < 1) a.splits = 1;
    const int kblocks = (K + BK - 1) / BK;
    if (a.grp_mode != kGroupNone) {
        if (!a.grp || a.groups < 1 || a.groups > kMaxGemmGroups || a.splits != 1) return -40;
        if (a.grp_mode == kGroupRows) {
            // a k-tail would run into the next group's rows of an MN-major B
            if (a_mn_major || (K % BK) != 0 || a.b_grp_rows < (b_mn_major ? K : N)) return -41;
        } else if (a.grp_mode == kGroupK) {
            if (!a_mn_major || !b_mn_major || a.epi != kEpiStoreF32 || a.col_group > 0) return -42;
            a.splits = a.groups;  // the split index of a tile is its group
        } else {
            return -43;
        }
    } else if (a.splits > kblocks) {
        return -5;
    }
    if (a.splits > 1 && a.epi != kEpiSplitPartial && a.grp_mode != kGroupK) return -6;
    if (a.col_group <= 0) a.col_group = N;
    if (a.col_group != N && (a.col_group % 32) != 0) return -7;
    // alignment needed by the vectorised epilogue
    if (a.epi == kEpiStoreBF16 || a.epi == kEpiGeluBF16 || a.epi == kEpiDGeluBF16) {
        if ((a.ldo % 8) != 0 || (reinterpret_cast<uintptr_t>(a.out) & 15)) return -8;
        if ((a.epi != kEpiStoreBF16) &&
            ((a.ld_aux % 8) != 0 || (reinterpret_cast<uintptr_t>(a.aux) & 15)))
            return -8;
    } else if (a.epi == kEpiStoreF32 || a.epi == kEpiResidF32) {
        // narrow or odd-strided fp32 outputs take the scalar store path
        a.scalar_store = ((a.ldo % 4) != 0 || (reinterpret_cast<uintptr_t>(a.out) & 15) ||
                          (a.group_stride % 4) != 0 || (a.out_grp_stride % 4) != 0) ? 1 : 0;
        if (a.epi == kEpiResidF32 &&
            ((a.ldr % 4) != 0 || (reinterpret_cast<uintptr_t>(a.resid) & 15)))
            a.scalar_store = 1;
    } else if (a.epi == kEpiSplitPartial) {
        if (reinterpret_cast<uintptr_t>(a.out) & 15) return -8;
    }
    const int num_m = (M + BM - 1) / BM;
    int bn = bn_hint;
    if (bn != 64 && bn != 128 && bn != 256) {
        // pick the tile width with the smallest estimated makespan
        double best = 1e30;
        const int cands[3] = {256, 128, 64};
        for (int i = 0; i < 3; ++i) {
            int c = cands[i];
            long long tiles = (long long)num_m * ((N + c - 1) / c) * a.splits;
            long long waves = (tiles + num_sms - 1) / num_sms;
            double cost = (double)waves * (c + 48);
            if (cost < best - 1e-9) {
                best = cost;
                bn = c;
            }
        }
    }
    plan->bn = bn;
    plan->args = a;
    int rc;
    if (!a_mn_major)
        rc = make_tmap_bf16(&plan->tmA, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, BK, BM);
    else
        rc = make_tmap_bf16(&plan->tmA, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, BK);
    if (rc) return -20 + rc;
    // a row-grouped B stacks `groups` blocks of b_grp_rows rows along its outer dimension
    const uint64_t b_rows = (a.grp_mode == kGroupRows)
                                ? (uint64_t)a.groups * (uint64_t)a.b_grp_rows
                                : (uint64_t)(b_mn_major ? K : N);
    if (!b_mn_major)
        rc = make_tmap_bf16(&plan->tmB, B, (uint64_t)K, b_rows, (uint64_t)ldb, BK, (uint32_t)bn);
    else
        rc = make_tmap_bf16(&plan->tmB, B, (uint64_t)N, b_rows, (uint64_t)ldb, 64, BK);
    if (rc) return -30 + rc;
    long long tiles = (long long)num_m * ((N + bn - 1) / bn) * a.splits;
    plan->grid = (int)(tiles < num_sms ? tiles : num_sms);
    plan->smem_bytes = bn == 256 ? GemmCfg<256>::SMEM : (bn == 128 ? GemmCfg<128>::SMEM : GemmCfg<64>::SMEM);
    return 0;
}

int gemm_run(const GemmPlan& p, cudaStream_t stream) {
    switch (p.bn) {
        case 256:
            return launch_bn<256>(p, stream);
        case 128:
            return launch_bn<128>(p, stream);
        case 64:
            return launch_bn<64>(p, stream);
        default:
            return -12;
    }
}

int gemm_splitk_reduce(const float* partial, int splits, int M, int N, float* out, long long ldo,
                       int col_group, long long group_stride, int accumulate,
                       cudaStream_t stream) {
    if (col_group <= 0) col_group = N;
    if ((N % 4) != 0 || (ldo % 4) != 0 || (col_group != N && (col_group % 4) != 0) ||
        (group_stride % 4) != 0) {
        const long long total = (long long)M * N;
        splitk_reduce_scalar_kernel<<<(int)((total + 255) / 256), 256, 0, stream>>>(
            partial, splits, M, N, out, ldo, col_group, group_stride, accumulate);
        return launch_status();
    }
    long long total4 = (long long)M * N / 4;
    int threads = 256;
    long long blocks = (total4 + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    splitk_reduce_kernel<<<(int)blocks, threads, 0, stream>>>(partial, splits, M, N, out, ldo,
                                                             col_group, group_stride, accumulate);
    return launch_status();
}

}  // namespace llmgpu
