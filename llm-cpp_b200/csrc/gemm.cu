// tcgen05 GEMM for sm_100a: persistent, warp-specialised, TMA-fed, fp32 accumulators in TMEM.
//
// Roles per CTA (256 threads, one CTA per SM):
//   warp 0      : TMA producer (one elected lane) filling a STAGES-deep smem ring
//   warp 1      : TMEM allocator + MMA issuer (one lane issues tcgen05.mma)
//   warps 4..7  : epilogue (tcgen05.ld from TMEM lanes 32*(warp%4).., fused epilogue, global stores)
// Two TMEM accumulators (2*BN columns) let the epilogue of tile i overlap the MMAs of tile i+1.
//
// Every CTA loads its own operand tiles with plain TMA loads.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <vector>
#include <algorithm>

#include "common.cuh"
#include "gemm.cuh"

namespace llmgpu {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kGemmThreads = 256;
// CTA-pair kernel: warp 0 TMA, warp 1 MMA, warps 4..11 epilogue (two warps per TMEM lane
// quarter, each draining half of a tile's columns)
constexpr int kPairThreads = 384;
constexpr int kPairEpiWarps = 8;
constexpr int kGroupM = 16;  // tile raster: groups of 16 m-blocks share B tiles in L2

template <int BN>
struct GemmCfg {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (BN == 256) ? 4 : (BN == 128 ? 6 : 8);
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 4 * 2 * 4096 + 256;
    static_assert((2 * STAGES + 4 + 8) * 8 + 4 <= 256, "barrier area");
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

// ---------------------------------------------------------------------------- epilogue
// Each epilogue warp owns 32 accumulator rows (TMEM lanes) and moves a tile out in chunks of
// 32 columns. With TMA outputs (args.tma_epi) values go registers -> a swizzled box of 32
// rows in shared memory -> one bulk tensor store (or reduce-add), so every global write is a
// full, coalesced line. Plain bf16 outputs and dGELU pack two chunks per 32 x 64 box
// (128-byte rows: half the bulk operations); fp32 outputs use 32 x 32 boxes, GELU's two bf16
// outputs 32 x 32 boxes with 64-byte rows. Inputs of the epilogue (residual, stored
// pre-activation) come in through TMA loads into the box they are combined in, one unit
// ahead. Two 4 KB boxes per warp alternate so the store of one unit overlaps the next.
// Outputs whose strides a tensor map cannot describe take the per-thread row stores of
// epi_store.
constexpr int kEpiSlotBytes = 4096;
constexpr int kEpiStageBytes = 4 * 2 * kEpiSlotBytes;
constexpr int kPairEpiStageBytes = kPairEpiWarps * 2 * kEpiSlotBytes;

// byte offset of 16-byte chunk `ch` of row r in a box of 128-byte rows (fp32, 128-byte
// swizzle: chunk ^= row % 8) or 64-byte rows (bf16, 64-byte swizzle: chunk ^= (row / 2) % 4)
__device__ __forceinline__ uint32_t box_off_f32(int r, int ch) {
    return (uint32_t)(r * 128 + ((ch ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint32_t box_off_bf16(int r, int ch) {
    return (uint32_t)(r * 64 + ((ch ^ ((r >> 1) & 3)) << 4));
}
__device__ __forceinline__ void box_put_f32(uint8_t* box, int r, const float* v) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch)
        *reinterpret_cast<float4*>(box + box_off_f32(r, ch)) =
            make_float4(v[4 * ch], v[4 * ch + 1], v[4 * ch + 2], v[4 * ch + 3]);
}
__device__ __forceinline__ void box_put_bf16(uint8_t* box, int r, const float* v) {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch)
        *reinterpret_cast<uint4*>(box + box_off_bf16(r, ch)) =
            make_uint4(pack_bf16x2(v[8 * ch], v[8 * ch + 1]), pack_bf16x2(v[8 * ch + 2], v[8 * ch + 3]),
                       pack_bf16x2(v[8 * ch + 4], v[8 * ch + 5]),
                       pack_bf16x2(v[8 * ch + 6], v[8 * ch + 7]));
}

struct EpiWarp {
    uint8_t* stage;   // this warp's two 4 KB boxes
    uint64_t* bar;    // [2]: completion of the input load into each box
    uint32_t phase;   // bit s: parity of bar[s]
    int slot;         // box of the next chunk
    uint32_t pend;    // bit s: an input load into box s not yet waited for
};

// Epilogues that read an input: the residual (fp32, a unit is one 32-column chunk) and the
// stored pre-activation of dGELU (bf16, a unit is two chunks in one 32 x 64 box). A unit's
// input is loaded one unit ahead, the first two before the accumulator is ready, so the
// HBM latency of the input is not paid once per chunk.
__device__ __forceinline__ bool epi_has_input(const GemmArgs& a) {
    return a.tma_epi && (a.epi == kEpiResidF32 || a.epi == kEpiDGeluBF16);
}
__device__ __forceinline__ int epi_unit_chunks(const GemmArgs& a) {
    return a.epi == kEpiDGeluBF16 ? 2 : 1;
}
// End of the chunks of [c_begin, c_end) a TMA epilogue writes: none when the rows are past
// M; none from the first chunk whose columns start at or past N.
__device__ __forceinline__ int epi_chunk_end(const GemmArgs& a, int row0, int n0, int c_begin,
                                             int c_end) {
    if (row0 >= a.M) return c_begin;
    const int lim = (a.N - n0 + 31) / 32;
    return c_end < lim ? c_end : (lim > c_begin ? lim : c_begin);
}
// lane 0: the 4 KB input box of the unit starting at column col0 into box s
__device__ __forceinline__ void epi_load_unit(const CUtensorMap* tmX, EpiWarp& w, int s,
                                              int col0, int row0) {
    mbar_arrive_expect_tx(&w.bar[s], (uint32_t)kEpiSlotBytes);
    tma_load_3d(w.stage + s * kEpiSlotBytes, tmX, &w.bar[s], col0, row0, 0);
    w.pend |= 1u << s;
}
// Issued before the accumulator wait: the inputs of the tile's first two units.
__device__ __forceinline__ void epilogue_prefetch(const GemmArgs& a, const CUtensorMap* tmX,
                                                  int row0, int n0, int lane, EpiWarp& w,
                                                  int c_begin, int c_end) {
    if (!epi_has_input(a)) return;
    const int ce = epi_chunk_end(a, row0, n0, c_begin, c_end);
    const int u = epi_unit_chunks(a);
    if (lane == 0 && ce > c_begin) {
        bulk_wait_group_read<0>();  // earlier stores have read both boxes
        epi_load_unit(tmX, w, w.slot, n0 + c_begin * 32, row0);
        if (c_begin + u < ce) epi_load_unit(tmX, w, w.slot ^ 1, n0 + (c_begin + u) * 32, row0);
    }
    __syncwarp();
}
// Error exit: wait (bounded) for input loads still landing in this warp's boxes.
__device__ __forceinline__ void epilogue_drain(const GemmArgs& a, int lane, EpiWarp& w) {
    if (lane == 0)
        for (int s = 0; s < 2; ++s)
            if (w.pend & (1u << s))
                mbar_wait_bounded(&w.bar[s], (w.phase >> s) & 1u, a.err, kDevTimeoutFull);
    __syncwarp();
}

// The input epilogues (epilogue_prefetch has issued the first two units' loads).
__device__ __forceinline__ void epilogue_input_tile(const GemmArgs& a, const CUtensorMap* tmO,
                                                    const CUtensorMap* tmX, uint32_t tbase,
                                                    bool empty, int row0, int n0, int lane,
                                                    EpiWarp& w, int c_begin, int c_end) {
    const int u = epi_unit_chunks(a);
    const int ce = epi_chunk_end(a, row0, n0, c_begin, c_end);
#pragma unroll 1
    for (int c = c_begin; c < ce; c += u) {
        uint32_t ra[32], rb[32];
        if (!empty) {
            tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), ra);
            if (u == 2) tmem_ld_32x32b_x32(tbase + (uint32_t)((c + 1) * 32), rb);
        }
        // the next unit's input goes into the box the previous unit stored from
        if (c > c_begin && c + u < ce) {
            if (lane == 0) {
                bulk_wait_group_read<0>();
                epi_load_unit(tmX, w, w.slot ^ 1, n0 + (c + u) * 32, row0);
            }
            __syncwarp();
        }
        if (!empty) {
            tmem_ld_wait();
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) ra[j] = rb[j] = 0u;
        }
        uint8_t* box = w.stage + w.slot * kEpiSlotBytes;
        mbar_wait_bounded(&w.bar[w.slot], (w.phase >> w.slot) & 1u, a.err, kDevTimeoutFull);
        w.phase ^= 1u << w.slot;
        w.pend &= ~(1u << w.slot);
        if (a.epi == kEpiResidF32) {
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
                float4* p = reinterpret_cast<float4*>(box + box_off_f32(lane, ch));
                float4 q = *p;
                q.x += __uint_as_float(ra[4 * ch]);
                q.y += __uint_as_float(ra[4 * ch + 1]);
                q.z += __uint_as_float(ra[4 * ch + 2]);
                q.w += __uint_as_float(ra[4 * ch + 3]);
                *p = q;
            }
        } else {
            // dGELU in place: 16-byte chunks 0-3 of a row hold columns c*32.., 4-7 the next 32
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
                uint4* p = reinterpret_cast<uint4*>(box + box_off_f32(lane, ch));
                const uint4 hp = *p;
                const uint32_t h[4] = {hp.x, hp.y, hp.z, hp.w};
                uint32_t o[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int j = 8 * (ch & 3) + 2 * k;
                    const float x0 = __uint_as_float(ch < 4 ? ra[j] : rb[j]);
                    const float x1 = __uint_as_float(ch < 4 ? ra[j + 1] : rb[j + 1]);
                    o[k] = pack_bf16x2(x0 * gelu_tanh_grad(bf16_lo(h[k])),
                                       x1 * gelu_tanh_grad(bf16_hi(h[k])));
                }
                *p = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_3d(tmO, box, n0 + c * 32, row0, 0);
            bulk_commit_group();
        }
        w.slot ^= 1;
    }
}

// Rotary embedding of one lane's 32 accumulator columns [col0, col0 + 32) of row m (a chunk
// never straddles a head: rope_hd and col0 are multiples of 32).
__device__ __forceinline__ void rope_chunk(const GemmArgs& a, int m, int col0, uint32_t (&r)[32]) {
    if (col0 >= a.rope_cols || m >= a.M) return;
    const int half = a.rope_hd >> 1;
    const float2* cs = a.rope + (long long)(m % a.rope_T) * half + ((col0 % a.rope_hd) >> 1);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const float2 w = cs[i];
        const float x0 = __uint_as_float(r[2 * i]), x1 = __uint_as_float(r[2 * i + 1]);
        r[2 * i] = __float_as_uint(x0 * w.x - x1 * w.y);
        r[2 * i + 1] = __float_as_uint(x0 * w.y + x1 * w.x);
    }
}

// One accumulator tile of one warp: rows [row0, row0+32), columns [n0, n0+NCOLS), TMEM
// columns from tbase. `empty`: the tile had no k-blocks (writes zeros).
template <int NCOLS>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& a, const CUtensorMap* tmO,
                                              const CUtensorMap* tmX, uint32_t tbase, bool empty,
                                              int row0, int n0, int split, int g, int lane,
                                              EpiWarp& w, int c_begin = 0,
                                              int c_end = NCOLS / 32) {
    if (epi_has_input(a)) {
        epilogue_input_tile(a, tmO, tmX, tbase, empty, row0, n0, lane, w, c_begin, c_end);
        return;
    }
    if (a.tma_epi && a.epi == kEpiStoreBF16) {
        // two chunks per 32 x 64 box (128-byte rows): half the bulk stores of 32 x 32 boxes.
        // A warp's chunk range has even length; a second chunk past N is clipped by the store.
        if (row0 >= a.M) return;
        const int lim = (a.N - n0 + 31) / 32;
        const int ce = c_end < lim ? c_end : lim;
#pragma unroll 1
        for (int c = c_begin; c < ce; c += 2) {
            uint32_t ra[32], rb[32];
            if (!empty) {
                tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), ra);
                tmem_ld_32x32b_x32(tbase + (uint32_t)((c + 1) * 32), rb);
                tmem_ld_wait();
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) ra[j] = rb[j] = 0u;
            }
            if (a.rope) {
                rope_chunk(a, row0 + lane, n0 + c * 32, ra);
                rope_chunk(a, row0 + lane, n0 + (c + 1) * 32, rb);
            }
            uint8_t* box = w.stage + w.slot * kEpiSlotBytes;
            if (lane == 0) bulk_wait_group_read<1>();  // this box's previous store has read it
            __syncwarp();
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                *reinterpret_cast<uint4*>(box + box_off_f32(lane, ch)) = make_uint4(
                    pack_bf16x2(__uint_as_float(ra[8 * ch]), __uint_as_float(ra[8 * ch + 1])),
                    pack_bf16x2(__uint_as_float(ra[8 * ch + 2]), __uint_as_float(ra[8 * ch + 3])),
                    pack_bf16x2(__uint_as_float(ra[8 * ch + 4]), __uint_as_float(ra[8 * ch + 5])),
                    pack_bf16x2(__uint_as_float(ra[8 * ch + 6]), __uint_as_float(ra[8 * ch + 7])));
                *reinterpret_cast<uint4*>(box + box_off_f32(lane, ch + 4)) = make_uint4(
                    pack_bf16x2(__uint_as_float(rb[8 * ch]), __uint_as_float(rb[8 * ch + 1])),
                    pack_bf16x2(__uint_as_float(rb[8 * ch + 2]), __uint_as_float(rb[8 * ch + 3])),
                    pack_bf16x2(__uint_as_float(rb[8 * ch + 4]), __uint_as_float(rb[8 * ch + 5])),
                    pack_bf16x2(__uint_as_float(rb[8 * ch + 6]), __uint_as_float(rb[8 * ch + 7])));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_3d(tmO, box, n0 + c * 32, row0, 0);
                bulk_commit_group();
            }
            w.slot ^= 1;
        }
        return;
    }
#pragma unroll 1
    for (int c = c_begin; c < c_end; ++c) {
        uint32_t r[32];
        if (!empty) {
            tmem_ld_32x32b_x32(tbase + (uint32_t)(c * 32), r);
            tmem_ld_wait();
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
        const int col0 = n0 + c * 32;
        if (row0 >= a.M || col0 >= a.N) continue;  // uniform across the warp
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (!a.tma_epi) {
            const long long obase = (a.grp_mode == kGroupK) ? g * a.out_grp_stride : 0;
            if (row0 + lane < a.M) epi_store(a, row0 + lane, col0, split, obase, v);
            continue;
        }
        uint8_t* box = w.stage + w.slot * kEpiSlotBytes;
        if (lane == 0) bulk_wait_group_read<1>();  // this box's previous store has read it
        __syncwarp();
        int x = col0, z = 0;
        bool reduce = false;
        switch (a.epi) {
            case kEpiStoreBF16:
                box_put_bf16(box, lane, v);
                break;
            case kEpiStoreF32:
                box_put_f32(box, lane, v);
                if (a.grp_mode == kGroupK) {
                    z = g;
                } else if (a.col_group != a.N) {
                    z = col0 / a.col_group;
                    x = col0 - z * a.col_group;
                }
                reduce = a.accumulate != 0;
                break;
            case kEpiSplitPartial:
                box_put_f32(box, lane, v);
                z = split;
                break;
            case kEpiGeluBF16: {
                box_put_bf16(box, lane, v);  // pre-activation -> aux
                float gv[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) gv[j] = gelu_tanh(v[j]);
                box_put_bf16(box + 2048, lane, gv);
                break;
            }
            default:
                break;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            if (a.epi == kEpiGeluBF16) {
                tma_store_3d(tmX, box, col0, row0, 0);
                tma_store_3d(tmO, box + 2048, col0, row0, 0);
            } else if (reduce) {
                tma_reduce_add_3d(tmO, box, x, row0, z);
            } else {
                tma_store_3d(tmO, box, x, row0, z);
            }
            bulk_commit_group();
        }
        w.slot ^= 1;
    }
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmO,
                        const __grid_constant__ CUtensorMap tmX, const GemmArgs args) {
    using Cfg = GemmCfg<BN>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
    uint8_t* sEpi = smem + STAGES * Cfg::STAGE_BYTES;  // 2 boxes per epilogue warp
    uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + kEpiStageBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* epi_bar = acc_empty + 2;  // two per epilogue warp
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_bar + 8);

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
        for (int i = 0; i < 8; ++i) mbar_init(&epi_bar[i], 1);
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
    pdl_enter();  // barriers, TMEM and descriptors are set up while the previous kernel ends
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
        EpiWarp ew{sEpi + q * 2 * kEpiSlotBytes, &epi_bar[2 * q], 0u, 0, 0u};
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int m_blk, n_blk, split, g, kb0, kb1;
            if (!tile_work(args, s_grp, t, num_m, num_n, tiles_mn, kblocks, m_blk, n_blk, split,
                           g, kb0, kb1))
                continue;
            const int m0 = m_blk * BM, n0 = n_blk * BN;
            epilogue_prefetch(args, &tmX, m0 + q * 32, n0, lane, ew, 0, BN / 32);
            if (!mbar_wait_bounded(&acc_full[acc], acc_phase, args.err, kDevTimeoutAcc)) {
                epilogue_drain(args, lane, ew);
                break;
            }
            tc_fence_after();
            const uint32_t tbase =
                tmem_base + (uint32_t)(acc * BN) + ((uint32_t)(q * 32) << 16);
            epilogue_tile<BN>(args, &tmO, &tmX, tbase, kb1 <= kb0, m0 + q * 32, n0, split, g,
                              lane, ew);
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
        if (lane == 0) bulk_wait_group_all();  // stores complete before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
}

// ---------------------------------------------------------------------------- CTA pairs
// 256 x 256 output tiles on a cluster of two CTAs (two SMs) sharing each tcgen05 MMA
// (cta_group::2). Per k-block each CTA stages its 128 rows of A and its 128 rows (N) of B,
// so an SM streams 32 KB per 128x256x64 of MMA work instead of 48 KB, and six stages fit.
// Each CTA holds rows [128*rank, 128*rank+128) of the tile in its own TMEM (two 256-column
// accumulators) and runs its own epilogue. The leader CTA (rank 0) issues every MMA; its
// commits arrive on the stage / accumulator barriers of both CTAs; both CTAs' loads count
// their bytes on the leader's stage barrier; the follower's epilogue arrives remotely on
// the leader's accumulator-free barrier.
struct PairCfg {
    static constexpr int BMP = 256;
    static constexpr int BN = 256;
    static constexpr int BNH = 128;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BNH * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = 5;
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + kPairEpiStageBytes + 256;
    // the last 256 bytes: stage, accumulator and epilogue barriers, then the TMEM address
    static_assert((2 * STAGES + 4 + 2 * kPairEpiWarps) * 8 + 4 <= 256, "barrier area");
};

// Bytes one CTA of a pair loads per k-block (A rows from am, B rows from bn); boxes wholly
// past M or N are not loaded (their rows or columns are discarded by the epilogue).
__device__ __forceinline__ uint32_t pair_stage_bytes(const GemmArgs& a, int am, int bn) {
    uint32_t bytes = 0;
    if (!a.a_mn_major)
        bytes += (am < a.M) ? (uint32_t)PairCfg::A_BYTES : 0u;
    else
        bytes += 8192u * ((am < a.M ? 1u : 0u) + (am + 64 < a.M ? 1u : 0u));
    if (!a.b_mn_major)
        bytes += (bn < a.N) ? (uint32_t)PairCfg::B_BYTES : 0u;
    else
        bytes += 8192u * ((bn < a.N ? 1u : 0u) + (bn + 64 < a.N ? 1u : 0u));
    return bytes;
}

// Launch parameters of the pair kernel for NG co-scheduled products (NG = 2: the data- and
// weight-gradient products of one layer, which read the same upstream gradient but not each
// other's results). With NG = 1 cluster c takes tiles c, c + clusters, ...; with NG = 2 the
// host's per-cluster lists in `sched` ([cluster][stride]: count, then items g << 24 | tile)
// balance the two products' tiles over the pairs.
//
// With `queue` set (NG = 2), the units are handed out at run time instead: the leader CTA's
// producer claims the next unit from queue[0] a few k-blocks before its current tile's loads
// end and publishes it through a ring of kItemSlots slots in both CTAs' shared memory, and
// every other role of the pair takes the units from the ring in the same order. Units are
// numbered longest first: all units of product q_first, then those of the other product
// (split-major tile order within a product). A pair whose SMs start late, held by another
// kernel such as a collective, takes fewer units. queue[1] counts the pairs that have
// finished claiming; the last one resets both counters for the next launch.
template <int NG>
struct PairParams {
    CUtensorMap tmA[NG];
    CUtensorMap tmB[NG];
    CUtensorMap tmO[NG];
    CUtensorMap tmX[NG];
    GemmArgs args[NG];
    const int* sched;
    int sched_stride;
    int* queue;
    int q_first;
    int q_total[2];
};

constexpr int kItemSlots = 4;
// roles that take each unit from the ring: the leader's MMA issuer and the follower's
// producer, and every epilogue warp of both CTAs
constexpr int kItemConsumers = 2 + 2 * kPairEpiWarps;
// k-blocks before the end of a tile's loads at which the leader claims its next unit (the
// claim's round trip to L2 overlaps these loads)
constexpr int kClaimAhead = 4;

// Unit number idx of the run-time queue as (product << 24 | tile), -1 past the last one.
template <int NG>
__device__ __forceinline__ int pair_queue_unit(const PairParams<NG>& P, int idx) {
    const int f = P.q_first, n0 = P.q_total[f];
    if (idx < n0) return (f << 24) | idx;
    idx -= n0;
    return idx < P.q_total[f ^ 1] ? (((f ^ 1) << 24) | idx) : -1;
}

// One role's view of the unit ring. Slot s of the ring carries units s, s + kItemSlots, ...;
// `full` (one per slot, in each CTA) completes when the leader's producer has written the
// slot in both CTAs, `empty` (one per slot, in the leader CTA) when all kItemConsumers roles
// have read it.
struct PairRing {
    uint64_t* full;
    uint64_t* empty;
    int* slot;
    uint32_t rank;
    int i;
    // A consumer's next unit; -1 when the list has ended or the wait gave up (error set).
    // With warp_wide, all 32 lanes take the unit and lane 0 releases the slot.
    __device__ __forceinline__ int take(int* err, bool warp_wide) {
        const int s = i % kItemSlots;
        const uint32_t parity = (uint32_t)(i / kItemSlots) & 1u;
        ++i;
        if (!mbar_wait_bounded_cluster(&full[s], parity, err, kDevTimeoutItem)) return -1;
        const int v = *reinterpret_cast<volatile int*>(&slot[s]);
        if (warp_wide) __syncwarp();
        if (!warp_wide || (threadIdx.x & 31) == 0) {
            if (rank == 0)
                mbar_arrive(&empty[s]);
            else
                mbar_arrive_cluster(mapa_shared(smem_u32(&empty[s]), 0));
        }
        return v;
    }
    // The leader producer publishes unit v (-1 ends every role's list) once the slot's
    // previous unit has been read by every consumer.
    __device__ __forceinline__ bool put(int v, int* err) {
        const int s = i % kItemSlots;
        if (i >= kItemSlots &&
            !mbar_wait_bounded(&empty[s], (uint32_t)(i / kItemSlots - 1) & 1u, err,
                               kDevTimeoutItem))
            return false;
        ++i;
        slot[s] = v;
        st_shared_cluster_u32(mapa_shared(smem_u32(&slot[s]), 1), (uint32_t)v);
        mbar_arrive(&full[s]);
        mbar_arrive_cluster(mapa_shared(smem_u32(&full[s]), 1));
        return true;
    }
};

// Tile geometry of one product on 256 x 256 pair tiles.
struct PairShape {
    int num_m, num_n, tiles_mn, kblocks;
};
__device__ __forceinline__ PairShape pair_shape(const GemmArgs& a) {
    PairShape s;
    s.num_m = (a.M + PairCfg::BMP - 1) / PairCfg::BMP;
    s.num_n = (a.N + PairCfg::BN - 1) / PairCfg::BN;
    s.tiles_mn = s.num_m * s.num_n;
    s.kblocks = (a.K + BK - 1) / BK;
    return s;
}

// The work items of cluster cid in order: product g, tile t of that product (split-major).
// With two products the items come from the cluster's list in the host-built table; the
// entry of the next item is loaded while the current one is processed, so no role waits on
// a global load at a tile boundary.
template <int NG>
struct PairItems {
    const int* list;
    int n, i, next;
    int cid, nclusters, total;
    __device__ __forceinline__ PairItems(const PairParams<NG>& P, int cid_, int ncl) {
        cid = cid_;
        nclusters = ncl;
        i = 0;
        if constexpr (NG == 1) {
            const PairShape s = pair_shape(P.args[0]);
            total = s.tiles_mn * P.args[0].splits;
            list = nullptr;
            n = next = 0;
        } else {
            total = 0;
            list = P.sched + (size_t)cid * P.sched_stride;
            n = list[0];
            next = n > 0 ? list[1] : 0;
        }
    }
    __device__ __forceinline__ bool get(int& g, int& t) {
        if constexpr (NG == 1) {
            g = 0;
            t = cid + i * nclusters;
            ++i;
            return t < total;
        } else {
            if (i >= n) return false;
            const int v = next;
            if (i + 1 < n) next = list[2 + i];
            ++i;
            g = v >> 24;
            t = v & 0xffffff;
            return true;
        }
    }
};

template <int NG>
__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ PairParams<NG> P) {
    using Cfg = PairCfg;
    constexpr int STAGES = Cfg::STAGES;
    constexpr int BN = Cfg::BN;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_u32 = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
    uint8_t* sEpi = smem + STAGES * Cfg::STAGE_BYTES;  // 2 boxes per epilogue warp
    uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + kPairEpiStageBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* epi_bar = acc_empty + 2;  // two per epilogue warp
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(epi_bar + 2 * kPairEpiWarps);

    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int cid = blockIdx.x >> 1;
    const int nclusters = gridDim.x >> 1;
    int* const err = P.args[0].err;
    // run-time unit queue (dual launches): ring barriers [full x kItemSlots, empty x
    // kItemSlots] and slots
    const bool dyn = NG == 2 && P.queue != nullptr;
    __shared__ __align__(8) uint64_t s_item_bar[2 * kItemSlots];
    __shared__ int s_item[kItemSlots];

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kItemSlots; ++s) {
            mbar_init(&s_item_bar[s], 1);
            mbar_init(&s_item_bar[kItemSlots + s], kItemConsumers);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 2 * 32 * kPairEpiWarps);  // epilogue threads, both CTAs
        }
        for (int i = 0; i < 2 * kPairEpiWarps; ++i) mbar_init(&epi_bar[i], 1);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        for (int g = 0; g < NG; ++g) {
            tma_prefetch_desc(&P.tmA[g]);
            tma_prefetch_desc(&P.tmB[g]);
        }
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish_pair();
    }
    pdl_enter();  // barriers, TMEM and descriptors are set up while the previous kernel ends
    // row-group table of a grouped product (single products only)
    __shared__ int s_grp[kMaxGemmGroups + 1];
    if (NG == 1 && P.args[0].grp_mode != kGroupNone)
        for (int i = threadIdx.x; i <= P.args[0].groups; i += blockDim.x) s_grp[i] = P.args[0].grp[i];
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // barriers of both CTAs initialised before any remote use
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs)
            const uint32_t full_leader = mapa_shared(smem_u32(&full[0]), 0);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int g, t;
            PairItems<NG> items(P, cid, nclusters);
            PairRing ring{s_item_bar, s_item_bar + kItemSlots, s_item, rank, 0};
            const bool claimer = dyn && leader;
            int pending = claimer ? atomicAdd(P.queue, 1) : 0;  // the leader's next unit
            while (ok) {
                if (dyn) {
                    int v;
                    if (leader) {
                        v = pair_queue_unit(P, pending);
                        if (!ring.put(v, err)) break;
                    } else {
                        v = ring.take(err, false);
                    }
                    if (v < 0) break;
                    g = v >> 24;
                    t = v & 0xffffff;
                } else if (!items.get(g, t)) {
                    break;
                }
                const GemmArgs& args = P.args[g];
                const PairShape sh = pair_shape(args);
                const CUtensorMap* tmA = &P.tmA[g];
                const CUtensorMap* tmB = &P.tmB[g];
                int m_blk, n_blk, split, gi, kb0, kb1;
                tile_work(args, s_grp, t, sh.num_m, sh.num_n, sh.tiles_mn, sh.kblocks, m_blk,
                          n_blk, split, gi, kb0, kb1);
                const int M = args.M, N = args.N;
                const int m0 = m_blk * Cfg::BMP, n0 = n_blk * BN;
                const int am = m0 + 128 * (int)rank, bn = n0 + Cfg::BNH * (int)rank;
                const uint32_t all_bytes = leader ? pair_stage_bytes(args, m0, n0) +
                                                        pair_stage_bytes(args, m0 + 128, n0 + Cfg::BNH)
                                                  : 0u;
                const int claim_at = kb1 - kClaimAhead > kb0 ? kb1 - kClaimAhead : kb0;
                if (claimer && kb1 <= kb0) pending = atomicAdd(P.queue, 1);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (claimer && kb == claim_at) pending = atomicAdd(P.queue, 1);
                    if (!mbar_wait_bounded_cluster(&empty[stage], phase ^ 1u, err,
                                                   kDevTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&full[stage], all_bytes);
                    const uint32_t fb = full_leader + 8u * (uint32_t)stage;
                    const int k0 = kb * BK;
                    uint8_t* a = sA + stage * Cfg::A_BYTES;
                    uint8_t* b = sB + stage * Cfg::B_BYTES;
                    if (!args.a_mn_major) {
                        if (am < M) tma_load_2d_pair(a, tmA, fb, k0, am);
                    } else {
                        if (am < M) tma_load_2d_pair(a, tmA, fb, am, k0);
                        if (am + 64 < M) tma_load_2d_pair(a + 8192, tmA, fb, am + 64, k0);
                    }
                    if (!args.b_mn_major) {
                        if (bn < N) tma_load_2d_pair(b, tmB, fb, k0, bn);
                    } else {
                        if (bn < N) tma_load_2d_pair(b, tmB, fb, bn, k0);
                        if (bn + 64 < N) tma_load_2d_pair(b + 8192, tmB, fb, bn + 64, k0);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // the last pair to finish claiming resets the counters for the next launch
            if (claimer && atomicAdd(P.queue + 1, 1) == nclusters - 1) {
                atomicExch(P.queue, 0);
                atomicExch(P.queue + 1, 0);
            }
            if (!ok) spin_ns(100000);  // error path: let copies in flight land first
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer (leader only)
            const uint32_t acc_full_peer = mapa_shared(smem_u32(&acc_full[0]), 1);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            int g, t;
            PairItems<NG> items(P, cid, nclusters);
            PairRing ring{s_item_bar, s_item_bar + kItemSlots, s_item, rank, 0};
            while (ok) {
                if (dyn) {
                    const int v = ring.take(err, false);
                    if (v < 0) break;
                    g = v >> 24;
                    t = v & 0xffffff;
                } else if (!items.get(g, t)) {
                    break;
                }
                const GemmArgs& args = P.args[g];
                const PairShape sh = pair_shape(args);
                const uint32_t idesc =
                    make_idesc_bf16(Cfg::BMP, BN, args.a_mn_major, args.b_mn_major);
                int m_blk, n_blk, split, gi, kb0, kb1;
                tile_work(args, s_grp, t, sh.num_m, sh.num_n, sh.tiles_mn, sh.kblocks, m_blk,
                          n_blk, split, gi, kb0, kb1);
                if (!mbar_wait_bounded_cluster(&acc_empty[acc], acc_phase ^ 1u, err,
                                               kDevTimeoutAccFree)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait_bounded_cluster(&full[stage], phase, err, kDevTimeoutFull)) {
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
                        umma_bf16_pair(d, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit_pair(&empty[stage], 0x3);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                if (kb1 > kb0) {
                    umma_commit_pair(&acc_full[acc], 0x3);
                } else {  // empty group: both epilogues write zeros
                    mbar_arrive(&acc_full[acc]);
                    mbar_arrive_cluster(acc_full_peer + 8u * (uint32_t)acc);
                }
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
        }
    } else if (warp >= 4) {
        // ---------------- epilogue warps (both CTAs): warp 4 + e drains TMEM lane quarter
        // e % 4, columns [half * BN/2, (half + 1) * BN/2) with half = e / 4
        const int e = warp - 4;
        const int q = e & 3, half = e >> 2;
        const uint32_t acc_empty_leader = mapa_shared(smem_u32(&acc_empty[0]), 0);
        EpiWarp ew{sEpi + e * 2 * kEpiSlotBytes, &epi_bar[2 * e], 0u, 0, 0u};
        int acc = 0;
        uint32_t acc_phase = 0;
        int g, t;
        PairItems<NG> items(P, cid, nclusters);
        PairRing ring{s_item_bar, s_item_bar + kItemSlots, s_item, rank, 0};
        while (true) {
            if (dyn) {
                const int v = ring.take(err, true);
                if (v < 0) break;
                g = v >> 24;
                t = v & 0xffffff;
            } else if (!items.get(g, t)) {
                break;
            }
            const GemmArgs& args = P.args[g];
            const PairShape sh = pair_shape(args);
            int m_blk, n_blk, split, gi, kb0, kb1;
            tile_work(args, s_grp, t, sh.num_m, sh.num_n, sh.tiles_mn, sh.kblocks, m_blk, n_blk,
                      split, gi, kb0, kb1);
            const int m0 = m_blk * Cfg::BMP + 128 * (int)rank, n0 = n_blk * BN;
            epilogue_prefetch(args, &P.tmX[g], m0 + q * 32, n0, lane, ew, half * (BN / 64),
                              (half + 1) * (BN / 64));
            if (!mbar_wait_bounded_cluster(&acc_full[acc], acc_phase, err, kDevTimeoutAcc)) {
                epilogue_drain(args, lane, ew);
                break;
            }
            tc_fence_after();
            const uint32_t tbase =
                tmem_base + (uint32_t)(acc * BN) + ((uint32_t)(q * 32) << 16);
            epilogue_tile<BN>(args, &P.tmO[g], &P.tmX[g], tbase, kb1 <= kb0, m0 + q * 32, n0,
                              split, gi, lane, ew, half * (BN / 64), (half + 1) * (BN / 64));
            tc_fence_before();
            if (leader)
                mbar_arrive(&acc_empty[acc]);
            else
                mbar_arrive_cluster(acc_empty_leader + 8u * (uint32_t)acc);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
        if (lane == 0) bulk_wait_group_all();  // stores complete before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // neither CTA leaves while the other may still touch its memory
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
}

__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int M, int N,
                                     float* __restrict__ out, long long ldo, int col_group,
                                     long long group_stride, int accumulate) {
    pdl_enter();
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

// The same reduction for a split count known at compile time: each thread takes two 4-column
// groups per pass with all 2 x S plane loads issued before the first add (the planes are
// summed in split order, as above).
template <int S>
__global__ void __launch_bounds__(256) splitk_reduce_s_kernel(
    const float* __restrict__ part, int M, int N, float* __restrict__ out, long long ldo,
    int col_group, long long group_stride, int accumulate) {
    pdl_enter();
    const long long total4 = (long long)M * N / 4;
    const float4* p4 = reinterpret_cast<const float4*>(part);
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total4;
         i += 2 * stride) {
        const long long i2 = i + stride;
        const bool two = i2 < total4;
        float4 a[S], b[S];
#pragma unroll
        for (int k = 0; k < S; ++k) {
            a[k] = p4[k * total4 + i];
            if (two) b[k] = p4[k * total4 + i2];
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (h == 1 && !two) break;
            const float4* v = h == 0 ? a : b;
            float4 s = v[0];
#pragma unroll
            for (int k = 1; k < S; ++k) {
                s.x += v[k].x;
                s.y += v[k].y;
                s.z += v[k].z;
                s.w += v[k].w;
            }
            const long long e = (h == 0 ? i : i2) * 4;
            const int m = (int)(e / N);
            const int n = (int)(e - (long long)m * N);
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
}

__global__ void splitk_reduce_scalar_kernel(const float* __restrict__ part, int splits, int M,
                                            int N, float* __restrict__ out, long long ldo,
                                            int col_group, long long group_stride,
                                            int accumulate) {
    pdl_enter();
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

// 3-D tensor map over an epilogue output or input: dims {x, y, z} with row stride `ys` and
// plane stride `zs` in bytes. Boxes are 32 rows of 32 fp32 or 32 bf16 columns, or (wide) 64
// bf16 columns; rows of 128 bytes take the 128-byte swizzle (the layout box_off_f32
// addresses), 64-byte rows the 64-byte one (box_off_bf16).
int make_tmap_box(CUtensorMap* tm, const void* ptr, bool f32, uint64_t x, uint64_t y, uint64_t z,
                  uint64_t ys, uint64_t zs, bool wide = false) {
    auto enc = get_encode_fn();
    if (!enc) return -1;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0 || (ys & 15) != 0 || (zs & 15) != 0)
        return -2;
    const bool rows128 = f32 || wide;
    cuuint64_t dims[3] = {x, y, z};
    cuuint64_t strides[2] = {ys, zs};
    cuuint32_t box[3] = {(!f32 && wide) ? 64u : 32u, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(tm, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                     const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     rows128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -4;
}

// Output (and epilogue input) tensor maps for the TMA epilogue; returns false when a stride
// or base address cannot be described (the per-thread store path is used then).
bool plan_tma_epilogue(GemmPlan* plan, const GemmArgs& a) {
    if (a.scalar_store) return false;
    const bool f32 = (a.epi == kEpiStoreF32 || a.epi == kEpiResidF32 || a.epi == kEpiSplitPartial);
    const uint64_t elt = f32 ? 4 : 2;
    const uint64_t ys = (uint64_t)a.ldo * elt;
    uint64_t x = (uint64_t)a.N, z = 1, zs = ys * (uint64_t)a.M;
    if (a.epi == kEpiStoreF32) {
        if (a.grp_mode == kGroupK) {
            z = (uint64_t)a.groups;
            zs = (uint64_t)a.out_grp_stride * 4;
        } else if (a.col_group != a.N) {
            x = (uint64_t)a.col_group;
            z = (uint64_t)(a.N / a.col_group);
            zs = (uint64_t)a.group_stride * 4;
        }
    } else if (a.epi == kEpiSplitPartial) {
        z = (uint64_t)a.splits;
        zs = (uint64_t)a.M * (uint64_t)a.N * 4;  // planes [split][M][N], ldo == N
        if (a.ldo != a.N) return false;
    }
    zs = (zs + 15) & ~(uint64_t)15;  // a single plane: any aligned stride
    if (z > 1 && ((a.epi == kEpiStoreF32 && ((a.grp_mode == kGroupK ? a.out_grp_stride
                                                                     : a.group_stride) * 4) % 16) ||
                  (a.epi == kEpiSplitPartial && ((uint64_t)a.M * a.N * 4) % 16)))
        return false;
    // plain bf16 outputs leave in 32 x 64 boxes (two chunks per store)
    if (make_tmap_box(&plan->tmO, a.out, f32, x, (uint64_t)a.M, z, ys, zs,
                      a.epi == kEpiStoreBF16 || a.epi == kEpiDGeluBF16))
        return false;
    if (a.epi == kEpiResidF32) {
        const uint64_t rs = (uint64_t)a.ldr * 4;
        if (make_tmap_box(&plan->tmX, a.resid, true, (uint64_t)a.N, (uint64_t)a.M, 1, rs,
                          (rs * a.M + 15) & ~(uint64_t)15))
            return false;
    } else if (a.epi == kEpiGeluBF16 || a.epi == kEpiDGeluBF16) {
        const uint64_t xs = (uint64_t)a.ld_aux * 2;
        if (make_tmap_box(&plan->tmX, a.aux, false, (uint64_t)a.N, (uint64_t)a.M, 1, xs,
                          (xs * a.M + 15) & ~(uint64_t)15, a.epi == kEpiDGeluBF16))
            return false;
    } else {
        plan->tmX = plan->tmO;
    }
    return true;
}

}  // namespace

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("LLMGPU_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

namespace {

template <int BN>
int launch_bn(const GemmPlan& p, cudaStream_t stream) {
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(gemm_bf16_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)GemmCfg<BN>::SMEM) != cudaSuccess)
            return -10;
        attr_set = true;
    }
    return launch_kernel_pdl(gemm_bf16_tc_kernel<BN>, p.grid, kGemmThreads, GemmCfg<BN>::SMEM,
                             stream, p.tmA, p.tmB, p.tmO, p.tmX, p.args);
}

int pair_set_attr() {
    static int rc = -1;
    static std::once_flag once;
    std::call_once(once, [] {
        rc = (cudaFuncSetAttribute(gemm_bf16_pair_kernel<1>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)PairCfg::SMEM) == cudaSuccess &&
              cudaFuncSetAttribute(gemm_bf16_pair_kernel<2>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)PairCfg::SMEM) == cudaSuccess)
                 ? 0
                 : -10;
    });
    return rc;
}

// Clusters of two that can be resident at once (one CTA per SM).
int pair_max_clusters(int num_sms) {
    static int n = -1;
    static std::once_flag once;
    std::call_once(once, [num_sms] {
        n = num_sms / 2;
        if (pair_set_attr()) return;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (num_sms / 2), 1, 1);
        cfg.blockDim = dim3(kPairThreads, 1, 1);
        cfg.dynamicSmemBytes = PairCfg::SMEM;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int c = 0;
        if (cudaOccupancyMaxActiveClusters(&c, gemm_bf16_pair_kernel<1>, &cfg) == cudaSuccess &&
            c > 0)
            n = c < n ? c : n;
        cudaGetLastError();
    });
    return n;
}

template <int NG>
int launch_pair_params(const PairParams<NG>& P, int grid, cudaStream_t stream) {
    if (pair_set_attr()) return -10;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kPairThreads, 1, 1);
    cfg.dynamicSmemBytes = PairCfg::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_bf16_pair_kernel<NG>, P);
    return e == cudaSuccess ? 0 : -(1000 + (int)e);
}

int launch_pair(const GemmPlan& p, cudaStream_t stream) {
    PairParams<1> P;
    P.tmA[0] = p.tmA;
    P.tmB[0] = p.tmB;
    P.tmO[0] = p.tmO;
    P.tmX[0] = p.tmX;
    P.args[0] = p.args;
    P.sched = nullptr;
    P.sched_stride = 0;
    P.queue = nullptr;
    P.q_first = 0;
    P.q_total[0] = P.q_total[1] = 0;
    return launch_pair_params<1>(P, p.grid, stream);
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
    const bool pair_ok = a.grp_mode != kGroupRows;  // a pair tile spans 256 rows of one group
    int bn = bn_hint;
    if (bn == kGemmPairTile && !pair_ok) return -44;
    if (bn != 64 && bn != 128 && bn != 256 && bn != kGemmPairTile) {
        // pick the tile with the smallest estimated makespan; a CTA pair streams a third
        // less operand data per MMA than one CTA with a 128x256 tile, and runs about
        // 1.6x faster per SM
        double best = 1e30;
        const int cands[4] = {kGemmPairTile, 256, 128, 64};
        for (int i = pair_ok ? 0 : 1; i < 4; ++i) {
            const int c = cands[i];
            double cost;
            if (c == kGemmPairTile) {
                const long long tiles = (long long)((M + 255) / 256) * ((N + 255) / 256) * a.splits;
                const int slots = pair_max_clusters(num_sms);
                const long long waves = (tiles + slots - 1) / slots;
                cost = (double)waves * (256 + 48) / 1.6;
            } else {
                const long long tiles = (long long)num_m * ((N + c - 1) / c) * a.splits;
                const long long waves = (tiles + num_sms - 1) / num_sms;
                cost = (double)waves * (c + 48);
            }
            if (cost < best - 1e-9) {
                best = cost;
                bn = c;
            }
        }
    }
    plan->bn = bn;
    a.tma_epi = 0;
    if (std::getenv("LLMGPU_GEMM_DIRECT_EPILOGUE") == nullptr) a.tma_epi = plan_tma_epilogue(plan, a) ? 1 : 0;
    if (!a.tma_epi) plan->tmO = plan->tmX = CUtensorMap{};
    // the rotary epilogue runs on the bf16 TMA store path only
    if (a.rope && (a.epi != kEpiStoreBF16 || !a.tma_epi || a.rope_T <= 0 || a.rope_hd <= 0 ||
                   (a.rope_hd % 32) != 0 || (a.rope_cols % 32) != 0))
        return -9;
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
    // a CTA of a pair stages 128 of the tile's 256 B rows
    const uint32_t b_box = (bn == kGemmPairTile) ? (uint32_t)PairCfg::BNH : (uint32_t)bn;
    if (!b_mn_major)
        rc = make_tmap_bf16(&plan->tmB, B, (uint64_t)K, b_rows, (uint64_t)ldb, BK, b_box);
    else
        rc = make_tmap_bf16(&plan->tmB, B, (uint64_t)N, b_rows, (uint64_t)ldb, 64, BK);
    if (rc) return -30 + rc;
    if (bn == kGemmPairTile) {
        const long long tiles = (long long)((M + 255) / 256) * ((N + 255) / 256) * a.splits;
        const int slots = pair_max_clusters(num_sms);
        plan->grid = 2 * (int)(tiles < slots ? tiles : slots);
        plan->smem_bytes = PairCfg::SMEM;
        return 0;
    }
    long long tiles = (long long)num_m * ((N + bn - 1) / bn) * a.splits;
    plan->grid = (int)(tiles < num_sms ? tiles : num_sms);
    plan->smem_bytes = bn == 256 ? GemmCfg<256>::SMEM : (bn == 128 ? GemmCfg<128>::SMEM : GemmCfg<64>::SMEM);
    return 0;
}

int gemm_pair_slots(int num_sms) { return pair_max_clusters(num_sms); }

// Longest-first list scheduling of the two products' tiles (split units included) over the
// resident pairs: each tile, longest first, goes to the pair with the least work so far
// (ties: the lower pair), and every pair runs its tiles in the order they were given.
// Cost of a tile: its k-blocks plus 4 for pipeline fill and epilogue.
namespace {

int pair_tile_cost(int kblocks) { return kblocks + 4; }

struct PairUnit {
    int cost, g, t;
};

// Units of one product on pair tiles, `splits` ways over K.
void pair_units(std::vector<PairUnit>& units, int g, int M, int N, int K, int splits) {
    const int num_m = (M + PairCfg::BMP - 1) / PairCfg::BMP;
    const int num_n = (N + PairCfg::BN - 1) / PairCfg::BN;
    const int kblocks = (K + BK - 1) / BK;
    const int tiles = num_m * num_n * splits;
    for (int t = 0; t < tiles; ++t) {
        const int split = t / (num_m * num_n);
        const int kb0 = (int)((long long)split * kblocks / splits);
        const int kb1 = (int)((long long)(split + 1) * kblocks / splits);
        units.push_back(PairUnit{pair_tile_cost(kb1 - kb0), g, t});
    }
}

// Longest-first assignment of `units` to `ncl` pairs; returns the largest pair load.
long long pair_lpt(std::vector<PairUnit>& units, int ncl, std::vector<std::vector<int>>* lists) {
    std::stable_sort(units.begin(), units.end(),
                     [](const PairUnit& x, const PairUnit& y) { return x.cost > y.cost; });
    std::vector<long long> load(ncl, 0);
    if (lists) lists->assign(ncl, {});
    for (const PairUnit& u : units) {
        int best = 0;
        for (int c = 1; c < ncl; ++c)
            if (load[c] < load[best]) best = c;
        load[best] += u.cost;
        if (lists) (*lists)[best].push_back((u.g << 24) | u.t);
    }
    return *std::max_element(load.begin(), load.end());
}

}  // namespace

// LLMGPU_GEMM_QUEUE: "0" keeps every dual launch on the host's per-pair lists, "1" puts
// every one on the run-time queue; unset, the caller decides.
int pair_queue_override() {
    static const int v = [] {
        const char* e = getenv("LLMGPU_GEMM_QUEUE");
        return (e && (e[0] == '0' || e[0] == '1')) ? e[0] - '0' : -1;
    }();
    return v;
}

int gemm_make_plan2(GemmPlan2* plan, const GemmPlan& p0, const GemmPlan& p1, int num_sms) {
    plan->sched = nullptr;
    plan->queue = nullptr;
    const GemmPlan* ps[2] = {&p0, &p1};
    std::vector<PairUnit> units;
    for (int g = 0; g < 2; ++g) {
        const GemmArgs& a = ps[g]->args;
        if (ps[g]->bn != kGemmPairTile || a.grp_mode != kGroupNone) return -50;
        const long long tiles = (long long)((a.M + PairCfg::BMP - 1) / PairCfg::BMP) *
                                ((a.N + PairCfg::BN - 1) / PairCfg::BN) * a.splits;
        if (tiles >= (1 << 24)) return -51;
        pair_units(units, g, a.M, a.N, a.K, a.splits);
    }
    const int ncl = std::min<int>(pair_max_clusters(num_sms), (int)units.size());
    // run-time queue order: the product with the longest units first
    int qcost[2] = {0, 0}, qtotal[2] = {0, 0};
    for (const PairUnit& u : units) {
        qcost[u.g] = std::max(qcost[u.g], u.cost);
        ++qtotal[u.g];
    }
    std::vector<std::vector<int>> lists;
    pair_lpt(units, ncl, &lists);
    size_t stride = 1;
    for (const auto& l : lists) stride = std::max(stride, l.size() + 1);
    // the per-pair lists, then the queue's two counters (zero between launches)
    std::vector<int> table((size_t)ncl * stride + 2, 0);
    for (int c = 0; c < ncl; ++c) {
        table[(size_t)c * stride] = (int)lists[c].size();
        for (size_t i = 0; i < lists[c].size(); ++i) table[(size_t)c * stride + 1 + i] = lists[c][i];
    }
    int* d = nullptr;
    if (cudaMalloc(&d, table.size() * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return -52;
    }
    if (cudaMemcpy(d, table.data(), table.size() * sizeof(int), cudaMemcpyHostToDevice) !=
        cudaSuccess) {
        cudaFree(d);
        cudaGetLastError();
        return -53;
    }
    plan->p[0] = p0;
    plan->p[1] = p1;
    plan->sched = d;
    plan->sched_stride = (int)stride;
    plan->queue = d + (size_t)ncl * stride;
    plan->q_first = qcost[1] > qcost[0] ? 1 : 0;
    plan->q_total[0] = qtotal[0];
    plan->q_total[1] = qtotal[1];
    plan->grid = 2 * ncl;
    return 0;
}

int gemm_run2(const GemmPlan2& plan, cudaStream_t stream, bool queue) {
    PairParams<2> P;
    for (int g = 0; g < 2; ++g) {
        P.tmA[g] = plan.p[g].tmA;
        P.tmB[g] = plan.p[g].tmB;
        P.tmO[g] = plan.p[g].tmO;
        P.tmX[g] = plan.p[g].tmX;
        P.args[g] = plan.p[g].args;
    }
    P.sched = plan.sched;
    P.sched_stride = plan.sched_stride;
    const int ov = pair_queue_override();
    P.queue = (ov < 0 ? queue : ov == 1) ? plan.queue : nullptr;
    P.q_first = plan.q_first;
    P.q_total[0] = plan.q_total[0];
    P.q_total[1] = plan.q_total[1];
    return launch_pair_params<2>(P, plan.grid, stream);
}

void gemm_free_plan2(GemmPlan2* plan) {
    if (plan->sched) cudaFree(plan->sched);
    plan->sched = nullptr;
    plan->queue = nullptr;
}

int gemm_run(const GemmPlan& p, cudaStream_t stream) {
    switch (p.bn) {
        case 256:
            return launch_bn<256>(p, stream);
        case 128:
            return launch_bn<128>(p, stream);
        case 64:
            return launch_bn<64>(p, stream);
        case kGemmPairTile:
            return launch_pair(p, stream);
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
        launch_kernel(splitk_reduce_scalar_kernel, (int)((total + 255) / 256), 256, 0, stream, partial, splits, M, N, out, ldo, col_group, group_stride, accumulate);
        return launch_status();
    }
    long long total4 = (long long)M * N / 4;
    int threads = 256;
    long long blocks2 = (total4 + 2 * threads - 1) / (2 * threads);
    if (blocks2 > 148 * 8) blocks2 = 148 * 8;
#define SR_LAUNCH(S)                                                                           \
    launch_kernel(splitk_reduce_s_kernel<S>, (int)blocks2, threads, 0, stream, partial, M, N, \
                  out, ldo, col_group, group_stride, accumulate)
    switch (splits) {
        case 2: SR_LAUNCH(2); return launch_status();
        case 3: SR_LAUNCH(3); return launch_status();
        case 4: SR_LAUNCH(4); return launch_status();
        case 6: SR_LAUNCH(6); return launch_status();
        case 8: SR_LAUNCH(8); return launch_status();
        default: break;
    }
#undef SR_LAUNCH
    long long blocks = (total4 + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    launch_kernel(splitk_reduce_kernel, (int)blocks, threads, 0, stream, partial, splits, M, N, out, ldo,
                                                             col_group, group_stride, accumulate);
    return launch_status();
}

}  // namespace llmgpu
