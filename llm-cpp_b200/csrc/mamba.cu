// Mamba block kernels (MambaBlock::forward/backward, src/mamba.cpp:36-166, 179-413):
// causal depthwise conv + SiLU, dt = clamp(softplus(xp[:, :R] dt_proj^T), 1e-3, 0.1), the
// selective scan h = exp(A dt) h + B x dt, y = C.h + D x, the SiLU(z) gate, and their
// backward. The in/x/out projections run on the tcgen05 GEMM (model.cu).
//
// Scan parallelisation: one thread per (sequence, channel d, state n); the L lanes of a
// channel (L = next power of two >= N) reduce C.h with shuffles. The forward saves h every
// kChunk steps; the backward walks chunks in reverse, recomputes the chunk's states from
// the saved one (instead of storing the T x D x N trajectory the reference keeps,
// src/mamba.cpp:215-229) and runs the reverse recurrence of src/mamba.cpp:277-308.
// All cross-channel and cross-sequence sums go through partial buffers reduced in a fixed
// order, so results are deterministic.
#include "common.cuh"
#include "mamba.cuh"

namespace llmgpu {

namespace {


__device__ __forceinline__ float silu_f(float v) { return __fdividef(v, 1.0f + __expf(-v)); }
__device__ __forceinline__ float sigmoid_f(float v) { return __fdividef(1.0f, 1.0f + __expf(-v)); }
__device__ __forceinline__ float silu_grad_f(float v) {
    const float s = sigmoid_f(v);
    return s * (1.0f + v * (1.0f - s));
}
// dt = clamp(softplus(x), 1e-3, 0.1) (src/mamba.cpp:120-135) and, for the backward, the
// derivative of that w.r.t. x: sigmoid(x) where softplus(x) lies inside the clamp, else 0
// (src/mamba.cpp:318-328). softplus(x) = log(1 + e) with e = e^x matters only where the clamp
// keeps it, e in [1.0005e-3, 0.10517]: there log(1 + e) is its alternating series to the
// e^8 term (remainder below 3e-9 relative, e < 0.11). Above e = 0.25 softplus exceeds 0.22
// and the clamp gives 0.1 whatever its value.
struct DtOf {
    float dt, ddt;
};
__device__ __forceinline__ DtOf dt_of(float x) {
    const float e = __expf(x);
    float q = -0.125f;
    q = fmaf(q, e, 1.0f / 7.0f);
    q = fmaf(q, e, -1.0f / 6.0f);
    q = fmaf(q, e, 0.2f);
    q = fmaf(q, e, -0.25f);
    q = fmaf(q, e, 1.0f / 3.0f);
    q = fmaf(q, e, -0.5f);
    q = fmaf(q, e, 1.0f);
    const float sp = e > 0.25f ? 1.0f : q * e;
    const bool inside = sp >= 0.001f && sp <= 0.1f;
    return {fminf(fmaxf(sp, 0.001f), 0.1f), inside ? __fdividef(e, 1.0f + e) : 0.f};
}

// ---------------------------------------------------------------- conv forward
// pre[t,d] = b[d] + sum_j w[d,j] x[t-(K-1)+j, d] within each sequence; u = silu(pre).
// A thread owns one channel over a run of kConvRows rows and slides a K-row window of x
// down it, so each x is read once; the loads of kConvBatch rows are issued together before
// their arithmetic. Taps that reach before the sequence start are skipped.
constexpr int kConvRows = 64;
constexpr int kConvBatch = 8;
template <int K>
__global__ void conv_fwd_kernel(const bf16* __restrict__ proj, long long ldp, int D, int T,
                                const float* __restrict__ w, const float* __restrict__ bias,
                                float* __restrict__ u32, bf16* __restrict__ u16, long long rows) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= D) return;
    const long long r0 = (long long)blockIdx.y * kConvRows;
    const int nr = (int)min((long long)kConvRows, rows - r0);
    float wk[K], win[K];  // win[j] = x[row - (K-1) + j]
#pragma unroll
    for (int j = 0; j < K; ++j) wk[j] = w[d * K + j];
    const float bs = bias[d];
    int t = (int)(r0 % T);
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {
        const int back = K - 1 - j;
        win[j] = t - back >= 0 ? __bfloat162float(proj[(r0 - back) * ldp + D + d]) : 0.f;
    }
    const bf16* xs = proj + r0 * ldp + D + d;
    for (int rb = 0; rb < nr; rb += kConvBatch) {
        float xg[kConvBatch];
#pragma unroll
        for (int q = 0; q < kConvBatch; ++q)
            xg[q] = rb + q < nr ? __bfloat162float(xs[(long long)(rb + q) * ldp]) : 0.f;
#pragma unroll
        for (int q = 0; q < kConvBatch; ++q) {
            win[K - 1] = xg[q];
            float acc = bs;
#pragma unroll
            for (int j = 0; j < K; ++j)
                if (t >= K - 1 - j) acc += wk[j] * win[j];
            if (rb + q < nr) {
                const float uv = silu_f(acc);
                const long long i = (r0 + rb + q) * D + d;
                u32[i] = uv;
                u16[i] = __float2bfloat16_rn(uv);
            }
#pragma unroll
            for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
            t = t + 1 == T ? 0 : t + 1;
        }
    }
}

// ---------------------------------------------------------------- scan staging
// A block of kScanWarps warps owns CPB = kScanWarps * 32 / L consecutive channels of one
// sequence; the L lanes of a channel hold S states each (state n*S + s in lane n): d_state
// 16 runs as 8 lanes x 2 states, and all (sequence, channel) pairs of a Mamba layer are
// resident at once (one state per lane, with twice the warps, measured slower: more
// instructions per state, and the scan is issue-bound at the bench shape). Time runs in chunks;
// the block loads a chunk's per-(step, channel) inputs and its per-(step, state) B and C
// into shared memory with coalesced row segments, double buffered: the loads of the next
// chunk are issued into registers before the recurrence of the current one runs, so the
// serial part of the scan does not wait on global memory.
constexpr int kScanWarps = 4;
template <int L, int S>
struct ScanTile {
    static constexpr int kThreads = kScanWarps * 32;
    static constexpr int kCPW = 32 / L;                 // channels per warp
    static constexpr int kCPB = kScanWarps * kCPW;      // channels per block
    static constexpr int kNS = L * S;                   // state slots per channel
    static constexpr int kTC = kScanChunk;              // steps per chunk
    static constexpr int kEPT = kTC * kCPB / kThreads;  // (step, channel) slots per thread
    static constexpr int kBPT = (kTC * kNS + kThreads - 1) / kThreads;  // (step, state) slots
    static_assert(kTC * kCPB % kThreads == 0, "chunk tile must split evenly over the block");
    static constexpr int kRow = kCPB + 1;               // padded row: lanes reading one channel
                                                        // at different steps hit distinct banks
};

// Sum of L values by a fixed pairwise tree (a short dependency chain; deterministic).
template <int L>
__device__ __forceinline__ float tree_sum(float (&v)[L]) {
#pragma unroll
    for (int w = L / 2; w >= 1; w >>= 1)
#pragma unroll
        for (int k = 0; k < w; ++k) v[k] += v[k + w];
    return v[0];
}

// ---------------------------------------------------------------- scan forward
// exp(A dt) = 2^((A log2 e) dt): A is scaled by log2 e once per thread and the power of two
// runs on the special-function unit (ex2.approx, flush-to-zero: decays below 2^-126 are 0).
constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float exp2_sfu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// A lane's S consecutive state values to shared memory (one 8-byte store for S = 2).
template <int S>
__device__ __forceinline__ void store_states(float* p, const float (&v)[S]) {
    if constexpr (S == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
        for (int s = 0; s < S; ++s) p[s] = v[s];
    }
}

// A lane's S consecutive state values from shared memory (one 8-byte load for S = 2).
template <int S>
__device__ __forceinline__ void load_states(const float* p, float (&v)[S]) {
    if constexpr (S == 2) {
        const float2 q = *reinterpret_cast<const float2*>(p);
        v[0] = q.x;
        v[1] = q.y;
    } else {
#pragma unroll
        for (int s = 0; s < S; ++s) v[s] = p[s];
    }
}

// The sequence is cut into gridDim.z segments of whole chunks, scanned side by side. The
// recurrence is linear, so a segment's states are its own scan from h = 0 plus the state
// entering it decayed by exp(A * (sum of dt so far in the segment)). PASS 0 scans each
// segment from zero and keeps only its final state and its dt sum (seg_h [B][P][D][N],
// seg_dt [B][P][D]); PASS 1 folds the earlier segments' results into the state entering its
// segment, then scans it again writing y, the gated output and the states every kScanChunk
// steps. With one segment, PASS 1 alone is the plain scan.
//
// Time runs in chunks of TF steps (two or one kScanChunk). The block stages a chunk's
// (dt, dt u) and (u, z) per (step, channel) and B, C per (step, state) in shared memory; the
// inputs of the next chunk are loaded into registers while the current one runs. Per step a lane does S
// states: a = 2^(A' dt), h = a h + B (dt u), p = sum_s C h. The L lanes of a channel then
// add their p through shared memory: lane n of a channel sums, for its steps n, n + L, ...,
// the L partials of that step (row pitch 33 floats: conflict-free) and writes y and the gate.
template <int L, int S, int PASS>
__global__ void __launch_bounds__(kScanWarps * 32) scan_fwd_kernel(
    const float* __restrict__ raw, const float* __restrict__ u, const float* __restrict__ xp,
    long long ldx, const float* __restrict__ alog, const float* __restrict__ dskip,
    const bf16* __restrict__ proj, long long ldp, float* __restrict__ y32,
    bf16* __restrict__ gated, float* __restrict__ hchk, float* __restrict__ seg_h,
    float* __restrict__ seg_dt, int T, int D, int N, int R) {
    using G = ScanTile<L, S>;
    constexpr int CPB = G::kCPB, CPW = G::kCPW, NT = G::kThreads, NS = G::kNS;
    // 32-step chunks (states saved at both 16-step boundaries); 16 for 32-channel blocks,
    // whose staging would not fit the 48 KB of static shared memory
    constexpr int TF = CPB <= 16 ? 2 * kScanChunk : kScanChunk;
    constexpr int EPT = TF * CPB / NT;            // (step, channel) items a thread stages
    constexpr int BPT = (TF * NS + NT - 1) / NT;  // (step, state) items a thread stages
    constexpr int KPER = TF / L;                  // steps whose output a lane writes
    static_assert(TF * CPB % NT == 0 && TF % L == 0, "chunk tile must split evenly");
    constexpr int P1 = PASS == 1 ? 2 : 1;
    __shared__ float2 sDU[2][TF][CPB];  // (dt, dt * u)
    __shared__ float2 sUZ[P1][PASS == 1 ? TF : 1][CPB];  // (u, z) for the outputs
    __shared__ __align__(16) float sB[2][TF][NS];
    __shared__ __align__(16) float sC[P1][PASS == 1 ? TF : 1][NS];
    __shared__ float sRed[PASS == 1 ? kScanWarps : 1][PASS == 1 ? TF : 1][33];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = lane % L, ch = lane / L, c = warp * CPW + ch;
    const int d0 = blockIdx.x * CPB, d = d0 + c;
    const int b = blockIdx.y;
    const bool chan = d < D;
    float A2[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const int k = n * S + s;
        A2[s] = (chan && k < N) ? alog[(long long)d * N + k] * kLog2e : 0.f;
    }
    const float Ds = chan ? dskip[d] : 0.f;
    const int nch = (T + TF - 1) / TF;
    const int nch16 = (T + kScanChunk - 1) / kScanChunk;

    float pr[EPT], pu[EPT], pz[EPT], pb[BPT], pc[BPT];
    auto fetch = [&](int t0) {
        const long long row0 = (long long)b * T + t0;  // the chunk's first token row
        const float* raw_c = raw + row0 * D + d0;
        const float* u_c = u + row0 * D + d0;
        const bf16* z_c = proj + row0 * ldp + d0;
        const float* b_c = xp + row0 * ldx + R;
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            const int idx = tid + e * NT, i = idx / CPB, cc = idx % CPB;
            const bool ok = t0 + i < T && d0 + cc < D;
            pr[e] = ok ? raw_c[i * D + cc] : 0.f;
            pu[e] = ok ? u_c[i * D + cc] : 0.f;
            if constexpr (PASS == 1) pz[e] = ok ? __bfloat162float(z_c[i * ldp + cc]) : 0.f;
        }
#pragma unroll
        for (int e = 0; e < BPT; ++e) {
            const int idx = tid + e * NT, i = idx / NS, k = idx % NS;
            const bool ok = idx < TF * NS && t0 + i < T && k < N;
            pb[e] = ok ? b_c[i * ldx + k] : 0.f;
            if constexpr (PASS == 1) pc[e] = ok ? b_c[i * ldx + N + k] : 0.f;
        }
    };
    auto stage = [&](int buf, int t0) {
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            const int idx = tid + e * NT, i = idx / CPB, cc = idx % CPB;
            const bool ok = t0 + i < T && d0 + cc < D;
            const float dt = ok ? dt_of(pr[e]).dt : 0.f;
            sDU[buf][i][cc] = make_float2(dt, dt * pu[e]);
            if constexpr (PASS == 1) sUZ[buf][i][cc] = make_float2(pu[e], pz[e]);
        }
#pragma unroll
        for (int e = 0; e < BPT; ++e) {
            const int idx = tid + e * NT;
            if (idx < TF * NS) {
                sB[buf][idx / NS][idx % NS] = pb[e];
                if constexpr (PASS == 1) sC[buf][idx / NS][idx % NS] = pc[e];
            }
        }
    };

    // this block's segment: chunks [k_begin, k_end)
    const int seg = blockIdx.z, nseg = gridDim.z;
    const int cps = (nch + nseg - 1) / nseg;
    const int k_begin = seg * cps, k_end = min(nch, k_begin + cps);
    float h[S];
#pragma unroll
    for (int s = 0; s < S; ++s) h[s] = 0.f;
    if (PASS == 1) {
        // the state entering the segment, from the earlier segments' zero-start scans
        for (int p = 0; p < seg; ++p) {
            const long long bp = (long long)b * nseg + p;
            const float dts = chan ? seg_dt[bp * D + d] : 0.f;
#pragma unroll
            for (int s = 0; s < S; ++s) {
                const int kk = n * S + s;
                const float he = (chan && kk < N) ? seg_h[(bp * D + d) * N + kk] : 0.f;
                h[s] = fmaf(exp2_sfu(A2[s] * dts), h[s], he);
            }
        }
    }
    float dtsum = 0.f;
    if (k_begin < k_end) fetch(k_begin * TF);
    for (int k = k_begin; k < k_end; ++k) {
        const int buf = k & 1, t0 = k * TF;
        stage(buf, t0);
        __syncthreads();
        if (k + 1 < k_end) fetch(t0 + TF);
        // steps past T were staged as dt = dt u = B = C = 0, which leaves h unchanged
        if constexpr (PASS == 0) {
#pragma unroll
            for (int i = 0; i < TF; ++i) {
                const float2 dd = sDU[buf][i][c];
                dtsum += dd.x;
#pragma unroll
                for (int s = 0; s < S; ++s)
                    h[s] = fmaf(exp2_sfu(A2[s] * dd.x), h[s], sB[buf][i][n * S + s] * dd.y);
            }
        } else {
            float p[TF];
#pragma unroll
            for (int i = 0; i < TF; ++i) {
                if (i % kScanChunk == 0 && t0 + i < T) {
                    const int k16 = (t0 + i) / kScanChunk;
#pragma unroll
                    for (int s = 0; s < S; ++s)
                        if (chan && n * S + s < N)
                            hchk[(((long long)b * nch16 + k16) * D + d) * N + n * S + s] = h[s];
                }
                const float2 dd = sDU[buf][i][c];
                float bv[S], cv[S];
                load_states<S>(&sB[buf][i][n * S], bv);
                load_states<S>(&sC[buf][i][n * S], cv);
                float acc = 0.f;
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    h[s] = fmaf(exp2_sfu(A2[s] * dd.x), h[s], bv[s] * dd.y);
                    acc = fmaf(cv[s], h[s], acc);
                }
                p[i] = acc;
            }
#pragma unroll
            for (int i = 0; i < TF; ++i) sRed[warp][i][lane] = p[i];
            __syncwarp();
#pragma unroll
            for (int jj = 0; jj < KPER; ++jj) {
                const int j = n + L * jj;
                float part[L];
#pragma unroll
                for (int m = 0; m < L; ++m) part[m] = sRed[warp][j][ch * L + m];
                float y = tree_sum<L>(part);
                if (chan && t0 + j < T) {
                    const long long row = (long long)b * T + t0 + j;
                    const float2 uz = sUZ[buf][j][c];
                    y = fmaf(Ds, uz.x, y);
                    y32[row * D + d] = y;
                    gated[row * D + d] = __float2bfloat16_rn(y * silu_f(uz.y));
                }
            }
            __syncwarp();  // the partials are read before the next chunk overwrites them
        }
    }
    if (PASS == 0) {
        const long long bp = (long long)b * nseg + seg;
#pragma unroll
        for (int s = 0; s < S; ++s)
            if (chan && n * S + s < N) seg_h[(bp * D + d) * N + n * S + s] = h[s];
        if (chan && n == 0) seg_dt[bp * D + d] = dtsum;
    }
}

// ---------------------------------------------------------------- scan backward
// Chunks of kScanChunk steps from the right. Per chunk a lane recomputes its states from the
// saved h (keeping the decays a and the states in registers), then runs the reverse
// recurrence: dh = dh' + dy C, dh' = dh a (for the step before), with per-lane sums over its
// S states G = sum dh B and H = sum (dh a h_prev) A, and per-state terms dB = dh (dt u) and
// dC = dy h. From the channel sums of G and H: du = G dt + dy D and ddt = H + G u. The L
// lanes of a channel add G and H through shared memory like the forward's outputs; the dB
// and dC terms go to a [channel][state] table and the block sums each (step, state) over its
// channels in a fixed order (partials per channel group, reduced by dbc_reduce_kernel).
template <int L, int S>
struct ScanBwdSmem {
    static constexpr int CPB = ScanTile<L, S>::kCPB, NS = ScanTile<L, S>::kNS;
    static constexpr int TC = kScanChunk;
    static constexpr size_t kDU = 0;                                      // float2 [2][TC][CPB]
    static constexpr size_t kGU = kDU + sizeof(float2) * 2 * TC * CPB;    // float2 [2][TC][CPB]
    static constexpr size_t kDf = kGU + sizeof(float2) * 2 * TC * CPB;    // float [2][TC][CPB]
    static constexpr size_t kB = kDf + sizeof(float) * 2 * TC * CPB;      // float [2][TC][NS]
    static constexpr size_t kC = kB + sizeof(float) * 2 * TC * NS;        // float [2][TC][NS]
    static constexpr size_t kRed = kC + sizeof(float) * 2 * TC * NS;      // float2 [W][TC][33]
    // dB/dC terms [2][TC][ROW]: a step's [channel][state] block, rows padded by 16 floats so
    // that the block sum's reads of consecutive (step, state) pairs fall in distinct banks
    static constexpr int ROW = CPB * NS + 16;
    static constexpr size_t kP = kRed + sizeof(float) * kScanWarps * 2 * TC * 33;
    static constexpr size_t kBytes = kP + sizeof(float) * 2 * TC * ROW;
    static_assert(kB % 16 == 0 && kRed % 8 == 0 && kP % 16 == 0, "table alignment");
};

// Three blocks per SM (at most 170 registers a thread): the bench's four sequences of 96
// channel groups make 384 blocks, which must all be resident.
template <int L, int S>
__global__ void __launch_bounds__(kScanWarps * 32, 3) scan_bwd_kernel(
    const float* __restrict__ raw, const float* __restrict__ u, const float* __restrict__ xp,
    long long ldx, const float* __restrict__ alog, const float* __restrict__ dskip,
    const bf16* __restrict__ proj, long long ldp, const float* __restrict__ y32,
    const float* __restrict__ dgated, const float* __restrict__ hchk, float* __restrict__ du,
    float* __restrict__ draw, bf16* __restrict__ dproj, float* __restrict__ dbc_part,
    float* __restrict__ da_part, float* __restrict__ dd_part, const float* __restrict__ seg_dh,
    const float* __restrict__ seg_dt, int T, int D, int N, int R) {
    using G = ScanTile<L, S>;
    using SM = ScanBwdSmem<L, S>;
    constexpr int CPB = G::kCPB, CPW = G::kCPW, NT = G::kThreads, NS = G::kNS;
    constexpr int TC = kScanChunk;
    constexpr int EPT = TC * CPB / NT, BPT = (TC * NS + NT - 1) / NT, KPER = TC / L;
    static_assert(TC * CPB % NT == 0 && TC % L == 0, "chunk tile must split evenly");
    extern __shared__ __align__(16) unsigned char scan_smem[];
    auto sDU = reinterpret_cast<float2(*)[TC][CPB]>(scan_smem + SM::kDU);  // (dt, dt u)
    auto sGU = reinterpret_cast<float2(*)[TC][CPB]>(scan_smem + SM::kGU);  // (dy, u)
    // d(dt)/d(dt_raw): sigmoid(dt_raw) where softplus(dt_raw) lies inside the clamp, else 0
    // (src/mamba.cpp:318-328)
    auto sDf = reinterpret_cast<float(*)[TC][CPB]>(scan_smem + SM::kDf);
    auto sB = reinterpret_cast<float(*)[TC][NS]>(scan_smem + SM::kB);
    auto sC = reinterpret_cast<float(*)[TC][NS]>(scan_smem + SM::kC);
    auto sRed = reinterpret_cast<float2(*)[TC][33]>(scan_smem + SM::kRed);  // (G, H) partials
    auto sP = reinterpret_cast<float(*)[TC][SM::ROW]>(scan_smem + SM::kP);  // [dB, dC]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = lane % L, ch = lane / L, c = warp * CPW + ch;
    const int d0 = blockIdx.x * CPB, d = d0 + c;
    const int b = blockIdx.y;
    const bool chan = d < D;
    float A[S], A2[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const int k = n * S + s;
        A[s] = (chan && k < N) ? alog[(long long)d * N + k] : 0.f;
        A2[s] = A[s] * kLog2e;
    }
    const float Ds = chan ? dskip[d] : 0.f;
    const int nch = (T + TC - 1) / TC;
    const long long BT = (long long)gridDim.y * T;

    float pr[EPT], pu[EPT], pg[EPT], pz[EPT], py[EPT], pb[BPT], pc[BPT], ph[S];
    auto fetch = [&](int t0) {
        // the state saved at the chunk's start, loaded a chunk ahead like the inputs
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const int kk = n * S + s;
            ph[s] = (chan && kk < N)
                        ? hchk[(((long long)b * nch + t0 / TC) * D + d) * N + kk] : 0.f;
        }
        const long long row0 = (long long)b * T + t0;  // the chunk's first token row
        const long long o0 = row0 * D + d0;
        const bf16* z_c = proj + row0 * ldp + d0;
        const float* b_c = xp + row0 * ldx + R;
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            const int idx = tid + e * NT, i = idx / CPB, cc = idx % CPB;
            const bool ok = t0 + i < T && d0 + cc < D;
            const long long o = o0 + i * D + cc;
            pr[e] = ok ? raw[o] : 0.f;
            pu[e] = ok ? u[o] : 0.f;
            pg[e] = ok ? dgated[o] : 0.f;
            pz[e] = ok ? __bfloat162float(z_c[i * ldp + cc]) : 0.f;
            py[e] = ok ? y32[o] : 0.f;
        }
#pragma unroll
        for (int e = 0; e < BPT; ++e) {
            const int idx = tid + e * NT, i = idx / NS, k = idx % NS;
            const bool ok = idx < TC * NS && t0 + i < T && k < N;
            pb[e] = ok ? b_c[i * ldx + k] : 0.f;
            pc[e] = ok ? b_c[i * ldx + N + k] : 0.f;
        }
    };
    // also writes the x_z gradient, which needs no scan state
    auto stage = [&](int buf, int t0) {
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            const int idx = tid + e * NT, i = idx / CPB, cc = idx % CPB;
            const bool ok = t0 + i < T && d0 + cc < D;
            const DtOf v = dt_of(pr[e]);
            const float dt = ok ? v.dt : 0.f;
            sDU[buf][i][cc] = make_float2(dt, dt * pu[e]);
            sGU[buf][i][cc] = make_float2(pg[e] * silu_f(pz[e]), pu[e]);  // d(loss)/d(y), u
            sDf[buf][i][cc] = ok ? v.ddt : 0.f;
            if (ok) {
                const long long row = (long long)b * T + t0 + i;
                dproj[row * ldp + d0 + cc] = __float2bfloat16_rn(pg[e] * py[e] * silu_grad_f(pz[e]));
            }
        }
#pragma unroll
        for (int e = 0; e < BPT; ++e) {
            const int idx = tid + e * NT;
            if (idx < TC * NS) {
                sB[buf][idx / NS][idx % NS] = pb[e];
                sC[buf][idx / NS][idx % NS] = pc[e];
            }
        }
    };

    // this block's segment: chunks [k_begin, k_end), walked from the right; dh entering it
    // from the right folds the later segments' zero-start results (scan_bwd_carry_kernel)
    const int seg = blockIdx.z, nseg = gridDim.z;
    const int cps = (nch + nseg - 1) / nseg;
    const int k_begin = seg * cps, k_end = min(nch, k_begin + cps);
    float dh_next[S], dA_acc[S];
#pragma unroll
    for (int s = 0; s < S; ++s) dh_next[s] = dA_acc[s] = 0.f;
    for (int p = nseg - 1; p > seg; --p) {
        const long long bp = (long long)b * nseg + p;
        const float dts = chan ? seg_dt[bp * D + d] : 0.f;
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const int kk = n * S + s;
            const float he = (chan && kk < N) ? seg_dh[(bp * D + d) * N + kk] : 0.f;
            dh_next[s] = fmaf(exp2_sfu(A2[s] * dts), dh_next[s], he);
        }
    }
    float dD_acc = 0.f;
    if (k_begin < k_end) fetch((k_end - 1) * TC);
    for (int k = k_end - 1; k >= k_begin; --k) {
        const int buf = k & 1, t0 = k * TC;
        stage(buf, t0);
        float h_start[S], as[S][TC], hs[S][TC];
#pragma unroll
        for (int s = 0; s < S; ++s) h_start[s] = ph[s];
        __syncthreads();
        if (k > k_begin) fetch(t0 - TC);
        // The chunk's decays and states, recomputed from the state saved at its start. Steps
        // past T were staged as dt = dt u = B = C = dy = 0: h and dh pass through them
        // unchanged and they add nothing to dA, dD, dB or dC; their du and ddt are not stored.
#pragma unroll
        for (int i = 0; i < TC; ++i) {
            const float2 dd = sDU[buf][i][c];
            float bv[S];
            load_states<S>(&sB[buf][i][n * S], bv);
#pragma unroll
            for (int s = 0; s < S; ++s) {
                as[s][i] = exp2_sfu(A2[s] * dd.x);
                hs[s][i] = fmaf(as[s][i], i > 0 ? hs[s][i - 1] : h_start[s], bv[s] * dd.y);
            }
        }
        // the reverse recurrence; per-lane G and H of every step, dB/dC terms per state
        float gl[TC], hl[TC];
#pragma unroll
        for (int i = TC - 1; i >= 0; --i) {
            const float2 dd = sDU[buf][i][c];
            const float2 gu = sGU[buf][i][c];
            float gs = 0.f, hsum = 0.f, tb[S], tc[S];
            float bv[S], cv[S];
            load_states<S>(&sB[buf][i][n * S], bv);
            load_states<S>(&sC[buf][i][n * S], cv);
#pragma unroll
            for (int s = 0; s < S; ++s) {
                const float Bv = bv[s], Cv = cv[s];
                const float h_prev = i > 0 ? hs[s][i - 1] : h_start[s];
                const float dh = fmaf(gu.x, Cv, dh_next[s]);
                tb[s] = dh * dd.y;        // dB term
                tc[s] = gu.x * hs[s][i];  // dC term
                gs = fmaf(dh, Bv, gs);
                dh_next[s] = dh * as[s][i];
                const float x = dh_next[s] * h_prev;
                hsum = fmaf(x, A[s], hsum);
                dA_acc[s] = fmaf(x, dd.x, dA_acc[s]);
            }
            // [channel][state] rows: a warp's lanes store 32 consecutive floats (S = 1) or
            // 8-byte pairs (S = 2), conflict-free either way
            store_states<S>(&sP[0][i][c * NS + n * S], tb);
            store_states<S>(&sP[1][i][c * NS + n * S], tc);
            gl[i] = gs;
            hl[i] = hsum;
        }
#pragma unroll
        for (int i = 0; i < TC; ++i) sRed[warp][i][lane] = make_float2(gl[i], hl[i]);
        __syncwarp();
#pragma unroll
        for (int jj = 0; jj < KPER; ++jj) {
            const int j = n + L * jj;
            float gp[L], hp[L];
#pragma unroll
            for (int m = 0; m < L; ++m) {
                const float2 v = sRed[warp][j][ch * L + m];
                gp[m] = v.x;
                hp[m] = v.y;
            }
            const float gsum = tree_sum<L>(gp), hsum = tree_sum<L>(hp);
            const float2 dd = sDU[buf][j][c];
            const float2 gu = sGU[buf][j][c];
            dD_acc = fmaf(gu.x, gu.y, dD_acc);
            if (chan && t0 + j < T) {
                const long long row = (long long)b * T + t0 + j;
                du[row * D + d] = fmaf(gsum, dd.x, gu.x * Ds);
                draw[row * D + d] = fmaf(gsum, gu.y, hsum) * sDf[buf][j][c];
            }
        }
        __syncthreads();
        // block partial over its channels (fixed order) -> dbc_part[blockIdx.x][2][B*T][N]
#pragma unroll
        for (int k0 = 0; k0 < 2 * TC * NS; k0 += NT) {
            const int kk = k0 + tid;
            const int kind = kk / (TC * NS), i = (kk / NS) % TC, nn = kk % NS;
            const int t = t0 + i;
            if (kk >= 2 * TC * NS || nn >= N || t >= T) continue;
            float v[CPB];
#pragma unroll
            for (int cc = 0; cc < CPB; ++cc) v[cc] = sP[kind][i][cc * NS + nn];
            const float sum = tree_sum<CPB>(v);
            const long long row = (long long)b * T + t;
            dbc_part[((long long)blockIdx.x * 2 + kind) * BT * N + row * N + nn] = sum;
        }
    }
    // dD over the channel's lanes (each lane summed its own steps)
#pragma unroll
    for (int o = L / 2; o >= 1; o >>= 1) dD_acc += __shfl_xor_sync(0xffffffffu, dD_acc, o);
    // per (sequence, segment) partials [B * nseg][D][N] and [B * nseg][D]
    const long long bs = (long long)b * nseg + seg;
#pragma unroll
    for (int s = 0; s < S; ++s)
        if (chan && n * S + s < N) da_part[(bs * D + d) * N + n * S + s] = dA_acc[s];
    if (n == 0 && chan) dd_part[bs * D + d] = dD_acc;
}

// dh entering each segment's left end from a zero carry at its right end, and the segment's
// dt sum: dh_t = dh_(t+1) exp(A dt_(t+1)) + dy_t C_t over the segment, from the right. These
// are what the segments to the left need to start their reverse scans from the true dh.
template <int L, int S>
__global__ void __launch_bounds__(kScanWarps * 32) scan_bwd_carry_kernel(
    const float* __restrict__ raw, const float* __restrict__ xp, long long ldx,
    const float* __restrict__ alog, const bf16* __restrict__ proj, long long ldp,
    const float* __restrict__ dgated, float* __restrict__ seg_dh, float* __restrict__ seg_dt,
    int T, int D, int N, int R) {
    using G = ScanTile<L, S>;
    constexpr int CPB = G::kCPB, TC = G::kTC, EPT = G::kEPT, NT = G::kThreads, RW = G::kRow;
    constexpr int NS = G::kNS, BPT = G::kBPT;
    __shared__ float sDt[2][TC][RW], sDy[2][TC][RW];
    __shared__ __align__(16) float sC[2][TC][NS];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = lane % L, c = warp * G::kCPW + lane / L;
    const int d0 = blockIdx.x * CPB, d = d0 + c;
    const int b = blockIdx.y;
    const bool chan = d < D;
    float A2[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const int k = n * S + s;
        A2[s] = (chan && k < N) ? alog[(long long)d * N + k] * kLog2e : 0.f;
    }
    const int nch = (T + TC - 1) / TC;
    float pr[EPT], pg[EPT], pz[EPT], pc[BPT];
    auto fetch = [&](int t0) {
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            const int idx = tid + e * NT, i = idx / CPB, dd = d0 + idx % CPB;
            const bool ok = t0 + i < T && dd < D;
            const long long row = (long long)b * T + t0 + i;
            pr[e] = ok ? raw[row * D + dd] : 0.f;
            pg[e] = ok ? dgated[row * D + dd] : 0.f;
            pz[e] = ok ? __bfloat162float(proj[row * ldp + dd]) : 0.f;
        }
#pragma unroll
        for (int e = 0; e < BPT; ++e) {
            const int idx = tid + e * NT, i = idx / NS, k = idx % NS;
            const bool ok = idx < TC * NS && t0 + i < T && k < N;
            const long long row = (long long)b * T + t0 + i;
            pc[e] = ok ? xp[row * ldx + R + N + k] : 0.f;
        }
    };
    auto stage = [&](int buf, int t0) {
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            const int idx = tid + e * NT, i = idx / CPB, cc = idx % CPB;
            const bool ok = t0 + i < T && d0 + cc < D;
            sDt[buf][i][cc] = ok ? dt_of(pr[e]).dt : 0.f;
            sDy[buf][i][cc] = pg[e] * silu_f(pz[e]);
        }
#pragma unroll
        for (int e = 0; e < BPT; ++e) {
            const int idx = tid + e * NT;
            if (idx < TC * NS) sC[buf][idx / NS][idx % NS] = pc[e];
        }
    };
    const int seg = blockIdx.z, nseg = gridDim.z;
    const int cps = (nch + nseg - 1) / nseg;
    const int k_begin = seg * cps, k_end = min(nch, k_begin + cps);
    float dh_next[S];
#pragma unroll
    for (int s = 0; s < S; ++s) dh_next[s] = 0.f;
    float dtsum = 0.f;
    if (k_begin < k_end) fetch((k_end - 1) * TC);
    for (int k = k_end - 1; k >= k_begin; --k) {
        const int buf = k & 1, t0 = k * TC;
        stage(buf, t0);
        __syncthreads();
        if (k > k_begin) fetch(t0 - TC);
#pragma unroll
        for (int i = TC - 1; i >= 0; --i) {
            const float dyv = sDy[buf][i][c], dt = sDt[buf][i][c];
            dtsum += dt;
#pragma unroll
            for (int s = 0; s < S; ++s)
                dh_next[s] = fmaf(dyv, sC[buf][i][n * S + s], dh_next[s]) * exp2_sfu(A2[s] * dt);
        }
    }
    const long long bp = (long long)b * nseg + seg;
#pragma unroll
    for (int s = 0; s < S; ++s)
        if (chan && n * S + s < N) seg_dh[(bp * D + d) * N + n * S + s] = dh_next[s];
    if (chan && n == 0) seg_dt[bp * D + d] = dtsum;
}

// dB, dC: sum over channel groups (fixed order) -> bf16 columns R.. of dxp
__global__ void dbc_reduce_kernel(const float* __restrict__ part, int groups, long long BT, int N,
                                  int R, bf16* __restrict__ dxp, long long ldx) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= BT * N) return;
    const long long row = i / N;
    const int n = (int)(i - row * N);
    float sb = 0.f, sc = 0.f;
    for (int g = 0; g < groups; ++g) {
        sb += part[(long long)g * 2 * BT * N + i];
        sc += part[(long long)g * 2 * BT * N + BT * N + i];
    }
    dxp[row * ldx + R + n] = __float2bfloat16_rn(sb);
    dxp[row * ldx + R + N + n] = __float2bfloat16_rn(sc);
}

// out[j] (+)= sum_b part[b][j]
__global__ void batch_reduce_kernel(const float* __restrict__ part, int B, long long n,
                                    float* __restrict__ out, int accumulate) {
    const long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (j >= n) return;
    float s = 0.f;
    for (int b = 0; b < B; ++b) s += part[(long long)b * n + j];
    out[j] = accumulate ? out[j] + s : s;
}


// conv backward, fused: g = (du_scan + du_xp) * silu'(pre) with pre recomputed from the x
// window; per-run partial sums of dconv_b and dconv_w; and dx_ssm[t,d] =
// sum_j g[t+(K-1-j), d] w[d,j] within the sequence, from a K-row window of g that runs K-1
// rows ahead of the row it completes (those halo rows are recomputed, not stored).
// Grid: D/256 x row runs of kConvRows; partials part[run][d][K+1].
template <int K>
__global__ void conv_bwd_kernel(const bf16* __restrict__ proj, long long ldp, int D, int T,
                                const float* __restrict__ w, const float* __restrict__ bias,
                                const float* __restrict__ du1, const float* __restrict__ du2,
                                float* __restrict__ part, bf16* __restrict__ dproj,
                                long long rows) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= D) return;
    const long long r0 = (long long)blockIdx.y * kConvRows;
    const int nr = (int)min((long long)kConvRows, rows - r0);
    const int nh = (int)min((long long)nr + K - 1, rows - r0);  // rows incl. the halo
    float wk[K], xw[K], gw[K];  // xw[j] = x[row'-(K-1)+j], gw[f] = g[row'-(K-1)+f]
#pragma unroll
    for (int j = 0; j < K; ++j) {
        wk[j] = w[d * K + j];
        gw[j] = 0.f;
    }
    const float bs = bias[d];
    int tp = (int)(r0 % T);  // position of row' in its sequence
    int tr = tp;             // position of the row the window completes next
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {
        const int back = K - 1 - j;
        xw[j] = tp - back >= 0 ? __bfloat162float(proj[(r0 - back) * ldp + D + d]) : 0.f;
    }
    float sb = 0.f, sw[K];
#pragma unroll
    for (int j = 0; j < K; ++j) sw[j] = 0.f;
    const bf16* xs = proj + r0 * ldp + D + d;
    for (int rb = 0; rb < nr + K - 1; rb += kConvBatch) {
        float xg[kConvBatch], gg[kConvBatch];
#pragma unroll
        for (int q = 0; q < kConvBatch; ++q) {
            const bool in = rb + q < nh;
            const long long i = (r0 + rb + q) * D + d;
            xg[q] = in ? __bfloat162float(xs[(long long)(rb + q) * ldp]) : 0.f;
            gg[q] = in ? du1[i] + du2[i] : 0.f;
        }
#pragma unroll
        for (int q = 0; q < kConvBatch; ++q) {
            const int r = rb + q;
            if (r >= nr + K - 1) break;
            xw[K - 1] = xg[q];
            float pre = bs;
#pragma unroll
            for (int j = 0; j < K; ++j)
                if (tp >= K - 1 - j) pre += wk[j] * xw[j];
            const float g = gg[q] * silu_grad_f(pre);
            if (r < nr) {
                sb += g;
#pragma unroll
                for (int j = 0; j < K; ++j)
                    if (tp >= K - 1 - j) sw[j] += g * xw[j];
            }
            // g[row'] enters the window; the row K-1 above row' is now complete
            gw[K - 1] = g;
            const int rr = r - (K - 1);
            if (rr >= 0) {
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < K; ++j) {
                    const int f = K - 1 - j;
                    if (tr + f < T) acc += gw[f] * wk[j];
                }
                dproj[(r0 + rr) * ldp + D + d] = __float2bfloat16_rn(acc);
                tr = tr + 1 == T ? 0 : tr + 1;
            }
#pragma unroll
            for (int j = 0; j < K - 1; ++j) {
                xw[j] = xw[j + 1];
                gw[j] = gw[j + 1];
            }
            tp = tp + 1 == T ? 0 : tp + 1;
        }
    }
    float* p = part + ((long long)blockIdx.y * D + d) * (K + 1);
    p[0] = sb;
#pragma unroll
    for (int j = 0; j < K; ++j) p[1 + j] = sw[j];
}

// conv weight/bias gradients: out_b[d] (+)= sum_blk part[blk][d][0], out_w[d,j] (+)= ...[1+j]
__global__ void conv_reduce_kernel(const float* __restrict__ part, int nblk, int D, int K,
                                   float* __restrict__ gw, float* __restrict__ gb, int accumulate) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= D * (K + 1)) return;
    const int d = i / (K + 1), j = i - d * (K + 1);
    float s = 0.f;
    for (int k = 0; k < nblk; ++k) s += part[((long long)k * D + d) * (K + 1) + j];
    float* o = j == 0 ? gb + d : gw + (long long)d * K + (j - 1);
    *o = accumulate ? *o + s : s;
}


// fp32 GEMM on the CUDA cores for the dt_rank-wide contractions of the dt path (the clamp
// mask after softplus needs fp32 operands): C = A B with A(m,k) = A[m*sam + k*sak] and
// B(k,n) = B[k*sbk + n*sbn]. 128 x BN output tile per block (8 x BN/16 per thread), k staged
// 16 at a time in double-buffered shared memory, the next stage's loads in flight during the
// current stage's math. blockIdx.z splits K into chunks of kchunk: with one chunk the tile
// goes straight to out (fp32, += when accumulate) or out16 (bf16); with several, to
// part[z][M][N] for a fixed-order reduction.
constexpr int kSgM = 128, kSgK = 16;
template <int BN>
__global__ void __launch_bounds__(256) sgemm_f32_kernel(
    const float* __restrict__ A, long long sam, long long sak, const float* __restrict__ Bm,
    long long sbk, long long sbn, int M, int N, int K, int kchunk, float* __restrict__ part,
    float* __restrict__ out, bf16* __restrict__ out16, long long ldo, int accumulate) {
    constexpr int TM = 8, TN = BN / 16;
    constexpr int AE = kSgM * kSgK / 256, BE = kSgK * BN / 256;
    static_assert(BN % 16 == 0 && kSgK * BN % 256 == 0, "B stage must split over the block");
    __shared__ __align__(16) float As[2][kSgK][kSgM + 4];
    __shared__ __align__(16) float Bs[2][kSgK][BN + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.x * kSgM, n0 = blockIdx.y * BN;
    const int kbeg = blockIdx.z * kchunk, kend = min(K, kbeg + kchunk);
    const bool a_kfast = sak == 1, b_nfast = sbn == 1;
    float ra[AE], rb[BE];
    auto gload = [&](int k0) {
#pragma unroll
        for (int e = 0; e < AE; ++e) {
            const int idx = tid + e * 256;
            const int mm = a_kfast ? idx / kSgK : idx % kSgM;
            const int kk = a_kfast ? idx % kSgK : idx / kSgM;
            const int m = m0 + mm, k = k0 + kk;
            ra[e] = (m < M && k < kend) ? A[(long long)m * sam + (long long)k * sak] : 0.f;
        }
#pragma unroll
        for (int e = 0; e < BE; ++e) {
            const int idx = tid + e * 256;
            const int nn = b_nfast ? idx % BN : idx / kSgK;
            const int kk = b_nfast ? idx / BN : idx % kSgK;
            const int n = n0 + nn, k = k0 + kk;
            rb[e] = (n < N && k < kend) ? Bm[(long long)k * sbk + (long long)n * sbn] : 0.f;
        }
    };
    auto sstore = [&](int buf) {
#pragma unroll
        for (int e = 0; e < AE; ++e) {
            const int idx = tid + e * 256;
            const int mm = a_kfast ? idx / kSgK : idx % kSgM;
            const int kk = a_kfast ? idx % kSgK : idx / kSgM;
            As[buf][kk][mm] = ra[e];
        }
#pragma unroll
        for (int e = 0; e < BE; ++e) {
            const int idx = tid + e * 256;
            const int nn = b_nfast ? idx % BN : idx / kSgK;
            const int kk = b_nfast ? idx / BN : idx % kSgK;
            Bs[buf][kk][nn] = rb[e];
        }
    };
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
    if (kbeg < kend) {
        gload(kbeg);
        sstore(0);
    }
    __syncthreads();
    int buf = 0;
    for (int k0 = kbeg; k0 < kend; k0 += kSgK) {
        const bool more = k0 + kSgK < kend;
        if (more) gload(k0 + kSgK);
#pragma unroll
        for (int kk = 0; kk < kSgK; ++kk) {
            float av[TM], bv[TN];
            const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * TM]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * TM + 4]);
            av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
            av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
#pragma unroll
            for (int j = 0; j < TN; ++j) bv[j] = Bs[buf][kk][tx * TN + j];
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] += av[i] * bv[j];
        }
        if (more) sstore(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
    const bool split = gridDim.z > 1;
    // whole 4-column groups of a plain fp32 output go out as one 16-byte store
    const bool vec = TN == 4 && !split && !out16 && !accumulate && n0 + tx * 4 + 4 <= N &&
                     (ldo & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int m = m0 + ty * TM + i;
        if (m >= M) continue;
        if (vec) {
            *reinterpret_cast<float4*>(out + (long long)m * ldo + n0 + tx * 4) =
                make_float4(acc[i][0], acc[i][1 % TN], acc[i][2 % TN], acc[i][3 % TN]);
            continue;
        }
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int n = n0 + tx * TN + j;
            if (n >= N) continue;
            if (split) {
                part[((long long)blockIdx.z * M + m) * N + n] = acc[i][j];
            } else if (out16) {
                out16[(long long)m * ldo + n] = __float2bfloat16_rn(acc[i][j]);
            } else {
                float* o = out + (long long)m * ldo + n;
                *o = accumulate ? *o + acc[i][j] : acc[i][j];
            }
        }
    }
}

// out (+)= sum_y part[y] (fixed order), fp32 [m*ldo + n] or, when out16 is given, bf16
__global__ void small_gemm_reduce_kernel(const float* __restrict__ part, int splits, int M, int N,
                                         float* __restrict__ out, bf16* __restrict__ out16,
                                         long long ldo, int accumulate) {
    const long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (e >= (long long)M * N) return;
    const int m = (int)(e / N), n = (int)(e - (long long)m * N);
    float s = 0.f;
    for (int y = 0; y < splits; ++y) s += part[(long long)y * M * N + e];
    if (out16) {
        out16[(long long)m * ldo + n] = __float2bfloat16_rn(s);
    } else {
        float* o = out + (long long)m * ldo + n;
        *o = accumulate ? *o + s : s;
    }
}

__global__ void convert_kernel(const float* __restrict__ src, long long lds, bf16* __restrict__ dst,
                               long long ldd, long long rows, int cols) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= rows * cols) return;
    const long long r = i / cols;
    const int c = (int)(i - r * cols);
    dst[r * ldd + c] = __float2bfloat16_rn(src[r * lds + c]);
}

template <int L, int S>
int launch_scan_fwd(const MambaDims& m, const float* raw, const float* u, const float* xp,
                    const float* alog, const float* dskip, const bf16* proj, float* y32,
                    bf16* gated, float* hchk, float* seg_work, cudaStream_t s) {
    constexpr int CPB = ScanTile<L, S>::kCPB;
    const int nseg = mamba_scan_segments(m.B, m.T, m.D, m.N);
    dim3 grid((m.D + CPB - 1) / CPB, m.B, nseg);
    float* seg_h = seg_work;
    float* seg_dt = seg_work + (size_t)m.B * nseg * m.D * m.N;
    if (nseg > 1) {
        scan_fwd_kernel<L, S, 0><<<grid, kScanWarps * 32, 0, s>>>(
            raw, u, xp, m.ldx, alog, dskip, proj, m.ldp, y32, gated, hchk, seg_h, seg_dt, m.T,
            m.D, m.N, m.R);
        int rc = launch_status();
        if (rc) return rc;
    }
    scan_fwd_kernel<L, S, 1><<<grid, kScanWarps * 32, 0, s>>>(raw, u, xp, m.ldx, alog, dskip, proj,
                                                              m.ldp, y32, gated, hchk, seg_h,
                                                              seg_dt, m.T, m.D, m.N, m.R);
    return launch_status();
}

template <int L, int S>
int launch_scan_bwd(const MambaDims& m, const float* raw, const float* u, const float* xp,
                    const float* alog, const float* dskip, const bf16* proj, const float* y32,
                    const float* dgated, const float* hchk, float* du, float* draw, bf16* dproj,
                    float* dbc_part, float* da_part, float* dd_part, float* seg_work,
                    cudaStream_t s) {
    constexpr int CPB = ScanTile<L, S>::kCPB;
    const int nseg = mamba_scan_segments(m.B, m.T, m.D, m.N);
    dim3 grid((m.D + CPB - 1) / CPB, m.B, nseg);
    float* seg_dh = seg_work;
    float* seg_dt = seg_work + (size_t)m.B * nseg * m.D * m.N;
    if (nseg > 1) {
        scan_bwd_carry_kernel<L, S><<<grid, kScanWarps * 32, 0, s>>>(
            raw, xp, m.ldx, alog, proj, m.ldp, dgated, seg_dh, seg_dt, m.T, m.D, m.N, m.R);
        int rc = launch_status();
        if (rc) return rc;
    }
    constexpr size_t smem = ScanBwdSmem<L, S>::kBytes;
    static bool attr = false;  // per instantiation
    if (!attr) {
        const cudaError_t e = cudaFuncSetAttribute(
            scan_bwd_kernel<L, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return -(1000 + (int)e);
        attr = true;
    }
    scan_bwd_kernel<L, S><<<grid, kScanWarps * 32, smem, s>>>(
        raw, u, xp, m.ldx, alog, dskip, proj, m.ldp, y32, dgated, hchk, du, draw, dproj, dbc_part,
        da_part, dd_part, seg_dh, seg_dt, m.T, m.D, m.N, m.R);
    return launch_status();
}

// Scan layout for d_state N: lanes per channel (L) and states per lane (S), L * S >= N;
// 0 when N is above 16 (the staging is sized for it).
int scan_layout(int N) { return N <= 4 ? 41 : N <= 8 ? 81 : N <= 16 ? 82 : 0; }
int scan_cpb(int layout) { return kScanWarps * (32 / (layout / 10)); }

}  // namespace

int small_gemm_f32(const float* A, long long sam, long long sak, const float* B, long long sbk,
                   long long sbn, int M, int N, int K, int ksplit, float* part, float* out,
                   bf16* out16, long long ldo, int accumulate, cudaStream_t s) {
    if (ksplit < 1 || M < 1 || N < 1 || K < 1) return -1;
    const int kchunk = ((K + ksplit - 1) / ksplit + kSgK - 1) / kSgK * kSgK;
    const int zs = (K + kchunk - 1) / kchunk;
    if (zs > 1 && !part) return -1;
    const bool narrow = N <= 48;  // the dt_rank-wide outputs fit one 48-column tile
    const int bn = narrow ? 48 : 64;
    dim3 grid((M + kSgM - 1) / kSgM, (N + bn - 1) / bn, zs);
    if (narrow)
        sgemm_f32_kernel<48><<<grid, 256, 0, s>>>(A, sam, sak, B, sbk, sbn, M, N, K, kchunk, part,
                                                  out, out16, ldo, accumulate);
    else
        sgemm_f32_kernel<64><<<grid, 256, 0, s>>>(A, sam, sak, B, sbk, sbn, M, N, K, kchunk, part,
                                                  out, out16, ldo, accumulate);
    int rc = launch_status();
    if (rc || zs == 1) return rc;
    const long long n = (long long)M * N;
    small_gemm_reduce_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(part, zs, M, N, out, out16, ldo,
                                                                    accumulate);
    return launch_status();
}

int convert_f32_bf16(const float* src, long long lds, bf16* dst, long long ldd, long long rows,
                     int cols, cudaStream_t s) {
    const long long n = rows * cols;
    convert_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(src, lds, dst, ldd, rows, cols);
    return launch_status();
}

int mamba_scan_groups(int D, int N) {
    const int layout = scan_layout(N);
    if (!layout) return 0;
    const int cpb = scan_cpb(layout);
    return (D + cpb - 1) / cpb;
}
int mamba_conv_blocks(long long rows) { return (int)((rows + kConvRows - 1) / kConvRows); }

template <int K>
int launch_conv_fwd(const MambaDims& m, const bf16* proj, const float* w, const float* bias,
                    float* u32, bf16* u16, cudaStream_t s) {
    const long long rows = (long long)m.B * m.T;
    dim3 grid((m.D + 255) / 256, mamba_conv_blocks(rows));
    conv_fwd_kernel<K><<<grid, 256, 0, s>>>(proj, m.ldp, m.D, m.T, w, bias, u32, u16, rows);
    return launch_status();
}

template <int K>
int launch_conv_bwd(const MambaDims& m, const bf16* proj, const float* w, const float* bias,
                    const float* du_scan, const float* du_xp, float* part, bf16* dproj,
                    cudaStream_t s) {
    const long long rows = (long long)m.B * m.T;
    dim3 grid((m.D + 255) / 256, mamba_conv_blocks(rows));
    conv_bwd_kernel<K><<<grid, 256, 0, s>>>(proj, m.ldp, m.D, m.T, w, bias, du_scan, du_xp, part,
                                            dproj, rows);
    return launch_status();
}

int mamba_conv_forward(const MambaDims& m, const bf16* proj, const float* w, const float* bias,
                       float* u32, bf16* u16, cudaStream_t s) {
    switch (m.K) {
        case 1: return launch_conv_fwd<1>(m, proj, w, bias, u32, u16, s);
        case 2: return launch_conv_fwd<2>(m, proj, w, bias, u32, u16, s);
        case 3: return launch_conv_fwd<3>(m, proj, w, bias, u32, u16, s);
        case 4: return launch_conv_fwd<4>(m, proj, w, bias, u32, u16, s);
        case 5: return launch_conv_fwd<5>(m, proj, w, bias, u32, u16, s);
        case 6: return launch_conv_fwd<6>(m, proj, w, bias, u32, u16, s);
        case 7: return launch_conv_fwd<7>(m, proj, w, bias, u32, u16, s);
        case 8: return launch_conv_fwd<8>(m, proj, w, bias, u32, u16, s);
        default: return -1;
    }
}

// raw = xp[:, :R] dt_proj^T, fp32 (rows x D, K = R)
int mamba_dt_forward(const MambaDims& m, const float* xp, const float* dt_proj, float* raw,
                     cudaStream_t s) {
    const int rows = m.B * m.T;
    return small_gemm_f32(xp, m.ldx, 1, dt_proj, 1, m.R, rows, m.D, m.R, 1, nullptr, raw, nullptr,
                          m.D, 0, s);
}

static int scan_channels_per_block(int N) {
    switch (scan_layout(N)) {
        case 41: return ScanTile<4, 1>::kCPB;
        case 81: return ScanTile<8, 1>::kCPB;
        case 82: return ScanTile<8, 2>::kCPB;
        default: return 1;
    }
}

static int device_sms() {
    static int sms = [] {
        int dev = 0, n = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        return n > 0 ? n : 148;
    }();
    return sms;
}

// Splitting the sequence costs a carry pass, so it only pays when the (channel group, sequence)
// grid leaves SMs idle: fewer blocks than SMs. Then enough segments of at least 32 chunks
// (512 steps) each to reach two blocks per SM, at most 8.
int mamba_scan_segments(int B, int T, int D, int N) {
    const int sms = device_sms();
    const int cpb = scan_channels_per_block(N);
    const long long blocks = (long long)B * ((D + cpb - 1) / cpb);
    if (blocks <= 0 || blocks >= sms) return 1;
    const int nch = (T + kScanChunk - 1) / kScanChunk;
    long long p = (2LL * sms + blocks - 1) / blocks;
    if (p > T / 512) p = T / 512;
    if (p > 8) p = 8;
    if (p > nch) p = nch;
    return p < 1 ? 1 : (int)p;
}
int mamba_scan_parts_max(int max_batch, int max_seq, int D, int N) {
    int best = 0;
    for (int b = 1; b <= max_batch; ++b) {
        const int parts = b * mamba_scan_segments(b, max_seq, D, N);
        best = parts > best ? parts : best;
    }
    return best;
}
size_t mamba_scan_seg_floats(int max_batch, int max_seq, int D, int N) {
    return (size_t)mamba_scan_parts_max(max_batch, max_seq, D, N) * D * (N + 1);
}

int mamba_scan_forward(const MambaDims& m, const float* raw, const float* u, const float* xp,
                       const float* alog, const float* dskip, const bf16* proj, float* y32,
                       bf16* gated, float* hchk, float* seg_work, cudaStream_t s) {
#define SF(L, S) \
    launch_scan_fwd<L, S>(m, raw, u, xp, alog, dskip, proj, y32, gated, hchk, seg_work, s)
    switch (scan_layout(m.N)) {
        case 41: return SF(4, 1);
        case 81: return SF(8, 1);
        case 82: return SF(8, 2);
        default: return -1;
    }
#undef SF
}

int mamba_scan_backward(const MambaDims& m, const float* raw, const float* u, const float* xp,
                        const float* alog, const float* dskip, const bf16* proj, const float* y32,
                        const float* dgated, const float* hchk, float* du, float* draw, bf16* dproj,
                        float* dbc_part, float* da_part, float* dd_part, float* seg_work,
                        cudaStream_t s) {
#define SB(L, S)                                                                             \
    launch_scan_bwd<L, S>(m, raw, u, xp, alog, dskip, proj, y32, dgated, hchk, du, draw, dproj, \
                          dbc_part, da_part, dd_part, seg_work, s)
    switch (scan_layout(m.N)) {
        case 41: return SB(4, 1);
        case 81: return SB(8, 1);
        case 82: return SB(8, 2);
        default: return -1;
    }
#undef SB
}

int mamba_reduce_dbc(const MambaDims& m, const float* dbc_part, bf16* dxp, cudaStream_t s) {
    const long long BT = (long long)m.B * m.T, n = BT * m.N;
    dbc_reduce_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(dbc_part, mamba_scan_groups(m.D, m.N),
                                                             BT, m.N, m.R, dxp, m.ldx);
    return launch_status();
}

int mamba_batch_reduce(const float* part, int B, long long n, float* out, int accumulate,
                       cudaStream_t s) {
    batch_reduce_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(part, B, n, out, accumulate);
    return launch_status();
}

int mamba_conv_backward(const MambaDims& m, const bf16* proj, const float* w, const float* bias,
                        const float* du_scan, const float* du_xp, float* part, bf16* dproj,
                        float* gw, float* gb, int accumulate, cudaStream_t s) {
    int rc;
    switch (m.K) {
        case 1: rc = launch_conv_bwd<1>(m, proj, w, bias, du_scan, du_xp, part, dproj, s); break;
        case 2: rc = launch_conv_bwd<2>(m, proj, w, bias, du_scan, du_xp, part, dproj, s); break;
        case 3: rc = launch_conv_bwd<3>(m, proj, w, bias, du_scan, du_xp, part, dproj, s); break;
        case 4: rc = launch_conv_bwd<4>(m, proj, w, bias, du_scan, du_xp, part, dproj, s); break;
        case 5: rc = launch_conv_bwd<5>(m, proj, w, bias, du_scan, du_xp, part, dproj, s); break;
        case 6: rc = launch_conv_bwd<6>(m, proj, w, bias, du_scan, du_xp, part, dproj, s); break;
        case 7: rc = launch_conv_bwd<7>(m, proj, w, bias, du_scan, du_xp, part, dproj, s); break;
        case 8: rc = launch_conv_bwd<8>(m, proj, w, bias, du_scan, du_xp, part, dproj, s); break;
        default: return -1;
    }
    if (rc) return rc;
    const long long rows = (long long)m.B * m.T;
    const int nr = m.D * (m.K + 1);
    conv_reduce_kernel<<<(nr + 255) / 256, 256, 0, s>>>(part, mamba_conv_blocks(rows), m.D, m.K, gw,
                                                        gb, accumulate);
    return launch_status();
}

}  // namespace llmgpu
