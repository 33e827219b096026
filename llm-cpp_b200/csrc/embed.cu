// Token/position embedding gather and its deterministic scatter-add backward.
#include "common.cuh"
#include "kernels.cuh"

namespace llmgpu {

namespace {

__device__ __forceinline__ int wrap_token(int tok, int V) {
    // ((tok % V) + V) % V, as src/model.cpp:152-153 clamps out-of-vocabulary ids
    int r = tok % V;
    return r < 0 ? r + V : r;
}

// `rope` (nullable): per position t, the (cos, sin) of every column pair (2j, 2j+1) as
// [T][C/2] float2, i.e. one float4 per group of four columns. With it the sum is rotated
// pairwise and scaled by rope_scale, as rope_cfg does to the embedding sum
// (src/model.cpp:81-104,158): (x0 cos - x1 sin, x0 sin + x1 cos) * scale.
__global__ void embed_fwd_kernel(const int32_t* __restrict__ tokens, const float* __restrict__ wte,
                                 const float* __restrict__ wpe, float* __restrict__ x, int B, int T,
                                 int C, int V, const float4* __restrict__ rope, float rope_scale) {
    pdl_enter();
    const int row = blockIdx.x;  // b*T + t
    const int t = row % T;
    const int tok = wrap_token(tokens[row], V);
    const float4* a = reinterpret_cast<const float4*>(wte + (long long)tok * C);
    const float4* p = reinterpret_cast<const float4*>(wpe + (long long)t * C);
    float4* o = reinterpret_cast<float4*>(x + (long long)row * C);
    const float4* r = rope ? rope + (long long)t * (C >> 2) : nullptr;
    for (int i = threadIdx.x; i < (C >> 2); i += blockDim.x) {
        float4 u = a[i], w = p[i];
        float4 v = make_float4(u.x + w.x, u.y + w.y, u.z + w.z, u.w + w.w);
        if (r) {
            const float4 cs = r[i];  // (cos, sin) of pair 2i, then of pair 2i+1
            v = make_float4((v.x * cs.x - v.y * cs.y) * rope_scale,
                            (v.x * cs.y + v.y * cs.x) * rope_scale,
                            (v.z * cs.z - v.w * cs.w) * rope_scale,
                            (v.z * cs.w + v.w * cs.z) * rope_scale);
        }
        o[i] = v;
    }
}

// Single-CTA bitonic sort of n <= 16384 keys (token << 32 | row) in shared memory.
__global__ void __launch_bounds__(1024) sort_keys_kernel(const int32_t* __restrict__ tokens, int n,
                                                         int V, uint64_t* __restrict__ keys) {
    pdl_enter();
    extern __shared__ uint64_t sk[];
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = threadIdx.x; i < np2; i += blockDim.x) {
        sk[i] = i < n ? (((uint64_t)wrap_token(tokens[i], V) << 32) | (uint32_t)i) : ~0ull;
    }
    __syncthreads();
    for (int size = 2; size <= np2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < np2; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    uint64_t a = sk[i], b = sk[j];
                    if ((a > b) == up) {
                        sk[i] = b;
                        sk[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) keys[i] = sk[i];
}

// Deterministic scatter-add of dx rows into wte_grad, balanced for skewed token
// frequencies (a Zipf batch repeats its most frequent id ~10% of the time).
// Sorted positions are cut into pieces: a piece starts where the token changes or at a
// multiple of kPiece. Stage 1 (one warp per piece start and 128-column slice) sums the
// piece's rows in row order; a piece that is a whole run is added to its token's row
// directly, otherwise its sum goes to scratch[piece start]. Stage 2 (one warp per run
// start of a multi-piece run) sums those piece partials in order and adds the total.
constexpr int kPiece = 16;

__device__ __forceinline__ uint32_t key_tok(const uint64_t* keys, int i) {
    return (uint32_t)(keys[i] >> 32);
}

// First index past `p` (within [p + 1, lim), lim <= p + 32) whose token is not `tok`: one key
// load per lane and a ballot instead of a chain of dependent loads. Whole warp.
__device__ __forceinline__ int run_end_within(const uint64_t* keys, int p, int lim, uint32_t tok,
                                              int lane) {
    const int q = p + 1 + lane;
    const bool same = q < lim && key_tok(keys, q) == tok;
    const unsigned m = __ballot_sync(0xffffffffu, same);  // a prefix of lanes: sorted keys
    return m == 0xffffffffu ? p + 33 : p + __ffs(~m);
}

__device__ __forceinline__ void add4(float4& a, const float4& v) {
    a.x += v.x;
    a.y += v.y;
    a.z += v.z;
    a.w += v.w;
}

__global__ void wte_grad_pieces(const uint64_t* __restrict__ keys, int n,
                                const float* __restrict__ dx, float* __restrict__ wte_grad,
                                float* __restrict__ scratch, int C) {
    pdl_enter();
    const int p = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int c = blockIdx.y * 128 + lane * 4;
    if (p >= n) return;  // whole warp
    const bool col = c < C;
    const uint32_t tok = key_tok(keys, p);
    const bool run_start = (p == 0) || key_tok(keys, p - 1) != tok;
    if (!run_start && (p % kPiece) != 0) return;  // not a piece start (whole warp)
    const int block_end = min(n, (p / kPiece + 1) * kPiece);
    const int e = run_end_within(keys, p, block_end, tok, lane);
    // the piece's rows in row order, four loads in flight
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (col) {
        int k = p;
        for (; k + 4 <= e; k += 4) {
            float4 v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int row = (int)(keys[k + j] & 0xffffffffu);
                v[j] = *reinterpret_cast<const float4*>(dx + (long long)row * C + c);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) add4(acc, v[j]);
        }
        for (; k < e; ++k) {
            const int row = (int)(keys[k] & 0xffffffffu);
            add4(acc, *reinterpret_cast<const float4*>(dx + (long long)row * C + c));
        }
    }
    const bool run_end = (e == n) || key_tok(keys, e) != tok;
    if (!col) return;
    if (run_start && run_end) {
        float4* g = reinterpret_cast<float4*>(wte_grad + (long long)tok * C + c);
        float4 o = *g;
        add4(o, acc);
        *g = o;
    } else {
        *reinterpret_cast<float4*>(scratch + (long long)p * C + c) = acc;
    }
}

__global__ void wte_grad_runs(const uint64_t* __restrict__ keys, int n,
                              const float* __restrict__ scratch, float* __restrict__ wte_grad,
                              int C) {
    pdl_enter();
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int c = blockIdx.y * 128 + lane * 4;
    if (r >= n) return;  // whole warp
    const uint32_t tok = key_tok(keys, r);
    if (r > 0 && key_tok(keys, r - 1) == tok) return;  // not a run start
    const int first_end = min(n, (r / kPiece + 1) * kPiece);
    if (first_end >= n || key_tok(keys, first_end) != tok) return;  // single-piece run
    // the run's further pieces start at first_end + k kPiece: count them 32 at a time, one
    // key load per lane (a frequent token's run has dozens of pieces)
    int pieces = 0;
    for (;;) {
        const int q = first_end + (pieces + lane) * kPiece;
        const bool same = q < n && key_tok(keys, q) == tok;
        const unsigned m = __ballot_sync(0xffffffffu, same);
        const int cnt = m == 0xffffffffu ? 32 : __ffs(~m) - 1;
        pieces += cnt;
        if (cnt < 32) break;
    }
    if (c >= C) return;
    // piece sums in piece order, four loads in flight
    float4 acc = *reinterpret_cast<const float4*>(scratch + (long long)r * C + c);
    int k = 0;
    for (; k + 4 <= pieces; k += 4) {
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            v[j] = *reinterpret_cast<const float4*>(
                scratch + (long long)(first_end + (k + j) * kPiece) * C + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) add4(acc, v[j]);
    }
    for (; k < pieces; ++k)
        add4(acc, *reinterpret_cast<const float4*>(
                      scratch + (long long)(first_end + k * kPiece) * C + c));
    float4* g = reinterpret_cast<float4*>(wte_grad + (long long)tok * C + c);
    float4 o = *g;
    add4(o, acc);
    *g = o;
}

__global__ void wpe_grad_kernel(const float* __restrict__ dx, float* __restrict__ wpe_grad, int B,
                                int T, int C, int accumulate) {
    pdl_enter();
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;  // over T*C/4
    if (i >= (long long)T * C / 4) return;
    const int t = (int)(i / (C / 4));
    const int c4 = (int)(i - (long long)t * (C / 4));
    float4 acc = accumulate ? reinterpret_cast<float4*>(wpe_grad + (long long)t * C)[c4]
                            : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int b = 0; b < B; ++b) {
        float4 v = reinterpret_cast<const float4*>(dx + ((long long)b * T + t) * C)[c4];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    reinterpret_cast<float4*>(wpe_grad + (long long)t * C)[c4] = acc;
}

}  // namespace

int embed_forward(const int32_t* tokens, const float* wte, const float* wpe, float* x, int B,
                  int T, int C, int V, cudaStream_t s, const float* rope, float rope_scale) {
    if ((C & 3) != 0) return -1;
    launch_kernel(embed_fwd_kernel, B * T, 128, 0, s, tokens, wte, wpe, x, B, T, C, V,
                                           reinterpret_cast<const float4*>(rope), rope_scale);
    return launch_status();
}

int embed_sort_keys(const int32_t* tokens, int n, int V, uint64_t* keys, cudaStream_t s) {
    if (n > 16384 || n <= 0) return -1;
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    const size_t smem = (size_t)np2 * sizeof(uint64_t);
    static bool set = false;
    if (!set) {
        cudaFuncSetAttribute(sort_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             16384 * 8);
        set = true;
    }
    launch_kernel(sort_keys_kernel, 1, 1024, smem, s, tokens, n, V, keys);
    return launch_status();
}

int embed_backward(const uint64_t* keys, const float* dx, float* wte_grad, float* wpe_grad, int B,
                   int T, int C, int accumulate_wpe, float* scratch, cudaStream_t s) {
    if ((C & 3) != 0) return -1;
    const int n = B * T;
    dim3 grid((n + 7) / 8, (C + 127) / 128);
    launch_kernel(wte_grad_pieces, grid, 256, 0, s, keys, n, dx, wte_grad, scratch, C);
    launch_kernel(wte_grad_runs, grid, 256, 0, s, keys, n, scratch, wte_grad, C);
    const long long m = (long long)T * C / 4;
    launch_kernel(wpe_grad_kernel, (int)((m + 255) / 256), 256, 0, s, dx, wpe_grad, B, T, C, accumulate_wpe);
    return launch_status();
}

}  // namespace llmgpu
