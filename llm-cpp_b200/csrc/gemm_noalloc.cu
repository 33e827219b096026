// Split-K GEMM entry point that allocates no device memory.
//
// Callers such as a custom allocator, a pre-reserved memory pool, or code running where
// any cudaMalloc would break a memory budget or an exclusive pool cannot hand
// llmgpu_op_gemm a freshly allocated split-K workspace. This variant keeps its split-K
// partial sums in a fixed file-scope device array instead, so the caller passes only
// inputs and outputs.
#include <cuda_runtime.h>

#include <mutex>

#include "gemm.cuh"
#include "llmgpu_ops.h"

using namespace llmgpu;

namespace {

// 4 Mi floats (16 MiB) of split-K partials. Every GPU that loads the library holds this
// array until the process exits. Contents persist between calls; every call overwrites
// the splits*M*N floats it uses before reading them, so nothing needs clearing.
constexpr long long kNoAllocScratchFloats = 4LL << 20;
__device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device. In host code the array's
// name is only a host-side stand-in; the device address comes from cudaGetSymbolAddress,
// queried once per device with that device current.
int scratch_for_current_device(float** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -102;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return -103;
        g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_scratch_ptr[dev];
    return 0;
}

int device_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
    return n > 0 ? n : 148;
}

}  // namespace

extern "C" int llmgpu_op_gemm_splitk_noalloc(const void* A, long long lda, int a_mn_major,
                                             const void* B, long long ldb, int b_mn_major, int M,
                                             int N, int K, float* out, long long ldo,
                                             int accumulate, int splits, int col_group,
                                             long long group_stride, int* err, void* stream) {
    if (M <= 0 || N <= 0 || K <= 0 || splits < 1 || !out) return -1;
    // the column-group rule of llmgpu_op_gemm (its plan sees col_group, this one's partial
    // tiles are ungrouped), so that both entry points accept the same arguments
    if (col_group > 0 && col_group != N && (col_group % 32) != 0) return -7;
    if ((long long)splits * M * N > kNoAllocScratchFloats) return -101;  // beyond the scratch
    float* scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    GemmArgs g{};
    g.epi = kEpiSplitPartial;
    g.out = scratch;
    g.ldo = N;
    g.splits = splits;
    g.col_group = N;
    g.err = err;
    GemmPlan plan;
    rc = gemm_make_plan(&plan, A, lda, a_mn_major, B, ldb, b_mn_major, M, N, K, g, 0,
                        device_sms());
    if (rc) return rc;
    if ((rc = gemm_run(plan, st))) return rc;
    return gemm_splitk_reduce(scratch, splits, M, N, out, ldo, col_group <= 0 ? N : col_group,
                              group_stride, accumulate, st);
}
