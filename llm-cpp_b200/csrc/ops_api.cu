// Kernel-level C ABI (include/llmgpu_ops.h): thin wrappers that run one kernel
// on caller-owned device buffers, used by the per-kernel parity tests.
#include <cuda_runtime.h>

#include "gemm.cuh"
#include "llmgpu_ops.h"

using namespace llmgpu;

static int device_num_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
    return n > 0 ? n : 148;
}

extern "C" int llmgpu_op_num_sms(void) { return device_num_sms(); }

extern "C" int llmgpu_op_gemm(const void* A, long long lda, int a_mn_major, const void* B,
                              long long ldb, int b_mn_major, int M, int N, int K, int epi,
                              void* out, long long ldo, int accumulate, const float* resid,
                              long long ldr, void* aux, long long ld_aux, int splits,
                              float* workspace, int col_group, long long group_stride, int bn,
                              int* err, void* stream) {
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    GemmArgs g{};
    g.epi = epi;
    g.accumulate = accumulate;
    g.out = out;
    g.ldo = ldo;
    g.col_group = col_group;
    g.group_stride = group_stride;
    g.resid = resid;
    g.ldr = ldr;
    g.aux = aux;
    g.ld_aux = ld_aux;
    g.splits = splits < 1 ? 1 : splits;
    g.err = err;
    if (g.splits > 1) {
        if (epi != kEpiStoreF32 || workspace == nullptr) return -100;
        g.epi = kEpiSplitPartial;
        g.out = workspace;
        g.ldo = N;
    }
    GemmPlan plan;
    int rc = gemm_make_plan(&plan, A, lda, a_mn_major, B, ldb, b_mn_major, M, N, K, g, bn,
                            device_num_sms());
    if (rc) return rc;
    rc = gemm_run(plan, st);
    if (rc) return rc;
    if (g.splits > 1)
        rc = gemm_splitk_reduce(workspace, g.splits, M, N, reinterpret_cast<float*>(out), ldo,
                                col_group <= 0 ? N : col_group, group_stride, accumulate, st);
    return rc;
}
