"""Per-kernel wrappers over the kernel-level C ABI (include/llmgpu_ops.h).

Arguments are torch CUDA tensors (used only as device allocations); every call
checks the status code and the device error word and raises on failure.
"""
import torch

from ._lib import load

EPI_BF16, EPI_F32, EPI_RESID, EPI_GELU, EPI_DGELU = 0, 1, 2, 3, 4


def _ptr(t):
    return 0 if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


class KernelError(RuntimeError):
    pass


def _check(rc, what):
    if rc != 0:
        raise KernelError(f"{what} failed with status {rc}")


def gemm(A, B, M, N, K, *, a_mn=False, b_mn=False, lda=None, ldb=None, epi=EPI_F32, out=None,
         ldo=None, accumulate=False, resid=None, ldr=None, aux=None, ld_aux=None, splits=1,
         col_group=0, group_stride=0, bn=0, err=None):
    """D[M,N] = A[M,K] @ B[N,K]^T on the tcgen05 GEMM kernel (bf16 in, fp32 acc)."""
    lib = load()
    dev = A.device
    if lda is None:
        lda = A.shape[-1]
    if ldb is None:
        ldb = B.shape[-1]
    if out is None:
        dt = torch.float32 if epi in (EPI_F32, EPI_RESID) else torch.bfloat16
        out = torch.zeros(M, N, dtype=dt, device=dev)
    if ldo is None:
        ldo = out.shape[-1]
    own_err = err is None
    if own_err:
        err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = None
    if splits > 1:
        ws = torch.empty(splits * M * N, dtype=torch.float32, device=dev)
    rc = lib.llmgpu_op_gemm(_ptr(A), lda, int(a_mn), _ptr(B), ldb, int(b_mn), M, N, K, epi,
                            _ptr(out), ldo, int(accumulate), _ptr(resid), ldr or 0, _ptr(aux),
                            ld_aux or 0, splits, _ptr(ws), col_group, group_stride, bn,
                            _ptr(err), _stream())
    _check(rc, "llmgpu_op_gemm")
    if own_err:
        torch.cuda.synchronize()
        if int(err.item()) != 0:
            raise KernelError(f"gemm device error code {int(err.item())}")
    return out
