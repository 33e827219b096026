"""The split-K GEMM entry point that allocates nothing (llmgpu_op_gemm_splitk_noalloc).

It serves callers that cannot call cudaMalloc (their memory comes from a pre-reserved pool
or a fixed budget) and keeps its split-K partials in a fixed array inside the library.
Checked through the C ABI against llmgpu_op_gemm with a caller-provided workspace, on two
calls in a row (the second reuses the array the first one left behind).
"""
import ctypes

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SCRATCH_FLOATS = 4 << 20


def _noalloc(lib):
    f = lib.llmgpu_op_gemm_splitk_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _rel(a, b):
    return float((a.double() - b.double()).norm() / (b.double().norm() + 1e-30))


def test_noalloc_splitk_matches_workspace_gemm(cuda):
    from llmgpu import load, ops
    lib = load()
    noalloc = _noalloc(lib)
    stream = torch.cuda.current_stream().cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    g = torch.Generator().manual_seed(21)
    # weight-gradient shape: X^T dY over 1024 tokens into three grouped [C, C] outputs,
    # then a plain one with accumulation, so the second call sees the first call's leftovers
    cases = [dict(M=128, N=384, K=1024, splits=4, group=128, acc=0),
             dict(M=256, N=192, K=2048, splits=6, group=0, acc=1)]
    for c in cases:
        M, N, K, S = c["M"], c["N"], c["K"], c["splits"]
        a = torch.randn(K, M, generator=g).to(torch.bfloat16).to(cuda)   # MN-major A
        b = torch.randn(K, N, generator=g).to(torch.bfloat16).to(cuda)   # MN-major B
        grouped = c["group"] > 0
        shape = (N // c["group"], M, c["group"]) if grouped else (M, N)
        ldo = c["group"] if grouped else N
        gs = M * c["group"] if grouped else 0
        base = torch.randn(*shape, generator=g).to(cuda)
        want = base.clone()
        ops.gemm(a, b, M, N, K, a_mn=True, b_mn=True, epi=ops.EPI_F32, out=want, ldo=ldo,
                 accumulate=bool(c["acc"]), splits=S, col_group=c["group"], group_stride=gs)
        got = base.clone()
        rc = noalloc(a.data_ptr(), M, 1, b.data_ptr(), N, 1, M, N, K, got.data_ptr(), ldo,
                     c["acc"], S, c["group"], gs, err.data_ptr(), stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert _rel(got, want) < 1e-5
        # and against a plain fp32 product of the same bf16 operands
        ref = a.float().t() @ b.float()
        if grouped:
            ref = ref.reshape(M, N // c["group"], c["group"]).permute(1, 0, 2)
        ref = ref + base if c["acc"] else ref
        assert _rel(got, ref) < 1e-5


def test_noalloc_rejects_what_the_workspace_gemm_rejects(cuda):
    """A column group that is neither N nor a multiple of 32 is refused by both entry points
    with the same status."""
    from llmgpu import load, ops
    lib = load()
    noalloc = _noalloc(lib)
    M, N, K, S, group = 64, 96, 256, 2, 48
    a = torch.zeros(K, M, dtype=torch.bfloat16, device=cuda)
    b = torch.zeros(K, N, dtype=torch.bfloat16, device=cuda)
    out = torch.zeros(N // group, M, group, device=cuda)
    ws = torch.zeros(S * M * N, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    rc_ws = lib.llmgpu_op_gemm(a.data_ptr(), M, 1, b.data_ptr(), N, 1, M, N, K, ops.EPI_F32,
                               out.data_ptr(), group, 0, None, 0, None, 0, S, ws.data_ptr(),
                               group, M * group, 0, None, stream)
    rc_na = noalloc(a.data_ptr(), M, 1, b.data_ptr(), N, 1, M, N, K, out.data_ptr(), group, 0, S,
                    group, M * group, None, stream)
    assert rc_ws == rc_na == -7


def test_noalloc_rejects_oversize(cuda):
    from llmgpu import load
    noalloc = _noalloc(load())
    out = torch.zeros(1, device=cuda)
    M, N, S = 2048, 1024, 4                          # 8 Mi floats > 4 Mi scratch
    assert S * M * N > SCRATCH_FLOATS
    rc = noalloc(out.data_ptr(), M, 1, out.data_ptr(), N, 1, M, N, 256, out.data_ptr(), N, 0, S,
                 0, 0, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == -101
