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


def _sync_check(rc, what):
    _check(rc, what)
    torch.cuda.synchronize()


def embed(tokens, wte, wpe, B, T):
    lib = load()
    C, V = wte.shape[1], wte.shape[0]
    x = torch.empty(B * T, C, dtype=torch.float32, device=wte.device)
    _sync_check(lib.llmgpu_op_embed(_ptr(tokens), _ptr(wte), _ptr(wpe), _ptr(x), B, T, C, V,
                                    _stream()), "embed")
    return x


def embed_bwd(tokens, dx, wte_grad, wpe_grad, B, T, accumulate_wpe=False):
    """wte_grad[tok mod V] += dx rows; wpe_grad (+)= the batch sum of dx rows (in place)."""
    lib = load()
    V, C = wte_grad.shape
    work = torch.empty(int(lib.llmgpu_op_embed_bwd_work(B, T, C)), dtype=torch.uint8,
                       device=dx.device)
    _sync_check(lib.llmgpu_op_embed_bwd(_ptr(tokens), _ptr(dx), _ptr(wte_grad), _ptr(wpe_grad),
                                        B, T, C, V, int(accumulate_wpe), _ptr(work), _stream()),
                "embed_bwd")


def norm_fwd(x, gamma, beta, rms=False):
    lib = load()
    rows, C = x.shape
    y = torch.empty(rows, C, dtype=torch.bfloat16, device=x.device)
    mean = torch.empty(rows, device=x.device)
    rstd = torch.empty(rows, device=x.device)
    _sync_check(lib.llmgpu_op_norm_fwd(_ptr(x), _ptr(gamma), _ptr(beta), _ptr(y), _ptr(mean),
                                       _ptr(rstd), rows, C, int(rms), _stream()), "norm_fwd")
    return y, mean, rstd


def norm_bwd(dy, x, gamma, mean, rstd, resid=None, rms=False, out=None):
    """dx = resid + the norm's input gradient; `out` (may be `resid` itself) receives dx."""
    lib = load()
    rows, C = x.shape
    dx = torch.empty_like(x) if out is None else out
    dx16 = torch.empty(rows, C, dtype=torch.bfloat16, device=x.device)
    dg, db, ds = (torch.empty(C, device=x.device) for _ in range(3))
    work = torch.empty(int(lib.llmgpu_op_norm_bwd_work(rows, C)), device=x.device)
    _sync_check(lib.llmgpu_op_norm_bwd(_ptr(dy), _ptr(x), _ptr(gamma), _ptr(mean), _ptr(rstd),
                                       _ptr(resid), _ptr(dx), _ptr(dx16), _ptr(dg), _ptr(db),
                                       _ptr(ds), _ptr(work), rows, C, int(rms), _stream()),
                "norm_bwd")
    return dx, dx16, dg, db, ds


def cross_entropy(logits16, V, tokens, scale, smoothing=0.0):
    lib = load()
    rows, Vp = logits16.shape
    loss = torch.empty(rows, device=logits16.device)
    _sync_check(lib.llmgpu_op_cross_entropy(_ptr(logits16), rows, V, Vp, _ptr(tokens),
                                            _ptr(loss), scale, smoothing, _stream()),
                "cross_entropy")
    return loss


def rope_table(T, hd, theta, device):
    """(cos, sin) of pos * theta^(-2j/hd), shape [T, hd/2, 2] fp32."""
    j = torch.arange(hd // 2, dtype=torch.float64)
    ang = torch.arange(T, dtype=torch.float64)[:, None] * theta ** (-2.0 * j / hd)[None, :]
    return torch.stack([ang.cos(), ang.sin()], -1).float().to(device).contiguous()


def attention_fwd(qkv, B, T, H, hd, rope=None, workspace=True):
    """Causal attention forward; with `workspace`, a head_dim below 64 runs zero-padded on the
    tcgen05 kernel (llmgpu_op_attention_fwd_ws), else on the mma.sync kernel."""
    lib = load()
    C = H * hd
    out = torch.empty(B * T, C, dtype=torch.bfloat16, device=qkv.device)
    lse = torch.empty(B, H, T, device=qkv.device)
    if workspace:
        nbytes = int(lib.llmgpu_op_attention_bwd_work(B, T, H, hd))
        work = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=qkv.device)
        rc = lib.llmgpu_op_attention_fwd_ws(_ptr(qkv), _ptr(out), _ptr(lse), B, T, H, hd,
                                            _ptr(rope), _ptr(work) if nbytes else None,
                                            _stream())
    else:
        rc = lib.llmgpu_op_attention_fwd(_ptr(qkv), _ptr(out), _ptr(lse), B, T, H, hd,
                                         _ptr(rope), _stream())
    _sync_check(rc, "attention_fwd")
    return out, lse


def attention_bwd(qkv, out, dout, lse, B, T, H, hd, rope=None):
    lib = load()
    dqkv = torch.zeros_like(qkv)
    dvec = torch.empty(B, H, T, device=qkv.device)
    nbytes = int(lib.llmgpu_op_attention_bwd_work(B, T, H, hd))
    work = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=qkv.device)
    _sync_check(lib.llmgpu_op_attention_bwd(_ptr(qkv), _ptr(out), _ptr(dout), _ptr(lse),
                                            _ptr(dvec), _ptr(dqkv), B, T, H, hd, _ptr(rope),
                                            _ptr(work), _stream()), "attention_bwd")
    return dqkv


def swiglu_fwd(h13, F):
    lib = load()
    rows = h13.shape[0]
    g = torch.empty(rows, F, dtype=torch.bfloat16, device=h13.device)
    _sync_check(lib.llmgpu_op_swiglu_fwd(_ptr(h13), _ptr(g), rows, F, _stream()), "swiglu_fwd")
    return g


def swiglu_bwd(dg, h13, F):
    lib = load()
    rows = h13.shape[0]
    d = torch.empty_like(h13)
    _sync_check(lib.llmgpu_op_swiglu_bwd(_ptr(dg), _ptr(h13), _ptr(d), rows, F, _stream()),
                "swiglu_bwd")
    return d


GROUP_ROWS, GROUP_K = 1, 2


def gemm_grouped(A, B, M, N, K, grp, groups, mode, *, a_mn=False, b_mn=False, lda=None,
                 ldb=None, epi=EPI_F32, out=None, ldo=None, accumulate=False, aux=None,
                 ld_aux=None, b_grp_rows=0, out_grp_stride=0):
    """Grouped (per-expert) GEMM; `grp` is an int32 device tensor of groups+1 row offsets."""
    lib = load()
    if lda is None:
        lda = A.shape[-1]
    if ldb is None:
        ldb = B.shape[-1]
    if ldo is None:
        ldo = out.shape[-1]
    err = torch.zeros(1, dtype=torch.int32, device=A.device)
    rc = lib.llmgpu_op_gemm_grouped(_ptr(A), lda, int(a_mn), _ptr(B), ldb, int(b_mn), M, N, K,
                                    epi, _ptr(out), ldo, int(accumulate), _ptr(aux), ld_aux or 0,
                                    _ptr(grp), groups, mode, b_grp_rows, out_grp_stride,
                                    _ptr(err), _stream())
    _check(rc, "llmgpu_op_gemm_grouped")
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise KernelError(f"grouped gemm device error code {int(err.item())}")
    return out


def moe_route(y, mean, rstd, gamma, beta, gate, B, T, k, rms=False):
    """Router: returns (probs [BT,E], idx [BT,k], wts [BT,k], ssum [BT])."""
    lib = load()
    C, E = gate.shape
    dev = y.device
    probs = torch.empty(B * T, E, dtype=torch.float32, device=dev)
    idx = torch.empty(B * T, k, dtype=torch.int32, device=dev)
    wts = torch.empty(B * T, k, dtype=torch.float32, device=dev)
    ssum = torch.empty(B * T, dtype=torch.float32, device=dev)
    _sync_check(lib.llmgpu_op_moe_route(_ptr(y), _ptr(mean), _ptr(rstd), _ptr(gamma), _ptr(beta),
                                        int(rms), _ptr(gate), B, T, C, E, k, _ptr(probs),
                                        _ptr(idx), _ptr(wts), _ptr(ssum), _stream()),
                "moe_route")
    return probs, idx, wts, ssum


def moe_dispatch(idx, B, T, E):
    """Dispatch: returns (grp [2E+1], row_of [BT,k], tok_of [BT*k + 128E])."""
    lib = load()
    k = idx.shape[1]
    dev = idx.device
    grp = torch.empty(2 * E + 1, dtype=torch.int32, device=dev)
    row_of = torch.empty(B * T, k, dtype=torch.int32, device=dev)
    tok_of = torch.empty(B * T * k + 128 * E, dtype=torch.int32, device=dev)
    _sync_check(lib.llmgpu_op_moe_dispatch(_ptr(idx), B, T, E, k, _ptr(grp), _ptr(row_of),
                                           _ptr(tok_of), _stream()), "moe_dispatch")
    return grp, row_of, tok_of
