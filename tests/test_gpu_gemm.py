"""tcgen05 GEMM kernel vs a torch fp32 reference of the same product.

The GEMM replaces the fp32 contractions of Tensor::matmul (src/tensor.cpp:229-321)
and the gradient loops of the blocks; here it is checked alone on bf16-rounded
inputs, so the only difference from the fp32 reference is accumulation order.
"""
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _mk(shape, gen, scale=1.0):
    return (torch.randn(*shape, generator=gen) * scale).to(torch.bfloat16)


def _ref(a, b, a_mn, b_mn):
    A = a.float().t() if a_mn else a.float()      # -> [M, K]
    B = b.float() if b_mn else b.float().t()      # -> [K, N]
    return A @ B


def _rel(x, y):
    return float((x.float() - y.float()).norm() / (y.float().norm() + 1e-30))


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("bn", [64, 128, 256, 512])  # 512: 256x256 tiles on a CTA pair
@pytest.mark.parametrize("M,N,K", [(256, 512, 192), (200, 100, 70), (128, 64, 64),
                                   (520, 300, 136), (1024, 768, 512)])
def test_gemm_majors_tiles(cuda, a_mn, b_mn, bn, M, N, K):
    from llmgpu import ops
    g = torch.Generator().manual_seed(M * 7 + N * 3 + K + 11 * bn + 2 * a_mn + b_mn)
    a = _mk((K, M) if a_mn else (M, K), g)
    b = _mk((K, N) if b_mn else (N, K), g)
    # pad leading dims to multiples of 8 elements (16-byte TMA strides)
    def pad(t):
        r, c = t.shape
        cp = (c + 7) // 8 * 8
        out = torch.zeros(r, cp, dtype=t.dtype)
        out[:, :c] = t
        return out
    ap, bp = pad(a).to(cuda), pad(b).to(cuda)
    out = torch.zeros(M, (N + 7) // 8 * 8, dtype=torch.float32, device=cuda)
    ops.gemm(ap, bp, M, N, K, a_mn=a_mn, b_mn=b_mn, epi=ops.EPI_F32, out=out, bn=bn)
    ref = _ref(a, b, a_mn, b_mn)
    got = out[:, :N].cpu()
    assert _rel(got, ref) < 1e-4, _rel(got, ref)


@pytest.mark.parametrize("bn", [0, 128, 256, 512])  # planner's choice, one CTA, CTA pair
@pytest.mark.parametrize("M,N,K", [(384, 320, 256),
                                   # several tiles per CTA or pair; the last tile column ends
                                   # inside a 32-column chunk and after an odd chunk count
                                   (8192, 968, 128)])
def test_gemm_epilogues(cuda, bn, M, N, K):
    from llmgpu import ops
    g = torch.Generator().manual_seed(5)
    a = _mk((M, K), g, 0.5).to(cuda)
    b = _mk((K, N), g, 0.5).to(cuda)          # MN-major B, like x @ W
    ref = a.float() @ b.float()
    # bf16 store
    o = ops.gemm(a, b, M, N, K, b_mn=True, bn=bn, epi=ops.EPI_BF16)
    assert _rel(o, ref) < 8e-3
    # residual add
    r = torch.randn(M, N, device=cuda)
    o = ops.gemm(a, b, M, N, K, b_mn=True, bn=bn, epi=ops.EPI_RESID, resid=r, ldr=N)
    assert _rel(o, ref + r) < 1e-5
    # accumulate
    base = torch.randn(M, N, device=cuda)
    o = base.clone()
    ops.gemm(a, b, M, N, K, b_mn=True, bn=bn, epi=ops.EPI_F32, out=o, accumulate=True)
    assert _rel(o, ref + base) < 1e-5
    # gelu + stored pre-activation
    h = torch.zeros(M, N, dtype=torch.bfloat16, device=cuda)
    o = ops.gemm(a, b, M, N, K, b_mn=True, bn=bn, epi=ops.EPI_GELU, aux=h, ld_aux=N)
    gelu = 0.5 * ref * (1 + torch.tanh(0.7978845608 * (ref + 0.044715 * ref ** 3)))
    assert _rel(h, ref) < 8e-3
    assert _rel(o, gelu) < 8e-3
    # gelu backward from the stored pre-activation
    hv = h.float()
    th = torch.tanh(0.7978845608 * (hv + 0.044715 * hv ** 3))
    dg = 0.5 * (1 + th) + 0.5 * hv * (1 - th * th) * 0.7978845608 * (1 + 3 * 0.044715 * hv * hv)
    o = ops.gemm(a, b, M, N, K, b_mn=True, bn=bn, epi=ops.EPI_DGELU, aux=h, ld_aux=N)
    assert _rel(o, ref * dg) < 8e-3


@pytest.mark.parametrize("bn", [0, 512])
def test_gemm_splitk_grouped(cuda, bn):
    """Weight-gradient shape: X^T dY with K = tokens, split over K, written into
    three adjacent [C, C] parameter gradients (Wq|Wk|Wv layout)."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(9)
    T, C = 1024, 128
    x = _mk((T, C), g).to(cuda)          # [tokens, C]  -> A MN-major
    dy = _mk((T, 3 * C), g).to(cuda)     # [tokens, 3C] -> B MN-major
    ref = x.float().t() @ dy.float()     # [C, 3C]
    out = torch.zeros(3, C, C, device=cuda)
    ops.gemm(x, dy, C, 3 * C, T, a_mn=True, b_mn=True, epi=ops.EPI_F32, out=out, ldo=C,
             splits=4, col_group=C, group_stride=C * C, bn=bn)
    want = torch.stack([ref[:, i * C:(i + 1) * C] for i in range(3)])
    assert _rel(out, want) < 1e-5


@pytest.mark.parametrize("bn", [256, 512])
def test_gemm_large_persistent(cuda, bn):
    """More tiles than SMs (or SM pairs): exercises the persistent tile loop and the
    double-buffered accumulator hand-off (across the two CTAs of a pair for 512)."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(3)
    M, N, K = 8192, 2304, 768
    a = _mk((M, K), g).to(cuda)
    b = _mk((N, K), g).to(cuda)
    o = ops.gemm(a, b, M, N, K, epi=ops.EPI_F32, bn=bn)
    ref = a.float() @ b.float().t()
    assert _rel(o, ref) < 1e-4


@pytest.mark.parametrize("K", [768, 3072])
def test_gemm_residual_step_shapes(cuda, K):
    """The training step's N = 768 products with the residual epilogue at 8192 token rows on
    CTA pairs (attention output, K 768; FFN down, K 3072): 96 pair tiles in two waves."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(K)
    M, N = 8192, 768
    a = _mk((M, K), g, 0.5).to(cuda)
    b = _mk((K, N), g, 0.5).to(cuda)          # MN-major B, like x @ W
    r = torch.randn(M, N, device=cuda)
    o = ops.gemm(a, b, M, N, K, b_mn=True, bn=512, epi=ops.EPI_RESID, resid=r, ldr=N)
    assert _rel(o, a.float() @ b.float() + r) < 1e-5
