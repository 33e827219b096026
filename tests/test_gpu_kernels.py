"""Per-kernel parity on the GPU: embedding gather (bit-exact), LayerNorm/RMSNorm forward and
backward, fused cross-entropy and causal attention forward/backward, each through the
kernel-level C ABI and checked against a plain fp32/fp64 reference of the same op."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


def test_embedding_gather_bit_exact(cuda):
    """x = wte[tok mod V] + wpe[t] (src/model.cpp:149-157), OOV ids wrap modulo V."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(0)
    B, T, C, V = 3, 37, 64, 101
    wte = torch.randn(V, C, generator=g).to(cuda)
    wpe = torch.randn(T, C, generator=g).to(cuda)
    tok = torch.randint(-300, 300, (B, T), generator=g, dtype=torch.int32)
    x = ops.embed(tok.to(cuda), wte, wpe, B, T)
    t = tok.long() % V
    want = wte.cpu()[t.reshape(-1)] + wpe.cpu().repeat(B, 1)
    assert torch.equal(x.cpu(), want)


@pytest.mark.parametrize("C", [96, 768])
@pytest.mark.parametrize("accumulate_wpe", [False, True])
def test_embedding_backward_repeated_ids(cuda, C, accumulate_wpe):
    """wte_grad[tok mod V] += dx rows, wpe_grad (+)= sum over the batch (src/model.cpp:314-322).
    One id fills 1500 of the 2048 rows (a run of 94 sixteen-row pieces: more than one
    32-piece window of the run search), the rest are random ids, negative and past V
    included; C 96 leaves lanes of the last column slice without a column."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(C + accumulate_wpe)
    B, T, V = 2, 1024, 300
    tok = torch.randint(-400, 700, (B * T,), generator=g, dtype=torch.int32)
    tok[torch.randperm(B * T, generator=g)[:1500]] = 7
    dx = torch.randn(B * T, C, generator=g)
    wte_g0 = torch.randn(V, C, generator=g)
    wpe_g0 = torch.randn(T, C, generator=g)
    wte_g, wpe_g = wte_g0.clone().to(cuda), wpe_g0.clone().to(cuda)
    ops.embed_bwd(tok.to(cuda), dx.to(cuda), wte_g, wpe_g, B, T, accumulate_wpe)
    want = wte_g0.double().index_add_(0, (tok.long() % V), dx.double())
    assert _rel(wte_g.cpu(), want) < 1e-6
    # the most repeated row: 1500 fp32 additions in pieces of 16
    assert torch.allclose(wte_g.cpu()[7].double(), want[7], rtol=0, atol=2e-4)
    # the batch sum over b in order (b = 0, then 1): exact in fp32
    d3 = dx.reshape(B, T, C)
    want_pe = (wpe_g0 + d3[0]) + d3[1] if accumulate_wpe else d3[0] + d3[1]
    assert torch.equal(wpe_g.cpu(), want_pe)


@pytest.mark.parametrize("rms", [False, True])
@pytest.mark.parametrize("C,rows", [(128, 300), (768, 300), (1024, 300),
                                    (768, 8192)])  # the GPT-2-small step's 8 x 1024 rows
def test_norm_forward_backward(cuda, rms, C, rows):
    from llmgpu import ops
    g = torch.Generator().manual_seed(C + rms + rows)
    x = (torch.randn(rows, C, generator=g) * 2 + 0.5).to(cuda)
    gamma = (1 + 0.1 * torch.randn(C, generator=g)).to(cuda)
    beta = (0.1 * torch.randn(C, generator=g)).to(cuda)
    y, mean, rstd = ops.norm_fwd(x, gamma, beta, rms)
    xd = x.double().requires_grad_(True)
    if rms:
        ref = xd / torch.sqrt((xd * xd).mean(-1, keepdim=True) + 1e-5) * gamma.double()
    else:
        mu = xd.mean(-1, keepdim=True)
        var = ((xd - mu) ** 2).mean(-1, keepdim=True)
        ref = (xd - mu) / torch.sqrt(var + 1e-5) * gamma.double() + beta.double()
    assert _rel(y.float(), ref.detach()) < 5e-3
    dy = torch.randn(rows, C, generator=g).to(cuda)
    resid = torch.randn(rows, C, generator=g).to(cuda)
    dx, dx16, dg, db, ds = ops.norm_bwd(dy, x, gamma, mean, rstd, resid, rms)
    ref.backward(dy.double())
    want_dx = xd.grad + resid.double()
    assert _rel(dx, want_dx) < 1e-5
    assert _rel(dx16.float(), want_dx) < 5e-3
    xh = (ref.detach() - (0 if rms else beta.double())) / gamma.double()
    assert _rel(dg, (dy.double() * xh).sum(0)) < 1e-5
    if not rms:
        assert _rel(db, dy.double().sum(0)) < 1e-5
    assert _rel(ds, want_dx.sum(0)) < 1e-5


@pytest.mark.parametrize("C,rows,form", [
    (64, 77, "none"), (512, 1001, "inplace"), (768, 8192, "inplace"), (768, 8192, "none"),
    (1024, 2049, "none"), (2048, 300, "inplace"), (1536, 600, "plain")])
def test_norm_backward_forms(cuda, C, rows, form):
    """The backward without an incoming residual gradient (the final norm), with dx written
    over the residual gradient it reads (the Mamba block), ragged last 8-row groups, and
    widths on both kernels (up to 1024 columns the shared-memory ring, above it the
    per-warp kernel)."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(C * 7 + rows)
    x = (torch.randn(rows, C, generator=g) * 1.5 - 0.25).to(cuda)
    gamma = (1 + 0.1 * torch.randn(C, generator=g)).to(cuda)
    beta = (0.1 * torch.randn(C, generator=g)).to(cuda)
    _, mean, rstd = ops.norm_fwd(x, gamma, beta, False)
    dy = torch.randn(rows, C, generator=g).to(cuda)
    resid = None if form == "none" else torch.randn(rows, C, generator=g).to(cuda)
    resid0 = None if resid is None else resid.clone()
    out = resid if form == "inplace" else None
    dx, _, dg, db, ds = ops.norm_bwd(dy, x, gamma, mean, rstd, resid, False, out=out)
    xd = x.double().requires_grad_(True)
    mu = xd.mean(-1, keepdim=True)
    xh = (xd - mu) / torch.sqrt(((xd - mu) ** 2).mean(-1, keepdim=True) + 1e-5)
    (xh * gamma.double() + beta.double()).backward(dy.double())
    want_dx = xd.grad + (0 if resid0 is None else resid0.double())
    if form == "inplace":
        assert dx.data_ptr() == resid.data_ptr()
    assert _rel(dx, want_dx) < 1e-5
    assert _rel(dg, (dy.double() * xh.detach()).sum(0)) < 1e-5
    assert _rel(db, dy.double().sum(0)) < 1e-5
    assert _rel(ds, want_dx.sum(0)) < 1e-5


# rows above the grid run several rows per CTA; a row wider than 110 KB (60032 bf16) runs
# one CTA per SM instead of two; label smoothing per src/loss.cpp:26-40
@pytest.mark.parametrize("V,Vp,rows,smoothing", [
    (256, 256, 64, 0.0), (50257, 50304, 64, 0.0), (300, 384, 64, 0.0),
    (50257, 50304, 700, 0.0), (60001, 60032, 400, 0.0), (256, 256, 300, 0.1),
    (50257, 50304, 333, 0.05), (300, 384, 64, 0.2)])
def test_cross_entropy(cuda, V, Vp, rows, smoothing):
    """loss = lse - logit[tgt]; dlogits = (softmax - y) * scale with y = 1 - smoothing at the
    target and smoothing / (V - 1) elsewhere, zero in padding (src/loss.cpp:6-40); targets
    are the tokens mod V."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(V + rows)
    logits = torch.zeros(rows, Vp)
    logits[:, :V] = torch.randn(rows, V, generator=g) * 2
    l16 = logits.to(torch.bfloat16)
    tok = torch.randint(-V, 2 * V, (rows,), generator=g, dtype=torch.int32)
    scale = 1.0 / rows
    d = l16.clone().to(cuda)
    loss = ops.cross_entropy(d, V, tok.to(cuda), scale, smoothing)
    lf = l16.float()[:, :V].double()
    tgt = tok.long() % V
    lse = torch.logsumexp(lf, -1)
    want_loss = lse - lf[torch.arange(rows), tgt]
    assert torch.allclose(loss.cpu().double(), want_loss, rtol=1e-4, atol=1e-4)
    p = torch.softmax(lf, -1)
    y = torch.full_like(p, smoothing / (V - 1) if smoothing > 0 else 0.0)
    y[torch.arange(rows), tgt] = 1.0 - smoothing
    want = (p - y) * scale
    got = d.cpu().float()
    assert _rel(got[:, :V], want) < 1e-2
    assert torch.count_nonzero(got[:, V:]) == 0


def _attn_ref(qkv, B, T, H, hd):
    C = H * hd
    q, k, v = qkv.double().reshape(B, T, 3, H, hd).permute(2, 0, 3, 1, 4)
    s = q @ k.transpose(-1, -2) / np.sqrt(np.float32(hd))
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=s.device), 1)
    s = s.masked_fill(mask, float("-inf"))
    a = torch.softmax(s, -1)
    o = a @ v
    return o.permute(0, 2, 1, 3).reshape(B * T, C), torch.logsumexp(s, -1)


@pytest.mark.parametrize("B,T,H,hd", [(2, 128, 4, 32), (1, 200, 2, 64), (2, 64, 12, 64),
                                      (1, 1024, 2, 64), (3, 33, 1, 32), (3, 300, 3, 64),
                                      (2, 1024, 12, 64), (2, 256, 3, 16), (1, 132, 2, 48)])
def test_attention_forward_backward(cuda, B, T, H, hd):
    from llmgpu import ops
    g = torch.Generator().manual_seed(T * H + hd)
    C = H * hd
    qkv = (torch.randn(B * T, 3 * C, generator=g)).to(torch.bfloat16).to(cuda)
    out, lse = ops.attention_fwd(qkv, B, T, H, hd)
    q = qkv.float().double().requires_grad_(True)
    ref, ref_lse = _attn_ref(q, B, T, H, hd)
    assert _rel(out.float(), ref.detach()) < 1e-2
    assert torch.allclose(lse.double(), ref_lse.detach(), atol=2e-3, rtol=1e-3)
    dout = torch.randn(B * T, C, generator=g).to(torch.bfloat16).to(cuda)
    dqkv = ops.attention_bwd(qkv, out, dout, lse, B, T, H, hd)
    ref.backward(dout.double())
    want = q.grad
    for part in range(3):
        sl = slice(part * C, (part + 1) * C)
        assert _rel(dqkv[:, sl].float(), want[:, sl]) < 2e-2, part


@pytest.mark.parametrize("B,T,H,hd", [(2, 128, 4, 32), (3, 33, 1, 32)])
def test_attention_padded_heads_match_mma_kernel(cuda, B, T, H, hd):
    """head_dim 32 on the tcgen05 kernel (heads zero-padded to 64) against the mma.sync
    kernel on the same inputs: the padded dims add nothing to scores or outputs."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(11 + T)
    qkv = torch.randn(B * T, 3 * H * hd, generator=g).to(torch.bfloat16).to(cuda)
    out_tc, lse_tc = ops.attention_fwd(qkv, B, T, H, hd)
    out_mma, lse_mma = ops.attention_fwd(qkv, B, T, H, hd, workspace=False)
    assert _rel(out_tc.float(), out_mma.float()) < 1e-2
    assert torch.allclose(lse_tc, lse_mma, atol=2e-3, rtol=1e-3)


def _rope_ref(x, B, T, H, hd, theta=10000.0):
    """Rotate pairs (2j, 2j+1) of each head by pos * theta^(-2j/hd); x: [B*T, H*hd]."""
    j = torch.arange(hd // 2, dtype=torch.float64, device=x.device)
    ang = torch.arange(T, dtype=torch.float64, device=x.device)[:, None] * theta ** (-2.0 * j / hd)
    c, s = ang.cos()[None, :, None, :], ang.sin()[None, :, None, :]
    v = x.reshape(B, T, H, hd // 2, 2)
    x0, x1 = v[..., 0], v[..., 1]
    return torch.stack([x0 * c - x1 * s, x0 * s + x1 * c], -1).reshape(B * T, H * hd)


@pytest.mark.parametrize("B,T,H,hd", [(2, 128, 4, 64), (1, 200, 2, 64), (2, 96, 2, 32)])
def test_attention_rope(cuda, B, T, H, hd):
    """RoPE applied per head to Q and K inside the attention kernels (config 3)."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(T + H)
    C = H * hd
    qkv = torch.randn(B * T, 3 * C, generator=g).to(torch.bfloat16).to(cuda)
    tab = ops.rope_table(T, hd, 10000.0, cuda)
    out, lse = ops.attention_fwd(qkv, B, T, H, hd, rope=tab)
    q = qkv.double().requires_grad_(True)
    rot = torch.cat([_rope_ref(q[:, :C], B, T, H, hd), _rope_ref(q[:, C:2 * C], B, T, H, hd),
                     q[:, 2 * C:]], 1)
    ref, _ = _attn_ref(rot, B, T, H, hd)
    assert _rel(out.float(), ref.detach()) < 1e-2
    dout = torch.randn(B * T, C, generator=g).to(torch.bfloat16).to(cuda)
    dqkv = ops.attention_bwd(qkv, out, dout, lse, B, T, H, hd, rope=tab)
    ref.backward(dout.double())
    for part in range(3):
        sl = slice(part * C, (part + 1) * C)
        assert _rel(dqkv[:, sl].float(), q.grad[:, sl]) < 2e-2, part


def test_swiglu_forward_backward(cuda):
    """gated = silu(h1) * h3 and its backward (src/transformer.cpp:22-30, 76-89)."""
    from llmgpu import ops
    g = torch.Generator().manual_seed(2)
    rows, F = 257, 704
    h13 = (torch.randn(rows, 2 * F, generator=g) * 2).to(torch.bfloat16).to(cuda)
    gated = ops.swiglu_fwd(h13, F)
    h = h13.double().requires_grad_(True)
    ref = torch.nn.functional.silu(h[:, :F]) * h[:, F:]
    assert _rel(gated.float(), ref.detach()) < 5e-3
    dg = torch.randn(rows, F, generator=g).to(torch.bfloat16).to(cuda)
    d = ops.swiglu_bwd(dg, h13, F)
    ref.backward(dg.double())
    assert _rel(d.float(), h.grad) < 5e-3
