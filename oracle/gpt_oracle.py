"""ORACLE — test infrastructure only. Never imported by the product path.

CPU restatement (numpy) of the reference's training step, `Trainer::train_step_accum`
(src/trainer.cpp:127-169): GPT forward (src/model.cpp:144-171), softmax cross-entropy
(src/loss.cpp:6-40), the manual backward (src/model.cpp:175-323 and the blocks), global-norm
clipping (src/optimizer.cpp:90-101) and AdamW (src/optimizer.cpp:53-89).

Pinned against the reference itself: tests/golden/ holds outputs of the unmodified reference
(oracle/_ref/ref_step, built by oracle/Makefile from the reference sources) and the
reference's own known-answer tests; tests/test_oracle_golden.py checks this restatement
against them.

Two configurations have no reference GPT path and are restatements built from reference
pieces (parity unpinned beyond those pieces):
  * ffn="swiglu" + rope_qk: the SILU FeedForward (src/transformer.cpp:22-30,41-119) with
    RoPE applied per head to Q and K using the pairing/frequencies of rope_cfg
    (src/model.cpp:81-104) with dim = head_dim;
  * moe: MoEFFN forward (src/moe.cpp:23-62) and aux loss (src/moe.cpp:64-75) in place of the
    FFN, with this restatement's own backward.

All arithmetic is float64 unless dtype=np.float32 is requested.
"""
from __future__ import annotations

import dataclasses
import struct
from typing import List

import numpy as np

GELU_K = float(np.sqrt(np.float32(2.0) / np.float32(3.14159265)))  # src/transformer.cpp:34
LN_EPS = 1e-5                                                          # include/llm/tensor.h:68


@dataclasses.dataclass
class Cfg:
    vocab: int
    n_layers: int
    n_heads: int
    n_embd: int
    block_size: int
    tied: bool = True
    rmsnorm: bool = False
    # Mamba (src/mamba.cpp); use_mamba => checkpoint v4
    mamba: bool = False
    d_inner: int = 0
    d_state: int = 16
    dt_rank: int = 0
    conv_kernel: int = 4
    # extensions (no reference GPT path)
    ffn: str = "gelu"          # "gelu" | "swiglu"
    ffn_hidden: int = 0        # 0 -> 4*n_embd
    rope_qk: bool = False
    rope_theta: float = 10000.0
    moe_experts: int = 0       # >0 replaces the FFN by MoEFFN
    moe_top_k: int = 2
    moe_aux_coef: float = 0.01
    # Config::pos_encoding (include/llm/model.h:15-33): "learned", "sinusoidal" (wpe init
    # only) or "rope" (rope_cfg on the embedding sum, with the options below; rope_theta
    # above is Config::rope_theta)
    pos_encoding: str = "learned"
    rope_scaling: float = 1.0
    rope_mode: int = 0
    yarn_alpha: float = 1.0
    yarn_beta: float = 32.0

    @property
    def hidden(self):
        return self.ffn_hidden or 4 * self.n_embd

    @property
    def di(self):
        return self.d_inner or 2 * self.n_embd

    @property
    def dr(self):
        return self.dt_rank or (self.n_embd + 15) // 16


# ----------------------------------------------------------------------------- parameters
def param_specs(cfg: Cfg):
    """(name, shape) in GPT::parameters() order (src/model.cpp:889-909)."""
    C, V = cfg.n_embd, cfg.vocab
    specs = [("wte", (V, C)), ("wpe", (cfg.block_size, C)), ("ln_f_gamma", (C,)),
             ("ln_f_beta", (C,))]
    if not cfg.tied:
        specs.append(("lm_head", (C, V)))
    for l in range(cfg.n_layers):
        p = f"blk{l}."
        if cfg.mamba:  # src/mamba.cpp:415-420
            D, N, R, K = cfg.di, cfg.d_state, cfg.dr, cfg.conv_kernel
            specs += [(p + "norm_w", (C,)), (p + "in_proj", (2 * D, C)),
                      (p + "conv_w", (D, 1, K)), (p + "conv_b", (D,)),
                      (p + "x_proj", (R + 2 * N, D)), (p + "dt_proj", (D, R)),
                      (p + "a_log", (D, N)), (p + "d", (D,)), (p + "out_proj", (C, D))]
            continue
        specs += [(p + "Wq", (C, C)), (p + "Wk", (C, C)), (p + "Wv", (C, C)), (p + "Wo", (C, C))]
        if cfg.moe_experts:
            E, H = cfg.moe_experts, 4 * C
            specs += [(p + "gate", (C, E)), (p + "W1e", (E, C, H)), (p + "W2e", (E, H, C))]
        elif cfg.ffn == "swiglu":  # FeedForward::parameters SILU order (src/transformer.cpp:272)
            H = cfg.hidden
            specs += [(p + "W1", (C, H)), (p + "W2", (H, C)), (p + "W3", (C, H)),
                      (p + "b1", (H,)), (p + "b2", (C,))]
        else:
            H = cfg.hidden
            specs += [(p + "W1", (C, H)), (p + "W2", (H, C)), (p + "b1", (H,)), (p + "b2", (C,))]
        specs += [(p + "ln1_gamma", (C,)), (p + "ln1_beta", (C,)), (p + "ln2_gamma", (C,)),
                  (p + "ln2_beta", (C,))]
    return specs


def init_params(cfg: Cfg, seed: int) -> List[np.ndarray]:
    """Seeded synthetic weights: N(0, 0.02^2) for matrices, zero biases, unit gains.

    Mamba: a_log[d, n] = -(n + 1) (negative A in the reference's exp(a_log * dt) convention,
    src/mamba.cpp:223), d = 1, conv bias 0, in/x/out projections N(0, 0.02^2),
    dt_proj N(0, 0.02^2)."""
    rng = np.random.default_rng(seed)
    out = []
    for name, shape in param_specs(cfg):
        base = name.split(".")[-1]
        if base in ("ln_f_gamma", "ln1_gamma", "ln2_gamma", "norm_w", "d"):
            a = np.ones(shape, np.float32)
        elif base in ("ln_f_beta", "ln1_beta", "ln2_beta", "b1", "b2", "conv_b"):
            a = np.zeros(shape, np.float32)
        elif base == "a_log":
            a = -np.tile(np.arange(1, shape[1] + 1, dtype=np.float32), (shape[0], 1))
        else:
            a = (rng.standard_normal(shape) * 0.02).astype(np.float32)
        out.append(a)
    if cfg.pos_encoding == "sinusoidal":
        out[1] = sinusoidal_wpe(cfg.block_size, cfg.n_embd)
    return out


def decay_flags(cfg: Cfg):
    """AdamW::default_decay: ndim > 1 (include/llm/optimizer.h:70-72)."""
    return [len(s) > 1 for _, s in param_specs(cfg)]


# ----------------------------------------------------------------------------- checkpoint
def write_ckpt(path: str, cfg: Cfg, params: List[np.ndarray]):
    """Binary checkpoint v3 (transformer) / v4 (mamba), src/model.cpp:568-635.

    The file always carries lm_head; when tied it holds wte^T (tie_weights)."""
    specs = param_specs(cfg)
    assert len(specs) == len(params)
    by = {n: p for (n, _), p in zip(specs, params)}

    def tensor(a):
        a = np.ascontiguousarray(a, np.float32)
        b = struct.pack("<Q", a.ndim) + b"".join(struct.pack("<Q", d) for d in a.shape)
        return b + struct.pack("<Q", a.size) + a.tobytes()

    with open(path, "wb") as f:
        f.write(struct.pack("<II", 0x4C4C4D00, 4 if cfg.mamba else 3))
        f.write(struct.pack("<5Q", cfg.vocab, cfg.n_layers, cfg.n_heads, cfg.n_embd,
                            cfg.block_size))
        lm = by["wte"].T if cfg.tied else by["lm_head"]
        for t in (by["wte"], by["wpe"], by["ln_f_gamma"], by["ln_f_beta"], lm):
            f.write(tensor(t))
        names = [n for n, _ in specs]
        if cfg.mamba:
            f.write(struct.pack("<4Q", cfg.di, cfg.d_state, cfg.dr, cfg.conv_kernel))
        f.write(struct.pack("<Q", cfg.n_layers))
        for l in range(cfg.n_layers):
            blk = [by[n] for n in names if n.startswith(f"blk{l}.")]
            f.write(struct.pack("<Q", len(blk)))
            for t in blk:
                f.write(tensor(t))


def read_ckpt(path: str, cfg: Cfg) -> List[np.ndarray]:
    """Reads a v3/v4 checkpoint written for `cfg` back into parameters() order."""
    with open(path, "rb") as f:
        buf = f.read()
    off = 0

    def u64():
        nonlocal off
        v = struct.unpack_from("<Q", buf, off)[0]
        off += 8
        return v

    magic, ver = struct.unpack_from("<II", buf, 0)
    off = 8
    assert magic == 0x4C4C4D00
    hdr = [u64() for _ in range(5)]
    assert hdr == [cfg.vocab, cfg.n_layers, cfg.n_heads, cfg.n_embd, cfg.block_size], hdr

    def tensor():
        nonlocal off
        nd = u64()
        shape = tuple(u64() for _ in range(nd))
        n = u64()
        a = np.frombuffer(buf, np.float32, n, off).reshape(shape).copy()
        off += 4 * n
        return a

    top = [tensor() for _ in range(5)]
    if ver >= 4:
        [u64() for _ in range(4)]
    nb = u64()
    blocks = []
    for _ in range(nb):
        npar = u64()
        blocks += [tensor() for _ in range(npar)]
    out = top[:4] + ([] if cfg.tied else [top[4]]) + blocks
    return out


# ----------------------------------------------------------------------------- primitives
def layernorm_fwd(x, g, b, eps=LN_EPS):
    """Tensor::layernorm (src/tensor.cpp:388-413)."""
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    y = (x - mu) / np.sqrt(var + eps) * g
    return y + b if b is not None else y


def layernorm_bwd(x, dy, g, eps=LN_EPS):
    """Tensor::layernorm_backward (src/tensor.cpp:556-602): (dx, dgamma, dbeta)."""
    C = x.shape[-1]
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    inv = 1.0 / np.sqrt(var + eps)
    xh = (x - mu) * inv
    dyg = dy * g
    dx = inv * (dyg - dyg.sum(-1, keepdims=True) / C - xh * (dyg * xh).sum(-1, keepdims=True) / C)
    return dx, (dy * xh).sum(0), dy.sum(0)


def rmsnorm_fwd(x, w, eps=LN_EPS):
    """Tensor::rmsnorm (src/tensor.cpp:604-623)."""
    ms = (x * x).mean(-1, keepdims=True)
    return x / np.sqrt(ms + eps) * w


def rmsnorm_bwd(x, dy, w, eps=LN_EPS):
    """Tensor::rmsnorm_backward (src/tensor.cpp:625-655): (dx, dw)."""
    C = x.shape[-1]
    ms = (x * x).mean(-1, keepdims=True)
    inv = 1.0 / np.sqrt(ms + eps)
    dot = (dy * w * x).sum(-1, keepdims=True)
    dx = dy * w * inv - x * (dot * inv ** 3 / C)
    return dx, (dy * x * inv).sum(0)


def gelu(v):
    """tanh GELU of FeedForward::forward (src/transformer.cpp:31-35)."""
    return 0.5 * v * (1.0 + np.tanh(GELU_K * (v + 0.044715 * v ** 3)))


def gelu_grad(v):
    """src/transformer.cpp:151-158."""
    th = np.tanh(GELU_K * (v + 0.044715 * v ** 3))
    return 0.5 * (1 + th) + 0.5 * v * (1 - th * th) * GELU_K * (1 + 3 * 0.044715 * v * v)


def silu(v):
    return v / (1.0 + np.exp(-v))


def silu_grad(v):
    s = 1.0 / (1.0 + np.exp(-v))
    return s * (1 + v * (1 - s))


def softmax(x):
    m = x.max(-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(-1, keepdims=True)


def ce_loss(logits, tgt):
    """cross_entropy_loss (src/loss.cpp:6-22): mean over rows of -log softmax[target]."""
    m = logits.max(-1, keepdims=True)
    lse = np.log(np.exp(logits - m).sum(-1)) + m[:, 0]
    return float((lse - logits[np.arange(len(tgt)), tgt]).mean())


def ce_backward(logits, tgt, smoothing=0.0):
    """cross_entropy_backward (src/loss.cpp:26-40): (softmax - y) / T."""
    T, V = logits.shape
    d = softmax(logits)
    off = smoothing / (V - 1) if (smoothing > 0 and V > 1) else 0.0
    y = np.full_like(d, off)
    y[np.arange(T), tgt] = 1.0 - smoothing
    return (d - y) / T


def rope_tables(T, hd, theta):
    """Angles pos * theta^(-i/hd) for even i (rope_cfg pairing, src/model.cpp:88-100)."""
    i = np.arange(0, hd, 2, dtype=np.float64)
    freq = theta ** (-i / hd)
    ang = np.arange(T, dtype=np.float64)[:, None] * freq[None, :]
    return np.cos(ang), np.sin(ang)


def rope_cfg_tables(T, C, theta, scaling, mode, alpha, beta):
    """rope_cfg (src/model.cpp:71-104) in its own float32 arithmetic: per position and column
    pair (i, i+1), i even, the (cos, sin) of pos * freq * yarn_alpha with freq = base^(-i/C),
    base = theta * scaling for NTK (mode 0); for YaRN (mode 1, scaling > 1) freq =
    ((1 - m)/scaling + m) * theta^(-i/C) with the ramp m of yarn_ramp and the output scale
    sqrt(1 + 0.1 ln scaling). Returns cos, sin [T, C//2] and the scale."""
    f = np.float32
    sc = f(1.0) if f(scaling) < f(1.0) else f(scaling)
    base = f(theta) * (sc if mode == 0 else f(1.0))
    yarn = mode == 1 and sc > f(1.0)
    scale = f(np.sqrt(f(1.0) + f(0.1) * f(np.log(sc)))) if yarn else f(1.0)
    i = np.arange(0, C - 1, 2).astype(f)
    expo = (-i / f(C)).astype(f)
    freq = np.power(base, expo).astype(f)
    if yarn:
        d = (i / f(C) * f(beta)).astype(f)
        low, high = f(beta) / f(2.0), f(beta)
        m = np.where(d < low, f(0.0), np.where(d > high, f(1.0), (d - low) / (high - low))).astype(f)
        freq = (((f(1.0) - m) / sc + m) * np.power(f(theta), expo)).astype(f)
    ang = (np.arange(T, dtype=f)[:, None] * freq[None, :] * f(alpha)).astype(f)
    return np.cos(ang), np.sin(ang), scale


def rope_cfg_apply(x, cos, sin, scale):
    """Rotates column pairs (2j, 2j+1) of x [T, C] and scales, as rope_cfg writes `out`."""
    out = x.copy()
    n = cos.shape[1]
    x0, x1 = x[:, 0:2 * n:2], x[:, 1:2 * n:2]
    out[:, 0:2 * n:2] = (x0 * cos - x1 * sin) * scale
    out[:, 1:2 * n:2] = (x0 * sin + x1 * cos) * scale
    return out


def sinusoidal_wpe(block_size, C):
    """GPT::GPT's sinusoidal wpe fill (src/model.cpp:34-41), float32."""
    f = np.float32
    pos = np.arange(block_size, dtype=f)[:, None]
    i = np.arange(C)
    angle = (pos / np.power(f(10000.0), ((2 * (i // 2)).astype(f) / f(C)).astype(f))).astype(f)
    return np.where(i % 2 == 0, np.sin(angle), np.cos(angle)).astype(f)


def rope_apply(x, cos, sin, inverse=False):
    """Rotate pairs (2j, 2j+1) of every head slice; x: [T, H, hd]."""
    x0, x1 = x[..., 0::2], x[..., 1::2]
    s = -sin if inverse else sin
    out = np.empty_like(x)
    out[..., 0::2] = x0 * cos[:, None, :] - x1 * s[:, None, :]
    out[..., 1::2] = x0 * s[:, None, :] + x1 * cos[:, None, :]
    return out


# ----------------------------------------------------------------------------- model
class Model:
    def __init__(self, cfg: Cfg, params: List[np.ndarray], dtype=np.float64):
        self.cfg = cfg
        self.dtype = dtype
        self.names = [n for n, _ in param_specs(cfg)]
        self.p = {n: np.asarray(a, dtype) for n, a in zip(self.names, params)}
        # MoE: optional routing given from outside, forced_routes[sequence][layer] = int
        # [T, k] expert indices, consumed one sequence per forward_backward call. Lets a
        # test evaluate the restatement under exactly the routing another implementation
        # chose (routing is a discrete decision that rounding upstream can flip near ties).
        self.forced_routes = None
        # TrainConfig::label_smoothing, applied by cross_entropy_backward (src/loss.cpp:26-40)
        self.smoothing = 0.0
        self._seq = 0
        self._layer = 0
        self._routes = None

    # ------------------------------------------------------------------ norms
    def _norm(self, x, g, b):
        return rmsnorm_fwd(x, g) if self.cfg.rmsnorm else layernorm_fwd(x, g, b)

    def _norm_bwd(self, x, dy, g):
        if self.cfg.rmsnorm:
            dx, dg = rmsnorm_bwd(x, dy, g)
            return dx, dg, np.zeros_like(dg)
        return layernorm_bwd(x, dy, g)

    # ------------------------------------------------------------------ attention
    def _attn_fwd(self, h, P):
        cfg = self.cfg
        T, C = h.shape
        H = cfg.n_heads
        hd = C // H
        q = (h @ P["Wq"]).reshape(T, H, hd)
        k = (h @ P["Wk"]).reshape(T, H, hd)
        v = (h @ P["Wv"]).reshape(T, H, hd)
        if cfg.rope_qk:
            cos, sin = rope_tables(T, hd, cfg.rope_theta)
            q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
        scale = 1.0 / np.sqrt(np.float32(hd))
        s = np.einsum("thd,shd->hts", q, k) * scale
        mask = np.triu(np.ones((T, T), bool), 1)
        s[:, mask] = -1e9                      # src/attention.cpp:79-82
        a = softmax(s)
        o = np.einsum("hts,shd->thd", a, v).reshape(T, C)
        cache = dict(q=q, k=k, v=v, a=a, o=o, mask=mask, scale=scale)
        return o @ P["Wo"], cache

    def _attn_bwd(self, h, dy, P, c, G):
        """MultiHeadAttention::backward (src/attention.cpp:183-363)."""
        cfg = self.cfg
        T, C = h.shape
        H = cfg.n_heads
        hd = C // H
        G["Wo"] += c["o"].T @ dy
        do = (dy @ P["Wo"].T).reshape(T, H, hd)
        a = c["a"]
        dv = np.einsum("hts,thd->shd", a, do)
        da = np.einsum("thd,shd->hts", do, c["v"])
        ds = a * (da - (da * a).sum(-1, keepdims=True)) * c["scale"]
        ds[:, c["mask"]] = 0.0
        dq = np.einsum("hts,shd->thd", ds, c["k"])
        dk = np.einsum("hts,thd->shd", ds, c["q"])
        if cfg.rope_qk:
            cos, sin = rope_tables(T, hd, cfg.rope_theta)
            dq, dk = rope_apply(dq, cos, sin, True), rope_apply(dk, cos, sin, True)
        dq, dk, dv = dq.reshape(T, C), dk.reshape(T, C), dv.reshape(T, C)
        G["Wq"] += h.T @ dq
        G["Wk"] += h.T @ dk
        G["Wv"] += h.T @ dv
        return dq @ P["Wq"].T + dk @ P["Wk"].T + dv @ P["Wv"].T

    # ------------------------------------------------------------------ FFN / MoE
    def _ffn_fwd(self, h, P):
        cfg = self.cfg
        if cfg.moe_experts:
            return self._moe_fwd(h, P)
        if cfg.ffn == "swiglu":
            h1, h3 = h @ P["W1"], h @ P["W3"]
            gated = silu(h1) * h3
            return gated @ P["W2"], dict(h1=h1, h3=h3, gated=gated)
        pre = h @ P["W1"]
        g = gelu(pre)
        return g @ P["W2"], dict(pre=pre, g=g)

    def _ffn_bwd(self, h, dy, P, c, G):
        cfg = self.cfg
        if cfg.moe_experts:
            return self._moe_bwd(h, dy, P, c, G)
        G["b2"] += dy.sum(0)
        if cfg.ffn == "swiglu":  # src/transformer.cpp:41-119
            G["W2"] += c["gated"].T @ dy
            dgated = dy @ P["W2"].T
            dh3 = dgated * silu(c["h1"])
            dh1 = dgated * c["h3"] * silu_grad(c["h1"])
            G["W1"] += h.T @ dh1
            G["W3"] += h.T @ dh3
            G["b1"] += dh1.sum(0)
            return dh1 @ P["W1"].T + dh3 @ P["W3"].T
        G["W2"] += c["g"].T @ dy           # src/transformer.cpp:120-183
        dh = (dy @ P["W2"].T) * gelu_grad(c["pre"])
        G["W1"] += h.T @ dh
        G["b1"] += dh.sum(0)
        return dh @ P["W1"].T

    def _route(self, h, gate):
        """Router of MoEFFN::forward (src/moe.cpp:225-242): softmax, top-k by descending
        probability (ties: lower expert index first), renormalised weights."""
        cfg = self.cfg
        probs = softmax(h @ gate)
        k = cfg.moe_top_k
        if self._routes is not None:
            idx = np.asarray(self._routes[self._layer], np.int64)
        else:
            # stable sort on -p keeps the lower index first among equal probabilities
            idx = np.argsort(-probs, axis=1, kind="stable")[:, :k]
        top = np.take_along_axis(probs, idx, 1)
        s = top.sum(1, keepdims=True)
        s = np.where(s < 1e-8, 1.0, s)
        return probs, idx, top / s, s

    def _moe_fwd(self, h, P):
        cfg = self.cfg
        T, C = h.shape
        probs, idx, w, s = self._route(h, P["gate"])
        out = np.zeros_like(h)
        ys = np.zeros((T, cfg.moe_top_k, C), h.dtype)
        pres = []
        for j in range(cfg.moe_top_k):
            e = idx[:, j]
            pre = np.einsum("tc,tch->th", h, P["W1e"][e])
            y = np.einsum("th,thc->tc", gelu(pre), P["W2e"][e])
            ys[:, j] = y
            pres.append(pre)
            out += w[:, j:j + 1] * y
        E = cfg.moe_experts
        load = probs.mean(0)
        mean = 1.0 / E
        aux = cfg.moe_aux_coef * ((load - mean) ** 2).sum() / (mean * mean * E)
        return out, dict(probs=probs, idx=idx, w=w, s=s, ys=ys, pres=pres, aux=aux)

    def _moe_bwd(self, h, dy, P, c, G):
        cfg = self.cfg
        T, C = h.shape
        E, k = cfg.moe_experts, cfg.moe_top_k
        probs, idx, w, s = c["probs"], c["idx"], c["w"], c["s"]
        dh = np.zeros_like(h)
        dw = np.einsum("tc,tjc->tj", dy, c["ys"])
        for j in range(k):
            e = idx[:, j]
            pre = c["pres"][j]
            dyj = w[:, j:j + 1] * dy
            g = gelu(pre)
            np.add.at(G["W2e"], e, np.einsum("th,tc->thc", g, dyj))
            dpre = np.einsum("tc,thc->th", dyj, P["W2e"][e]) * gelu_grad(pre)
            np.add.at(G["W1e"], e, np.einsum("tc,th->tch", h, dpre))
            dh += np.einsum("th,tch->tc", dpre, P["W1e"][e])
        # renormalisation w_j = p_j / S over the selected experts
        top = np.take_along_axis(probs, idx, 1)
        dtop = dw / s - (dw * top).sum(1, keepdims=True) / (s * s)
        dprobs = np.zeros_like(probs)
        np.put_along_axis(dprobs, idx, dtop, 1)
        # aux loss: coef * sum_e (load_e - 1/E)^2 / ((1/E)^2 E), load = mean_t probs
        mean = 1.0 / E
        load = probs.mean(0)
        dprobs += cfg.moe_aux_coef * 2.0 * (load - mean) / (mean * mean * E) / T
        dscores = probs * (dprobs - (dprobs * probs).sum(1, keepdims=True))
        G["gate"] += h.T @ dscores
        dh += dscores @ P["gate"].T
        return dh

    # ------------------------------------------------------------------ mamba
    def _mamba_fwd(self, x, P):
        """MambaBlock::forward (src/mamba.cpp:60-166), keeping the backward's intermediates."""
        cfg = self.cfg
        T = x.shape[0]
        D, N, R, K = cfg.di, cfg.d_state, cfg.dr, cfg.conv_kernel
        normed = rmsnorm_fwd(x, P["norm_w"]) if cfg.rmsnorm else layernorm_fwd(x, P["norm_w"], None)
        proj = normed @ P["in_proj"].T
        xz, xs = proj[:, :D], proj[:, D:]
        w = P["conv_w"].reshape(D, K)
        pre = np.tile(P["conv_b"], (T, 1))
        for j in range(K):
            sh = K - 1 - j
            pre[sh:] += xs[:T - sh] * w[:, j]
        u = silu(pre)
        xp = u @ P["x_proj"].T
        raw = xp[:, :R] @ P["dt_proj"].T
        sp = np.log1p(np.exp(raw))
        dt = np.clip(sp, 0.001, 0.1)
        Bm, Cm = xp[:, R:R + N], xp[:, R + N:]
        A = P["a_log"]
        hs = np.zeros((T, D, N), x.dtype)
        h = np.zeros((D, N), x.dtype)
        for t in range(T):
            a = np.exp(A * dt[t][:, None])
            h = a * h + Bm[t][None, :] * (u[t] * dt[t])[:, None]
            hs[t] = h
        y = np.einsum("tdn,tn->td", hs, Cm) + P["d"] * u
        gate = silu(xz)
        gated = gate * y
        out = x + gated @ P["out_proj"].T
        cache = dict(normed=normed, xz=xz, xs=xs, pre=pre, u=u, xp=xp, raw=raw, sp=sp, dt=dt,
                     Bm=Bm, Cm=Cm, hs=hs, y=y, gate=gate, gated=gated)
        return out, cache

    def _mamba_bwd(self, x, dout, P, c, G):
        """MambaBlock::backward (src/mamba.cpp:179-413)."""
        cfg = self.cfg
        T = x.shape[0]
        D, N, R, K = cfg.di, cfg.d_state, cfg.dr, cfg.conv_kernel
        A = P["a_log"]
        dgated = dout @ P["out_proj"]
        G["out_proj"] += dout.T @ c["gated"]
        dgate = dgated * c["y"]
        dY = dgated * c["gate"]
        dxz = dgate * silu_grad(c["xz"])
        u, dt, Bm, Cm, hs = c["u"], c["dt"], c["Bm"], c["Cm"], c["hs"]
        G["d"] += (dY * u).sum(0)
        du = dY * P["d"]
        dB = np.zeros((T, N), x.dtype)
        dC = np.einsum("td,tdn->tn", dY, hs)
        ddt = np.zeros((T, D), x.dtype)
        dA = np.zeros((D, N), x.dtype)
        dh_next = np.zeros((D, N), x.dtype)
        for t in range(T - 1, -1, -1):
            a = np.exp(A * dt[t][:, None])
            h_prev = hs[t - 1] if t > 0 else np.zeros((D, N), x.dtype)
            dh = dh_next + dY[t][:, None] * Cm[t][None, :]
            dB[t] = (dh * (u[t] * dt[t])[:, None]).sum(0)
            du[t] += (dh * Bm[t][None, :]).sum(1) * dt[t]
            dA += dh * h_prev * a * dt[t][:, None]
            ddt[t] = (dh * h_prev * a * A).sum(1) + (dh * Bm[t][None, :]).sum(1) * u[t]
            dh_next = dh * a
        G["a_log"] += dA
        dxp = np.zeros_like(c["xp"])
        dxp[:, R:R + N] += dB
        dxp[:, R + N:] += dC
        inr = ((c["sp"] >= 0.001) & (c["sp"] <= 0.1)).astype(x.dtype)
        draw = ddt * inr / (1.0 + np.exp(-c["raw"]))
        dxp[:, :R] += draw @ P["dt_proj"]
        G["dt_proj"] += draw.T @ c["xp"][:, :R]
        du_total = du + dxp @ P["x_proj"]
        G["x_proj"] += dxp.T @ u
        dpre = du_total * silu_grad(c["pre"])
        w = P["conv_w"].reshape(D, K)
        G["conv_b"] += dpre.sum(0)
        dxs = np.zeros((T, D), x.dtype)
        dw = np.zeros((D, K), x.dtype)
        for j in range(K):
            sh = K - 1 - j
            dxs[:T - sh] += dpre[sh:] * w[:, j]
            dw[:, j] += (dpre[sh:] * c["xs"][:T - sh]).sum(0)
        G["conv_w"] += dw.reshape(D, 1, K)
        dproj = np.concatenate([dxz, dxs], 1)
        dn = dproj @ P["in_proj"]
        G["in_proj"] += dproj.T @ c["normed"]
        if cfg.rmsnorm:
            dx, dg = rmsnorm_bwd(x, dn, P["norm_w"])
        else:
            dx, dg, _ = layernorm_bwd(x, dn, P["norm_w"])
        G["norm_w"] += dg
        return dx + dout

    # ------------------------------------------------------------------ whole model
    def _blk(self, l):
        pre = f"blk{l}."
        return {n[len(pre):]: v for n, v in self.p.items() if n.startswith(pre)}

    def _embed(self, tok):
        """wte[tok] + wpe[t] (src/model.cpp:149-157), rotated by rope_cfg under RoPE (:158).
        The backward scatters the gradient of the rotated sum into wte/wpe as it is
        (src/model.cpp:314-322): the reference does not rotate it back."""
        cfg, p = self.cfg, self.p
        x = p["wte"][tok] + p["wpe"][:len(tok)]
        if cfg.pos_encoding == "rope":
            cos, sin, sc = rope_cfg_tables(len(tok), cfg.n_embd, cfg.rope_theta, cfg.rope_scaling,
                                           cfg.rope_mode, cfg.yarn_alpha, cfg.yarn_beta)
            x = rope_cfg_apply(x, cos.astype(x.dtype), sin.astype(x.dtype), x.dtype.type(sc))
        return x

    def logits(self, tokens):
        """GPT::forward (src/model.cpp:140-171): logits [T, V] of one sequence."""
        cfg = self.cfg
        tok = np.asarray(tokens, np.int64) % cfg.vocab
        p = self.p
        x = self._embed(tok)
        self._routes = None
        for l in range(cfg.n_layers):
            P = self._blk(l)
            self._layer = l
            if cfg.mamba:
                x, _ = self._mamba_fwd(x, P)
                continue
            h1 = self._norm(x, P["ln1_gamma"], P["ln1_beta"])
            att, _ = self._attn_fwd(h1, P)
            y = x + att
            f, _ = self._ffn_fwd(self._norm(y, P["ln2_gamma"], P["ln2_beta"]), P)
            x = y + f
        hid = self._norm(x, p["ln_f_gamma"], p["ln_f_beta"])
        return hid @ (p["wte"].T if cfg.tied else p["lm_head"])

    def forward_backward(self, tokens):
        """One sequence: loss and gradients (dict name -> array), src/model.cpp:144-323."""
        cfg = self.cfg
        T = len(tokens)
        V, C = cfg.vocab, cfg.n_embd
        tok = np.asarray(tokens, np.int64) % V
        p = self.p
        x = self._embed(tok)
        G = {n: np.zeros_like(a) for n, a in p.items()}
        xs, caches = [], []
        aux_total = 0.0
        self._routes = None
        if self.forced_routes is not None:
            self._routes = self.forced_routes[self._seq]
            self._seq += 1
        for l in range(cfg.n_layers):
            P = self._blk(l)
            xs.append(x)
            self._layer = l
            if cfg.mamba:
                x, c = self._mamba_fwd(x, P)
                caches.append(c)
                continue
            h1 = self._norm(x, P["ln1_gamma"], P["ln1_beta"])
            att, ca = self._attn_fwd(h1, P)
            y = x + att
            h2 = self._norm(y, P["ln2_gamma"], P["ln2_beta"])
            f, cf = self._ffn_fwd(h2, P)
            if cfg.moe_experts:
                aux_total += cf["aux"]
            caches.append(dict(h1=h1, ca=ca, y=y, h2=h2, cf=cf))
            x = y + f
        hid = self._norm(x, p["ln_f_gamma"], p["ln_f_beta"])
        lm = p["wte"].T if cfg.tied else p["lm_head"]
        logits = hid @ lm
        loss = ce_loss(logits, tok) + aux_total
        dlog = ce_backward(logits, tok, self.smoothing)
        dlm = hid.T @ dlog
        if cfg.tied:
            G["wte"] += dlm.T
        else:
            G["lm_head"] += dlm
        dhid = dlog @ lm.T
        dx, dg, db = self._norm_bwd(x, dhid, p["ln_f_gamma"])
        G["ln_f_gamma"] += dg
        G["ln_f_beta"] += db
        for l in range(cfg.n_layers - 1, -1, -1):
            P = self._blk(l)
            Gl = _View(G, f"blk{l}.")
            c = caches[l]
            if cfg.mamba:
                dx = self._mamba_bwd(xs[l], dx, P, c, Gl)
                continue
            dh2 = self._ffn_bwd(c["h2"], dx, P, c["cf"], Gl)
            dyn, dg2, db2 = self._norm_bwd(c["y"], dh2, P["ln2_gamma"])
            Gl["ln2_gamma"] += dg2
            Gl["ln2_beta"] += db2
            dy = dx + dyn
            dh1 = self._attn_bwd(c["h1"], dy, P, c["ca"], Gl)
            dxn, dg1, db1 = self._norm_bwd(xs[l], dh1, P["ln1_gamma"])
            Gl["ln1_gamma"] += dg1
            Gl["ln1_beta"] += db1
            dx = dy + dxn
        np.add.at(G["wte"], tok, dx)
        G["wpe"][:T] += dx
        return loss, G, logits


class _View:
    """Prefix view of the gradient dict, so block code can use local names."""

    def __init__(self, G, prefix):
        self.G, self.prefix = G, prefix

    def __getitem__(self, k):
        return self.G[self.prefix + k]

    def __setitem__(self, k, v):
        self.G[self.prefix + k] = v


# ----------------------------------------------------------------------------- trainer
@dataclasses.dataclass
class AdamWState:
    """Adam/AdamW state (src/optimizer.cpp:53-89)."""
    lr: float = 3e-4
    b1: float = 0.9
    b2: float = 0.95
    eps: float = 1e-8
    wd: float = 0.1
    t: int = 0
    m: list = None
    v: list = None


def clip_by_global_norm(grads, max_norm):
    """src/optimizer.cpp:90-101: scales in place, returns the pre-clip norm."""
    total = float(np.sqrt(sum(float((g.astype(np.float64) ** 2).sum()) for g in grads)))
    if total > max_norm and total > 0:
        s = max_norm / total
        for g in grads:
            g *= s
    return total


def adamw_step(params, grads, st: AdamWState, decay):
    """AdamW::step (src/optimizer.cpp:78-89) -> Adam::step (:54-71)."""
    if st.m is None:
        st.m = [np.zeros_like(g) for g in grads]
        st.v = [np.zeros_like(g) for g in grads]
    for p, d in zip(params, decay):
        if d:
            p -= st.lr * st.wd * p
    st.t += 1
    c1 = 1.0 - st.b1 ** st.t
    c2 = 1.0 - st.b2 ** st.t
    for p, g, m, v in zip(params, grads, st.m, st.v):
        m *= st.b1
        m += (1 - st.b1) * g
        v *= st.b2
        v += (1 - st.b2) * g * g
        p -= st.lr * (m / c1) / (np.sqrt(v / c2) + st.eps)


def train_step(model: Model, batch, st: AdamWState, clip=1.0):
    """Trainer::train_step_accum with K = len(batch) micro-batches (src/trainer.cpp:127-169).

    Returns (per-sequence losses, raw mean grads (pre-clip), grad norm after clipping,
    skipped)."""
    names = model.names
    acc = [np.zeros_like(model.p[n]) for n in names]
    losses = []
    for seq in batch:
        loss, G, _ = model.forward_backward(seq)
        losses.append(loss)
        for a, n in zip(acc, names):
            a += G[n]
    K = len(batch)
    raw = [a / K for a in acc]
    grads = [g.copy() for g in raw]
    if not all(np.isfinite(g).all() for g in grads):
        return losses, raw, 0.0, True
    clip_by_global_norm(grads, clip)
    gnorm = float(np.sqrt(sum(float((g.astype(np.float64) ** 2).sum()) for g in grads)))
    params = [model.p[n] for n in names]
    adamw_step(params, grads, st, decay_flags(model.cfg))
    return losses, raw, gnorm, False


# ----------------------------------------------------------------------------- inputs
def zipf_tokens(vocab, n, seed, s=1.1):
    """Token ids with P(rank k) proportional to k^-s over the whole vocabulary."""
    rng = np.random.default_rng(seed)
    pk = np.arange(1, vocab + 1, dtype=np.float64) ** (-s)
    pk /= pk.sum()
    return rng.choice(vocab, size=n, p=pk).astype(np.int32)


def uniform_tokens(vocab, n, seed):
    return np.random.default_rng(seed).integers(0, vocab, size=n).astype(np.int32)


def selective_scan(x, A, B, C, dt, D_skip, h0):
    """selective_scan_sequential (src/mamba_scan.cpp:11-70) with the layout of
    include/llm/mamba_scan.h:7-20: x, dt [T, D]; A, h0 [D, N]; B, C [T, N]; D_skip [D].
    Returns (y [T, D], h_final [D, N])."""
    T = x.shape[0]
    h = np.array(h0, dtype=np.float64)
    y = np.zeros(x.shape, np.float64)
    for t in range(T):
        a = np.exp(A * dt[t][:, None])
        h = a * h + B[t][None, :] * (x[t] * dt[t])[:, None]
        y[t] = (h * C[t][None, :]).sum(1) + D_skip * x[t]
    return y, h
