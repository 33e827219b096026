"""Pins the numpy oracle (oracle/gpt_oracle.py) before it is trusted:

* against outputs of the unmodified reference training step (tests/golden/*.npz, made by
  tests/golden/make_golden.py from oracle/_ref/ref_step), and
* against the reference's own known-answer tests for this path.
"""
import os

import numpy as np
import pytest

from oracle import golden
from oracle import gpt_oracle as go

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
# training-step fixtures (moe_forward.npz holds a single MoE FFN: tests/test_oracle_moe.py)
CASES = sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz") and not f.startswith("moe_"))


def _load(name):
    return golden.load(os.path.join(GOLDEN, name + ".npz"))


def _split(cfg, flat):
    out, off = [], 0
    for _, s in go.param_specs(cfg):
        n = int(np.prod(s))
        out.append(flat[off:off + n].reshape(s))
        off += n
    assert off == flat.size
    return out


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference(name):
    z, meta, cfg = _load(name)
    B, T, steps = meta["B"], meta["T"], meta["steps"]
    model = go.Model(cfg, _split(cfg, z["init"]))
    hp = meta["hp"]
    st = go.AdamWState(lr=hp["lr"], b1=hp["b1"], b2=hp["b2"], eps=hp["eps"], wd=hp["wd"])
    toks = z["tokens"].reshape(steps, B, T)
    losses, gnorms = [], []
    for s in range(steps):
        l, raw, gn, skipped = go.train_step(model, list(toks[s]), st, clip=hp["clip"])
        assert not skipped
        losses += l
        gnorms.append(gn)
        if s == 0:
            raw0 = raw
    assert np.allclose(losses, z["losses"], rtol=1e-5, atol=0), (losses, z["losses"])
    assert np.allclose(gnorms, z["gnorm"], rtol=1e-4)
    ref_g = _split(cfg, z["grads"])
    for (n, _), g, r in zip(go.param_specs(cfg), raw0, ref_g):
        if np.linalg.norm(r) == 0:
            assert np.linalg.norm(g) < 1e-12, n
        else:
            assert _rel(g, r) < 1e-4, (n, _rel(g, r))
    # Post-AdamW weights. A zero-initialised tensor (biases, LayerNorm betas) holds only the
    # Adam steps, lr*m/(sqrt(v)+eps) per entry, which for gradients near eps magnify the
    # fp32-vs-fp64 gradient difference; its tolerance is therefore looser.
    ref_p = _split(cfg, z["params"])
    init = _split(cfg, z["init"])
    for (n, _), r, p0 in zip(go.param_specs(cfg), ref_p, init):
        tol = 1e-4 if not np.any(p0) else 1e-5
        assert _rel(model.p[n], r) < tol, (n, _rel(model.p[n], r))


def test_golden_covers_both_dt_clamp_branches():
    """The Mamba fixture must exercise the in-range and clamped dt paths
    (src/mamba.cpp:318-328), else dt_proj gradients would be trivially zero."""
    z, meta, cfg = _load("mamba_rms")
    g = _split(cfg, z["grads"])
    names = [n for n, _ in go.param_specs(cfg)]
    assert np.linalg.norm(g[names.index("blk0.dt_proj")]) > 0


def test_scan_known_answer():
    """tests/test_mamba_scan.cpp:10-39: x=1, A=-0.5, dt=0.1, B=0.1, C=1, D=1 -> y[0]=1.04."""
    T, D, N = 4, 8, 4
    y, _ = go.selective_scan(np.ones((T, D)), np.full((D, N), -0.5), np.full((T, N), 0.1),
                             np.ones((T, N)), np.full((T, D), 0.1), np.ones(D), np.zeros((D, N)))
    assert abs(y[0, 0] - 1.04) < 0.005


def test_scan_lcg_random_chunked_equivalence():
    """tests/test_mamba_scan.cpp:55-83 (LCG-random inputs, T in {33,129}, nonzero h0):
    the sequential scan equals a chunked two-pass scan within 1e-4."""
    rng = [0x1234567]

    def rnd():
        rng[0] = (rng[0] * 1664525 + 1013904223) & 0xFFFFFFFF
        return (rng[0] >> 8) / float(1 << 24) - 0.5

    for TT in (33, 129):
        DD, NN = 16, 4
        xx = np.array([rnd() for _ in range(TT * DD)]).reshape(TT, DD)
        AA = np.array([-0.5 + 0.5 * rnd() for _ in range(DD * NN)]).reshape(DD, NN)
        BB = np.array([rnd() for _ in range(TT * NN)]).reshape(TT, NN)
        CC = np.array([rnd() for _ in range(TT * NN)]).reshape(TT, NN)
        dd = np.array([0.05 + 0.05 * (rnd() + 0.5) for _ in range(TT * DD)]).reshape(TT, DD)
        Ds = np.array([rnd() for _ in range(DD)])
        hh = np.array([0.1 * rnd() for _ in range(DD * NN)]).reshape(DD, NN)
        ys, _ = go.selective_scan(xx, AA, BB, CC, dd, Ds, hh)
        # chunked: 4 chunks (8 when T >= 256), prefix-combined (src/mamba_scan.cpp:94-148)
        nch = min(TT, 4)
        ch = (TT + nch - 1) // nch
        h = hh.copy()
        yp = np.zeros_like(ys)
        for c in range(nch):
            s, e = c * ch, min(TT, (c + 1) * ch)
            yc, h = go.selective_scan(xx[s:e], AA, BB[s:e], CC[s:e], dd[s:e], Ds, h)
            yp[s:e] = yc
        assert np.abs(ys - yp).max() < 1e-4


def test_ce_backward_known_answer():
    """tests/test_ce_backward.cpp:7-24: dlogits = (softmax - onehot)/T, rows sum to 0."""
    logits = np.array([[1, 0, -1, 0.5], [0, 0, 0, 0]], np.float64)
    d = go.ce_backward(logits, np.array([0, 2]))
    p = go.softmax(logits)
    y = np.zeros_like(p)
    y[0, 0] = y[1, 2] = 1
    assert np.allclose(d, (p - y) / 2, atol=1e-7)
    assert abs(d[0].sum()) < 1e-7
    ds = go.ce_backward(logits, np.array([0, 2]), 0.1)
    assert abs(ds[0].sum()) < 1e-7 and ds[0, 0] > d[0, 0]


def test_adamw_decay_known_answer():
    """tests/test_adamw.cpp:13-23: zero grad, lr 0.1, wd 0.01 -> 2-D weight 0.999, 1-D kept."""
    w2, b1 = np.ones((2, 2)), np.ones(2)
    st = go.AdamWState(lr=0.1, b1=0.9, b2=0.999, eps=1e-8, wd=0.01)
    go.adamw_step([w2, b1], [np.zeros((2, 2)), np.zeros(2)], st, [True, False])
    assert abs(w2[0, 0] - 0.999) < 1e-7 and abs(b1[0] - 1.0) < 1e-12


def test_clip_known_answer():
    """tests/test_clip_norm.cpp: norm 5 clipped to 1; norm 0.5 untouched."""
    g = [np.array([3.0, 4.0]), np.array([0.0])]
    assert abs(go.clip_by_global_norm(g, 1.0) - 5.0) < 1e-6
    assert abs(np.sqrt(sum((x ** 2).sum() for x in g)) - 1.0) < 1e-6
    g3 = [np.array([0.3, 0.4])]
    assert abs(go.clip_by_global_norm(g3, 1.0) - 0.5) < 1e-6 and g3[0][0] == 0.3


def test_checkpoint_roundtrip(tmp_path):
    """v3/v4 layout written and read back (src/model.cpp:568-811)."""
    for name in CASES:
        z, meta, cfg = _load(name)
        p = _split(cfg, z["init"])
        f = tmp_path / (name + ".bin")
        go.write_ckpt(str(f), cfg, p)
        q = go.read_ckpt(str(f), cfg)
        assert all(np.array_equal(a, b) for a, b in zip(p, q))
