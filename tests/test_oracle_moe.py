"""Pins the MoE part of the numpy oracle (oracle/gpt_oracle.py) before it is trusted.

* Forward and aux loss against the unmodified reference MoEFFN (tests/golden/moe_forward.npz,
  made by tests/golden/make_golden_moe.py from oracle/_ref/ref_moe): random rows, all-zero
  rows whose probabilities tie across every expert, and large rows with peaked routing.
* The backward (the reference has none, src/moe.cpp) against central finite differences of
  the oracle's own float64 forward.
"""
import json
import os

import numpy as np

from oracle import gpt_oracle as go

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _model(C, E, k, coef):
    cfg = go.Cfg(vocab=16, n_layers=1, n_heads=1, n_embd=C, block_size=8, moe_experts=E,
                 moe_top_k=k, moe_aux_coef=coef)
    return go.Model(cfg, go.init_params(cfg, seed=0))


def test_moe_forward_matches_reference():
    z = np.load(os.path.join(GOLDEN, "moe_forward.npz"))
    meta = json.loads(str(z["meta"]))
    m = _model(meta["C"], meta["E"], meta["k"], meta["coef"])
    P = dict(gate=z["gate"].astype(np.float64), W1e=z["w1"].astype(np.float64),
             W2e=z["w2"].astype(np.float64))
    out, c = m._moe_fwd(z["x"].astype(np.float64), P)
    ref = z["out"].astype(np.float64)
    err = np.abs(out - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err
    assert abs(c["aux"] - float(z["aux"])) <= 1e-5 * abs(float(z["aux"])) + 1e-9
    # all-zero rows: uniform probabilities, so the two lowest expert indices are chosen
    for r in meta["zero_rows"]:
        assert list(c["idx"][r]) == [0, 1]


def _loss(m, h, P, R):
    out, c = m._moe_fwd(h, P)
    return float((out * R).sum() + c["aux"])


def test_moe_backward_finite_differences():
    C, E, k, T = 8, 4, 2, 6
    m = _model(C, E, k, 0.05)
    rng = np.random.default_rng(7)
    P = dict(gate=rng.standard_normal((C, E)) * 0.7, W1e=rng.standard_normal((E, C, 4 * C)) * 0.3,
             W2e=rng.standard_normal((E, 4 * C, C)) * 0.3)
    h = rng.standard_normal((T, C))
    R = rng.standard_normal((T, C))
    out, c = m._moe_fwd(h, P)
    G = {n: np.zeros_like(v) for n, v in P.items()}
    dh = m._moe_bwd(h, R, P, c, G)
    eps = 1e-6
    checks = [("h", h, dh)] + [(n, P[n], G[n]) for n in ("gate", "W1e", "W2e")]
    for name, arr, grad in checks:
        flat = arr.reshape(-1)
        for i in rng.choice(flat.size, size=12, replace=False):
            old = flat[i]
            flat[i] = old + eps
            lp = _loss(m, h, P, R)
            flat[i] = old - eps
            lm = _loss(m, h, P, R)
            flat[i] = old
            fd = (lp - lm) / (2 * eps)
            an = grad.reshape(-1)[i]
            assert abs(fd - an) <= 1e-6 + 1e-5 * abs(fd), (name, i, fd, an)
