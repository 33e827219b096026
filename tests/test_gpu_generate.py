"""Inference on the training kernels: the last position's logits (llmgpu_forward_logits)
against the oracle's forward, and greedy generation built on them."""
import numpy as np
import pytest

from oracle import gpt_oracle as go

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("tied,rms", [(True, False), (False, True)])
def test_forward_logits_match_oracle(cuda, tied, rms):
    from llmgpu.trainer import Trainer, make_config
    cfg = go.Cfg(vocab=256, n_layers=2, n_heads=4, n_embd=128, block_size=64, tied=tied,
                 rmsnorm=rms)
    params = go.init_params(cfg, seed=4)
    B, T = 3, 40
    tr = Trainer(make_config(vocab_size=cfg.vocab, n_layers=cfg.n_layers, n_heads=cfg.n_heads,
                             n_embd=cfg.n_embd, block_size=cfg.block_size,
                             weight_tying=cfg.tied, use_rmsnorm=cfg.rmsnorm), B, T)
    for i, p in enumerate(params):
        tr.set_param(i, p)
    toks = np.random.default_rng(8).integers(0, cfg.vocab, size=(B, T)).astype(np.int32)
    got = tr.forward_logits(toks)
    model = go.Model(cfg, params)
    every = np.stack([model.logits(list(toks[b])) for b in range(B)])
    want = every[:, T - 1]
    # bf16 operands and bf16 logits on the device, fp64 in the oracle
    assert got.shape == (B, cfg.vocab)
    assert _rel(got, want) < 2e-2, _rel(got, want)
    # every position (GPT::forward's [T, V]): llmgpu_forward_logits_all
    allg = tr.forward_logits_all(toks)
    assert allg.shape == (B, T, cfg.vocab)
    assert _rel(allg, every) < 2e-2, _rel(allg, every)
    np.testing.assert_array_equal(allg[:, T - 1], got)
    # the loss path is untouched: eval_loss after forward_logits is the same as before it
    l0 = tr.eval_loss(toks)
    tr.forward_logits(toks)
    assert tr.eval_loss(toks) == l0

    # greedy generation: each new token is the argmax of the logits of its prefix
    prompt = [int(t) for t in toks[0, :10]]
    out = tr.generate(prompt, 6)
    assert out[:10] == prompt and len(out) == 16
    for k in range(10, 16):
        lg = tr.forward_logits(np.asarray(out[:k], np.int32)[None, :])[0]
        assert out[k] == int(np.argmax(lg))
