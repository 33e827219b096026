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


@pytest.mark.parametrize("tied,rms,pos", [(True, False, "learned"), (False, True, "rope"),
                                          (True, False, "sinusoidal")])
def test_kv_decode_matches_full_forward(cuda, tied, rms, pos):
    """KV-cached decoding (llmgpu_decode_prefill / llmgpu_decode_step, the incremental path of
    GPT::generate, src/attention.cpp:104-181): after a prompt, each teacher-forced token's
    logits equal the full forward's logits at that position, against the oracle and against
    the device's own full forward."""
    from llmgpu.trainer import Trainer, make_config
    cfg = go.Cfg(vocab=256, n_layers=2, n_heads=4, n_embd=128, block_size=64, tied=tied,
                 rmsnorm=rms, pos_encoding=pos, rope_scaling=2.0 if pos == "rope" else 1.0)
    params = go.init_params(cfg, seed=14)
    B, T0, n = 2, 10, 30
    tr = Trainer(make_config(vocab_size=cfg.vocab, n_layers=cfg.n_layers, n_heads=cfg.n_heads,
                             n_embd=cfg.n_embd, block_size=cfg.block_size, weight_tying=cfg.tied,
                             use_rmsnorm=cfg.rmsnorm,
                             pos_encoding={"learned": 0, "sinusoidal": 1, "rope": 2}[pos],
                             rope_scaling=cfg.rope_scaling), B, cfg.block_size)
    for i, p in enumerate(params):
        tr.set_param(i, p)
    toks = np.random.default_rng(15).integers(0, cfg.vocab, size=(B, T0 + n)).astype(np.int32)
    got = [tr.decode_prefill(toks[:, :T0])]
    for t in range(T0, T0 + n):
        got.append(tr.decode_step(toks[:, t]))
        assert tr.decode_position() == t + 1
    got = np.stack(got, 1)                                   # [B, n + 1, V]: positions T0-1 ..
    full = tr.forward_logits_all(toks)[:, T0 - 1:]           # the device's full forward
    model = go.Model(cfg, params)
    want = np.stack([model.logits(list(toks[b]))[T0 - 1:] for b in range(B)])
    assert _rel(got, want) < 2e-2, _rel(got, want)
    assert _rel(got, full) < 2e-2, _rel(got, full)
    # greedy generation through the caches picks the argmax of the full forward's logits
    prompt = [int(t) for t in toks[0, :T0]]
    out = tr.generate(prompt, 8)
    for k in range(T0, T0 + 8):
        lg = tr.forward_logits(np.asarray(out[:k], np.int32)[None, :])[0]
        srt = np.sort(lg)
        if srt[-1] - srt[-2] > 1e-2:  # away from near-ties of bf16 logits
            assert out[k] == int(np.argmax(lg)), k
    tr.close()


def test_kv_decode_refuses_uncovered_configurations(cuda):
    """SwiGLU (an extension without a reference generate path) has no KV-cached decode:
    the call reports it, and generate falls back to the full forward."""
    from llmgpu.trainer import LlmgpuError, Trainer, make_config
    tr = Trainer(make_config(vocab_size=128, n_layers=1, n_heads=2, n_embd=64, block_size=32,
                             use_rmsnorm=True, ffn_swiglu=True, ffn_hidden=128,
                             weight_tying=False), 1, 32)
    with pytest.raises(LlmgpuError):
        tr.decode_reset(1)
    assert not tr.decode_supported()
    assert len(tr.generate([1, 2, 3], 4)) == 7
    tr.close()
