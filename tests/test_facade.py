"""The C++ façade (include/llm/*.h): a program written against the reference's C++ training
API (tests/facade/train_tiny.cpp) compiles unchanged against the façade headers and links
with libllmgpu.so. Without a usable device it fails cleanly (std::runtime_error from the
GPT constructor); on a B200 its steps equal the C ABI's bit for bit."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from oracle import gpt_oracle as go

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
LIBDIR = os.path.join(ROOT, "llm-cpp_b200")
APP = os.path.join(ROOT, "tests", "facade", "train_tiny.cpp")
CFG = go.Cfg(vocab=256, n_layers=2, n_heads=4, n_embd=128, block_size=64)


def _build(tmp_path):
    if not os.path.exists(os.path.join(LIBDIR, "libllmgpu.so")):
        pytest.skip("libllmgpu.so not built")
    exe = str(tmp_path / "train_tiny")
    cxx = shutil.which("g++") or "g++"
    subprocess.run([cxx, "-O2", "-std=c++17", "-Wall", "-Werror", "-I" + os.path.join(ROOT, "include"),
                    APP, "-L" + LIBDIR, "-lllmgpu", "-Wl,-rpath," + LIBDIR, "-o", exe],
                   check=True, capture_output=True, text=True)
    return exe


def _inputs(tmp_path, steps, T):
    params = go.init_params(CFG, seed=41)
    ck = str(tmp_path / "init.bin")
    go.write_ckpt(ck, CFG, params)
    toks = go.uniform_tokens(CFG.vocab, steps * T, seed=42)
    tk = str(tmp_path / "tokens.i32")
    toks.tofile(tk)
    return ck, tk, toks


def test_facade_compiles_and_fails_cleanly_without_a_device(tmp_path):
    import torch
    exe = _build(tmp_path)
    if torch.cuda.is_available():
        pytest.skip("a device is present: the GPU test covers the run")
    ck, tk, _ = _inputs(tmp_path, 2, 16)
    r = subprocess.run([exe, str(tmp_path / "out"), tk, "2", "16", ck], capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 3, (r.returncode, r.stdout, r.stderr)
    assert r.stderr.startswith("error: GPT: "), r.stderr


@pytest.mark.gpu
def test_facade_steps_equal_the_c_abi(cuda, tmp_path):
    from llmgpu import feed
    from llmgpu.trainer import Trainer, make_config
    exe = _build(tmp_path)
    steps, T = 6, 64
    ck, tk, toks = _inputs(tmp_path, steps, T)
    out = str(tmp_path / "run")
    r = subprocess.run([exe, out, tk, str(steps), str(T), ck], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, (r.stdout, r.stderr)
    rd = lambda ext: np.fromfile(out + ext, np.float32)  # noqa: E731
    losses, lrs, gnorms, flat = rd(".losses"), rd(".lr"), rd(".gnorm"), rd(".params")
    # the learning rates are CosineScheduler(3e-4, 2, 10, 3e-5) at steps 0..5
    sched = feed.CosineScheduler(3e-4, 2, 10, 3e-5)
    for s in range(steps):
        assert abs(lrs[s] - sched.get_lr(s)) <= 2e-6 * max(abs(sched.get_lr(s)), 1e-12) + 1e-12
    # the same steps through the C ABI, with the learning rates the façade used
    tr = Trainer(make_config(vocab_size=256, n_layers=2, n_heads=4, n_embd=128, block_size=64),
                 1, 64)
    tr.set_adamw(lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1)
    tr.set_train(grad_clip=1.0)
    tr.load_binary(ck)
    for s in range(steps):
        tr.set_lr(float(lrs[s]))
        loss, gn, skipped = tr.train_step(toks[s * T:(s + 1) * T].reshape(1, T))
        assert not skipped
        assert np.float32(loss) == losses[s], (s, loss, losses[s])
        assert np.float32(gn) == gnorms[s], (s, gn, gnorms[s])
    want = np.concatenate([p.ravel() for p in tr.params()])
    np.testing.assert_array_equal(flat, want)
    # the train state the façade saved loads into a C-ABI context with the same weights
    tr2 = Trainer(make_config(vocab_size=256, n_layers=2, n_heads=4, n_embd=128, block_size=64),
                  1, 64)
    tr2.load_train_state(out + ".state")
    np.testing.assert_array_equal(np.concatenate([p.ravel() for p in tr2.params()]), want)
    tr.close()
    tr2.close()
