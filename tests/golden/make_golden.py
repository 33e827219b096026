"""Generates the golden fixtures of tests/golden/ from the UNMODIFIED reference.

For each case it writes seeded synthetic weights as a v3/v4 checkpoint plus an int32
token file, runs oracle/_ref/ref_step (the reference's own Trainer::train_step_accum,
compiled from the reference sources by oracle/Makefile) and stores inputs and outputs
in <case>.npz:
  init      float32 flat initial parameters (GPT::parameters() order)
  tokens    int32 [steps*B*T]
  losses    float32 [steps*B]   per-micro-batch loss
  grads     float32 flat        raw mean gradient of step 1 (pre-clip)
  params    float32 flat        parameters after `steps` optimizer steps
  gnorm     float32 [steps]     Trainer::last_grad_norm()
  meta      json string         config and hyper-parameters

Run from the repository root (needs the reference sources to build oracle/_ref):
    make -C oracle ref && python tests/golden/make_golden.py
"""
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
sys.path.insert(0, ROOT)
from oracle import gpt_oracle as go  # noqa: E402

REF = os.path.join(ROOT, "oracle", "_ref", "ref_step")

# Transformer cases use head_dim 32 so that the device kernels can run them directly.
CASES = {
    # LayerNorm + GELU FFN + tied head: the transformer path of configs 1 and 2
    "gpt_ln_gelu_tied": dict(cfg=dict(vocab=64, n_layers=2, n_heads=1, n_embd=32, block_size=16),
                             B=3, T=16, steps=2, seed=1, tok_seed=0),
    # RMSNorm + untied lm_head
    "gpt_rms_untied": dict(cfg=dict(vocab=48, n_layers=1, n_heads=1, n_embd=32, block_size=12,
                                    tied=False, rmsnorm=True),
                           B=2, T=12, steps=2, seed=2, tok_seed=3),
    # T > 128: the forward takes flash_attention_full (src/attention.cpp:68-75)
    "gpt_flash_t136": dict(cfg=dict(vocab=32, n_layers=1, n_heads=1, n_embd=32, block_size=136),
                           B=1, T=136, steps=1, seed=4, tok_seed=5),
    # Mamba blocks (checkpoint v4), RMSNorm; larger x_proj/dt_proj so that softplus(dt)
    # falls both inside and outside the clamp range [1e-3, 0.1]
    "mamba_rms": dict(cfg=dict(vocab=40, n_layers=2, n_heads=1, n_embd=16, block_size=12,
                               rmsnorm=True, mamba=True, d_inner=32, d_state=4, dt_rank=2,
                               conv_kernel=4),
                      B=2, T=12, steps=2, seed=6, tok_seed=7, dt_scale=True),
}
HP = dict(lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, clip=1.0)


def make_init(cfg, seed, dt_scale=False):
    params = go.init_params(cfg, seed)
    if dt_scale:
        rng = np.random.default_rng(seed + 100)
        for (n, s), i in zip(go.param_specs(cfg), range(len(params))):
            if n.endswith("in_proj"):
                params[i] = (rng.standard_normal(s) * 0.5).astype(np.float32)
            if n.endswith("x_proj"):
                params[i] = (rng.standard_normal(s) * 1.0).astype(np.float32)
            if n.endswith("dt_proj"):
                params[i] = (rng.standard_normal(s) * 3.0).astype(np.float32)
    return params


def run_case(name, spec, outdir):
    cfg = go.Cfg(**spec["cfg"])
    B, T, steps = spec["B"], spec["T"], spec["steps"]
    params = make_init(cfg, spec["seed"], spec.get("dt_scale", False))
    tokens = go.uniform_tokens(cfg.vocab, steps * B * T, spec["tok_seed"])
    with tempfile.TemporaryDirectory() as td:
        ck = os.path.join(td, "model.bin")
        tk = os.path.join(td, "tokens.i32")
        go.write_ckpt(ck, cfg, params)
        tokens.tofile(tk)
        args = [REF, ck, tk, str(B), str(T), td, f"steps={steps}",
                f"tied={int(cfg.tied)}", f"rmsnorm={int(cfg.rmsnorm)}"]
        args += [f"{k}={v}" for k, v in HP.items()]
        env = dict(os.environ, OMP_NUM_THREADS="1")
        subprocess.run(args, check=True, env=env, stdout=subprocess.DEVNULL)
        rd = lambda f: np.fromfile(os.path.join(td, f), np.float32)  # noqa: E731
        out = dict(init=np.concatenate([p.ravel() for p in params]), tokens=tokens,
                   losses=rd("losses.f32"), grads=rd("grads.f32"), params=rd("params.f32"),
                   gnorm=rd("gnorm.f32"))
    meta = dict(cfg=spec["cfg"], B=B, T=T, steps=steps, hp=HP)
    np.savez_compressed(os.path.join(outdir, name + ".npz"), meta=json.dumps(meta), **out)
    print(name, "loss0", out["losses"][0], "n_params", out["params"].size)


def main():
    outdir = os.path.dirname(os.path.abspath(__file__))
    for name, spec in CASES.items():
        run_case(name, spec, outdir)


if __name__ == "__main__":
    main()
