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

Cases marked compact (the config-1 step, 840 K parameters) store no `init` (it is
regenerated from meta["seed"] by gpt_oracle.init_params and checked against meta["init_sha256"])
and store `params_delta` = params - init instead of `params`; oracle/golden.py reads both forms.

Run from the repository root (needs the reference sources to build oracle/_ref):
    make -C oracle ref && python tests/golden/make_golden.py [case ...]
"""
import hashlib
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
    # several heads: the per-head slicing of MultiHeadAttention (src/attention.cpp:35-102,
    # 183-363) at head_dim 32 and 64 (the tcgen05 attention path), naive and flash forward
    "gpt_mh4_hd32": dict(cfg=dict(vocab=96, n_layers=1, n_heads=4, n_embd=128, block_size=64),
                         B=3, T=64, steps=2, seed=8, tok_seed=9, compact=True),
    "gpt_mh2_hd64_t200": dict(cfg=dict(vocab=80, n_layers=1, n_heads=2, n_embd=128,
                                       block_size=200),
                              B=2, T=200, steps=1, seed=10, tok_seed=11, compact=True),
    # Config::pos_encoding = RoPE: rope_cfg on the embedding sum (src/model.cpp:81-104,158),
    # NTK base scaling and the YaRN ramp with its attention scale
    "gpt_rope_ntk": dict(cfg=dict(vocab=64, n_layers=2, n_heads=2, n_embd=64, block_size=48,
                                  pos_encoding="rope", rope_theta=10000.0, rope_scaling=2.0,
                                  rope_mode=0),
                         B=2, T=48, steps=2, seed=12, tok_seed=13, compact=True),
    "gpt_rope_yarn": dict(cfg=dict(vocab=64, n_layers=1, n_heads=2, n_embd=64, block_size=40,
                                   tied=False, rmsnorm=True, pos_encoding="rope",
                                   rope_theta=500.0, rope_scaling=4.0, rope_mode=1,
                                   yarn_alpha=1.5, yarn_beta=32.0),
                          B=2, T=40, steps=2, seed=14, tok_seed=15, compact=True),
    "mamba_rope": dict(cfg=dict(vocab=40, n_layers=1, n_heads=1, n_embd=16, block_size=12,
                                rmsnorm=True, mamba=True, d_inner=32, d_state=4, dt_rank=2,
                                conv_kernel=4, pos_encoding="rope", rope_scaling=3.0),
                       B=2, T=12, steps=1, seed=16, tok_seed=17),
    # the tiny char-level configuration exactly: 4 layers, n_embd 128, 4 heads, vocab 256,
    # T 128, batch 8, ids uniform over [0, 256) from PCG64 seed 0, weights from seed 1
    "gpt_config1": dict(cfg=dict(vocab=256, n_layers=4, n_heads=4, n_embd=128, block_size=128),
                        B=8, T=128, steps=1, seed=1, tok_seed=0, compact=True, threads=8),
}
POS = {"learned": 0, "sinusoidal": 1, "rope": 2}
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
                f"tied={int(cfg.tied)}", f"rmsnorm={int(cfg.rmsnorm)}",
                f"pos={POS[cfg.pos_encoding]}", f"rope_theta={cfg.rope_theta!r}",
                f"rope_scaling={cfg.rope_scaling!r}", f"rope_mode={cfg.rope_mode}",
                f"yarn_alpha={cfg.yarn_alpha!r}", f"yarn_beta={cfg.yarn_beta!r}"]
        args += [f"{k}={v}" for k, v in HP.items()]
        env = dict(os.environ, OMP_NUM_THREADS=str(spec.get("threads", 1)))
        subprocess.run(args, check=True, env=env, stdout=subprocess.DEVNULL)
        rd = lambda f: np.fromfile(os.path.join(td, f), np.float32)  # noqa: E731
        init = np.concatenate([p.ravel() for p in params])
        out = dict(init=init, tokens=tokens, losses=rd("losses.f32"), grads=rd("grads.f32"),
                   params=rd("params.f32"), gnorm=rd("gnorm.f32"))
    meta = dict(cfg=spec["cfg"], B=B, T=T, steps=steps, hp=HP)
    if spec.get("compact"):
        meta.update(seed=spec["seed"], init_sha256=hashlib.sha256(init.tobytes()).hexdigest())
        out["params_delta"] = out.pop("params") - init
        del out["init"]
    np.savez_compressed(os.path.join(outdir, name + ".npz"), meta=json.dumps(meta), **out)
    print(name, "loss0", out["losses"][0], "n_params", out["grads"].size)


def main():
    outdir = os.path.dirname(os.path.abspath(__file__))
    names = sys.argv[1:] or list(CASES)
    for name in names:
        run_case(name, CASES[name], outdir)


if __name__ == "__main__":
    main()
