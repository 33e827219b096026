"""Dual GEMM launches hand their tiles to the CTA pairs at run time (a device counter and a
ring of work units in shared memory) in data-parallel contexts, and run the host's per-pair
lists otherwise; LLMGPU_GEMM_QUEUE=1 / 0 forces either. Which pair computes a tile must not
change any result: every output element is written by one tile, and split-K pieces go to
fixed partial slots summed in a fixed order. Two processes, one per setting, train the same
steps from the same weights and must end bit-identical; the profiled step must show dual
launches, and the later steps show that the counters were reset after each launch."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))

SCRIPT = r"""
import hashlib, json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from llmgpu.trainer import Trainer, make_config
B, T = 4, 1024
c = make_config(vocab_size=2048, n_layers=2, n_heads=12, n_embd=768, block_size=T)
tr = Trainer(c, B, T)
tr.set_adamw(lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1)
tr.set_train(grad_clip=1.0)
rng = np.random.default_rng(11)
for i in range(tr.num_params()):
    p = tr.get_param(i)
    tr.set_param(i, (rng.standard_normal(p.shape) * 0.02).astype(np.float32))
losses = []
tr.set_profile(True)
for s in range(3):
    toks = rng.integers(0, 2048, size=(B, T)).astype(np.int32)
    loss, gn, _ = tr.train_step(toks)
    losses.append(float(loss).hex())
    if s == 0:
        shapes, _ = tr.gemm_last_step()
        tr.set_profile(False)
h = hashlib.sha256()
for i in range(tr.num_params()):
    h.update(np.ascontiguousarray(tr.get_param(i)).tobytes())
print(json.dumps({"losses": losses, "params": h.hexdigest(),
                  "dual": int((shapes[:, 3] > 0).sum())}))
tr.close()
"""


def _run(queue):
    env = dict(os.environ, LLMGPU_GEMM_QUEUE=str(queue))
    out = subprocess.run([sys.executable, "-c", SCRIPT,
                          os.path.join(ROOT, "llm-cpp_b200", "python")],
                         env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_run_time_tile_queue_matches_host_lists(cuda):
    dyn = _run(1)
    fixed = _run(0)
    assert dyn["dual"] >= 4, dyn  # each layer's backward GEMM pairs share launches
    assert dyn["losses"] == fixed["losses"]
    assert dyn["params"] == fixed["params"]
