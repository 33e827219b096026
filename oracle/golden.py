"""ORACLE — test infrastructure only. Reads the golden fixtures of tests/golden/.

A fixture holds the inputs and outputs of the unmodified reference training step
(tests/golden/make_golden.py). Compact fixtures omit the initial parameters, which are
regenerated from the stored seed and checked against the stored SHA-256, and store the
parameter change of the step instead of the parameters.
"""
import hashlib
import json

import numpy as np

from . import gpt_oracle as go


def load(path):
    """Returns (arrays dict with init/tokens/losses/grads/params/gnorm, meta dict, Cfg)."""
    z = np.load(path)
    meta = json.loads(str(z["meta"]))
    cfg = go.Cfg(**meta["cfg"])
    out = {k: z[k] for k in z.files if k != "meta"}
    if "init" not in out:
        init = np.concatenate([p.ravel() for p in go.init_params(cfg, meta["seed"])])
        if hashlib.sha256(init.tobytes()).hexdigest() != meta["init_sha256"]:
            raise RuntimeError(f"{path}: regenerated initial parameters differ from the fixture's")
        out["init"] = init
    if "params_delta" in out:
        out["params"] = out["init"] + out.pop("params_delta")
    return out, meta, cfg
