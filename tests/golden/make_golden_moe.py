"""Generates tests/golden/moe_forward.npz from the UNMODIFIED reference MoEFFN.

Runs oracle/_ref/ref_moe (MoEFFN::forward and MoEFFN::aux_loss, src/moe.cpp:23-75, built
from the reference sources by oracle/Makefile) on seeded synthetic weights and inputs:
distinct weights per expert, random rows, all-zero rows (uniform routing probabilities:
every expert ties, so the lower indices must win) and large rows (peaked routing).
Stores gate [C,E], W1 [E,C,4C], W2 [E,4C,C], x [T,C], out [T,C], aux and meta.

Run from the repository root:
    make -C oracle ref && python tests/golden/make_golden_moe.py
"""
import json
import os
import subprocess
import tempfile

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
REF = os.path.join(ROOT, "oracle", "_ref", "ref_moe")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "moe_forward.npz")


def main():
    C, E, k, T, coef = 16, 8, 2, 24, 0.01
    H = 4 * C
    rng = np.random.default_rng(2024)
    gate = (rng.standard_normal((C, E)) * 0.5).astype(np.float32)
    w1 = (rng.standard_normal((E, C, H)) * 0.1).astype(np.float32)
    w2 = (rng.standard_normal((E, H, C)) * 0.1).astype(np.float32)
    x = rng.standard_normal((T, C)).astype(np.float32)
    x[3] = 0.0
    x[11] = 0.0
    x[17] *= 6.0
    x[20] *= 6.0
    with tempfile.TemporaryDirectory() as d:
        fin, fout = os.path.join(d, "in.bin"), os.path.join(d, "out.bin")
        np.concatenate([gate.ravel(), w1.ravel(), w2.ravel(), x.ravel()]).tofile(fin)
        subprocess.run([REF, fin, fout, str(C), str(E), str(k), str(T), repr(coef)], check=True)
        res = np.fromfile(fout, np.float32)
    out, aux = res[:T * C].reshape(T, C), res[T * C]
    meta = dict(C=C, E=E, k=k, T=T, coef=coef, zero_rows=[3, 11], large_rows=[17, 20])
    np.savez_compressed(OUT, gate=gate, w1=w1, w2=w2, x=x, out=out, aux=np.float32(aux),
                        meta=json.dumps(meta))
    print("wrote", OUT, "aux", aux)


if __name__ == "__main__":
    main()
