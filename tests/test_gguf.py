"""GGUF F32 export/import (llmgpu.gguf) against the reference's own save_gguf / load_gguf,
run by oracle/_ref/ref_gguf on the same parameters (passed as a reference binary
checkpoint): the files must be byte-identical, and each side must read the other's."""
import os
import subprocess

import numpy as np
import pytest

from llmgpu import gguf
from oracle import gpt_oracle as go

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
REF = os.path.join(ROOT, "oracle", "_ref", "ref_gguf")


def _ref(*args):
    if not os.path.exists(REF):
        pytest.skip("oracle/_ref/ref_gguf not built (needs the reference sources)")
    subprocess.run([REF, *map(str, args)], check=True, capture_output=True)


@pytest.mark.parametrize("tied,rms", [(True, False), (False, True)])
def test_gguf_matches_reference(tmp_path, tied, rms):
    cfg = go.Cfg(vocab=96, n_layers=2, n_heads=4, n_embd=64, block_size=48, tied=tied,
                 rmsnorm=rms)
    params = go.init_params(cfg, seed=5)
    shapes = [p.shape for p in params]
    ckpt = tmp_path / "model.bin"
    go.write_ckpt(str(ckpt), cfg, params)
    args = (cfg.vocab, cfg.n_layers, cfg.n_heads, cfg.n_embd, cfg.block_size, int(tied), int(rms))
    ref_file, our_file = tmp_path / "ref.gguf", tmp_path / "ours.gguf"
    _ref("save", *args, ckpt, ref_file)
    gguf.write_gguf(str(our_file), params)
    assert our_file.read_bytes() == ref_file.read_bytes()
    arrays, kvs = gguf.read_gguf(str(ref_file), shapes)
    assert kvs["llm.tensor_count"] == str(len(params))
    assert all(np.array_equal(a, p) for a, p in zip(arrays, params))
    back = tmp_path / "back.bin"
    _ref("load", *args, our_file, back)
    assert all(np.array_equal(a, p) for a, p in zip(go.read_ckpt(str(back), cfg), params))


def test_gguf_rejects_a_shape_mismatch(tmp_path):
    f = tmp_path / "x.gguf"
    gguf.write_gguf(str(f), [np.zeros((4, 3), np.float32), np.ones((2, 3), np.float32)])
    with pytest.raises(ValueError):
        gguf.read_gguf(str(f), [(4, 3), (3, 3)])
    with pytest.raises(ValueError):
        gguf.read_gguf(str(f), [(4, 3)])


@pytest.mark.parametrize("qtype", [0, 8, 4, 12])
def test_quantized_gguf_matches_reference(tmp_path, qtype):
    cfg = go.Cfg(vocab=96, n_layers=2, n_heads=4, n_embd=64, block_size=48)
    params = go.init_params(cfg, seed=9)
    # an evenly spread block (both signs, the extremes at +-1) and an all-zero block
    params[0].ravel()[:32] = np.linspace(-1, 1, 32, dtype=np.float32)
    params[0].ravel()[32:64] = 0.0
    big = next(i for i, p in enumerate(params) if i > 1 and p.size >= 1024)
    params[big].ravel()[3] = np.nan     # non-finite values: NaN and inf in separate blocks
    params[big].ravel()[700] = np.inf
    ckpt = tmp_path / "model.bin"
    go.write_ckpt(str(ckpt), cfg, params)
    ref_file, our_file = tmp_path / "ref.gguf", tmp_path / "ours.gguf"
    _ref("quant", cfg.vocab, cfg.n_layers, cfg.n_heads, cfg.n_embd, cfg.block_size, 1, 0, ckpt,
         ref_file, qtype)
    gguf.write_gguf_quant(str(our_file), params, qtype)
    assert our_file.read_bytes() == ref_file.read_bytes()
    # decoding: the values the reference's load_gguf puts into its model
    back = tmp_path / "back.bin"
    _ref("load", cfg.vocab, cfg.n_layers, cfg.n_heads, cfg.n_embd, cfg.block_size, 1, 0,
         our_file, back)
    want = go.read_ckpt(str(back), cfg)
    got, _ = gguf.read_gguf(str(our_file), [p.shape for p in params])
    for a, b in zip(got, want):
        assert np.array_equal(a, b, equal_nan=True)


def test_unknown_quant_type_is_refused(tmp_path):
    with pytest.raises(ValueError):
        gguf.write_gguf_quant(str(tmp_path / "q.gguf"), [np.zeros((2, 2), np.float32)], 5)
