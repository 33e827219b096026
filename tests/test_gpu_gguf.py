"""GGUF export of the model on the device and import into a second one: the parameters come
back exactly, and the reloaded model gives the same loss."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_gguf_round_trip_on_device(cuda, tmp_path):
    from llmgpu import gguf
    from llmgpu.trainer import Trainer, make_config
    cfg = make_config(vocab_size=256, n_layers=2, n_heads=4, n_embd=128, block_size=64)
    B, T = 2, 64
    toks = np.random.default_rng(3).integers(0, 256, size=(B, T)).astype(np.int32)
    a = Trainer(cfg, B, T)
    a.train_step(toks)  # move the weights away from the initialisation
    path = str(tmp_path / "model.gguf")
    gguf.save_gguf(a, path)
    b = Trainer(cfg, B, T)
    gguf.load_gguf(b, path)
    for i in range(a.num_params()):
        assert np.array_equal(a.get_param(i), b.get_param(i)), a.param_info(i)[0]
    assert a.eval_loss(toks) == b.eval_loss(toks)
