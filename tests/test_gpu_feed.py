"""The device feed (pinned, double-buffered H2D on a copy stream) trains exactly like the
host-copy step: same tokens, same deterministic kernels, so the same losses bit for bit."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_device_feed_matches_host_copies(cuda, tmp_path):
    from llmgpu import feed
    from llmgpu.trainer import Trainer, make_config
    cfg = make_config(vocab_size=256, n_layers=2, n_heads=4, n_embd=128, block_size=64)
    B, T = 4, 64
    toks = np.random.default_rng(7).integers(0, 256, size=20 * B * T).astype(np.int32)
    ds = feed.Dataset(toks, T)
    sched = feed.CosineScheduler(1e-3, 2, 10, 1e-4)
    runs = []
    for device_feed in (True, False):
        tr = Trainer(cfg, B, T)
        tr.set_adamw(lr=1e-3)
        log = feed.MetricsLogger(str(tmp_path / f"m{int(device_feed)}.jsonl"))
        runs.append(feed.train(tr, ds, B, T, 8, scheduler=sched, logger=log,
                               device_feed=device_feed))
    assert len(runs[0]) == 8
    assert runs[0] == runs[1]
    assert all(np.isfinite(runs[0]))
    assert len((tmp_path / "m1.jsonl").read_text().splitlines()) == 8


def test_rollback_restores_the_snapshot(cuda):
    """Trainer.snapshot_params / rollback_if_nonfinite (src/trainer.cpp:234-246): a non-finite
    loss restores the snapshot's parameters and halves the learning rate; a finite one
    changes nothing."""
    from llmgpu.trainer import Trainer, make_config
    cfg = make_config(vocab_size=256, n_layers=2, n_heads=4, n_embd=128, block_size=64)
    B, T = 4, 64
    toks = np.random.default_rng(11).integers(0, 256, size=(B, T)).astype(np.int32)
    tr = Trainer(cfg, B, T)
    tr.set_adamw(lr=1e-3)
    tr.snapshot_params()
    before = [tr.get_param(i).copy() for i in range(tr.num_params())]
    first_loss, _, _ = tr.train_step(toks)
    assert any(not np.array_equal(a, tr.get_param(i)) for i, a in enumerate(before))
    assert tr.rollback_if_nonfinite(1.0) is False
    assert tr.rollback_if_nonfinite(float("nan")) is True
    assert all(np.array_equal(a, tr.get_param(i)) for i, a in enumerate(before))
    assert tr.get_lr() == pytest.approx(5e-4)
    # the restored parameters give the first step's loss again
    again, _, _ = tr.train_step(toks)
    assert again == first_loss
