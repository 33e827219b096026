"""The data feed's host side against the reference's own feed code.

oracle/_ref/ref_feed links the reference's CosineScheduler, Dataset, DataLoader,
PrefetchLoader and MetricsLogger unmodified (oracle/ref_feed.cpp) and prints what they
produce; llmgpu.feed must produce the same.
"""
import json
import os
import subprocess

import numpy as np
import pytest

from llmgpu import feed

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
REF = os.path.join(ROOT, "oracle", "_ref", "ref_feed")


def _ref(*args):
    if not os.path.exists(REF):
        pytest.skip("oracle/_ref/ref_feed not built (needs the reference sources)")
    return subprocess.run([REF, *args], check=True, capture_output=True, text=True).stdout


def test_cosine_scheduler_matches_reference():
    n = 0
    for line in _ref("lr").splitlines():
        if not line.startswith("lr "):
            continue
        _, base, warm, mx, mn, cyc, step, val = line.split()
        s = feed.CosineScheduler(float(base), int(warm), int(mx), float(mn), int(cyc))
        got, want = s.get_lr(int(step)), float(val)
        assert abs(got - want) <= 2e-6 * abs(want) + 1e-12, (line, got)
        n += 1
    assert n > 500


def _runs(text, tag):
    out = []
    for line in text.splitlines():
        f = line.split()
        if f[0] == tag:
            assert int(f[1]) == len(f) - 2
            out.append([int(x) for x in f[2:]])
    return out


@pytest.mark.parametrize("content", [b"To be, or not to be:\nthat is the question.\n\xc3\xa9\xff\x00z",
                                     b""])
@pytest.mark.parametrize("bs", [7, 16])
def test_dataset_and_loaders_match_reference(tmp_path, content, bs):
    p = tmp_path / "text.txt"
    p.write_bytes(content)
    out = _ref("data", str(p), str(bs))
    ds = feed.Dataset.from_file(str(p), bs)
    assert _runs(out, "tokens") == [ds.tokens.tolist()]
    dl = feed.DataLoader(ds, bs)
    got = []
    while dl.has_next():
        got.append(dl.next_batch()[0].tolist())
    assert got == _runs(out, "loader")
    for prefetch in (2, 0):
        pl = feed.PrefetchLoader(ds, bs, prefetch)
        got = []
        while True:
            b = pl.next()
            if not b:
                break
            got.append(b[0].tolist())
        pl.close()
        assert got == _runs(out, "prefetch")


def test_metrics_logger_matches_reference(tmp_path):
    ref_path, our_path = tmp_path / "ref.jsonl", tmp_path / "ours.jsonl"
    _ref("log", str(ref_path))
    log = feed.MetricsLogger(str(our_path))
    log.log_step(1, 2.3614869, 10.60655, 3e-4, 0.8754321, 756960.19)
    log.log_step(20, 0.125, 1.1331485, 1.5e-5, 12.5, 1e-3)
    log.log_step(300, 7.0, 1096.6332, 0.0, 0.0, 0.0)
    assert our_path.read_text() == ref_path.read_text()
    for line in our_path.read_text().splitlines():
        json.loads(line)


def test_shuffled_loader_covers_the_same_runs():
    ds = feed.Dataset(np.arange(1000), 0)
    a = feed.DataLoader(ds, 64, shuffle=True, seed=3)
    b = feed.DataLoader(ds, 64)
    assert sorted(a.order.tolist()) == b.order.tolist()
    assert a.order.tolist() != b.order.tolist()
    c = feed.DataLoader(ds, 64, shuffle=True, seed=3)
    assert a.order.tolist() == c.order.tolist()  # seeded


def test_step_scheduler_matches_reference():
    n = 0
    for line in _ref("lr").splitlines():
        if not line.startswith("steplr"):
            continue
        _, base, size, gamma, step, val = line.split()
        got = feed.StepScheduler(float(base), int(size), float(gamma)).get_lr(int(step))
        want = float(val)
        assert got == pytest.approx(want, rel=1e-7, abs=1e-30), line
        n += 1
    assert n > 100


@pytest.mark.parametrize("block,eos,ratio", [(8, 0, 0.9), (5, 50256, 0.5), (64, 7, 1.0)])
def test_pack_and_split_match_reference(tmp_path, block, eos, ratio):
    p = tmp_path / "text.txt"
    p.write_bytes(b"Some text to pack into rows, with a ragged tail.\n" * 3)
    out = _ref("pack", str(p), str(block), str(eos), str(ratio))
    rows, mask = feed.pack_with_eos(feed.Dataset.from_file(str(p)).tokens, block, eos)
    assert rows.tolist() == _runs(out, "row")
    assert mask.tolist() == _runs(out, "mask")
    tr, va = feed.train_val_split(feed.Dataset.from_file(str(p)).tokens, ratio, 7)
    assert [tr.tolist()] == _runs(out, "train") and [va.tolist()] == _runs(out, "val")
