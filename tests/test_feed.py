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


def test_samplers_match_reference():
    from llmgpu import sampling
    rows, n = [], 0
    gen = [3, 7, 7, 49, 0, 3, 3]
    for line in _ref("sample").splitlines():
        f = line.split()
        if f[0] == "logits":
            rows.append(np.array([float(v) for v in f[1:]], np.float32))
        elif f[0] in ("temp", "topk", "topp"):
            r, t, seed, want = int(f[1]), float(f[2]), int(f[3]), int(f[4])
            l = rows[r]
            if f[0] == "temp":
                got = sampling.sample_temperature_seeded(l, t, seed)
            elif f[0] == "topk":
                got = sampling.sample_top_k_seeded(l, 5 + seed % 7, t, seed)
            else:
                got = sampling.sample_top_p_seeded(l, np.float32(0.5) + np.float32(0.01) * np.float32(seed), t, seed)
            assert got == want, line
            n += 1
        elif f[0] == "greedy":
            assert sampling.sample_greedy(rows[int(f[1])]) == int(f[2])
        elif f[0] == "reppen":
            want = np.array([float(v) for v in f[1:]], np.float32)
            assert np.array_equal(sampling.apply_repetition_penalty(rows[-1], gen, 1.3), want)
        elif f[0] == "freqpres":
            want = np.array([float(v) for v in f[1:]], np.float32)
            assert np.array_equal(sampling.apply_freq_presence(rows[-1], gen, 0.25, 0.5), want)
    assert n == 6 * 3 * 40 * 3


def test_generate_loop_with_a_stand_in_model():
    """sampling.generate over a fixed logits function (no GPU): greedy follows argmax,
    seeded sampling is reproducible, eos stops, the context window is the last max_seq."""
    from llmgpu import sampling
    V = 32
    seen = []

    def logits(ctx):
        seen.append(ctx.shape[1])
        r = np.random.default_rng(int(ctx.sum()) + ctx.shape[1])
        return r.standard_normal((1, V)).astype(np.float32)

    out = sampling.generate(logits, [1, 2, 3], 5, max_seq=4, vocab=V)
    assert len(out) == 8 and max(seen) == 4
    for k in range(3, 8):
        assert out[k] == sampling.sample_greedy(logits(np.asarray(out[:k][-4:], np.int32)[None]))
    a = sampling.generate(logits, [5], 6, 16, V, temperature=0.9, top_k=5, seed=3)
    b = sampling.generate(logits, [5], 6, 16, V, temperature=0.9, top_k=5, seed=3)
    assert a == b
    c = sampling.generate(logits, [5], 20, 16, V, temperature=1.0, top_p=0.9, eos_id=a[1])
    assert len(c) >= 2 and (len(c) == 21 or c[-1] == a[1])
    # an empty prompt starts from zero logits (uniform), as GPT::generate does
    assert sampling.generate(logits, [], 1, 16, V) == [0]


def test_shared_generator_stream_matches_reference():
    """MT19937.uniform_int / canonical: std::uniform_int_distribution and
    std::discrete_distribution drawing from one std::mt19937(42), interleaved."""
    from llmgpu import sampling
    rng = sampling.MT19937(42)
    n = 0
    for line in _ref("rng").splitlines():
        f = line.split()
        if f[0] == "uni":
            assert rng.uniform_int(0, int(f[2]) - 1) == int(f[3]), line
        else:
            i = int(f[1])
            w = [float((j * 31 + i) % 11 + 1) for j in range(17)]
            assert sampling._discrete_draw(w, rng.canonical()) == int(f[2]), line
        n += 1
    assert n == 400


@pytest.mark.parametrize("opts", [
    dict(temp=0.0, top_k=0, top_p=1.0, rep=1.0, prompt=[3, 1, 4, 1, 5]),
    dict(temp=0.8, top_k=0, top_p=1.0, rep=1.0, prompt=[3, 1, 4]),
    dict(temp=1.3, top_k=7, top_p=1.0, rep=1.0, prompt=[2, 7]),
    dict(temp=0.9, top_k=0, top_p=0.8, rep=1.0, prompt=[9]),
    dict(temp=1.0, top_k=0, top_p=1.0, rep=1.4, prompt=[5, 5, 6]),
    dict(temp=0.7, top_k=3, top_p=1.0, rep=1.2, prompt=[]),
])
def test_generate_matches_reference(tmp_path, opts):
    """sampling.generate, run over the oracle's logits, picks the reference's GPT::generate
    tokens (one std::mt19937(42) stream; uniform pick among the top k; top-p with the
    global seed; zero logits for an empty prompt; repetition penalty)."""
    import sys
    sys.path.insert(0, ROOT)
    from llmgpu import sampling
    from oracle import gpt_oracle as go
    cfg = go.Cfg(vocab=40, n_layers=1, n_heads=2, n_embd=32, block_size=32)
    params = go.init_params(cfg, seed=21)
    params[0] = params[0] * 50.0  # sharp logits: the top-k order has no near-ties
    ck = str(tmp_path / "m.bin")
    go.write_ckpt(ck, cfg, params)
    n = 12
    line = _ref("generate", ck, str(opts["temp"]), str(opts["top_k"]), str(opts["top_p"]),
                str(opts["rep"]), str(n), *[str(t) for t in opts["prompt"]]).split()
    want = [int(t) for t in line[2:]]
    model = go.Model(cfg, params)
    got = sampling.generate(lambda ctx: model.logits(ctx[0])[-1:], opts["prompt"], n,
                            cfg.block_size, cfg.vocab, temperature=opts["temp"],
                            top_k=opts["top_k"], top_p=opts["top_p"], rep_penalty=opts["rep"])
    assert got == want


def test_train_loop_with_a_stand_in_trainer(tmp_path):
    """feed.train on the host path (no GPU): each step gets the next B runs of T tokens,
    the scheduler's rate for that step is set first, a short tail ends the loop, and one
    metrics line is written per step."""
    B, T = 3, 8
    toks = np.arange(10 * B * T + 5, dtype=np.int32)

    class Stand:
        def __init__(self):
            self.lrs, self.blocks = [], []

        def set_lr(self, lr):
            self.lrs.append(lr)

        def train_step(self, block):
            self.blocks.append(np.array(block))
            return float(len(self.blocks)), 0.5, False

        def get_lr(self):
            return self.lrs[-1] if self.lrs else 3e-4

        def eval_loss(self, tokens):
            self.evaluated = tokens.copy()
            return 1.25

    st = Stand()
    sched = feed.CosineScheduler(1e-3, 2, 20, 1e-4)
    log = tmp_path / "m.jsonl"
    losses = feed.train(st, feed.Dataset(toks), B, T, 100, scheduler=sched,
                        logger=feed.MetricsLogger(str(log)), device_feed=False)
    assert len(losses) == 10  # 10 full steps; the 5-token tail is not a full run
    for s, blk in enumerate(st.blocks):
        assert np.array_equal(blk, toks[s * B * T:(s + 1) * B * T].reshape(B, T))
    assert st.lrs == [sched.get_lr(s) for s in range(10)]
    lines = [json.loads(x) for x in log.read_text().splitlines()]
    assert [x["step"] for x in lines] == list(range(10)) and lines[3]["loss"] == 4
    st2 = Stand()
    printed = []
    assert len(feed.train(st2, feed.Dataset(toks), B, T, 4, device_feed=False,
                          val_ds=feed.Dataset(toks[:300]), eval_interval=2,
                          print_fn=printed.append)) == 4
    assert printed == ["[trainer] step 0 loss 1 lr 0.0003", "[trainer] val loss 1.25",
                       "[trainer] step 2 loss 3 lr 0.0003", "[trainer] val loss 1.25"]
    assert np.array_equal(st2.evaluated, toks[:128][None, :])  # Trainer::evaluate's window
