"""World-size-2 data-parallel semantics on CPU (gloo), with the oracle as the model.

The device path shards the global batch over ranks (B sequences each) and all-reduces the
mean gradient before a replicated clip + AdamW. That must equal the reference's
train_step_accum over world*B sequences (src/trainer.cpp:127-169) and mean_reduce_grads
(src/trainer.cpp:171-182). Here two gloo ranks run the oracle on their shards, average the
flat gradients with all_reduce, step, and must end with the single-process result.
"""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from oracle import gpt_oracle as go
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = go.Cfg(vocab=64, n_layers=1, n_heads=2, n_embd=32, block_size=16)
    params = go.init_params(cfg, seed=3)
    toks = go.uniform_tokens(64, 4 * 16, seed=4).reshape(4, 16)
    model = go.Model(cfg, params)
    names = [n for n, _ in go.param_specs(cfg)]
    shard = toks[rank * 2:(rank + 1) * 2]
    acc = [np.zeros_like(model.p[n]) for n in names]
    for seq in shard:
        _, G, _ = model.forward_backward(seq)
        for a, n in zip(acc, names):
            a += G[n]
    flat = torch.from_numpy(np.concatenate([a.ravel() / len(shard) for a in acc]))
    dist.all_reduce(flat)
    flat /= world
    grads, off = [], 0
    for n in names:
        k = model.p[n].size
        grads.append(flat[off:off + k].numpy().reshape(model.p[n].shape).copy())
        off += k
    go.clip_by_global_norm(grads, 1.0)
    go.adamw_step([model.p[n] for n in names], grads, go.AdamWState(), go.decay_flags(cfg))
    q.put((rank, np.concatenate([model.p[n].ravel() for n in names])))
    dist.destroy_process_group()


def test_two_rank_mean_allreduce_equals_accumulation():
    import multiprocessing as mp
    from oracle import gpt_oracle as go
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = go.Cfg(vocab=64, n_layers=1, n_heads=2, n_embd=32, block_size=16)
    model = go.Model(cfg, go.init_params(cfg, seed=3))
    toks = go.uniform_tokens(64, 4 * 16, seed=4).reshape(4, 16)
    go.train_step(model, list(toks), go.AdamWState(), clip=1.0)
    want = np.concatenate([model.p[n].ravel() for n, _ in go.param_specs(cfg)])
    np.testing.assert_allclose(out[0], want, rtol=0, atol=1e-9)
    np.testing.assert_array_equal(out[0], out[1])


def _watch_worker(rank, world, port, die_after, q):
    """Runs PeerWatch arrivals for steps 0..4; rank 1 exits abruptly after `die_after` steps."""
    import datetime
    import time
    import torch.distributed as dist
    from llmgpu.dist import PeerLost, PeerWatch
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=30))
    watch = PeerWatch(store, rank, world, timeout_s=2.0)
    for step in range(5):
        if rank == 1 and die_after is not None and step == die_after:
            os._exit(0)  # a peer that stops between steps, with nothing in flight
        t0 = time.time()
        try:
            watch.arrive(step)
        except PeerLost as e:
            q.put((rank, "lost", e.step, e.ranks, time.time() - t0))
            return
    q.put((rank, "ok", 5, [], 0.0))
    if rank == 0:
        time.sleep(1.0)  # the store's host outlives the peers' last calls


def _run_watch(die_after):
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_watch_worker, args=(r, 2, port, die_after, q)) for r in range(2)]
    for p in procs:
        p.start()
    n = 2 if die_after is None else 1
    out = [q.get(timeout=120) for _ in range(n)]
    for p in procs:
        p.join(timeout=60)
    return out, procs


def test_peer_watch_all_ranks_arrive():
    out, procs = _run_watch(None)
    assert sorted(o[:2] for o in out) == [(0, "ok"), (1, "ok")]
    assert all(p.exitcode == 0 for p in procs)


def test_peer_watch_finds_a_killed_peer():
    """Rank 1 exits after two steps: rank 0's arrival at step 2 raises PeerLost([1]) after
    the 2 s bound instead of waiting for good (host-side detection, no device involved)."""
    out, procs = _run_watch(2)
    rank, what, step, ranks, waited = out[0]
    assert (rank, what, step, ranks) == (0, "lost", 2, [1])
    assert 1.5 < waited < 20.0
    assert procs[0].exitcode == 0
