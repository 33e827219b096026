"""Data parallelism on 2 GPUs: one process per GPU, NCCL all-reduce (average) of the flat
gradient arena inside llmgpu_train_step.

After two steps on different shards, both ranks must hold identical weights, and those must
match a single GPU training on the concatenated batch (train_step_accum with K = world*B,
src/trainer.cpp:127-169) up to the all-reduce's summation order.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

CFG = dict(vocab_size=256, n_layers=2, n_heads=4, n_embd=128, block_size=64)
B, T = 2, 64


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tokens(world):
    rng = np.random.default_rng(5)
    return rng.integers(0, CFG["vocab_size"], size=(2, world * B, T)).astype(np.int32)


def _worker(rank, world, port, q):
    import datetime
    import sys
    import torch.distributed as dist
    root = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    sys.path.insert(0, os.path.join(root, "llm-cpp_b200", "python"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from llmgpu.trainer import Trainer, make_config, unique_id
    obj = [unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    tr = Trainer(make_config(**CFG), B, T, rank=rank, world=world, uid=obj[0])
    tr.set_adamw()
    tr.set_train(grad_clip=1.0)
    toks = _tokens(world)
    tr.train_step(toks[0, rank * B:(rank + 1) * B])
    grads = [tr.get_grad(i) for i in range(tr.num_params())]
    tr.train_step(toks[1, rank * B:(rank + 1) * B])
    q.put((rank, grads, [tr.get_param(i) for i in range(tr.num_params())]))
    tr.close()
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_data_parallel_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, grads, params = q.get(timeout=300)
        res[rank] = (grads, params)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # replicated optimizer: every rank ends with the same weights, bit for bit
    for a, b in zip(res[0][1], res[1][1]):
        np.testing.assert_array_equal(a, b)
    # the all-reduced gradient equals the single-GPU gradient of the whole global batch
    from llmgpu.trainer import Trainer, make_config
    torch.cuda.set_device(0)
    one = Trainer(make_config(**CFG), world * B, T)
    one.set_adamw()
    one.set_train(grad_clip=1.0)
    one.train_step(_tokens(world)[0])
    for i, a in enumerate(res[0][0]):
        b = one.get_grad(i)
        rel = np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b), 1e-30)
        assert rel < 1e-3, (one.param_info(i)[0], rel)
    one.close()


def _stall_worker(rank, world, port, q):
    """Two steps together; then rank 1 leaves between steps (its process exits with nothing in
    flight) while rank 0 (a) finds it missing through PeerWatch before launching again, (b)
    ends its communicator with nothing in flight and (c) gets an error at once for the next
    step, with its parameters still readable."""
    import datetime
    import sys
    import time
    import torch.distributed as dist
    root = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    sys.path.insert(0, os.path.join(root, "llm-cpp_b200", "python"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from llmgpu.dist import PeerLost, PeerWatch
    from llmgpu.trainer import LlmgpuError, Trainer, make_config, unique_id
    obj = [unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    tr = Trainer(make_config(**CFG), B, T, rank=rank, world=world, uid=obj[0])
    tr.set_adamw()
    tr.set_train(grad_clip=1.0)
    watch = PeerWatch(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=5.0,
                      prefix="t/step")
    toks = _tokens(world)
    for s in range(2):
        watch.arrive(s)
        tr.train_step(toks[s, rank * B:(rank + 1) * B])  # returns with the step complete
    if rank == 1:
        q.put((rank, {}))
        q.close()
        q.join_thread()
        os._exit(0)  # gone between steps: no kernel or collective of this rank in flight
    res = {}
    t0 = time.time()
    try:
        watch.arrive(2)
        res["watch"] = "arrived"
    except PeerLost as e:
        res["watch"] = ("lost", e.ranks, time.time() - t0)
    if res["watch"] != "arrived":
        tr.abort_comm()  # nothing in flight: step 2 has not been launched
    t0 = time.time()
    try:
        tr.train_step(toks[0, :B])
        res["step"] = "completed"
    except LlmgpuError as e:
        res["step"] = ("error", str(e), time.time() - t0)
    res["param_ok"] = bool(np.isfinite(tr.get_param(0)).all())
    tr.close()
    q.put((rank, res))


def test_lost_peer_is_found_between_steps():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_stall_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=400) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    r0 = res[0]
    assert r0["watch"][0] == "lost" and r0["watch"][1] == [1], r0
    assert r0["step"][0] == "error" and "aborted" in r0["step"][1], r0
    assert r0["step"][2] < 1.0, r0
    assert r0["param_ok"]
