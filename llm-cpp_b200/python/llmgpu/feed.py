"""Data feed and training loop around the device step.

Host-side mirror of the reference's feed and loop, with the reference's names and
semantics:
- `CosineScheduler` (src/scheduler.cpp:13-28): linear warmup, then a cosine from base_lr to
  min_lr, optionally restarted `cycles` times; fp32 arithmetic as the reference does it.
  `StepScheduler` (:29-33): base_lr * gamma^(step // step_size).
- `pack_with_eos`, `train_val_split` (src/dataset.cpp:86-115): rows of block_size tokens, the
  last padded with eos_id, with 1/0 masks; a contiguous split at floor(n * train_ratio).
- `Dataset` (src/dataset.cpp:41-58): a flat token stream; `get_batch(idx, n)` is the run
  tokens[idx:idx+n] (shorter at the end). `Dataset.from_file` reads a text file the way the
  reference does with its default tokenizer, which has no merges: one id per byte.
- `DataLoader` (src/dataset.cpp:59-84): runs starting every `batch_size` tokens, in order
  or shuffled with a seed (a numpy permutation: the same set of runs as the reference, not
  the same order as its std::shuffle).
- `PrefetchLoader` (src/prefetch.cpp): a worker thread keeps up to `prefetch` runs ready.
- `MetricsLogger` (src/logging.cpp:49-55): one JSON line per step with the same fields and
  number formatting (6 significant digits).
- `train` (src/trainer.cpp:23-36): the loop. One device step takes B runs of T tokens (the
  reference's train_step_accum over B sequences), with the learning rate of
  `scheduler.get_lr(step)` set before it, as Trainer::train_step_accum does; every
  eval_interval steps the step's loss and rate are printed, with `evaluate` on a
  validation set when one is given.
- `evaluate` (Trainer::evaluate): the loss of the dataset's first min(n, 128) tokens as one
  sequence.

`DeviceFeed` is what the device adds: each step's [B, T] token block is staged in pinned
host memory and copied to the GPU on a copy stream while the previous step runs; the step's
stream waits for that copy only.
"""
import collections
import math
import threading

import numpy as np

_F32 = np.float32


class CosineScheduler:
    """get_lr(step) of the reference's CosineScheduler, in float32."""

    def __init__(self, base_lr, warmup, max_iters, min_lr=0.0, cycles=1):
        self.base_lr = _F32(base_lr)
        self.warmup = int(warmup)
        self.max_iters = int(max_iters)
        self.min_lr = _F32(min_lr)
        self.cycles = int(cycles) if cycles > 0 else 1

    def get_lr(self, step):
        step = int(step)
        if step < self.warmup:
            return float(_F32(self.base_lr * _F32(step)) / _F32(max(self.warmup, 1)))
        span = self.max_iters - self.warmup
        if span <= 0:
            return float(self.min_lr)
        if self.cycles > 1:
            cyc_len = span // self.cycles
            if cyc_len <= 0:
                cyc_len = span
            progress = _F32((step - self.warmup) % cyc_len) / _F32(cyc_len)
        else:
            progress = min(_F32(step - self.warmup) / _F32(span), _F32(1.0))
        c = np.cos(_F32(3.14159265) * _F32(progress), dtype=_F32)
        return float(self.min_lr + (self.base_lr - self.min_lr) * _F32(0.5) * (_F32(1.0) + c))


class StepScheduler:
    """get_lr(step) of the reference's StepScheduler: the power in double, the product in
    float, as std::pow(float, int) and the float return give it."""

    def __init__(self, base_lr, step_size, gamma):
        self.base_lr, self.step_size, self.gamma = _F32(base_lr), int(step_size), _F32(gamma)

    def get_lr(self, step):
        return float(_F32(float(self.base_lr) * float(self.gamma) ** (int(step) // self.step_size)))


def pack_with_eos(tokens, block_size, eos_id):
    """(input rows, mask rows): the tokens in rows of block_size, the last row padded with
    eos_id and masked 0 there."""
    t = np.asarray(tokens, dtype=np.int32).ravel()
    n = -(-t.size // block_size)
    rows = np.full((n, block_size), eos_id, np.int32)
    mask = np.zeros((n, block_size), np.int32)
    rows.ravel()[:t.size] = t
    mask.ravel()[:t.size] = 1
    return rows, mask


def train_val_split(tokens, train_ratio, seed=0):
    """(train, val): the first floor(n * train_ratio) tokens and the rest (the seed is unused,
    as in the reference)."""
    t = np.asarray(tokens, dtype=np.int32).ravel()
    k = int(t.size * float(train_ratio))
    return t[:k], t[k:]


class Dataset:
    """A flat stream of token ids."""

    # what the reference trains on when its text file is missing or empty
    _STUB = "To be, or not to be, that is the question.\n" * 1024

    def __init__(self, tokens, block_size=0):
        self.tokens = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        if self.tokens.size == 0:
            self.tokens = np.zeros(256, np.int32)
        self.block_size = int(block_size)

    @classmethod
    def from_file(cls, path, block_size=0):
        try:
            with open(path, "rb") as f:
                data = f.read()
        except OSError:
            data = b""
        if not data:
            data = cls._STUB.encode()
        return cls(np.frombuffer(data, dtype=np.uint8).astype(np.int32), block_size)

    def size(self):
        return int(self.tokens.size)

    def get_batch(self, idx, batch_size):
        return self.tokens[idx:idx + batch_size]


class DataLoader:
    def __init__(self, ds, batch_size, shuffle=False, seed=0):
        self.ds, self.batch_size, self.shuffle, self.seed = ds, int(batch_size), shuffle, seed
        self._build_order()

    def _build_order(self):
        self.order = np.arange(0, self.ds.size(), self.batch_size, dtype=np.int64)
        if self.shuffle:
            self.order = np.random.default_rng(self.seed).permutation(self.order)
        self.cursor = 0

    def has_next(self):
        return self.cursor < len(self.order)

    def next_batch(self):
        """[run] or [] when the runs are used up."""
        if not self.has_next():
            return []
        b = self.ds.get_batch(int(self.order[self.cursor]), self.batch_size)
        self.cursor += 1
        return [b]

    def reset(self):
        self._build_order()


class PrefetchLoader:
    """Runs in order, produced by a worker thread up to `prefetch` ahead (prefetch 0: made
    on demand). next() returns [run] or [] at the end."""

    def __init__(self, ds, batch_size, prefetch=2):
        self.ds, self.batch_size, self.prefetch = ds, int(batch_size), int(prefetch)
        self._cursor = 0
        self._queue = collections.deque()
        self._cv = threading.Condition()
        self._done = False
        self._stop = False
        self._worker = None
        if self.prefetch > 0:
            self._worker = threading.Thread(target=self._run, daemon=True)
            self._worker.start()

    def _run(self):
        while True:
            with self._cv:
                self._cv.wait_for(lambda: self._stop or len(self._queue) < self.prefetch)
                if self._stop:
                    return
                if self._cursor >= self.ds.size():
                    self._done = True
                    self._cv.notify_all()
                    return
                cur = self._cursor
                self._cursor += self.batch_size
            batch = self.ds.get_batch(cur, self.batch_size)  # outside the lock
            with self._cv:
                self._queue.append(batch)
                if self._cursor >= self.ds.size():
                    self._done = True
                self._cv.notify_all()

    def next(self):
        if self.prefetch == 0:
            if self._cursor >= self.ds.size():
                return []
            b = self.ds.get_batch(self._cursor, self.batch_size)
            self._cursor += self.batch_size
            return [b]
        with self._cv:
            self._cv.wait_for(lambda: self._queue or self._done)
            if not self._queue:
                return []
            b = self._queue.popleft()
            self._cv.notify_all()
            return [b]

    def has_next(self):
        with self._cv:
            return bool(self._queue) or self._cursor < self.ds.size()

    def close(self):
        with self._cv:
            self._stop = True
            self._cv.notify_all()
        if self._worker is not None:
            self._worker.join()


def _num(x):
    """A float as the reference's ostream writes it (6 significant digits, %g style)."""
    return format(float(_F32(x)), ".6g")


class MetricsLogger:
    def __init__(self, path):
        self.path = path

    def log_step(self, step, loss, ppl, lr, grad_norm, tokens_sec):
        with open(self.path, "a") as f:
            f.write('{"step":%d,"loss":%s,"ppl":%s,"lr":%s,"grad_norm":%s,"tokens_sec":%s}\n'
                    % (int(step), _num(loss), _num(ppl), _num(lr), _num(grad_norm),
                       _num(tokens_sec)))


class DeviceFeed:
    """Double-buffered token blocks on the device for Trainer.train_step_device.

    put(i, block) stages step i's int32 [B, T] block in pinned memory and starts its copy on
    the feed's stream once the step that last read that device buffer has finished; get(i)
    makes the trainer's stream wait for the copy and returns the device tensor; release(i),
    called after step i is launched, marks the buffer as read when that step completes."""

    def __init__(self, trainer, B, T, depth=2):
        import torch
        self.torch = torch
        self.B, self.T, self.depth = B, T, depth
        dev = torch.device("cuda", torch.cuda.current_device())
        self.host = [torch.empty((B, T), dtype=torch.int32).pin_memory() for _ in range(depth)]
        self.dev = [torch.empty((B, T), dtype=torch.int32, device=dev) for _ in range(depth)]
        self.copy_stream = torch.cuda.Stream(device=dev)
        self.step_stream = torch.cuda.ExternalStream(trainer.stream(), device=dev)
        self.copied = [torch.cuda.Event() for _ in range(depth)]
        self.read = [torch.cuda.Event() for _ in range(depth)]
        self._staged = [False] * depth
        self._launched = [False] * depth

    def put(self, i, block):
        s = i % self.depth
        if self._staged[s]:
            self.copied[s].synchronize()  # the pinned buffer's last copy has left it
        self.host[s].numpy()[...] = np.asarray(block, dtype=np.int32).reshape(self.B, self.T)
        with self.torch.cuda.stream(self.copy_stream):
            if self._launched[s]:
                self.copy_stream.wait_event(self.read[s])
            self.dev[s].copy_(self.host[s], non_blocking=True)
            self.copied[s].record(self.copy_stream)
        self._staged[s] = True

    def get(self, i):
        s = i % self.depth
        self.step_stream.wait_event(self.copied[s])
        return self.dev[s]

    def release(self, i):
        s = i % self.depth
        self.read[s].record(self.step_stream)
        self._launched[s] = True


def evaluate(trainer, dataset):
    """Trainer::evaluate: the loss of the first min(n, 128) tokens, one sequence."""
    t = dataset.tokens[:128]
    if t.size == 0:
        return 0.0
    return trainer.eval_loss(t[None, :])


def train(trainer, dataset, B, T, max_iters, scheduler=None, logger=None, prefetch=2,
          device_feed=True, log_every=1, val_ds=None, eval_interval=500, print_fn=print):
    """Trainer::train over the device step: each step takes the next B runs of T tokens
    (a short last run ends the loop), sets lr = scheduler.get_lr(step) first, and logs loss,
    perplexity, lr, grad norm and tokens/s. Returns the list of step losses."""
    import time
    loader = PrefetchLoader(dataset, T, prefetch)
    feed = DeviceFeed(trainer, B, T) if device_feed else None

    def next_block():
        runs = []
        for _ in range(B):
            r = loader.next()
            if not r or len(r[0]) < T:
                return None
            runs.append(r[0])
        return np.stack(runs)

    losses = []
    try:
        block = next_block()
        if block is not None and feed:
            feed.put(0, block)
        step = 0
        while block is not None and step < max_iters:
            nxt = next_block() if step + 1 < max_iters else None
            if scheduler is not None:
                trainer.set_lr(scheduler.get_lr(step))
            t0 = time.perf_counter()
            if feed:
                if nxt is not None:
                    feed.put(step + 1, nxt)  # copies while this step runs
                dev = feed.get(step)
                loss, gn, _ = trainer.train_step_device(dev.data_ptr(), B, T)
                feed.release(step)
            else:
                loss, gn, _ = trainer.train_step(block)
            dt = time.perf_counter() - t0
            losses.append(loss)
            lr = scheduler.get_lr(step) if scheduler is not None else trainer.get_lr()
            if logger is not None and step % max(log_every, 1) == 0:
                ppl = math.exp(min(loss, 80.0))
                logger.log_step(step, loss, ppl, lr, gn, B * T / dt if dt > 0 else 0.0)
            if print_fn is not None and eval_interval > 0 and step % eval_interval == 0:
                print_fn(f"[trainer] step {step} loss {_num(loss)} lr {_num(lr)}")
                if val_ds is not None:
                    print_fn(f"[trainer] val loss {_num(evaluate(trainer, val_ds))}")
            block = nxt
            step += 1
    finally:
        loader.close()
    return losses
