"""Host-side failure detection for data-parallel ranks (one process per GPU).

The reference has no collectives: its data parallelism is mean_reduce_grads over shards in
one process (src/trainer.cpp:171-182), so there is no peer to lose. Here every rank is its
own process, and two mechanisms keep a lost peer from hanging the others:

* inside a step, the library bounds every wait for a collective (llmgpu_set_comm_timeout):
  past the bound it aborts the communicator and the step returns LLMGPU_E_NCCL;
* between steps, PeerWatch (below) lets every rank announce the step it is about to run in
  a shared key-value store (torch.distributed's TCPStore or FileStore) and wait, with a
  bound, for every peer's announcement of the same step. A peer that exited, crashed or
  stopped is found there, before any kernel or collective of the next step is launched,
  and the caller gets PeerLost naming the ranks that did not arrive.
"""
import datetime


class PeerLost(RuntimeError):
    """A peer rank did not arrive at a step within the bound."""

    def __init__(self, step, ranks):
        self.step = step
        self.ranks = list(ranks)
        super().__init__(f"rank(s) {self.ranks} did not arrive at step {step}")


class PeerWatch:
    """Per-step arrival check of `world` ranks over a torch.distributed Store."""

    def __init__(self, store, rank, world, timeout_s=30.0, prefix="llmgpu/step"):
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.timeout = datetime.timedelta(seconds=float(timeout_s))
        self.prefix = prefix

    def _key(self, step, rank):
        return f"{self.prefix}/{step}/{rank}"

    def arrive(self, step):
        """Announces `step` and returns once every peer has announced it; raises PeerLost
        with the missing ranks after the timeout."""
        self.store.set(self._key(step, self.rank), "1")
        peers = [r for r in range(self.world) if r != self.rank]
        try:
            self.store.wait([self._key(step, r) for r in peers], self.timeout)
        except Exception:  # the store's timeout error (its type differs between stores)
            missing = [r for r in peers if not self._has(self._key(step, r))]
            raise PeerLost(step, missing or peers) from None
        if step >= 2:  # every peer is past step - 1: nobody waits on step - 2 any more
            try:
                self.store.delete_key(self._key(step - 2, self.rank))
            except Exception:
                pass

    def _has(self, key):
        try:
            return bool(self.store.check([key]))
        except Exception:
            return False
