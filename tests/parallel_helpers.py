"""In-process stand-ins for the multi-rank exchange, used by tests.

``ThreadExchange`` lets several ranks run as threads of one process (each
driving its own backend), exchanging torch tensors through shared memory with
the same semantics as ``leo_b200.parallel.TorchExchange``.
"""

from __future__ import annotations

import threading


class ThreadWorld:
    def __init__(self, world: int):
        self.world = world
        self.barrier = threading.Barrier(world, timeout=600)
        self.slots: dict = {}
        self.lock = threading.Lock()
        self.mail: dict = {}
        self.cond = threading.Condition()

    def exchange(self, rank: int) -> "ThreadExchange":
        return ThreadExchange(self, rank)


class ThreadExchange:
    def __init__(self, world: ThreadWorld, rank: int):
        self.w = world
        self.rank = rank
        self.world = world.world

    def _sync(self):
        import torch

        if torch.cuda.is_available():
            torch.cuda.synchronize()

    def all_gather_object(self, obj) -> list:
        with self.w.lock:
            self.w.slots[("obj", self.rank)] = obj
        self.w.barrier.wait()
        out = [self.w.slots[("obj", r)] for r in range(self.world)]
        self.w.barrier.wait()
        return out

    def all_reduce_max(self, tensor) -> None:
        import torch

        self._sync()
        with self.w.lock:
            self.w.slots[("max", self.rank)] = tensor.clone()
        self._sync()
        self.w.barrier.wait()
        acc = self.w.slots[("max", 0)].clone()
        for r in range(1, self.world):
            acc = torch.maximum(acc, self.w.slots[("max", r)])
        tensor.copy_(acc)
        self._sync()
        self.w.barrier.wait()

    def send(self, tensor, dst: int) -> None:
        self._sync()
        with self.w.cond:
            self.w.mail.setdefault((self.rank, dst), []).append(tensor.clone())
            self._sync()
            self.w.cond.notify_all()

    def recv(self, tensor, src: int) -> None:
        with self.w.cond:
            ok = self.w.cond.wait_for(lambda: self.w.mail.get((src, self.rank)), timeout=600)
            if not ok:
                raise TimeoutError("recv timed out")
            item = self.w.mail[(src, self.rank)].pop(0)
        tensor.copy_(item)
        self._sync()

    def broadcast(self, tensor, src: int) -> None:
        self._sync()
        if self.rank == src:
            with self.w.lock:
                self.w.slots[("bcast",)] = tensor.clone()
            self._sync()
        self.w.barrier.wait()
        if self.rank != src:
            tensor.copy_(self.w.slots[("bcast",)])
            self._sync()
        self.w.barrier.wait()


def run_ranks(world: int, fn):
    """Runs fn(rank, exchange) on `world` threads; re-raises the first error."""
    tw = ThreadWorld(world)
    results = [None] * world
    errors = []

    def body(r):
        try:
            results[r] = fn(r, tw.exchange(r))
        except BaseException as e:  # noqa: BLE001 - reported to the caller
            errors.append(e)
            tw.barrier.abort()

    threads = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=900)
    if errors:
        raise errors[0]
    return results
