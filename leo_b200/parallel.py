"""Exact logical-batch data parallelism over several GPUs.

The reference's ``MultiGpuBatchTrainer::train_story_batch``
(crates/leo-cli/src/training.rs:1212-1420) splits a logical batch of stories
into contiguous work-balanced ranges, one per device
(``work_balanced_story_ranges``, training.rs:926-964), runs each range as
independent story lanes, flattens every story's sparse delta back into
canonical story order and applies ONE flat FP64 mean (parallel.rs:715-798),
then replays serially on the canonical model.  The result equals one device
running the whole batch.

Here one process drives one GPU (``torch.distributed``, NCCL between GPUs) and
the batch-end merge is exchanged instead of gathered:

* per-story reports, losses and keyed context deltas are all-gathered (small,
  host objects);
* for each fixed tensor, element marks are MAX-all-reduced so every rank
  builds the same sorted merge list; the FP64 sum over stories in story order
  is a scan over ranks -- rank r receives rank r - 1's partial sums, adds its
  own lanes' deltas in lane order and sends them on -- so the addition order
  is exactly the single-device story order; the last rank forms the merged
  values and broadcasts them;
* every rank runs the identical serial replay (no post-replay broadcast).

``exchange_fixed_tensors`` is written against a small backend protocol so the
host logic is testable on CPU (gloo) with a stand-in backend.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Protocol, Sequence

import numpy as np

from .ctypes_types import FIXED_TENSORS, LeoB200BatchReport, LeoB200ShardStory, LeoB200StorySummary


def story_work(story: bytes) -> int:
    """training.rs:917-923: targets of a story (bytes + 1; 0 when empty)."""
    return 0 if len(story) == 0 else len(story) + 1


def work_balanced_story_ranges(stories: Sequence[bytes], shards: int) -> list[tuple[int, int]]:
    """``work_balanced_story_ranges`` (training.rs:926-964): contiguous
    [start, end) ranges, at most ``shards`` of them, balancing story work."""
    shard_count = min(shards, len(stories))
    if shard_count == 0:
        return []
    ranges: list[tuple[int, int]] = []
    start = 0
    remaining = sum(story_work(s) for s in stories)
    for shard_index in range(shard_count):
        remaining_shards = shard_count - shard_index
        if remaining_shards == 1:
            ranges.append((start, len(stories)))
            break
        max_end = len(stories) - (remaining_shards - 1)
        target = -(-remaining // remaining_shards)  # div_ceil
        end = start
        assigned = 0
        while end < max_end:
            next_work = story_work(stories[end])
            if end > start and assigned >= target:
                break
            assigned += next_work
            end += 1
        if end == start:
            end += 1
            assigned = story_work(stories[start])
        ranges.append((start, end))
        start = end
        remaining = max(remaining - assigned, 0)
    return ranges


class Exchange(Protocol):
    """The collectives the sharded merge needs."""

    rank: int
    world: int

    def all_gather_object(self, obj) -> list: ...
    def all_reduce_max(self, tensor) -> None: ...
    def send(self, tensor, dst: int) -> None: ...
    def recv(self, tensor, src: int) -> None: ...
    def broadcast(self, tensor, src: int) -> None: ...


class TorchExchange:
    """torch.distributed collectives: device tensors on ``group`` (NCCL
    between GPUs, or gloo on CPU), host objects on ``host_group`` (gloo)."""

    def __init__(self, group=None, host_group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.host_group = host_group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def _settle(self, tensor) -> None:
        # The backend's own stream reads these buffers next: finish the collective first.
        if tensor.is_cuda:
            import torch

            torch.cuda.current_stream(tensor.device).synchronize()

    def all_gather_object(self, obj) -> list:
        out = [None] * self.world
        self.dist.all_gather_object(out, obj, group=self.host_group)
        return out

    def all_reduce_max(self, tensor) -> None:
        self.dist.all_reduce(tensor, op=self.dist.ReduceOp.MAX, group=self.group)
        self._settle(tensor)

    def send(self, tensor, dst: int) -> None:
        self.dist.send(tensor, self._global(dst), group=self.group)
        self._settle(tensor)

    def recv(self, tensor, src: int) -> None:
        self.dist.recv(tensor, self._global(src), group=self.group)
        self._settle(tensor)

    def broadcast(self, tensor, src: int) -> None:
        self.dist.broadcast(tensor, self._global(src), group=self.group)
        self._settle(tensor)

    def _global(self, rank: int) -> int:
        return rank if self.group is None else self.dist.get_global_rank(self.group, rank)


class LocalExchange:
    """A world of one rank: every collective is the identity."""

    rank = 0
    world = 1

    def all_gather_object(self, obj) -> list:
        return [obj]

    def all_reduce_max(self, tensor) -> None:
        pass

    def send(self, tensor, dst: int) -> None:
        raise RuntimeError("a one-rank exchange has no peer")

    def recv(self, tensor, src: int) -> None:
        raise RuntimeError("a one-rank exchange has no peer")

    def broadcast(self, tensor, src: int) -> None:
        pass


class TensorBackend(Protocol):
    """Rank-local steps of the fixed-tensor merge (``leo_b200_shard_*``)."""

    def tensor_elements(self, tensor: int) -> int: ...
    def empty(self, count: int, dtype: str): ...
    def marks(self, tensor: int, out) -> None: ...
    def plan(self, tensor: int, marks) -> int: ...
    def accumulate(self, tensor: int, partial, first: bool) -> None: ...
    def finalize(self, tensor: int, partial, values) -> None: ...
    def commit(self, tensor: int, values) -> None: ...


def exchange_fixed_tensors(backend: TensorBackend, ex: Exchange) -> int:
    """The exact batch-end merge of every fixed tensor across ranks; returns
    fixed_parameter_updates (merged elements).  An error on any rank is raised
    on every rank, after the collectives of that tensor completed."""
    updates = 0
    last = ex.world - 1
    for t in range(FIXED_TENSORS):
        marks = backend.empty(backend.tensor_elements(t), "uint8")
        backend.marks(t, marks)
        ex.all_reduce_max(marks)
        count = backend.plan(t, marks)
        updates += count
        if count == 0:
            continue
        partial = backend.empty(count, "float64")
        status = backend.empty(1, "int32")
        status.zero_()
        if ex.rank > 0:
            ex.recv(status, ex.rank - 1)
            ex.recv(partial, ex.rank - 1)
        error = None
        if int(status.item()) == 0:
            try:
                backend.accumulate(t, partial, ex.rank == 0)
            except Exception as e:  # carried to every rank below
                error = e
                status.fill_(1)
        if ex.rank < last:
            ex.send(status, ex.rank + 1)
            ex.send(partial, ex.rank + 1)
        values = backend.empty(count, "float32")
        if ex.rank == last and int(status.item()) == 0:
            try:
                backend.finalize(t, partial, values)
            except Exception as e:
                error = e
                status.fill_(2)
        ex.broadcast(status, last)
        if int(status.item()) != 0:
            raise error if error is not None else RuntimeError(
                f"batch-end merge of fixed tensor {t} failed on another rank")
        ex.broadcast(values, last)
        backend.commit(t, values)
    return updates


@dataclass
class ShardResult:
    report: LeoB200BatchReport
    summaries: list
    losses: list


class DeviceTensorBackend:
    """``TensorBackend`` over a ``GpuBackend`` with torch tensors as buffers."""

    def __init__(self, gpu):
        import torch

        self.gpu = gpu
        self.torch = torch
        self.device = torch.device(f"cuda:{gpu.device}")

    def _lib(self):
        from . import native

        return native.lib()

    def _check(self, rc: int) -> None:
        from . import native

        native.check(rc)

    def tensor_elements(self, tensor: int) -> int:
        n = C.c_size_t()
        self._check(self._lib().leo_b200_shard_tensor_elements(self.gpu.handle, tensor, C.byref(n)))
        return n.value

    def empty(self, count: int, dtype: str):
        return self.torch.empty(max(count, 1), dtype=getattr(self.torch, dtype), device=self.device)

    def marks(self, tensor: int, out) -> None:
        self._check(self._lib().leo_b200_shard_marks(self.gpu.handle, tensor, out.data_ptr()))

    def plan(self, tensor: int, marks) -> int:
        n = C.c_uint32()
        self._check(self._lib().leo_b200_shard_plan(self.gpu.handle, tensor, marks.data_ptr(), C.byref(n)))
        return n.value

    def accumulate(self, tensor: int, partial, first: bool) -> None:
        self._check(self._lib().leo_b200_shard_accumulate(self.gpu.handle, tensor, partial.data_ptr(), int(first)))

    def finalize(self, tensor: int, partial, values) -> None:
        self._check(self._lib().leo_b200_shard_finalize(self.gpu.handle, tensor, partial.data_ptr(),
                                                        values.data_ptr()))

    def commit(self, tensor: int, values) -> None:
        self._check(self._lib().leo_b200_shard_commit(self.gpu.handle, tensor, values.data_ptr()))


def sharded_story_batch(gpu, ex: Exchange, stories: list[bytes], permission: int) -> ShardResult:
    """One logical batch over ``ex.world`` ranks; every rank passes the same
    ``stories`` and ends with the same canonical model."""
    from . import native
    from .backend import pack

    L = native.lib()
    if len(stories) < 2:
        result = gpu.train_story_batch(stories, permission)
        return ShardResult(result.report, result.summaries, result.losses)
    ranges = work_balanced_story_ranges(stories, ex.world)
    first, end = ranges[ex.rank] if ex.rank < len(ranges) else (len(stories), len(stories))
    data, offsets = pack(stories)
    native.check(L.leo_b200_shard_begin(gpu.handle, data.ctypes.data, offsets.ctypes.data, len(stories), first,
                                        end - first, permission))
    count = end - first
    records = (LeoB200ShardStory * max(count, 1))()
    local_targets = sum(story_work(s) for s in stories[first:end])
    losses = np.zeros(max(local_targets, 1), dtype=np.float32)
    ctx_bytes = C.c_size_t()
    native.check(L.leo_b200_shard_local(gpu.handle, records, losses.ctypes.data, C.byref(ctx_bytes)))
    ctx = np.zeros(max(ctx_bytes.value, 1), dtype=np.uint8)
    native.check(L.leo_b200_shard_context(gpu.handle, ctx.ctypes.data, ctx.size))
    # Per-story context blobs: u32 count, then count entries of (16 + 4 D) bytes.
    entry = 16 + 4 * gpu.config.context_embedding_dim
    blobs, pos = [], 0
    for _ in range(count):
        n = int(np.frombuffer(ctx[pos:pos + 4].tobytes(), dtype=np.uint32)[0])
        size = 4 + n * entry
        blobs.append(ctx[pos:pos + size].tobytes())
        pos += size
    local = (first, [bytes(r) for r in records[:count]], losses[:local_targets].tobytes(), blobs)
    gathered = sorted(ex.all_gather_object(local), key=lambda item: item[0])
    all_records = (LeoB200ShardStory * len(stories))()
    all_losses, all_ctx, ctx_offsets = [], [], [0]
    i = 0
    for _, recs, loss_bytes, story_blobs in gathered:
        for r in recs:
            C.memmove(C.byref(all_records[i]), r, C.sizeof(LeoB200ShardStory))
            i += 1
        all_losses.append(np.frombuffer(loss_bytes, dtype=np.float32))
        for b in story_blobs:
            all_ctx.append(b)
            ctx_offsets.append(ctx_offsets[-1] + len(b))
    if i != len(stories):
        raise RuntimeError("sharded batch: story reports do not cover the batch")
    updates = exchange_fixed_tensors(DeviceTensorBackend(gpu), ex)
    loss_arr = np.concatenate(all_losses) if all_losses else np.zeros(1, np.float32)
    ctx_arr = np.frombuffer(b"".join(all_ctx) or b"\0", dtype=np.uint8).copy()
    off_arr = np.array(ctx_offsets, dtype=np.uint64)
    report = LeoB200BatchReport()
    summaries = (LeoB200StorySummary * len(stories))()
    out_losses = np.zeros(max(sum(story_work(s) for s in stories), 1), dtype=np.float32)
    native.check(L.leo_b200_shard_finish(gpu.handle, all_records, loss_arr.ctypes.data, ctx_arr.ctypes.data,
                                         off_arr.ctypes.data, updates, C.byref(report), summaries,
                                         out_losses.ctypes.data))
    split, k = [], 0
    for s in stories:
        n = story_work(s)
        split.append(out_losses[k:k + n].copy())
        k += n
    return ShardResult(report, list(summaries), split)
