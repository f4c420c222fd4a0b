"""GPU backend over the C ABI, mirroring the reference's backend contract.

``GpuBackend`` exposes the parts of ``RuntimeBackend``
(crates/leo-core/src/backend.rs:351-475) that the story-batch path uses, with
the same names and argument meaning:

* ``train_story_batch(stories, permission)`` -- the trainer's whole batch
  (crates/leo-cli/src/training.rs:1539-1727): the device story pass, the
  batch-end mean merge and the serial canonical replay, fused;
* ``training_story_batch`` / ``training_story_batch_deltas`` --
  backend.rs:457-474 (no replay; the second keeps each story's delta);
* ``begin_document`` / ``reset_transient_state`` / ``training_step_batch`` /
  ``advance_frozen_batch`` -- the canonical runtime step by step
  (backend.rs:391-431);
* ``enable_parameter_tracking`` / ``parameter_changes`` /
  ``synchronize_packed_model`` -- backend.rs:358-359, 374-376;
* ``synchronize_model()`` / ``model`` -- backend.rs:355-357;
* ``replace_model(model)`` -- ``model_mut`` followed by a canonical upload.

Errors raise :class:`leo_b200.native.LeoError`; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import native
from .configs import Config
from .ctypes_types import (
    CHANGE_LISTS,
    DELTA_TENSORS,
    FROZEN,
    OUTPUT_CLASSES,
    TRAINING,
    UNSUPPORTED,
    LeoB200BatchReport,
    LeoB200PackedUpdate,
    LeoB200ParameterChanges,
    LeoB200ParameterChangeSizes,
    LeoB200Statistics,
    LeoB200StoryDeltas,
    LeoB200StoryDeltaSizes,
    LeoB200StorySummary,
)
from .model import HostModel


@dataclass
class BatchResult:
    report: LeoB200BatchReport
    summaries: list[LeoB200StorySummary]
    losses: list[np.ndarray]


@dataclass
class DeviceStoryBatchReport:
    """DeviceStoryBatchReport (backend.rs:331-336): per-story initial-pass
    losses (``story_metrics``' losses), summaries, replay ranges and the merge
    counts."""

    story_losses: list[np.ndarray]
    story_summaries: list[LeoB200StorySummary]
    replay_ranges: list[list[tuple[int, int]]]
    merge: LeoB200BatchReport


# Tensor order of a story delta (SparseModelDelta, parallel.rs:411-420).
DELTA_NAMES = ("threshold", "recurrent_weight", "input_weight", "output_weight", "output_bias",
               "context_output_weight")


@dataclass
class StoryDelta:
    """One story's SparseModelDelta (parallel.rs:411-459): per tensor, sorted
    indices (output weights as output * neuron_count + neuron) and nonzero
    deltas; keyed context deltas (order, key, observation increment,
    embedding delta); the statistics delta and the revision increment."""

    tensors: dict[str, tuple[np.ndarray, np.ndarray]]
    context_orders: np.ndarray
    context_keys: np.ndarray
    context_observation_increments: np.ndarray
    context_embedding_deltas: np.ndarray  # [entries, embedding_dim]
    statistics: LeoB200Statistics
    revision_increment: int
    changes: "ParameterChanges | None" = None  # the story's tracked indices (story_changes, backend.rs:348)


class StoryDeltaBuffers:
    """Host arrays behind one ``LeoB200StoryDeltas`` (CSR over stories),
    allocated from a ``LeoB200StoryDeltaSizes`` or packed from story deltas."""

    def __init__(self, sizes: LeoB200StoryDeltaSizes):
        n, d = int(sizes.stories), int(sizes.embedding_dim)
        self.sizes = sizes
        self.offsets = [np.zeros(n + 1, np.uint64) for _ in range(DELTA_TENSORS)]
        self.indices = [np.zeros(max(int(sizes.entries[t]), 1), np.uint32) for t in range(DELTA_TENSORS)]
        self.deltas = [np.zeros(max(int(sizes.entries[t]), 1), np.float32) for t in range(DELTA_TENSORS)]
        ce = max(int(sizes.context_entries), 1)
        self.context_offsets = np.zeros(n + 1, np.uint64)
        self.orders, self.keys = np.zeros(ce, np.uint32), np.zeros(ce, np.uint64)
        self.obs, self.emb = np.zeros(ce, np.uint32), np.zeros(ce * max(d, 1), np.float32)
        self.stats = (LeoB200Statistics * max(n, 1))()
        self.revisions = np.zeros(max(n, 1), np.uint64)
        self.change_offsets = [np.zeros(n + 1, np.uint64) for _ in range(CHANGE_LISTS)]
        self.change_indices = [np.zeros(max(int(sizes.changes[i]), 1), np.uint32) for i in range(CHANGE_LISTS)]
        self.dirty = np.zeros(max(n, 1), np.uint32)
        c = LeoB200StoryDeltas()
        for t in range(DELTA_TENSORS):
            c.offsets[t] = self.offsets[t].ctypes.data
            c.indices[t] = self.indices[t].ctypes.data
            c.deltas[t] = self.deltas[t].ctypes.data
        c.context_offsets = self.context_offsets.ctypes.data
        c.context_orders = self.orders.ctypes.data
        c.context_keys = self.keys.ctypes.data
        c.context_observation_increments = self.obs.ctypes.data
        c.context_embedding_deltas = self.emb.ctypes.data
        c.statistics = C.addressof(self.stats)
        c.revision_increments = self.revisions.ctypes.data
        for i in range(CHANGE_LISTS):
            c.change_offsets[i] = self.change_offsets[i].ctypes.data
            c.change_indices[i] = self.change_indices[i].ctypes.data
        c.dirty_flags = self.dirty.ctypes.data
        self.c = c

    @classmethod
    def pack(cls, deltas: list["StoryDelta"], embedding_dim: int) -> "StoryDeltaBuffers":
        sizes = LeoB200StoryDeltaSizes()
        sizes.stories = len(deltas)
        sizes.embedding_dim = embedding_dim
        for t, name in enumerate(DELTA_NAMES):
            sizes.entries[t] = sum(len(sd.tensors[name][0]) for sd in deltas)
        sizes.context_entries = sum(len(sd.context_keys) for sd in deltas)
        b = cls(sizes)
        d = embedding_dim
        for t, name in enumerate(DELTA_NAMES):
            at = 0
            for s, sd in enumerate(deltas):
                idx, val = sd.tensors[name]
                b.offsets[t][s] = at
                b.indices[t][at:at + len(idx)] = idx
                b.deltas[t][at:at + len(idx)] = val
                at += len(idx)
            b.offsets[t][len(deltas)] = at
        at = 0
        for s, sd in enumerate(deltas):
            k = len(sd.context_keys)
            b.context_offsets[s] = at
            b.orders[at:at + k] = sd.context_orders
            b.keys[at:at + k] = sd.context_keys
            b.obs[at:at + k] = sd.context_observation_increments
            b.emb[at * d:(at + k) * d] = np.asarray(sd.context_embedding_deltas, np.float32).reshape(-1)
            C.memmove(C.byref(b.stats[s]), C.byref(sd.statistics), C.sizeof(LeoB200Statistics))
            b.revisions[s] = sd.revision_increment
            at += k
        b.context_offsets[len(deltas)] = at
        return b

    def unpack(self) -> list["StoryDelta"]:
        n, d = int(self.sizes.stories), int(self.sizes.embedding_dim)
        out = []
        for s in range(n):
            tensors = {}
            for t, name in enumerate(DELTA_NAMES):
                lo, hi = int(self.offsets[t][s]), int(self.offsets[t][s + 1])
                tensors[name] = (self.indices[t][lo:hi].copy(), self.deltas[t][lo:hi].copy())
            lo, hi = int(self.context_offsets[s]), int(self.context_offsets[s + 1])
            stats = LeoB200Statistics()
            C.memmove(C.byref(stats), C.byref(self.stats[s]), C.sizeof(stats))
            lists = [self.change_indices[i][int(self.change_offsets[i][s]):int(self.change_offsets[i][s + 1])].copy()
                     for i in range(CHANGE_LISTS)]
            changes = ParameterChanges(*lists, bool(self.dirty[s] & 1), bool(self.dirty[s] & 2))
            out.append(StoryDelta(tensors, self.orders[lo:hi].copy(), self.keys[lo:hi].copy(), self.obs[lo:hi].copy(),
                                  self.emb[lo * d:hi * d].reshape(hi - lo, d).copy(), stats,
                                  int(self.revisions[s]), changes))
        return out


@dataclass
class DeviceStoryBatchDeltaReport(DeviceStoryBatchReport):
    """DeviceStoryBatchDeltaReport (backend.rs:342-349)."""

    story_deltas: list[StoryDelta]


@dataclass
class ParameterChanges:
    """ParameterChanges (runtime.rs:38-46), indices sorted."""

    threshold: np.ndarray
    recurrent_weight: np.ndarray
    input_weight: np.ndarray
    output_neurons: np.ndarray
    context_slots: np.ndarray
    output_bias_dirty: bool
    context_output_dirty: bool


@dataclass
class PackedSparseModelUpdate:
    """PackedSparseModelUpdate (parallel.rs:78-97): canonical values at the
    changed indices, output rows by neuron."""

    threshold_indices: np.ndarray
    threshold_values: np.ndarray
    recurrent_indices: np.ndarray
    recurrent_values: np.ndarray
    input_indices: np.ndarray
    input_values: np.ndarray
    output_neurons: np.ndarray
    output_values_by_neuron: np.ndarray
    context_slots: np.ndarray
    context_keys: np.ndarray
    context_observations: np.ndarray
    context_embeddings: np.ndarray
    output_bias: np.ndarray | None
    context_output_weights: np.ndarray | None
    generation: int
    parameter_revision: int
    statistics: LeoB200Statistics

    @classmethod
    def from_model(cls, model: HostModel, changes: ParameterChanges) -> "PackedSparseModelUpdate":
        """PackedSparseModelUpdate::from_model (parallel.rs:100-194)."""
        a = model.arrays
        n = model.config.neuron_count
        d = model.config.context_embedding_dim

        def pick(name, idx):
            idx = np.asarray(idx, dtype=np.uint32)
            if idx.size and int(idx.max()) >= a[name].size:
                raise native.LeoError(f"{name} sparse index is outside the model")
            return idx, a[name][idx.astype(np.int64)].astype(np.float32)

        ti, tv = pick("threshold", changes.threshold)
        ri, rv = pick("recurrent_weight", changes.recurrent_weight)
        ii, iv = pick("input_weight", changes.input_weight)
        on = np.asarray(changes.output_neurons, dtype=np.uint32)
        if on.size and int(on.max()) >= n:
            raise native.LeoError("output neuron sparse index is outside the model")
        ow = a["output_weight"].reshape(OUTPUT_CLASSES, n)[:, on.astype(np.int64)].T.copy()
        cs = np.asarray(changes.context_slots, dtype=np.uint32)
        if cs.size and int(cs.max()) >= a["context_keys"].size:
            raise native.LeoError("context sparse slot is outside the model")
        ci = cs.astype(np.int64)
        emb = a["context_embeddings"].reshape(-1, d)[ci].copy() if d else np.zeros((cs.size, 0), np.float32)
        stats = LeoB200Statistics()
        C.memmove(C.byref(stats), C.byref(model.statistics), C.sizeof(stats))
        return cls(ti, tv, ri, rv, ii, iv, on, ow.reshape(-1).astype(np.float32), cs,
                   a["context_keys"][ci].copy(), a["context_observations"][ci].copy(), emb.reshape(-1),
                   a["output_bias"].copy() if changes.output_bias_dirty else None,
                   a["context_output_weight"].copy() if changes.context_output_dirty else None,
                   model.generation, model.parameter_revision, stats)

    def apply_to_model(self, model: HostModel) -> None:
        """PackedSparseModelUpdate::apply_to_model (parallel.rs:196-300) on a host model."""
        a = model.arrays
        n = model.config.neuron_count
        d = model.config.context_embedding_dim
        for name, idx, val in (("threshold", self.threshold_indices, self.threshold_values),
                               ("recurrent_weight", self.recurrent_indices, self.recurrent_values),
                               ("input_weight", self.input_indices, self.input_values)):
            if idx.size and int(idx.max()) >= a[name].size:
                raise native.LeoError(f"{name} packed sparse index is outside model")
            a[name][idx.astype(np.int64)] = val
        on = self.output_neurons.astype(np.int64)
        if on.size and int(on.max()) >= n:
            raise native.LeoError("output packed sparse index is outside model")
        a["output_weight"].reshape(OUTPUT_CLASSES, n)[:, on] = self.output_values_by_neuron.reshape(-1,
                                                                                                   OUTPUT_CLASSES).T
        ci = self.context_slots.astype(np.int64)
        a["context_keys"][ci] = self.context_keys
        a["context_observations"][ci] = self.context_observations
        if d:
            a["context_embeddings"].reshape(-1, d)[ci] = self.context_embeddings.reshape(-1, d)
        if self.output_bias is not None:
            a["output_bias"][:] = self.output_bias
        if self.context_output_weights is not None:
            a["context_output_weight"][:] = self.context_output_weights
        model.generation = self.generation
        model.parameter_revision = self.parameter_revision
        stats = LeoB200Statistics()
        C.memmove(C.byref(stats), C.byref(self.statistics), C.sizeof(stats))
        model.statistics = stats


def pack(stories: list[bytes]) -> tuple[np.ndarray, np.ndarray]:
    offsets = np.zeros(len(stories) + 1, dtype=np.uint64)
    offsets[1:] = np.cumsum([len(s) for s in stories])
    data = np.frombuffer(b"".join(stories), dtype=np.uint8).copy() if stories else np.zeros(1, np.uint8)
    if data.size == 0:
        data = np.zeros(1, np.uint8)
    return data, offsets


class GpuBackend:
    """One CUDA device holding a canonical model and up to ``max_lanes`` story lanes."""

    def __init__(self, model: HostModel, device: int = 0, max_lanes: int = 64):
        if model.config.replay_stateful_batch:
            # Streaming replay (one trajectory carried across the selected
            # ranges, crates/leo-cli/src/training.rs:74-90) is a different
            # replay policy from the serial canonical replay built here.
            raise native.LeoError("replay.stateful_batch is not supported by this backend")
        self.config: Config = model.config
        self.device = device
        self.model = model.copy()
        handle = C.c_void_p()
        hm = self.model.view()
        native.check(native.lib().leo_b200_open(device, C.byref(hm), max_lanes, C.byref(handle)))
        self.handle = handle
        self.max_lanes = max_lanes

    def close(self) -> None:
        if getattr(self, "handle", None):
            native.lib().leo_b200_close(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def __enter__(self) -> "GpuBackend":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    # ---------------------------------------------------------------- model
    def synchronize_model(self) -> HostModel:
        hm = self.model.view()
        native.check(native.lib().leo_b200_download_model(self.handle, C.byref(hm)))
        self.model.absorb_scalars(hm)
        return self.model

    def replace_model(self, model: HostModel) -> None:
        self.model = model.copy()
        hm = self.model.view()
        native.check(native.lib().leo_b200_upload_canonical(self.handle, C.byref(hm)))

    def state_digest(self) -> bytes:
        out = (C.c_uint8 * 32)()
        native.check(native.lib().leo_b200_state_digest(self.handle, out))
        return bytes(out)

    @property
    def canonical_tick(self) -> int:
        return native.lib().leo_b200_canonical_tick(self.handle)

    @canonical_tick.setter
    def canonical_tick(self, tick: int) -> None:
        native.check(native.lib().leo_b200_set_canonical_tick(self.handle, tick))

    def set_cluster_sizes(self, story: int = 0, replay: int = 0) -> None:
        native.check(native.lib().leo_b200_set_cluster_sizes(self.handle, story, replay))

    def set_hub_threshold(self, min_in_degree: int, cta_events: int = 0, thread_events: int = 0) -> None:
        native.check(native.lib().leo_b200_set_hub_threshold(self.handle, min_in_degree, cta_events, thread_events))

    def hub_plan(self) -> tuple[int, int]:
        hubs, events = C.c_uint32(), C.c_uint64()
        native.check(native.lib().leo_b200_hub_count(self.handle, C.byref(hubs), C.byref(events)))
        return hubs.value, events.value

    def set_segment_capacity_limit(self, limit: int) -> None:
        """Diagnostic cap on every target's event segment (0: the exact bound)."""
        native.check(native.lib().leo_b200_set_segment_capacity_limit(self.handle, limit))

    def set_story_chunk(self, steps: int) -> None:
        native.check(native.lib().leo_b200_set_story_chunk(self.handle, steps))

    def set_device_context_merge(self, enable: bool) -> None:
        native.check(native.lib().leo_b200_set_device_context_merge(self.handle, 1 if enable else 0))

    def perf_stats(self):
        from .ctypes_types import LeoB200PerfStats

        st = LeoB200PerfStats()
        native.check(native.lib().leo_b200_perf_stats(self.handle, C.byref(st)))
        return st

    def reset_perf_stats(self) -> None:
        native.check(native.lib().leo_b200_reset_perf_stats(self.handle))

    def device_bytes(self) -> int:
        return native.lib().leo_b200_device_bytes(self.handle)

    # ---------------------------------------------------------------- batches
    def train_story_batch(self, stories: list[bytes], permission: int = TRAINING) -> BatchResult:
        """The trainer's whole batch: story pass, mean merge, serial replay
        (crates/leo-cli/src/training.rs:1539-1727)."""
        data, offsets = pack(stories)
        report = LeoB200BatchReport()
        summaries = (LeoB200StorySummary * max(len(stories), 1))()
        total = sum(len(s) + 1 for s in stories if s)
        losses = np.zeros(max(total, 1), dtype=np.float32)
        native.check(native.lib().leo_b200_train_story_batch(
            self.handle, data.ctypes.data, offsets.ctypes.data, len(stories), permission, C.byref(report),
            summaries, losses.ctypes.data))
        return BatchResult(report, list(summaries)[: len(stories)], _split(losses, stories))

    def batch_begin(self, stories: list[bytes], permission: int = TRAINING) -> None:
        self._pending = stories
        data, offsets = pack(stories)
        native.check(native.lib().leo_b200_batch_begin(self.handle, data.ctypes.data, offsets.ctypes.data,
                                                        len(stories), permission))

    def batch_steps(self, count: int) -> int:
        done = C.c_uint32()
        native.check(native.lib().leo_b200_batch_steps(self.handle, count, C.byref(done)))
        return done.value

    def batch_finish(self) -> BatchResult:
        stories = self._pending
        report = LeoB200BatchReport()
        summaries = (LeoB200StorySummary * max(len(stories), 1))()
        total = sum(len(s) + 1 for s in stories if s)
        losses = np.zeros(max(total, 1), dtype=np.float32)
        native.check(native.lib().leo_b200_batch_finish(self.handle, C.byref(report), summaries, losses.ctypes.data))
        return BatchResult(report, list(summaries)[: len(stories)], _split(losses, stories))

    # ---------------------------------------------------------------- RuntimeBackend, trait-shaped
    def _trait_batch(self, entry, stories, permission, *extra):
        data, offsets = pack(stories)
        report = LeoB200BatchReport()
        summaries = (LeoB200StorySummary * max(len(stories), 1))()
        total = sum(len(s) + 1 for s in stories if s)
        losses = np.zeros(max(total, 1), dtype=np.float32)
        counts = np.zeros(max(len(stories), 1), dtype=np.uint32)
        # At most ceil(len * fraction) targets are replayed, in ranges of at
        # least one target: bounded by the targets of the batch.
        ranges = np.zeros(2 * max(total, 1), dtype=np.uint64)
        rc = entry(self.handle, data.ctypes.data, offsets.ctypes.data, len(stories), permission, C.byref(report),
                   summaries, losses.ctypes.data, ranges.ctypes.data, counts.ctypes.data, *extra)
        if rc == UNSUPPORTED:
            return None
        native.check(rc)
        story_ranges, k = [], 0
        for c in counts[: len(stories)]:
            story_ranges.append([(int(ranges[2 * j]), int(ranges[2 * j + 1])) for j in range(k, k + int(c))])
            k += int(c)
        return report, list(summaries)[: len(stories)], _split(losses, stories), story_ranges

    def training_story_batch(self, stories: list[bytes], permission: int = TRAINING) -> DeviceStoryBatchReport | None:
        """RuntimeBackend::training_story_batch (backend.rs:457-463): every
        story on its own lane and the device-local mean merged into the
        canonical model and every lane; the caller replays.  None for fewer
        than two stories (backend.rs:587-589)."""
        out = self._trait_batch(native.lib().leo_b200_training_story_batch, stories, permission)
        if out is None:
            return None
        report, summaries, losses, ranges = out
        return DeviceStoryBatchReport(losses, summaries, ranges, report)

    def training_story_batch_deltas(self, stories: list[bytes],
                                    permission: int = TRAINING) -> DeviceStoryBatchDeltaReport | None:
        """RuntimeBackend::training_story_batch_deltas (backend.rs:468-474):
        each story's private delta against the canonical model, which stays
        unchanged."""
        sizes = LeoB200StoryDeltaSizes()
        out = self._trait_batch(native.lib().leo_b200_training_story_batch_deltas, stories, permission,
                                C.byref(sizes))
        if out is None:
            return None
        report, summaries, losses, ranges = out
        buffers = StoryDeltaBuffers(sizes)
        native.check(native.lib().leo_b200_story_deltas(self.handle, C.byref(buffers.c)))
        return DeviceStoryBatchDeltaReport(losses, summaries, ranges, report, buffers.unpack())

    def begin_document(self) -> None:
        """RuntimeBackend::begin_document (backend.rs:391; runtime.rs:353-355)."""
        native.check(native.lib().leo_b200_begin_document(self.handle))

    def reset_transient_state(self) -> None:
        """RuntimeBackend::reset_transient_state (backend.rs:402; runtime.rs:365-435)."""
        native.check(native.lib().leo_b200_reset_transient_state(self.handle))

    @staticmethod
    def _steps(steps):
        symbols = np.asarray([s for s, _ in steps], dtype=np.uint32)
        targets = np.asarray([-1 if t is None else t for _, t in steps], dtype=np.int32)
        return symbols, targets

    def training_step_batch(self, steps, permission: int = TRAINING) -> list[tuple[float | None, int]]:
        """RuntimeBackend::training_step_batch (backend.rs:413-421): serial
        steps ``(input_symbol, target_symbol or None)`` of the open document on
        the canonical model; per step (loss or None, active neurons)."""
        symbols, targets = self._steps(steps)
        losses = np.zeros(max(len(steps), 1), np.float32)
        active = np.zeros(max(len(steps), 1), np.uint32)
        native.check(native.lib().leo_b200_training_step_batch(self.handle, symbols.ctypes.data, targets.ctypes.data,
                                                                len(steps), permission, losses.ctypes.data,
                                                                active.ctypes.data))
        return [(None if t is None else float(losses[i]), int(active[i])) for i, (_, t) in enumerate(steps)]

    def advance_frozen_batch(self, steps) -> None:
        """RuntimeBackend::advance_frozen_batch (backend.rs:428-431)."""
        symbols, targets = self._steps(steps)
        native.check(native.lib().leo_b200_advance_frozen_batch(self.handle, symbols.ctypes.data,
                                                                 targets.ctypes.data, len(steps)))

    def enable_parameter_tracking(self) -> None:
        """RuntimeBackend::enable_parameter_tracking (backend.rs:358)."""
        native.check(native.lib().leo_b200_enable_parameter_tracking(self.handle))

    def parameter_changes(self) -> ParameterChanges:
        """RuntimeBackend::parameter_changes (backend.rs:359), indices sorted."""
        sizes = LeoB200ParameterChangeSizes()
        native.check(native.lib().leo_b200_parameter_changes(self.handle, C.byref(sizes), None))
        names = ("threshold", "recurrent_weight", "input_weight", "output_neurons", "context_slots")
        arrays = {k: np.zeros(max(int(getattr(sizes, k)), 1), np.uint32) for k in names}
        out = LeoB200ParameterChanges(*(arrays[k].ctypes.data for k in names))
        native.check(native.lib().leo_b200_parameter_changes(self.handle, C.byref(sizes), C.byref(out)))
        return ParameterChanges(*(arrays[k][: int(getattr(sizes, k))].copy() for k in names),
                                bool(sizes.output_bias_dirty), bool(sizes.context_output_dirty))

    def synchronize_packed_model(self, update: PackedSparseModelUpdate) -> None:
        """RuntimeBackend::synchronize_packed_model (backend.rs:374-376)."""
        u, keep = self._packed(update)  # keep: the arrays u points at, alive through the call
        native.check(native.lib().leo_b200_synchronize_packed_model(self.handle, C.byref(u)))
        del keep

    def commit_packed_host_model(self, update: PackedSparseModelUpdate) -> None:
        """RuntimeBackend::commit_packed_host_model (backend.rs:385-387): the
        same writes, the tracking window left open."""
        u, keep = self._packed(update)
        native.check(native.lib().leo_b200_commit_packed_host_model(self.handle, C.byref(u)))
        del keep

    @staticmethod
    def _packed(update: PackedSparseModelUpdate):
        """The C view of a packet and the arrays it points at (kept alive by the caller)."""
        keep = []

        def ptr(a, dtype):
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype=dtype)
            keep.append(a)
            return a.ctypes.data if a.size else None

        u = LeoB200PackedUpdate()
        u.threshold_indices = ptr(update.threshold_indices, np.uint32)
        u.threshold_values = ptr(update.threshold_values, np.float32)
        u.threshold_count = len(update.threshold_indices)
        u.recurrent_indices = ptr(update.recurrent_indices, np.uint32)
        u.recurrent_values = ptr(update.recurrent_values, np.float32)
        u.recurrent_count = len(update.recurrent_indices)
        u.input_indices = ptr(update.input_indices, np.uint32)
        u.input_values = ptr(update.input_values, np.float32)
        u.input_count = len(update.input_indices)
        u.output_neurons = ptr(update.output_neurons, np.uint32)
        u.output_values_by_neuron = ptr(update.output_values_by_neuron, np.float32)
        u.output_count = len(update.output_neurons)
        u.context_slots = ptr(update.context_slots, np.uint32)
        u.context_keys = ptr(update.context_keys, np.uint64)
        u.context_observations = ptr(update.context_observations, np.uint32)
        u.context_embeddings = ptr(update.context_embeddings, np.float32)
        u.context_count = len(update.context_slots)
        u.output_bias = ptr(update.output_bias, np.float32)
        u.context_output_weights = ptr(update.context_output_weights, np.float32)
        u.generation = update.generation
        u.parameter_revision = update.parameter_revision
        u.statistics = update.statistics
        return u, keep

    # ---------------------------------------------------------------- inspection
    CANONICAL_LANE = 0xFFFFFFFF

    def lane_model(self, lane: int) -> HostModel:
        m = HostModel(self.config)
        hm = m.view()
        native.check(native.lib().leo_b200_lane_model(self.handle, lane, C.byref(hm)))
        return m

    def lane_array(self, lane: int, name: str, dtype=np.float32, capacity: int | None = None) -> np.ndarray:
        cap = capacity or max(64 * self.config.neuron_count * max(self.config.synapses_per_neuron, 4), 1 << 16)
        buf = np.zeros(cap, dtype=np.uint8)
        written = C.c_size_t()
        native.check(native.lib().leo_b200_lane_array(self.handle, lane, name.encode(), buf.ctypes.data, cap,
                                                       C.byref(written)))
        return buf[: written.value].view(dtype).copy()


def _split(losses: np.ndarray, stories: list[bytes]) -> list[np.ndarray]:
    out, k = [], 0
    for s in stories:
        n = len(s) + 1 if s else 0
        out.append(losses[k:k + n].copy())
        k += n
    return out
