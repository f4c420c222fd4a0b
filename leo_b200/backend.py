"""GPU backend over the C ABI, mirroring the reference's backend contract.

``GpuBackend`` exposes the parts of ``RuntimeBackend``
(crates/leo-core/src/backend.rs:351-475) that the story-batch path uses, with
the same names and argument meaning:

* ``training_story_batch(stories, permission)`` -- backend.rs:457-463 together
  with the batch-end mean merge and serial replay of
  crates/leo-cli/src/training.rs:1539-1727;
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
from .ctypes_types import LeoB200BatchReport, LeoB200HostModel, LeoB200StorySummary, TRAINING
from .model import HostModel


@dataclass
class BatchResult:
    report: LeoB200BatchReport
    summaries: list[LeoB200StorySummary]
    losses: list[np.ndarray]


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
    def training_story_batch(self, stories: list[bytes], permission: int = TRAINING) -> BatchResult:
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
