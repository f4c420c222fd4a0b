"""TEST INFRASTRUCTURE ONLY: ctypes binding of the parity oracle.

The oracle (``oracle/leo_oracle.cpp``) restates the reference CPU backend.  This
module is imported only by ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``, as the checker or
the timed CPU baseline -- never by the product package.
"""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

from leo_b200.configs import Config
from leo_b200.ctypes_types import (
    LeoB200BatchReport,
    LeoB200HostModel,
    LeoB200Statistics,
    LeoB200StepMetrics,
    OUTPUT_CLASSES,
    SYMBOL_COUNT,
)

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "libleo_oracle.so"
_lib: C.CDLL | None = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        vp, sz, u64, i64 = C.c_void_p, C.c_size_t, C.c_uint64, C.c_int64
        L.leo_oracle_last_error.restype = C.c_char_p
        L.leo_oracle_config_validate.argtypes = [vp]
        L.leo_oracle_model_initialize.restype = vp
        L.leo_oracle_model_initialize.argtypes = [vp, C.c_int]
        L.leo_oracle_model_from_host.restype = vp
        L.leo_oracle_model_from_host.argtypes = [vp]
        L.leo_oracle_model_free.argtypes = [vp]
        L.leo_oracle_model_clone.restype = vp
        L.leo_oracle_model_clone.argtypes = [vp]
        L.leo_oracle_model_view.argtypes = [vp, vp]
        L.leo_oracle_model_set_scalars.argtypes = [vp, u64, u64, vp]
        L.leo_oracle_model_validate.argtypes = [vp]
        L.leo_oracle_training_state_hash.argtypes = [vp, vp]
        L.leo_oracle_model_state_hash.argtypes = [vp, vp]
        L.leo_oracle_sha256.argtypes = [vp, sz, vp]
        L.leo_oracle_resolve_context_slot.argtypes = [vp, sz, u64, C.c_int, C.POINTER(i64), C.POINTER(u64)]
        L.leo_oracle_runtime_new.restype = vp
        L.leo_oracle_runtime_new.argtypes = [vp]
        L.leo_oracle_runtime_free.argtypes = [vp]
        L.leo_oracle_runtime_model.restype = vp
        L.leo_oracle_runtime_model.argtypes = [vp]
        for name in ("model_changed", "begin_document", "finish_document", "reset", "enable_tracking"):
            getattr(L, f"leo_oracle_runtime_{name}").argtypes = [vp]
        L.leo_oracle_runtime_tick.restype = u64
        L.leo_oracle_runtime_tick.argtypes = [vp]
        L.leo_oracle_runtime_set_tick.argtypes = [vp, u64]
        L.leo_oracle_runtime_step.argtypes = [vp, C.c_uint32, i64, C.c_int, vp]
        L.leo_oracle_runtime_array.argtypes = [vp, C.c_char_p, C.POINTER(vp), C.POINTER(sz), C.POINTER(sz)]
        L.leo_oracle_train_story_batch.argtypes = [vp, vp, vp, sz, C.c_int, sz, vp, vp, vp, vp]
        L.leo_oracle_mean_of_models.argtypes = [vp, vp, sz, C.c_int]
        L.leo_oracle_sparse_mean_apply.argtypes = [vp, sz, vp, vp, vp, sz, C.c_float, C.c_float, C.POINTER(sz)]
        L.leo_oracle_select_replay_ranges.argtypes = [C.c_void_p, sz, C.c_float, sz, vp, sz, C.POINTER(sz)]
        L.leo_oracle_select_block.argtypes = [vp, vp, sz, sz, sz, sz, vp, vp, C.POINTER(sz), C.POINTER(C.c_float)]
        L.leo_oracle_global_order.argtypes = [vp, vp, sz, sz, sz, vp]
        L.leo_oracle_story_deltas.restype = vp
        L.leo_oracle_story_deltas.argtypes = [vp, vp, vp, sz, C.c_int, sz]
        L.leo_oracle_runtime_delta.restype = vp
        L.leo_oracle_runtime_delta.argtypes = [vp, vp, C.c_int]
        L.leo_oracle_deltas_free.argtypes = [vp]
        L.leo_oracle_deltas_sizes.argtypes = [vp, sz, vp]
        L.leo_oracle_deltas_copy.argtypes = [vp, sz, vp]
        L.leo_oracle_apply_story_deltas.argtypes = [vp, vp, vp, C.c_int, vp]
        L.leo_oracle_runtime_parameter_changes.argtypes = [vp, vp, vp]
        L.leo_oracle_last_story_changes.argtypes = [vp, vp, vp]
        _lib = L
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(lib().leo_oracle_last_error().decode())


_DTYPES = {
    "threshold": np.float32, "excitability": np.float32, "neuron_type": np.uint8,
    "recurrent_target": np.uint32, "recurrent_branch": np.uint8, "recurrent_delay": np.uint8,
    "recurrent_weight": np.float32, "input_target": np.uint32, "input_branch": np.uint8,
    "input_weight": np.float32, "output_weight": np.float32, "output_bias": np.float32,
    "context_keys": np.uint64, "context_embeddings": np.float32, "context_observations": np.uint32,
    "context_output_weight": np.float32,
}


def array_sizes(cfg: Config) -> dict[str, int]:
    n, s, f, d = cfg.neuron_count, cfg.synapses_per_neuron, cfg.input_fanout, cfg.context_embedding_dim
    ctx = cfg.context_slots
    return {
        "threshold": n, "excitability": n, "neuron_type": n,
        "recurrent_target": n * s, "recurrent_branch": n * s, "recurrent_delay": n * s, "recurrent_weight": n * s,
        "input_target": SYMBOL_COUNT * f, "input_branch": SYMBOL_COUNT * f, "input_weight": SYMBOL_COUNT * f,
        "output_weight": OUTPUT_CLASSES * n, "output_bias": OUTPUT_CLASSES,
        "context_keys": ctx, "context_embeddings": ctx * d, "context_observations": ctx,
        "context_output_weight": OUTPUT_CLASSES * d,
    }


class OracleModel:
    """An oracle-owned model; ``arrays()`` gives numpy views of its storage."""

    def __init__(self, handle: int, config: Config, owned: bool = True):
        self.handle = handle
        self.config = config
        self.owned = owned

    @classmethod
    def initialize(cls, config: Config, topology: int) -> "OracleModel":
        cc = config.to_c()
        h = lib().leo_oracle_model_initialize(C.byref(cc), topology)
        if not h:
            raise RuntimeError(lib().leo_oracle_last_error().decode())
        return cls(h, config)

    @classmethod
    def from_arrays(cls, config: Config, arrays: dict[str, np.ndarray], generation: int = 0,
                    revision: int = 0, statistics: LeoB200Statistics | None = None) -> "OracleModel":
        hm = LeoB200HostModel()
        hm.config = config.to_c()
        hm.generation = generation
        hm.parameter_revision = revision
        if statistics is not None:
            hm.statistics = statistics
        keep = {}
        for name, dt in _DTYPES.items():
            a = np.ascontiguousarray(arrays[name], dtype=dt)
            keep[name] = a
            ctype = getattr(LeoB200HostModel, name).offset  # noqa: F841 (field exists)
            setattr(hm, name, a.ctypes.data_as(type(getattr(hm, name))))
        h = lib().leo_oracle_model_from_host(C.byref(hm))
        if not h:
            raise RuntimeError(lib().leo_oracle_last_error().decode())
        return cls(h, config)

    def __del__(self):
        if getattr(self, "owned", False) and self.handle:
            lib().leo_oracle_model_free(self.handle)
            self.handle = None

    def clone(self) -> "OracleModel":
        return OracleModel(lib().leo_oracle_model_clone(self.handle), self.config)

    def view(self) -> LeoB200HostModel:
        hm = LeoB200HostModel()
        lib().leo_oracle_model_view(self.handle, C.byref(hm))
        return hm

    def arrays(self) -> dict[str, np.ndarray]:
        hm = self.view()
        out = {}
        for name, size in array_sizes(self.config).items():
            ptr = getattr(hm, name)
            out[name] = np.ctypeslib.as_array(ptr, shape=(size,)) if size else np.zeros(0, _DTYPES[name])
        return out

    def scalars(self) -> tuple[int, int, LeoB200Statistics]:
        hm = self.view()
        return hm.generation, hm.parameter_revision, hm.statistics

    def set_scalars(self, generation: int, revision: int, stats: LeoB200Statistics) -> None:
        lib().leo_oracle_model_set_scalars(self.handle, generation, revision, C.byref(stats))

    def validate(self) -> None:
        _check(lib().leo_oracle_model_validate(self.handle))

    def training_state_hash(self) -> bytes:
        out = (C.c_uint8 * 32)()
        lib().leo_oracle_training_state_hash(self.handle, out)
        return bytes(out)

    def model_state_hash(self) -> bytes:
        out = (C.c_uint8 * 32)()
        lib().leo_oracle_model_state_hash(self.handle, out)
        return bytes(out)


class OracleRuntime:
    """CPU runtime (runtime.rs:112-186) over a private copy of a model."""

    def __init__(self, model: OracleModel):
        h = lib().leo_oracle_runtime_new(model.handle)
        if not h:
            raise RuntimeError(lib().leo_oracle_last_error().decode())
        self.handle = h
        self.config = model.config
        self.model = OracleModel(lib().leo_oracle_runtime_model(h), model.config, owned=False)

    def __del__(self):
        if getattr(self, "handle", None):
            lib().leo_oracle_runtime_free(self.handle)
            self.handle = None

    def step(self, symbol: int, target: int | None, permission: int) -> LeoB200StepMetrics:
        m = LeoB200StepMetrics()
        _check(lib().leo_oracle_runtime_step(self.handle, symbol, -1 if target is None else target, permission,
                                            C.byref(m)))
        return m

    def begin_document(self) -> None:
        lib().leo_oracle_runtime_begin_document(self.handle)

    def finish_document(self) -> None:
        lib().leo_oracle_runtime_finish_document(self.handle)

    def reset(self) -> None:
        lib().leo_oracle_runtime_reset(self.handle)

    def enable_tracking(self) -> None:
        lib().leo_oracle_runtime_enable_tracking(self.handle)

    def model_changed(self) -> None:
        lib().leo_oracle_runtime_model_changed(self.handle)

    @property
    def tick(self) -> int:
        return lib().leo_oracle_runtime_tick(self.handle)

    @tick.setter
    def tick(self, value: int) -> None:
        lib().leo_oracle_runtime_set_tick(self.handle, value)

    def array(self, name: str) -> np.ndarray:
        ptr, es, cnt = C.c_void_p(), C.c_size_t(), C.c_size_t()
        _check(lib().leo_oracle_runtime_array(self.handle, name.encode(), C.byref(ptr), C.byref(es), C.byref(cnt)))
        n = cnt.value
        if n == 0:
            return np.zeros(0, dtype=np.uint64 if es.value == 8 else np.float32)
        buf = (C.c_uint8 * (n * es.value)).from_address(ptr.value)
        raw = np.frombuffer(buf, dtype=np.uint8).copy()
        if name in ("refractory_until", "branch_last_tick", "neuron_last_tick", "rec_last_tick", "input_last_tick"):
            return raw.view(np.uint64)
        if es.value == 8:
            return raw.view(np.uint64)
        if name == "context_history":
            return raw.view(np.uint32)
        return raw.view(np.float32)

    def train_story_batch(self, stories: list[bytes], permission: int, threads: int = 0):
        data = np.frombuffer(b"".join(stories), dtype=np.uint8).copy()
        offsets = np.zeros(len(stories) + 1, dtype=np.uint64)
        offsets[1:] = np.cumsum([len(s) for s in stories])
        report = LeoB200BatchReport()
        total_targets = sum(len(s) + 1 for s in stories if s)  # an empty story has no steps
        losses = np.zeros(max(total_targets, 1), dtype=np.float32)
        max_ranges = total_targets + len(stories)
        ranges = np.zeros(2 * max(max_ranges, 1), dtype=np.uint64)
        counts = np.zeros(len(stories), dtype=np.uint64)
        _check(lib().leo_oracle_train_story_batch(
            self.handle, data.ctypes.data, offsets.ctypes.data, len(stories), permission, threads,
            C.byref(report), losses.ctypes.data, ranges.ctypes.data, counts.ctypes.data))
        split, k = [], 0
        for i in range(len(stories)):
            c = int(counts[i])
            split.append([(int(ranges[2 * (k + j)]), int(ranges[2 * (k + j) + 1])) for j in range(c)])
            k += c
        return report, losses[:total_targets], split


    def story_deltas(self, stories: list[bytes], permission: int, threads: int = 0):
        """Each story's tracked delta against this runtime's model (the CPU
        branch's workers, training.rs:1667-1695); the model is unchanged."""
        data = np.frombuffer(b"".join(stories), dtype=np.uint8).copy() if any(stories) else np.zeros(1, np.uint8)
        offsets = np.zeros(len(stories) + 1, dtype=np.uint64)
        offsets[1:] = np.cumsum([len(s) for s in stories])
        h = lib().leo_oracle_story_deltas(self.handle, data.ctypes.data, offsets.ctypes.data, len(stories),
                                          permission, threads)
        deltas = _take_deltas(h, self.config.context_embedding_dim)
        # each story's tracked ParameterChanges (lists sorted)
        from leo_b200.backend import ParameterChanges

        n = len(stories)
        counts = np.zeros(max(n * 5, 1), np.uint64)
        dirty = np.zeros(max(n, 1), np.uint32)
        _check(lib().leo_oracle_last_story_changes(counts.ctypes.data, dirty.ctypes.data, None))
        per_list = [np.zeros(max(int(counts[l::5][:n].sum()), 1), np.uint32) for l in range(5)]
        table = (C.c_void_p * 5)(*[a.ctypes.data for a in per_list])
        _check(lib().leo_oracle_last_story_changes(None, None, table))
        at = [0] * 5
        for s, d in enumerate(deltas):
            lists = []
            for l in range(5):
                c = int(counts[s * 5 + l])
                lists.append(per_list[l][at[l]:at[l] + c].copy())
                at[l] += c
            d.changes = ParameterChanges(*lists, bool(dirty[s] & 1), bool(dirty[s] & 2))
        return deltas

    def delta_against(self, base: OracleModel, tracked: bool):
        """SparseModelDelta::between_tracked (with this runtime's parameter
        changes) or ::between of this runtime's model against ``base``."""
        h = lib().leo_oracle_runtime_delta(base.handle, self.handle, 1 if tracked else 0)
        return _take_deltas(h, self.config.context_embedding_dim)[0]

    def parameter_changes(self):
        """Runtime::parameter_changes (runtime.rs:322-333), in first-change order."""
        from leo_b200.backend import ParameterChanges
        from leo_b200.ctypes_types import LeoB200ParameterChanges, LeoB200ParameterChangeSizes

        sizes = LeoB200ParameterChangeSizes()
        _check(lib().leo_oracle_runtime_parameter_changes(self.handle, C.byref(sizes), None))
        names = ("threshold", "recurrent_weight", "input_weight", "output_neurons", "context_slots")
        arrays = {k: np.zeros(max(int(getattr(sizes, k)), 1), np.uint32) for k in names}
        out = LeoB200ParameterChanges(*(arrays[k].ctypes.data for k in names))
        _check(lib().leo_oracle_runtime_parameter_changes(self.handle, C.byref(sizes), C.byref(out)))
        return ParameterChanges(*(arrays[k][: int(getattr(sizes, k))].copy() for k in names),
                                bool(sizes.output_bias_dirty), bool(sizes.context_output_dirty))


def _take_deltas(h, embedding_dim: int):
    from leo_b200.backend import StoryDeltaBuffers
    from leo_b200.ctypes_types import LeoB200StoryDeltaSizes

    if not h:
        raise RuntimeError(lib().leo_oracle_last_error().decode())
    try:
        sizes = LeoB200StoryDeltaSizes()
        _check(lib().leo_oracle_deltas_sizes(h, embedding_dim, C.byref(sizes)))
        buffers = StoryDeltaBuffers(sizes)
        _check(lib().leo_oracle_deltas_copy(h, embedding_dim, C.byref(buffers.c)))
        return buffers.unpack()
    finally:
        lib().leo_oracle_deltas_free(h)


def apply_story_deltas(model: OracleModel, deltas, sum_instead: bool = False) -> LeoB200BatchReport:
    """apply_mean_deltas / apply_sum_deltas (parallel.rs:694-798) of story
    deltas (``leo_b200.backend.StoryDelta``) produced from ``model``."""
    from leo_b200.backend import StoryDeltaBuffers

    buffers = StoryDeltaBuffers.pack(list(deltas), model.config.context_embedding_dim)
    merge = LeoB200BatchReport()
    _check(lib().leo_oracle_apply_story_deltas(model.handle, C.byref(buffers.sizes), C.byref(buffers.c),
                                               1 if sum_instead else 0, C.byref(merge)))
    return merge


def select_block(candidates, keep: int, rotation: int, neuron_count: int):
    """A block's winners [(value, neuron)] in rank order and its cutoff
    (runtime.rs:964-997) from candidates [(value, neuron)]."""
    values = np.asarray([v for v, _ in candidates] or [0.0], dtype=np.float32)
    neurons = np.asarray([n for _, n in candidates] or [0], dtype=np.uint32)
    winners = np.zeros(max(len(candidates), 1), np.uint32)
    wvals = np.zeros(max(len(candidates), 1), np.float32)
    count, cutoff = C.c_size_t(), C.c_float()
    lib().leo_oracle_select_block(values.ctypes.data, neurons.ctypes.data, len(candidates), keep, rotation,
                                  neuron_count, winners.ctypes.data, wvals.ctypes.data, C.byref(count),
                                  C.byref(cutoff))
    return [(float(wvals[i]), int(winners[i])) for i in range(count.value)], float(cutoff.value)


def global_order(candidates, rotation: int, neuron_count: int) -> list:
    """Candidates [(value, neuron)] in the global cap's rank order (runtime.rs:1014-1030)."""
    values = np.asarray([v for v, _ in candidates] or [0.0], dtype=np.float32)
    neurons = np.asarray([n for _, n in candidates] or [0], dtype=np.uint32)
    order = np.zeros(max(len(candidates), 1), np.uint32)
    lib().leo_oracle_global_order(values.ctypes.data, neurons.ctypes.data, len(candidates), rotation, neuron_count,
                                  order.ctypes.data)
    return [candidates[int(i)] for i in order[: len(candidates)]]


def select_replay_ranges(losses: np.ndarray, fraction: float, segment: int) -> list[tuple[int, int]]:
    losses = np.ascontiguousarray(losses, dtype=np.float32)
    out = np.zeros(2 * (len(losses) + 1), dtype=np.uint64)
    cnt = C.c_size_t()
    lib().leo_oracle_select_replay_ranges(losses.ctypes.data, len(losses), fraction, segment, out.ctypes.data,
                                          len(losses) + 1, C.byref(cnt))
    return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(cnt.value)]


def sparse_mean_apply(target: np.ndarray, indices: np.ndarray, deltas: np.ndarray, offsets: np.ndarray,
                      lo: float, hi: float) -> int:
    """apply_sparse_scaled (parallel.rs:975-1022) + clamp, in place on ``target``."""
    t = np.ascontiguousarray(target, dtype=np.float32)
    idx = np.ascontiguousarray(indices, dtype=np.uint32)
    dl = np.ascontiguousarray(deltas, dtype=np.float32)
    off = np.ascontiguousarray(offsets, dtype=np.uint64)
    updates = C.c_size_t()
    _check(lib().leo_oracle_sparse_mean_apply(t.ctypes.data, t.size, idx.ctypes.data, dl.ctypes.data, off.ctypes.data,
                                              off.size - 1, lo, hi, C.byref(updates)))
    target[...] = t
    return updates.value


def shuffled_story_order(count: int, seed: int, pass_index: int) -> np.ndarray:
    """shuffled_story_order (crates/leo-cli/src/training/dataset.rs:9-13)."""
    out = np.zeros(max(count, 1), dtype=np.uint64)
    lib().leo_oracle_shuffled_story_order(C.c_uint64(count), C.c_uint64(seed % 2**64), C.c_uint64(pass_index % 2**64),
                                          out.ctypes.data_as(C.c_void_p))
    return out[:count]


def sha256(data: bytes) -> bytes:
    out = (C.c_uint8 * 32)()
    buf = np.frombuffer(data, dtype=np.uint8).copy() if data else np.zeros(1, np.uint8)
    lib().leo_oracle_sha256(buf.ctypes.data, len(data), out)
    return bytes(out)
