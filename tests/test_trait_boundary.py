"""The trait-shaped boundary (RuntimeBackend, crates/leo-core/src/backend.rs:
351-475): story deltas, the canonical runtime step by step, parameter tracking
and the packed sparse sync.

CPU tests port the reference's delta-algebra tests
(crates/leo-core/src/parallel.rs:1406-1497, 1583-1640) onto the oracle and the
host packet type; GPU tests drive the reference trainer's own loop
(crates/leo-cli/src/training.rs:1584-1660, 1833-1945) through the C ABI and
check it against the oracle and the golden fixtures bit for bit.
"""

import ctypes as C
import hashlib
import json
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
GOLDEN = json.loads((HERE / "golden" / "story_batches.json").read_text())
CASES = {c["name"]: c for c in GOLDEN["cases"]}

BEGIN, END = 256, 257


def _stories(case):
    import sys

    from leo_b200.configs import WORKLOADS

    sys.path.insert(0, str(HERE / "golden"))
    from make_golden import case_stories

    return WORKLOADS[case["workload"]], case_stories(case)


def _test_model(oracle_lib):
    from leo_b200.configs import WORKLOADS

    w = WORKLOADS["test"]
    return oracle_lib.OracleModel.initialize(w.config, w.topology)


def _same_delta(a, b):
    from leo_b200.backend import DELTA_NAMES

    for name in DELTA_NAMES:
        ia, da = a.tensors[name]
        ib, db = b.tensors[name]
        assert np.array_equal(ia, ib), name
        assert np.array_equal(da.view(np.uint32), db.view(np.uint32)), name
    order_a = np.lexsort((a.context_keys, a.context_orders))
    order_b = np.lexsort((b.context_keys, b.context_orders))
    assert np.array_equal(a.context_orders[order_a], b.context_orders[order_b])
    assert np.array_equal(a.context_keys[order_a], b.context_keys[order_b])
    assert np.array_equal(a.context_observation_increments[order_a], b.context_observation_increments[order_b])
    assert np.array_equal(a.context_embedding_deltas[order_a].view(np.uint32),
                          b.context_embedding_deltas[order_b].view(np.uint32))
    for field, _ in type(a.statistics)._fields_:
        assert getattr(a.statistics, field) == getattr(b.statistics, field), field
    assert a.revision_increment == b.revision_increment


# ---------------------------------------------------------------- CPU: oracle and host packets
def test_tracked_delta_matches_full_delta_for_one_worker_story(oracle_lib):
    """parallel.rs:1405-1424."""
    from leo_b200.ctypes_types import TRAINING

    base = _test_model(oracle_lib)
    rt = oracle_lib.OracleRuntime(base)
    rt.enable_tracking()
    rt.begin_document()
    rt.step(BEGIN, ord("A"), TRAINING)
    rt.step(ord("A"), END, TRAINING)
    rt.finish_document()
    _same_delta(rt.delta_against(base, tracked=True), rt.delta_against(base, tracked=False))


def test_device_sparse_snapshot_matches_tracked_worker_delta(oracle_lib):
    """parallel.rs:1426-1497: a delta built from the tracked VALUES (what a
    device exports: trained values at the changed indices minus the base)
    equals between_tracked."""
    from leo_b200.backend import StoryDelta
    from leo_b200.ctypes_types import TRAINING

    base = _test_model(oracle_lib)
    rt = oracle_lib.OracleRuntime(base)
    rt.enable_tracking()
    rt.begin_document()
    for symbol, target in ((BEGIN, ord("A")), (ord("A"), ord("B")), (ord("B"), END)):
        rt.step(symbol, target, TRAINING)
    rt.finish_document()
    changes = rt.parameter_changes()
    b, t = base.arrays(), rt.model.arrays()
    n = base.config.neuron_count

    def selected(name, idx):
        idx = np.sort(np.asarray(idx, dtype=np.int64))
        d = (t[name][idx] - b[name][idx]).astype(np.float32)
        keep = d != 0
        return idx[keep].astype(np.uint32), d[keep]

    out_idx = np.sort(np.concatenate([np.arange(257, dtype=np.int64) * n + o for o in changes.output_neurons])
                      if len(changes.output_neurons) else np.zeros(0, np.int64))
    tensors = {
        "threshold": selected("threshold", changes.threshold),
        "recurrent_weight": selected("recurrent_weight", changes.recurrent_weight),
        "input_weight": selected("input_weight", changes.input_weight),
        "output_weight": selected("output_weight", out_idx),
        "output_bias": selected("output_bias", np.arange(257) if changes.output_bias_dirty else []),
        "context_output_weight": selected("context_output_weight",
                                          np.arange(t["context_output_weight"].size)
                                          if changes.context_output_dirty else []),
    }
    expected = rt.delta_against(base, tracked=True)
    observed = StoryDelta(tensors, expected.context_orders, expected.context_keys,
                          expected.context_observation_increments, expected.context_embedding_deltas,
                          expected.statistics, expected.revision_increment)
    _same_delta(observed, expected)
    # The context rows of the changed slots reproduce the keyed context deltas.
    d = base.config.context_embedding_dim
    emb_b = b["context_embeddings"].reshape(-1, d)
    emb_t = t["context_embeddings"].reshape(-1, d)
    for slot in changes.context_slots:
        key = t["context_keys"][slot]
        if b["context_keys"][slot] != key:
            continue  # a slot allocated to a new key: its delta is against no base row
        hit = np.nonzero(expected.context_keys == key)[0]
        delta = (emb_t[slot] - emb_b[slot]).astype(np.float32)
        inc = int(t["context_observations"][slot]) - int(b["context_observations"][slot])
        if hit.size:
            assert np.array_equal(expected.context_embedding_deltas[hit[0]].view(np.uint32), delta.view(np.uint32))
            assert int(expected.context_observation_increments[hit[0]]) == max(inc, 0)
        else:
            assert not delta.any() and inc <= 0


def test_packed_sparse_update_reproduces_selected_canonical_rows(native_lib):
    """parallel.rs:1583-1640 on the host packet type."""
    from leo_b200.backend import ParameterChanges, PackedSparseModelUpdate
    from leo_b200.configs import WORKLOADS
    from leo_b200.model import HostModel

    w = WORKLOADS["test"]
    base = HostModel.initialize(w.config, w.topology)
    canonical = base.copy()
    a = canonical.arrays
    n = w.config.neuron_count
    a["threshold"][0] += np.float32(0.125)
    a["recurrent_weight"][0] *= np.float32(0.5)
    a["input_weight"][0] += np.float32(0.03125)
    for output in range(257):
        a["output_weight"][output * n] += np.float32(output * 1.0e-6)
    a["output_bias"][0] += np.float32(0.25)
    a["context_keys"][0] = 42
    a["context_observations"][0] = 7
    a["context_embeddings"][0] = np.float32(-0.125)
    a["context_output_weight"][0] += np.float32(0.0625)
    canonical.parameter_revision += 3
    canonical.statistics.processed_stories = 9
    changes = ParameterChanges(*(np.array([0], np.uint32) for _ in range(5)), True, True)
    packet = PackedSparseModelUpdate.from_model(canonical, changes)
    replica = base.copy()
    packet.apply_to_model(replica)
    for name in ("threshold", "recurrent_weight", "input_weight", "output_weight", "output_bias", "context_keys",
                 "context_observations", "context_embeddings", "context_output_weight"):
        assert np.array_equal(replica.arrays[name], canonical.arrays[name]), name
    assert replica.parameter_revision == canonical.parameter_revision
    assert replica.statistics.processed_stories == 9
    assert replica.training_state_hash() == canonical.training_state_hash()


def test_packed_sparse_update_rejects_an_index_outside_the_model(native_lib):
    from leo_b200.backend import ParameterChanges, PackedSparseModelUpdate
    from leo_b200.configs import WORKLOADS
    from leo_b200.model import HostModel
    from leo_b200.native import LeoError

    w = WORKLOADS["test"]
    m = HostModel.initialize(w.config, w.topology)
    bad = ParameterChanges(np.array([w.config.neuron_count], np.uint32), *(np.zeros(0, np.uint32) for _ in range(4)),
                           False, False)
    with pytest.raises(LeoError, match="outside the model"):
        PackedSparseModelUpdate.from_model(m, bad)


def test_oracle_story_deltas_mean_is_the_batch_merge(oracle_lib):
    """The CPU branch's merge is the mean of the tracked story deltas: with
    replay off, apply_mean_deltas of rt.story_deltas reproduces
    train_story_batch's model exactly."""
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import TRAINING

    case = CASES["test"]
    w, batches = _stories(case)
    cfg = replace(w.config, replay_fraction=0.0)
    merged = oracle_lib.OracleModel.initialize(cfg, w.topology)
    fused = oracle_lib.OracleRuntime(merged.clone())
    by_deltas = merged.clone()
    for batch in batches:
        rt = oracle_lib.OracleRuntime(by_deltas)
        deltas = rt.story_deltas(batch, TRAINING)
        assert len(deltas) == len(batch)
        report = oracle_lib.apply_story_deltas(by_deltas, deltas)
        fused_report, _, _ = fused.train_story_batch(batch, TRAINING)
        assert fused_report.replay_steps == 0
        assert by_deltas.training_state_hash() == fused.model.training_state_hash()
        assert report.fixed_parameter_updates == fused_report.fixed_parameter_updates
        assert report.context_keys == fused_report.context_keys


def test_trait_entry_points_are_exported(native_lib):
    for name in ("leo_b200_training_story_batch", "leo_b200_training_story_batch_deltas", "leo_b200_story_deltas",
                 "leo_b200_begin_document", "leo_b200_reset_transient_state", "leo_b200_training_step_batch",
                 "leo_b200_advance_frozen_batch", "leo_b200_enable_parameter_tracking",
                 "leo_b200_parameter_changes", "leo_b200_synchronize_packed_model"):
        assert hasattr(native_lib, name), name


# ---------------------------------------------------------------- GPU: through the C ABI
@pytest.mark.gpu
@pytest.mark.parametrize("name", ["test", "test-8", "baseline1"])
def test_gpu_story_deltas_match_oracle(native_lib, oracle_lib, name):
    """Each story's exported delta (training_story_batch_deltas) equals the
    oracle worker's between_tracked delta bit for bit, and its story_changes
    the worker's tracked parameter_changes; the canonical model is
    unchanged by the call, and the oracle's apply_mean_deltas of the GPU's
    deltas reproduces the GPU's own merge (training_story_batch)."""
    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    case = CASES[name]
    w, batches = _stories(case)
    model = HostModel.initialize(w.config, w.topology)
    oracle_model = oracle_lib.OracleModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as gpu:
        for i, batch in enumerate(batches):
            before = gpu.state_digest()
            rep = gpu.training_story_batch_deltas(batch, TRAINING)
            assert gpu.state_digest() == before, f"batch {i}: the deltas call changed the canonical model"
            expected = oracle_lib.OracleRuntime(oracle_model).story_deltas(batch, TRAINING)
            assert len(rep.story_deltas) == len(expected) == len(batch)
            for s, (got, want) in enumerate(zip(rep.story_deltas, expected)):
                try:
                    _same_delta(got, want)
                    # story_changes: the indices the story's lane tracked, as the worker's parameter_changes
                    for field in ("threshold", "recurrent_weight", "input_weight", "output_neurons", "context_slots"):
                        assert np.array_equal(getattr(got.changes, field), getattr(want.changes, field)), field
                    assert got.changes.output_bias_dirty == want.changes.output_bias_dirty
                    assert got.changes.context_output_dirty == want.changes.context_output_dirty
                except AssertionError as e:
                    raise AssertionError(f"batch {i} story {s}: {e}") from e
            merged = gpu.training_story_batch(batch, TRAINING)
            assert merged is not None
            oracle_report = oracle_lib.apply_story_deltas(oracle_model, rep.story_deltas)
            assert gpu.state_digest() == oracle_model.training_state_hash(), f"batch {i}"
            assert merged.merge.fixed_parameter_updates == oracle_report.fixed_parameter_updates
            assert merged.merge.context_keys == oracle_report.context_keys


def _replay_range(gpu, story: bytes, start: int, end: int, permission: int) -> tuple[int, int]:
    """replay_target_range (training.rs:1848-1955) through the trait calls."""
    end = min(end, len(story) + 1)
    gpu.begin_document()
    nxt, prefix_steps, target_steps = start, 0, 0
    if nxt > 0:
        prefix = [(BEGIN, None)] + [(b, None) for b in story[: nxt - 1]]
        gpu.advance_frozen_batch(prefix)
        prefix_steps = len(prefix)
    targets = []
    if nxt == 0:
        targets.append((BEGIN, story[0]))
        nxt = 1
    targets += [(story[p - 1], story[p] if p < len(story) else END) for p in range(nxt, end)]
    metrics = gpu.training_step_batch(targets, permission)
    target_steps = len(metrics)
    gpu.reset_transient_state()
    return prefix_steps, target_steps


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["test", "test-8", "baseline1", "baseline2-short"])
def test_gpu_caller_driven_replay_matches_golden(native_lib, name):
    """The reference trainer's GPU loop (training.rs:1584-1660) driven through
    the trait calls -- device batch without replay, tracking, the serial replay
    of every story's ranges with begin_document / advance_frozen_batch /
    training_step_batch, then parameter_changes and synchronize_packed_model --
    ends every batch at the fused path's golden state hash, tick and counts."""
    from leo_b200.backend import GpuBackend, PackedSparseModelUpdate
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    case = CASES[name]
    w, batches = _stories(case)
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as gpu:
        for i, (rec, batch) in enumerate(zip(case["batches"], batches)):
            rep = gpu.training_story_batch(batch, TRAINING)
            assert rep is not None
            losses = np.concatenate(rep.story_losses).astype("<f4")
            assert hashlib.sha256(losses.tobytes()).hexdigest() == rec["losses_sha256"], f"batch {i}"
            assert [[list(r) for r in s] for s in rep.replay_ranges] == rec["replay_ranges"], f"batch {i}"
            gpu.enable_parameter_tracking()
            prefix_total = target_total = segments = 0
            for story, ranges in zip(batch, rep.replay_ranges):
                for start, end in ranges:
                    if not story or start >= end or start > len(story):
                        continue
                    p, t = _replay_range(gpu, story, start, end, TRAINING)
                    prefix_total += p
                    target_total += t
                segments += len(ranges)
            assert segments == rec["report"]["replay_segments"], f"batch {i}"
            assert target_total == rec["report"]["replay_steps"], f"batch {i}"
            assert prefix_total == rec["report"]["replay_prefix_steps"], f"batch {i}"
            if target_total:
                changes = gpu.parameter_changes()
                update = PackedSparseModelUpdate.from_model(gpu.synchronize_model(), changes)
                gpu.synchronize_packed_model(update)
            assert gpu.state_digest().hex() == rec["state_hash"], f"batch {i}"
            assert gpu.canonical_tick == rec["canonical_tick"], f"batch {i}"
            m = gpu.synchronize_model()
            assert m.parameter_revision == rec["parameter_revision"]
            for k, v in rec["statistics"].items():
                assert getattr(m.statistics, k) == v, (i, k)


@pytest.mark.gpu
def test_gpu_parameter_tracking_matches_oracle(native_lib, oracle_lib):
    """Changed-index sets of the canonical runtime's steps equal the oracle
    runtime's tracked sets (as sets: the device reports them sorted)."""
    from leo_b200.backend import GpuBackend
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import FROZEN, TRAINING
    from leo_b200.model import HostModel

    w = WORKLOADS["test"]
    model = HostModel.initialize(w.config, w.topology)
    om = oracle_lib.OracleModel.initialize(w.config, w.topology)
    rt = oracle_lib.OracleRuntime(om)
    story = b"the quick brown fox jumps over the lazy dog"
    steps = [(BEGIN, story[0])] + [(story[p - 1], story[p] if p < len(story) else END)
                                   for p in range(1, len(story) + 1)]
    with GpuBackend(model, device=0, max_lanes=4) as gpu:
        gpu.enable_parameter_tracking()
        rt.enable_tracking()
        for doc in range(2):
            gpu.begin_document()
            rt.begin_document()
            gpu.advance_frozen_batch(steps[:5])
            for s, t in steps[:5]:
                rt.step(s, t, FROZEN)
            got = gpu.training_step_batch(steps[5:], TRAINING)
            for (s, t), (loss, active) in zip(steps[5:], got):
                m = rt.step(s, t, TRAINING)
                assert np.float32(loss).view(np.uint32) == np.float32(m.loss).view(np.uint32)
                assert active == m.active_neurons
        a, b = gpu.parameter_changes(), rt.parameter_changes()
        for field in ("threshold", "recurrent_weight", "input_weight", "output_neurons", "context_slots"):
            assert np.array_equal(getattr(a, field), np.sort(getattr(b, field))), field
        assert a.output_bias_dirty == b.output_bias_dirty
        assert a.context_output_dirty == b.context_output_dirty
        assert gpu.state_digest() == rt.model.training_state_hash()
        assert gpu.canonical_tick == rt.tick


@pytest.mark.gpu
def test_gpu_packed_sync_reaches_every_lane(native_lib):
    """synchronize_packed_model writes the packet into the canonical model and
    every resident lane; the next batch starts from it."""
    from leo_b200.backend import GpuBackend, ParameterChanges, PackedSparseModelUpdate
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    case = CASES["test"]
    w, batches = _stories(case)
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=4) as gpu:
        gpu.training_story_batch(batches[0], TRAINING)  # makes the lanes resident
        target = gpu.synchronize_model().copy()
        n = w.config.neuron_count
        target.arrays["threshold"][3] += np.float32(0.25)
        target.arrays["output_weight"][7 * n + 5] -= np.float32(0.5)
        target.arrays["output_bias"][1] += np.float32(0.125)
        changes = ParameterChanges(np.array([3], np.uint32), np.zeros(0, np.uint32), np.zeros(0, np.uint32),
                                   np.array([5], np.uint32), np.zeros(0, np.uint32), True, False)
        gpu.synchronize_packed_model(PackedSparseModelUpdate.from_model(target, changes))
        assert gpu.state_digest() == target.training_state_hash()
        for lane in range(4):
            lm = gpu.lane_model(lane)
            for name in ("threshold", "output_weight", "output_bias"):
                assert np.array_equal(lm.arrays[name], target.arrays[name]), (lane, name)


@pytest.mark.gpu
def test_gpu_training_story_batch_declines_one_story(native_lib):
    """backend.rs:587-589: a single story is not a device batch (None); the
    deltas variant takes it."""
    from leo_b200.backend import GpuBackend
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    w = WORKLOADS["test"]
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=2) as gpu:
        before = gpu.state_digest()
        assert gpu.training_story_batch([b"abc"], TRAINING) is None
        assert gpu.state_digest() == before
        rep = gpu.training_story_batch_deltas([b"abc"], TRAINING)
        assert rep is not None and len(rep.story_deltas) == 1
        assert gpu.state_digest() == before


def test_story_delta_buffers_round_trip(native_lib):
    """The CSR layout a caller hands to leo_b200_story_deltas / the oracle's
    apply: packing story deltas and unpacking them gives them back."""
    from leo_b200.backend import DELTA_NAMES, StoryDelta, StoryDeltaBuffers
    from leo_b200.ctypes_types import LeoB200Statistics

    rng = np.random.default_rng(5)
    d = 3
    deltas = []
    for s in range(4):
        tensors = {}
        for name in DELTA_NAMES:
            k = int(rng.integers(0, 6))
            idx = np.sort(rng.choice(1000, size=k, replace=False)).astype(np.uint32)
            tensors[name] = (idx, rng.standard_normal(k).astype(np.float32))
        m = int(rng.integers(0, 3))
        stats = LeoB200Statistics()
        stats.processed_bytes = 10 * s
        stats.training_loss_sum = 0.5 * s
        deltas.append(StoryDelta(tensors, rng.integers(1, 5, m).astype(np.uint32),
                                 rng.integers(1, 2**63, m, dtype=np.uint64), rng.integers(0, 3, m).astype(np.uint32),
                                 rng.standard_normal((m, d)).astype(np.float32), stats, s + 1))
    back = StoryDeltaBuffers.pack(deltas, d).unpack()
    assert len(back) == len(deltas)
    for a, b in zip(deltas, back):
        for name in DELTA_NAMES:
            assert np.array_equal(a.tensors[name][0], b.tensors[name][0])
            assert np.array_equal(a.tensors[name][1], b.tensors[name][1])
        assert np.array_equal(a.context_keys, b.context_keys)
        assert np.array_equal(a.context_orders, b.context_orders)
        assert np.array_equal(a.context_observation_increments, b.context_observation_increments)
        assert np.array_equal(a.context_embedding_deltas, b.context_embedding_deltas)
        assert a.statistics.processed_bytes == b.statistics.processed_bytes
        assert a.statistics.training_loss_sum == b.statistics.training_loss_sum
        assert a.revision_increment == b.revision_increment


@pytest.mark.gpu
def test_gpu_tracking_window_keeps_earlier_changes_for_the_lanes(native_lib):
    """Canonical steps before enable_parameter_tracking still reach the story
    lanes: a batch after (steps, enable) matches a batch after the steps alone."""
    from leo_b200.backend import GpuBackend
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    case = CASES["test"]
    w, batches = _stories(case)
    story = b"a story for the canonical runtime"
    steps = [(BEGIN, story[0])] + [(story[p - 1], story[p] if p < len(story) else END)
                                   for p in range(1, len(story) + 1)]
    digests = []
    for enable in (False, True):
        model = HostModel.initialize(w.config, w.topology)
        with GpuBackend(model, device=0, max_lanes=4) as gpu:
            gpu.train_story_batch(batches[0], TRAINING)  # lanes resident
            gpu.begin_document()
            gpu.training_step_batch(steps, TRAINING)
            if enable:
                gpu.enable_parameter_tracking()
                assert len(gpu.parameter_changes().threshold) == 0
            gpu.train_story_batch(batches[1], TRAINING)
            digests.append(gpu.state_digest())
    assert digests[0] == digests[1]


@pytest.mark.gpu
def test_gpu_commit_packed_host_model_keeps_the_tracking_window(native_lib):
    """commit_packed_host_model writes the packet like synchronize_packed_model
    but leaves the tracked changes in the window; synchronize closes it."""
    from leo_b200.backend import GpuBackend, ParameterChanges, PackedSparseModelUpdate
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    w = WORKLOADS["test"]
    story = b"tracked steps before a commit"
    steps = [(BEGIN, story[0])] + [(story[p - 1], story[p] if p < len(story) else END)
                                   for p in range(1, len(story) + 1)]
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=2) as gpu:
        gpu.enable_parameter_tracking()
        gpu.begin_document()
        gpu.training_step_batch(steps, TRAINING)
        before = gpu.parameter_changes()
        assert len(before.threshold) > 0
        target = gpu.synchronize_model().copy()
        target.arrays["output_bias"][2] += np.float32(0.5)
        none = np.zeros(0, np.uint32)
        packet = PackedSparseModelUpdate.from_model(target, ParameterChanges(none, none, none, none, none, True,
                                                                             False))
        gpu.commit_packed_host_model(packet)
        after = gpu.parameter_changes()
        assert np.array_equal(after.threshold, before.threshold)
        assert gpu.state_digest() == target.training_state_hash()
        gpu.synchronize_packed_model(packet)
        assert len(gpu.parameter_changes().threshold) == 0
        assert gpu.state_digest() == target.training_state_hash()
