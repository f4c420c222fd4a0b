"""GPU parity against the oracle (CPU restatement of the reference CPU backend).

Tolerance: exact.  The kernels keep the CPU's FP32 operation order, so lane
state after every step, the merged canonical model after every batch, and
the training_state_hash must be bit-identical (max-abs 0, relative 0).
"""

import numpy as np
import pytest

from leo_b200.configs import WORKLOADS
from leo_b200.ctypes_types import FROZEN, PROVISIONAL, TRAINING, VERIFIED
from leo_b200.synthetic import story_stream
from parity_helpers import compare_lane, story_steps

pytestmark = pytest.mark.gpu


def _backend(model, lanes):
    from leo_b200.backend import GpuBackend

    return GpuBackend(model, device=0, max_lanes=lanes)


def _models(name, oracle_lib):
    from leo_b200.model import HostModel

    wl = WORKLOADS[name]
    hm = HostModel.initialize(wl.config, wl.topology)
    om = oracle_lib.OracleModel.from_arrays(wl.config, hm.arrays)
    return wl, hm, om


@pytest.mark.parametrize("name,steps", [("test", 40), ("baseline1", 60)])
def test_lane_state_matches_oracle_every_step(name, steps, native_lib, oracle_lib):
    wl, hm, om = _models(name, oracle_lib)
    stories = story_stream(11, 2, steps, steps + 5)
    backend = _backend(hm, 2)
    backend.batch_begin(stories, TRAINING)
    runtimes = []
    for story in stories:
        rt = oracle_lib.OracleRuntime(om)
        rt.enable_tracking()
        rt.begin_document()
        runtimes.append(rt)
    schedules = [story_steps(s) for s in stories]
    for s in range(steps):
        backend.batch_steps(1)
        for lane, (rt, sched) in enumerate(zip(runtimes, schedules)):
            sym, tgt = sched[s]
            rt.step(sym, tgt, TRAINING)
            bad = compare_lane(backend, lane, rt, params=(s % 10 == 9))
            assert not bad, f"{name} lane {lane} step {s}: " + "; ".join(bad[:6])
    backend.close()


@pytest.mark.parametrize("name,count,lo,hi", [("test", 4, 8, 40), ("probe", 4, 40, 120), ("baseline1", 4, 64, 160)])
def test_story_batch_matches_oracle_state_hash(name, count, lo, hi, native_lib, oracle_lib):
    wl, hm, om = _models(name, oracle_lib)
    stories = story_stream(3, count, lo, hi)
    backend = _backend(hm, count)
    canonical = oracle_lib.OracleRuntime(om)
    for batch in range(2):
        result = backend.train_story_batch(stories, TRAINING)
        report, losses, ranges = canonical.train_story_batch(stories, TRAINING)
        got = np.concatenate(result.losses)
        assert np.array_equal(got.view(np.uint32), losses.view(np.uint32)), f"batch {batch}: losses differ"
        assert result.report.replay_steps == report.replay_steps
        assert result.report.replay_prefix_steps == report.replay_prefix_steps
        assert result.report.fixed_parameter_updates == report.fixed_parameter_updates
        assert result.report.context_keys == report.context_keys
        gm = backend.synchronize_model()
        cm = canonical.model.arrays()
        bad = [k for k in gm.arrays if not np.array_equal(gm.arrays[k].view(np.uint8), cm[k].view(np.uint8))]
        assert not bad, f"batch {batch}: canonical tensors differ: {bad}"
        assert backend.state_digest() == canonical.model.training_state_hash(), f"batch {batch}: digest differs"
        assert backend.canonical_tick == canonical.tick
    backend.close()


def test_single_story_batch_trains_canonical_directly(native_lib, oracle_lib):
    wl, hm, om = _models("test", oracle_lib)
    story = story_stream(5, 1, 30, 30)
    backend = _backend(hm, 2)
    canonical = oracle_lib.OracleRuntime(om)
    for _ in range(2):
        backend.train_story_batch(story, TRAINING)
        canonical.train_story_batch(story, TRAINING)
        assert backend.state_digest() == canonical.model.training_state_hash()
        assert backend.canonical_tick == canonical.tick
    backend.close()


@pytest.mark.parametrize("permission", [FROZEN, PROVISIONAL, VERIFIED], ids=["frozen", "provisional", "verified"])
def test_story_batch_permissions_match_oracle(permission, native_lib, oracle_lib):
    """Non-training permissions (permission.rs:24-31): frozen batches learn
    nothing and count no story; provisional and verified scale learning by
    their strength.  Losses, report, tensors, digest and tick against the oracle."""
    wl, hm, om = _models("test", oracle_lib)
    stories = story_stream(5, 4, 8, 40)
    backend = _backend(hm, 4)
    canonical = oracle_lib.OracleRuntime(om)
    for batch in range(2):
        result = backend.train_story_batch(stories, permission)
        report, losses, ranges = canonical.train_story_batch(stories, permission)
        got = np.concatenate(result.losses)
        assert np.array_equal(got.view(np.uint32), losses.view(np.uint32)), f"batch {batch}: losses differ"
        assert result.report.replay_steps == report.replay_steps
        assert result.report.fixed_parameter_updates == report.fixed_parameter_updates
        gm = backend.synchronize_model()
        cm = canonical.model.arrays()
        bad = [k for k in gm.arrays if not np.array_equal(gm.arrays[k].view(np.uint8), cm[k].view(np.uint8))]
        assert not bad, f"batch {batch}: canonical tensors differ: {bad}"
        assert backend.state_digest() == canonical.model.training_state_hash(), f"batch {batch}: digest differs"
        assert backend.canonical_tick == canonical.tick
    backend.close()


def test_edge_case_stories_match_oracle(native_lib, oracle_lib):
    """An empty story, a one-byte story, arbitrary bytes 0-255 and a story
    longer than 4,096 steps in one batch, then a single-story frozen batch:
    losses, report, tensors, digest and tick against the oracle."""
    wl, hm, om = _models("test", oracle_lib)
    rng = np.random.default_rng(7)
    stories = [b"", b"x", bytes(rng.integers(0, 256, 300, dtype=np.uint8)),
               bytes(rng.integers(32, 127, 5000, dtype=np.uint8))]
    backend = _backend(hm, 4)
    canonical = oracle_lib.OracleRuntime(om)
    for batch, permission in ((stories, TRAINING), ([stories[2]], FROZEN)):
        result = backend.train_story_batch(batch, permission)
        report, losses, ranges = canonical.train_story_batch(batch, permission)
        got = np.concatenate(result.losses) if result.losses else np.zeros(0, np.float32)
        assert np.array_equal(got.view(np.uint32), losses.view(np.uint32)), "losses differ"
        assert result.report.replay_steps == report.replay_steps
        assert result.report.replay_prefix_steps == report.replay_prefix_steps
        gm = backend.synchronize_model()
        cm = canonical.model.arrays()
        bad = [k for k in gm.arrays if not np.array_equal(gm.arrays[k].view(np.uint8), cm[k].view(np.uint8))]
        assert not bad, f"canonical tensors differ: {bad}"
        assert backend.state_digest() == canonical.model.training_state_hash()
        assert backend.canonical_tick == canonical.tick
    backend.close()


def test_replace_model_restarts_from_the_given_model(native_lib, oracle_lib):
    """replace_model (leo_b200_upload_canonical: the trait's model_mut /
    synchronize flow) puts a host model back on the device and into every
    lane: training the same batch again from the initial model and tick gives
    the same digest; a batch wider than the lanes reserved at open is refused."""
    from leo_b200.native import LeoError

    wl, hm, om = _models("test", oracle_lib)
    stories = story_stream(9, 4, 8, 40)
    backend = _backend(hm, 4)
    backend.train_story_batch(stories, TRAINING)
    first = backend.state_digest()
    backend.train_story_batch(stories, TRAINING)  # moves the lanes and canonical model on
    assert backend.state_digest() != first
    backend.replace_model(hm)
    backend.canonical_tick = 0
    backend.train_story_batch(stories, TRAINING)
    assert backend.state_digest() == first
    with pytest.raises(LeoError, match="lanes"):
        backend.train_story_batch(stories + stories, TRAINING)
    backend.close()
