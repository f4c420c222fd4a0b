"""Golden story-batch fixtures (``tests/golden/story_batches.json``, made by
``tests/golden/make_golden.py`` from the oracle).

The CPU test pins the oracle and the synthetic story generator against the
committed records; the GPU test checks the product path through the public
``GpuBackend.train_story_batch`` (the C-ABI ``leo_b200_train_story_batch``)
against the same records: bit-exact state hash, per-target losses, batch
report counts, revision, statistics and canonical tick.
"""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
GOLDEN = json.loads((HERE / "golden" / "story_batches.json").read_text())
CASES = {c["name"]: c for c in GOLDEN["cases"]}


def _stories(case):
    import sys

    from leo_b200.configs import WORKLOADS

    sys.path.insert(0, str(HERE / "golden"))
    from make_golden import case_stories

    return WORKLOADS[case["workload"]], case_stories(case)


@pytest.mark.parametrize("name", sorted(CASES))
def test_synthetic_stories_match_golden(name):
    case = CASES[name]
    _, batches = _stories(case)
    for rec, batch in zip(case["batches"], batches):
        assert hashlib.sha256(b"".join(batch)).hexdigest() == rec["stories_sha256"]
        assert [len(s) for s in batch] == rec["story_lengths"]


# The baseline3-sized and the bench-scale ("-full") cases take the oracle
# minutes to an hour; their fixtures are the oracle's output when
# make_golden.py writes them, and they are checked against the GPU below.
ORACLE_RECHECK = sorted(n for n in CASES if not n.startswith("baseline3") and not n.endswith("-full"))


@pytest.mark.parametrize("name", ORACLE_RECHECK)
def test_oracle_matches_golden(oracle_lib, name):
    from leo_b200.ctypes_types import TRAINING

    case = CASES[name]
    w, batches = _stories(case)
    rt = oracle_lib.OracleRuntime(oracle_lib.OracleModel.initialize(w.config, w.topology))
    assert rt.model.training_state_hash().hex() == case["initial_state_hash"]
    for rec, batch in zip(case["batches"], batches):
        report, losses, ranges = rt.train_story_batch(batch, TRAINING, 0)
        assert rt.model.training_state_hash().hex() == rec["state_hash"]
        assert hashlib.sha256(losses.astype("<f4").tobytes()).hexdigest() == rec["losses_sha256"]
        assert [[list(r) for r in s] for s in ranges] == rec["replay_ranges"]
        for k, v in rec["report"].items():
            assert int(getattr(report, k)) == v, k
        assert rt.tick == rec["canonical_tick"]


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_gpu_story_batch_matches_golden(native_lib, name):
    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    case = CASES[name]
    w, batches = _stories(case)
    model = HostModel.initialize(w.config, w.topology)
    assert model.training_state_hash().hex() == case["initial_state_hash"]
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as backend:
        for i, (rec, batch) in enumerate(zip(case["batches"], batches)):
            result = backend.train_story_batch(batch, TRAINING)
            assert backend.state_digest().hex() == rec["state_hash"], f"batch {i}"
            losses = np.concatenate(result.losses).astype("<f4")
            assert hashlib.sha256(losses.tobytes()).hexdigest() == rec["losses_sha256"], f"batch {i}"
            for k, v in rec["report"].items():
                assert int(getattr(result.report, k)) == v, (i, k)
            assert backend.canonical_tick == rec["canonical_tick"]
            m = backend.synchronize_model()
            assert m.parameter_revision == rec["parameter_revision"]
            for k, v in rec["statistics"].items():
                got = getattr(m.statistics, k)
                assert (got == v) if k != "training_loss_sum" else got == pytest.approx(v, rel=0, abs=0), (i, k)


@pytest.mark.gpu
@pytest.mark.parametrize("geometry,case_name", [
    ((1, 1, 64), "baseline1"), ((4, 16, 64), "baseline1"), ((0, 2, 7), "baseline1"), ((0, 0, 1), "baseline1"),
    ((0, 0xFFFFFFFF, 32), "baseline1"), ((0, 0xFFFFFFFF, 32), "baseline3-short"), ((2, 0xFFFFFFFF, 16), "test-8"),
], ids=["fixed1", "fixed4-replay16", "adaptive-chunk7", "adaptive-chunk1", "whole-gpu-replay",
        "whole-gpu-replay-hubs", "whole-gpu-replay-test8"])
def test_gpu_result_does_not_depend_on_geometry(native_lib, geometry, case_name):
    """Cluster sizes and the adaptive story-pass chunking change only how the
    work is spread over SMs: the golden state hashes hold for every geometry."""
    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    story_c, replay_c, chunk = geometry
    case = CASES[case_name]
    w, batches = _stories(case)
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as backend:
        backend.set_cluster_sizes(story_c, replay_c)
        backend.set_story_chunk(chunk)
        for i, (rec, batch) in enumerate(zip(case["batches"], batches)):
            backend.train_story_batch(batch, TRAINING)
            assert backend.state_digest().hex() == rec["state_hash"], f"batch {i}"


@pytest.mark.gpu
@pytest.mark.parametrize("case_name,min_in_degree,cta_events,thread_events", [
    ("baseline1", 1, 0, 0), ("baseline1", 1, 1, 1), ("baseline1", 1, 0, 1), ("test-8", 1, 1, 1),
    ("baseline2-short", 32, 2, 1), ("baseline3-short", 0, 1, 1), ("baseline3-short", 0, 0, 0),
    ("baseline3-short", 0, 2048, 1), ("baseline2-short", 32, 2048, 2),
], ids=["baseline1-all-hubs-default", "baseline1-all-hubs-cta", "baseline1-all-hubs-warp", "test8-all-hubs-cta",
        "baseline2-hubs", "baseline3-cta", "baseline3-default", "baseline3-warp-wide", "baseline2-warp-wide"])
def test_gpu_hub_path_matches_golden(native_lib, case_name, min_in_degree, cta_events, thread_events):
    """Hub targets (contiguous per-hub event buffers sorted by event order)
    give the same results as per-target event lists, on the thread-level,
    warp-level (register sort up to 256 keys, shared-memory sort above) and
    CTA-level sort, whichever neurons are hubs."""
    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    case = CASES[case_name]
    w, batches = _stories(case)
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as backend:
        backend.set_hub_threshold(min_in_degree, cta_events, thread_events)
        hubs, _ = backend.hub_plan()
        assert hubs > 0
        for i, (rec, batch) in enumerate(zip(case["batches"], batches)):
            backend.train_story_batch(batch, TRAINING)
            assert backend.state_digest().hex() == rec["state_hash"], f"batch {i}"


@pytest.mark.gpu
@pytest.mark.parametrize("case_name", ["test", "baseline1", "baseline2-short", "baseline3-short", "test-8"])
@pytest.mark.parametrize("device_merge", [True, False], ids=["device-context-merge", "host-context-merge"])
def test_gpu_context_merge_site_matches_golden(native_lib, case_name, device_merge):
    """The batch-end keyed context merge gives the golden hashes whether it
    runs on the device (per-order slot tables in shared memory) or on the host
    mirror, and the merged key count in the report is the same."""
    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    case = CASES[case_name]
    w, batches = _stories(case)
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as backend:
        backend.set_device_context_merge(device_merge)
        for i, (rec, batch) in enumerate(zip(case["batches"], batches)):
            result = backend.train_story_batch(batch, TRAINING)
            assert backend.state_digest().hex() == rec["state_hash"], f"batch {i}"
            assert int(result.report.context_keys) == rec["report"]["context_keys"], f"batch {i}"


@pytest.mark.gpu
def test_gpu_event_capacity_overrun_is_an_error(native_lib):
    """A step whose events overrun a target's event segment fails the batch
    with LeoError: the extra events are dropped without a write past the
    segment and the kernel's capacity flag becomes the error.  (The planned
    capacities are exact bounds; the diagnostic limit forces the overrun.)"""
    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel
    from leo_b200.native import LeoError

    case = CASES["baseline1"]
    w, batches = _stories(case)
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as backend:
        backend.set_segment_capacity_limit(1)
        with pytest.raises(LeoError, match="event capacity"):
            backend.train_story_batch(batches[0], TRAINING)
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as backend:
        backend.set_segment_capacity_limit(1 << 20)  # above every exact bound: no effect
        backend.train_story_batch(batches[0], TRAINING)
        assert backend.state_digest().hex() == case["batches"][0]["state_hash"]
