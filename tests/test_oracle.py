"""The oracle pinned against the reference's own known-answer tests, on CPU.

``oracle/known_answer_tests.cpp`` ports every unit test of the reference that
pins this path (learning.rs, runtime.rs, parallel.rs, model.rs, config.rs,
artifact.rs and the training.rs batch/replay tests); this file runs it and adds
property checks of the batch semantics the GPU path is compared against.
"""

import subprocess
from pathlib import Path

import numpy as np
import pytest

from leo_b200.configs import TEST, WORKLOADS
from leo_b200.ctypes_types import TOPOLOGY_REFERENCE, TRAINING

ORACLE = Path(__file__).resolve().parents[1] / "oracle"


def test_reference_known_answer_tests_pass(oracle_lib):
    subprocess.run(["make", "-s", "-C", str(ORACLE), "known_answer_tests"], check=True)
    proc = subprocess.run([str(ORACLE / "known_answer_tests")], capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith(("PASS", "FAIL"))]
    assert len(lines) >= 30
    assert all(ln.startswith("PASS") for ln in lines), [ln for ln in lines if ln.startswith("FAIL")]
    assert "OK: 0 failure(s)" in proc.stdout


def test_sha256_published_vectors(oracle_lib):
    """SHA-256 (artifact.rs:265 checks the empty-input vector) against
    hashlib on the padding boundaries."""
    import hashlib

    assert oracle_lib.sha256(b"").hex() == "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"
    assert oracle_lib.sha256(b"abc") == hashlib.sha256(b"abc").digest()
    for n in (0, 1, 55, 56, 63, 64, 65, 1000):
        data = bytes((i * 7 + 3) & 0xFF for i in range(n))
        assert oracle_lib.sha256(data) == hashlib.sha256(data).digest()


@pytest.mark.parametrize("fraction,segment", [(0.3, 8), (0.3, 32), (0.1, 4), (1.0, 16), (0.0, 8)])
def test_replay_ranges_properties(oracle_lib, fraction, segment):
    """select_replay_ranges (training.rs:1782-1830): ranges are sorted,
    disjoint, inside the story and cover about ``fraction`` of the targets."""
    rng = np.random.default_rng(segment + int(fraction * 100))
    for n in (0, 1, 7, 64, 300):
        losses = rng.gamma(2.0, 1.0, size=n).astype(np.float32)
        ranges = oracle_lib.select_replay_ranges(losses, fraction, segment)
        if n == 0 or fraction == 0.0:
            assert ranges == []
            continue
        prev_end = 0
        covered = 0
        for s, e in ranges:
            assert 0 <= s < e <= n
            assert s >= prev_end
            prev_end = e
            covered += e - s
        budget = int(np.ceil(np.float64(np.float32(fraction)) * n))
        assert covered <= max(budget, segment) + segment


def test_story_batch_is_independent_of_thread_count(oracle_lib):
    """Stories run independently until the batch end (docs/SEMANTICS.md:54):
    one thread or one per story gives the same canonical state."""
    from leo_b200.synthetic import story_stream

    stories = story_stream(3, 4, 8, 40)
    hashes = []
    for threads in (1, 4):
        model = oracle_lib.OracleModel.initialize(TEST, TOPOLOGY_REFERENCE)
        rt = oracle_lib.OracleRuntime(model)
        report, losses, ranges = rt.train_story_batch(stories, TRAINING, threads)
        hashes.append((rt.model.training_state_hash(), losses.tobytes(), ranges))
    assert hashes[0] == hashes[1]


def test_story_batch_changes_model_and_counts(oracle_lib):
    from leo_b200.synthetic import story_stream

    w = WORKLOADS["test"]
    stories = story_stream(w.story_seed, w.workers, w.min_story_bytes, w.max_story_bytes)
    model = oracle_lib.OracleModel.initialize(w.config, w.topology)
    before = model.training_state_hash()
    rt = oracle_lib.OracleRuntime(model)
    report, losses, ranges = rt.train_story_batch(stories, TRAINING, 0)
    assert rt.model.training_state_hash() != before
    assert len(losses) == sum(len(s) + 1 for s in stories)
    assert np.all(np.isfinite(losses)) and np.all(losses >= 0)
    gen, rev, stats = rt.model.scalars()
    assert rev > 0
    rt.model.validate()
