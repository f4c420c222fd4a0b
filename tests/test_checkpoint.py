"""``PSCLS100`` checkpoints of the host model (``leo_b200.checkpoint``).

CPU: the reference's own checkpoint tests (crates/leo-format/tests/checkpoint.rs
and the unit tests at crates/leo-format/src/lib.rs:1185-1229), the
configuration TOML tests (crates/leo-core/src/config.rs:525-583), rejection of
every damaged field ``decode_model`` checks, and a model trained by the oracle
on a golden case surviving save/load with its golden training-state hash.
GPU: a model trained through ``GpuBackend`` is synchronized, checkpointed,
loaded into a fresh backend and trained on; every batch keeps the golden hash.
"""

import hashlib
import json
import struct
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest

from leo_b200 import checkpoint as ck
from leo_b200.configs import PROBE, TEST, ConfigurationError, config_from_toml, config_to_toml
from leo_b200.ctypes_types import TOPOLOGY_REFERENCE
from leo_b200.model import HostModel
from leo_b200.native import LeoError

HERE = Path(__file__).resolve().parent
REFERENCE_CONFIGS = Path("/root/reference/configs")


def sample_model() -> HostModel:
    return HostModel.initialize(TEST, TOPOLOGY_REFERENCE)


def sample_checkpoint() -> bytearray:
    return bytearray(ck.encode_model(sample_model()))


def descriptor(i: int) -> int:
    return ck.HEADER_SIZE + i * ck.DESCRIPTOR_SIZE


def reseal(data: bytearray) -> bytearray:
    """Recompute every section digest and the header digest after an edit."""
    for i in range(12):
        d = descriptor(i)
        off, length = struct.unpack_from("<QQ", data, d + 48)
        if off + length <= len(data):
            data[d + 72:d + 104] = hashlib.sha256(bytes(data[off:off + length])).digest()
    data[ck.HEADER_DIGEST_OFFSET:ck.HEADER_SIZE] = bytes(32)
    data[ck.HEADER_DIGEST_OFFSET:ck.HEADER_SIZE] = hashlib.sha256(bytes(data[:ck.HEADER_SIZE])).digest()
    return data


def section(data: bytearray, kind: int) -> tuple[int, int, int]:
    for i in range(12):
        d = descriptor(i)
        if struct.unpack_from("<I", data, d)[0] == kind:
            off, length = struct.unpack_from("<QQ", data, d + 48)
            return d, off, length
    raise KeyError(kind)


# ---------------------------------------------------------------- crates/leo-format/tests/checkpoint.rs

def test_checkpoint_round_trip_preserves_tensors(tmp_path):
    model = sample_model()
    model.parameter_revision = 23
    model.statistics.persistent_ticks = 17
    model.statistics.active_neurons_sum = 51
    model.arrays["input_weight"][0] = 0.75
    model.arrays["context_keys"][0] = 42
    model.arrays["context_embeddings"][0] = 0.5
    model.arrays["context_output_weight"][0] = -0.25
    model.arrays["context_observations"][0] = 7
    path = tmp_path / "roundtrip.pscls"
    ck.save_model_atomic(path, model, False)
    before = ck.checkpoint_hash(path)
    loaded = ck.load_model(path)
    assert loaded.generation == model.generation
    assert loaded.parameter_revision == 23
    for name in model.arrays:
        assert np.array_equal(loaded.arrays[name], model.arrays[name]), name
    assert loaded.statistics.persistent_ticks == 17
    assert loaded.statistics.active_neurons_sum / loaded.statistics.persistent_ticks == 3.0
    assert loaded.config == model.config
    assert loaded.training_state_hash() == model.training_state_hash()
    assert ck.checkpoint_hash(path) == before
    assert not Path(f"{path}.tmp").exists()


def test_rolling_checkpoint_keeps_only_current_and_previous_model(tmp_path):
    model = sample_model()
    path = tmp_path / "rolling.pscls"
    ck.save_model_atomic(path, model, False)
    for revision in range(1, 5):
        model.parameter_revision = revision
        ck.commit_model_rolling(path, model, 1)
    assert ck.load_model(path).generation == 4
    assert ck.load_model(path).parameter_revision == 4
    for gen in (0, 1, 2):
        assert not ck.generation_path(path, gen).exists()
    assert ck.generation_path(path, 3).exists()
    assert ck.load_model(ck.generation_path(path, 3)).parameter_revision == 3


def test_corrupted_checkpoint_is_rejected(tmp_path):
    path = tmp_path / "corrupt.pscls"
    ck.save_model_atomic(path, sample_model(), False)
    data = bytearray(path.read_bytes())
    data[32] ^= 0xFF
    path.write_bytes(bytes(data))
    with pytest.raises(ck.CheckpointCorrupt):
        ck.load_model(path)


def test_checkpoint_holds_only_the_model(tmp_path):
    """The file is a function of the host model alone: a copy written after a
    trip through a second HostModel is byte-identical (worker state has no
    place in it, crates/leo-format/tests/checkpoint.rs:63-85)."""
    model = sample_model()
    a, b = tmp_path / "a.pscls", tmp_path / "b.pscls"
    ck.save_model_atomic(a, model, False)
    ck.save_model_atomic(b, ck.load_model(a).copy(), False)
    assert a.read_bytes() == b.read_bytes()


# ---------------------------------------------------------------- crates/leo-format/src/lib.rs unit tests

def test_duplicate_section_descriptors_are_rejected():
    data = sample_checkpoint()
    data[descriptor(1):descriptor(1) + 4] = data[descriptor(0):descriptor(0) + 4]
    with pytest.raises(ck.CheckpointCorrupt):
        ck.decode_model(bytes(data))
    with pytest.raises(ck.CheckpointCorrupt, match="duplicate"):
        ck.decode_model(bytes(reseal(data)))


def test_overlapping_section_ranges_are_rejected():
    data = sample_checkpoint()
    data[descriptor(1) + 48:descriptor(1) + 56] = data[descriptor(0) + 48:descriptor(0) + 56]
    with pytest.raises(ck.CheckpointCorrupt):
        ck.decode_model(bytes(data))
    with pytest.raises(ck.CheckpointCorrupt, match="overlapping"):
        ck.decode_model(bytes(reseal(data)))


def test_statistics_require_every_persisted_field():
    with pytest.raises(ck.CheckpointCorrupt):
        ck._decode_statistics(memoryview(bytes(8 * 8)))


def test_input_projection_requires_complete_weight_tensor():
    data = sample_checkpoint()
    d, off, length = section(data, ck.INPUT_PROJECTION)
    # fan-out, 4 targets, 4 branches, and a weight vector that claims 4 but ends early
    payload = struct.pack("<QQ4IQ4BQ", 2, 4, 0, 1, 2, 3, 4, 0, 0, 2, 3, 4) + struct.pack("<f", 1.0)
    data[off:off + length] = bytes(length)
    data[off:off + len(payload)] = payload
    struct.pack_into("<Q", data, d + 56, len(payload))
    with pytest.raises(ck.CheckpointCorrupt, match="truncated"):
        ck.decode_model(bytes(reseal(data)))


# ---------------------------------------------------------------- every check of decode_model

@pytest.mark.parametrize("edit,error,match", [
    (lambda d: d.__setitem__(slice(0, 8), b"PSCLS099"), ck.CheckpointIncompatible, "magic"),
    (lambda d: struct.pack_into("<I", d, 8, 2), ck.CheckpointIncompatible, "format version"),
    (lambda d: struct.pack_into("<I", d, 12, 0x04030201), ck.CheckpointIncompatible, "endianness"),
    (lambda d: d.__setitem__(60, 1), ck.CheckpointCorrupt, "reserved"),
    (lambda d: struct.pack_into("<I", d, 24, 11), ck.CheckpointCorrupt, "section count"),
    (lambda d: struct.pack_into("<I", d, 28, 1), ck.CheckpointCorrupt, "flags"),
    (lambda d: struct.pack_into("<Q", d, 40, 3), ck.CheckpointCorrupt, "CONFIG header pointer"),
    (lambda d: struct.pack_into("<Q", d, 16, 9), ck.CheckpointCorrupt, "generation metadata"),
    (lambda d: struct.pack_into("<I", d, descriptor(2) + 4, 2), ck.CheckpointIncompatible, "schema version"),
    (lambda d: struct.pack_into("<I", d, descriptor(4) + 8, 1), ck.CheckpointCorrupt, "invalid dtype"),
    (lambda d: struct.pack_into("<I", d, descriptor(4) + 12, 2), ck.CheckpointCorrupt, "rank/shape"),
    (lambda d: struct.pack_into("<I", d, descriptor(3) + 64, 32), ck.CheckpointCorrupt, "alignment"),
    (lambda d: struct.pack_into("<I", d, descriptor(3) + 68, 1), ck.CheckpointIncompatible, "compressed"),
    (lambda d: struct.pack_into("<Q", d, descriptor(5) + 48, struct.unpack_from("<Q", d, descriptor(5) + 48)[0] + 8),
     ck.CheckpointCorrupt, "byte range"),
    (lambda d: struct.pack_into("<Q", d, descriptor(11) + 56, 10 ** 9), ck.CheckpointCorrupt, "byte range"),
    (lambda d: d.__setitem__(descriptor(0) + 110, 1), ck.CheckpointCorrupt, "descriptor reserved"),
    (lambda d: struct.pack_into("<I", d, descriptor(6), 13), ck.CheckpointCorrupt, "unknown checkpoint section"),
    (lambda d: struct.pack_into("<I", d, descriptor(6) + 8, 9), ck.CheckpointCorrupt, "unknown checkpoint dtype"),
    (lambda d: struct.pack_into("<Q", d, descriptor(7) + 16, 256), ck.CheckpointCorrupt, "shape mismatch"),
])
def test_damaged_header_and_descriptors_are_rejected(edit, error, match):
    data = sample_checkpoint()
    edit(data)
    with pytest.raises(error, match=match):
        ck.decode_model(bytes(reseal(data)))


def test_section_digest_mismatch_is_rejected():
    data = sample_checkpoint()
    _, off, _ = section(data, ck.OUTPUT_BIAS)
    data[off + 9] ^= 1
    with pytest.raises(ck.CheckpointCorrupt, match="SHA-256 mismatch in OutputBias"):
        ck.decode_model(bytes(data))


def test_header_digest_mismatch_is_rejected():
    data = sample_checkpoint()
    data[ck.HEADER_DIGEST_OFFSET] ^= 1
    with pytest.raises(ck.CheckpointCorrupt, match="header SHA-256"):
        ck.decode_model(bytes(data))


def test_semantics_contract_must_be_current():
    data = sample_checkpoint()
    _, off, _ = section(data, ck.SEMANTICS)
    struct.pack_into("<I", data, off + 8, 2)  # execution semantics v2
    with pytest.raises(ck.CheckpointIncompatible, match="semantics"):
        ck.decode_model(bytes(reseal(data)))


def test_trailing_payload_bytes_are_rejected():
    data = sample_checkpoint()
    d, off, length = section(data, ck.RECURRENT_WEIGHTS)
    n = struct.unpack_from("<Q", data, off)[0]
    struct.pack_into("<Q", data, off, n - 1)  # one weight left over
    with pytest.raises(ck.CheckpointCorrupt, match="trailing"):
        ck.decode_model(bytes(reseal(data)))


def test_truncated_files_are_rejected():
    data = sample_checkpoint()
    _, off, length = section(data, ck.SEMANTICS)
    for cut in (0, 64, ck.HEADER_SIZE + 100, off + length - 1):
        with pytest.raises(ck.CheckpointError):
            ck.decode_model(bytes(data[:cut]))
    # the zero padding after the last payload is not part of any section
    assert ck.decode_model(bytes(data[:off + length])).generation == 0


def test_mismatched_capacity_is_an_invalid_model():
    data = sample_checkpoint()
    _, off, _ = section(data, ck.RECURRENT_TARGETS)
    struct.pack_into("<Q", data, off, TEST.synapses_per_neuron + 1)
    with pytest.raises(LeoError, match="dimensions are incompatible"):
        ck.decode_model(bytes(reseal(data)))


def test_invalid_config_text_is_rejected():
    data = sample_checkpoint()
    d, off, length = section(data, ck.CONFIG)
    text = bytes(data[off:off + length]).replace(b"block_count = 8", b"block_count = 9")
    data[off:off + length] = text
    with pytest.raises(ConfigurationError, match="block_count"):
        ck.decode_model(bytes(reseal(data)))


def test_layout_offsets_and_alignment():
    data = sample_checkpoint()
    assert data[:8] == b"PSCLS100"
    previous_end = (ck.HEADER_SIZE + 12 * ck.DESCRIPTOR_SIZE + 63) // 64 * 64
    for kind in range(1, 13):
        d, off, length = section(data, kind)
        assert d == descriptor(kind - 1)
        assert off % 64 == 0 and off == (previous_end + 63) // 64 * 64
        previous_end = off + length
    assert len(data) == (previous_end + 63) // 64 * 64
    assert struct.unpack_from("<QQ", data, 32) == section(data, ck.CONFIG)[1:]


# ---------------------------------------------------------------- generations

def test_commit_keeps_previous_generation_and_rollback_restores_it(tmp_path):
    model = sample_model()
    path = tmp_path / "nested" / "model.pscls"
    ck.save_model_atomic(path, model, False)
    assert ck.read_generation(path) == 0
    model.parameter_revision = 5
    ck.commit_model(path, model)
    assert model.generation == 1 and ck.read_generation(path) == 1
    assert ck.generation_path(path, 0).exists()
    restored = ck.rollback_model(path, 0)
    assert restored.generation == 0 and restored.parameter_revision == 0
    assert ck.read_generation(path) == 0
    assert ck.generation_path(path, 1).exists()  # the replaced file is kept as its generation
    with pytest.raises(ck.CheckpointCorrupt, match="not found"):
        ck.rollback_model(path, 7)


def test_failed_commit_restores_generation(tmp_path):
    model = sample_model()
    target = tmp_path / "is_a_directory"
    target.mkdir()
    with pytest.raises(OSError):
        ck.commit_model(target, model)
    assert model.generation == 0


def test_prune_ignores_unrelated_files(tmp_path):
    model = sample_model()
    path = tmp_path / "m.pscls"
    ck.save_model_atomic(path, model, False)
    (tmp_path / "m.pscls.genx").write_bytes(b"")
    (tmp_path / "m.pscls.gen").write_bytes(b"")
    (tmp_path / "other.pscls.gen000000").write_bytes(b"")
    for _ in range(3):
        ck.commit_model_rolling(path, model, 0)
    assert sorted(p.name for p in tmp_path.iterdir()) == ["m.pscls", "m.pscls.gen", "m.pscls.genx",
                                                          "other.pscls.gen000000"]


# ---------------------------------------------------------------- configuration text

def test_integrated_configuration_round_trips():
    config = replace(PROBE, membrane_reset_fraction=0.2, inhibitory_learning_rate=0.00003, context_max_order=6,
                     context_embedding_dim=12, context_slots_per_order=512, context_probe_limit=3,
                     context_dropout_rate=0.25, end_document_weight=6.0, plasticity_window=4,
                     replay_segment_bytes=32, replay_stateful_batch=True)
    decoded = config_from_toml(config_to_toml(config))
    assert decoded == config
    assert decoded.replay_stateful_batch is True


def test_replay_fraction_zero_disables_replay():
    assert config_from_toml(config_to_toml(replace(PROBE, replay_fraction=0.0))).replay_fraction == 0.0


def test_standard_toml_escaping_round_trips_model_names():
    config = replace(PROBE, name='Leo # "v1"\nreference\\\t\x01')
    assert config_from_toml(config_to_toml(config)).name == config.name


def test_unknown_architecture_switches_are_rejected():
    text = config_to_toml(PROBE).replace("[learning]\n", "[learning]\nunexpected_field = true\n")
    with pytest.raises(ConfigurationError, match="unexpected_field"):
        config_from_toml(text)
    with pytest.raises(ConfigurationError, match="unknown field"):
        config_from_toml(config_to_toml(PROBE) + "\n[extra]\nx = 1\n")


def test_defaulted_keys_may_be_absent_and_others_may_not():
    text = config_to_toml(PROBE).replace("plasticity_window = 1\n", "").replace("stateful_batch = false\n", "")
    assert config_from_toml(text) == PROBE
    with pytest.raises(ConfigurationError, match="missing field 'seed'"):
        config_from_toml(config_to_toml(PROBE).replace("seed = 1337\n", ""))


@pytest.mark.parametrize("old,new", [("seed = 1337", "seed = -1"), ("seed = 1337", "seed = 1.5"),
                                     ("stateful_batch = false", "stateful_batch = 0"),
                                     ('name = "Leo-probe"', "name = 3"),
                                     ("confidence_observations = 8", "confidence_observations = 4294967296"),
                                     ('name = "Leo-probe"', 'name = "  "'),
                                     ("teaching_replays = 1", "teaching_replays = 0"),
                                     ("early_stop_checks = 3", "early_stop_checks = 0"),
                                     ("minimum_relative_improvement = 0.005", "minimum_relative_improvement = -1.0"),
                                     ("[model]", "[model")])
def test_invalid_values_are_rejected(old, new):
    text = config_to_toml(PROBE)
    assert old in text
    with pytest.raises(ConfigurationError):
        config_from_toml(text.replace(old, new))


def test_integers_are_accepted_for_float_fields():
    text = config_to_toml(PROBE).replace("weight_max = 1.0", "weight_max = 1")
    assert config_from_toml(text) == PROBE


def test_stateful_batch_models_are_refused_by_the_backend():
    """A checkpoint may carry the streaming-replay switch; the backend only
    implements serial canonical replay and says so before touching a device."""
    from leo_b200.backend import GpuBackend

    model = HostModel.initialize(replace(TEST, replay_stateful_batch=True), TOPOLOGY_REFERENCE)
    with pytest.raises(LeoError, match="stateful_batch"):
        GpuBackend(model)


@pytest.mark.skipif(not REFERENCE_CONFIGS.exists(), reason="reference configs are not on this machine")
@pytest.mark.parametrize("name,want", [("test.toml", TEST), ("probe.toml", PROBE)])
def test_reference_config_files_parse_to_the_named_configs(name, want):
    assert config_from_toml((REFERENCE_CONFIGS / name).read_text()) == want


# ---------------------------------------------------------------- trained model through the oracle

GOLDEN = json.loads((HERE / "golden" / "story_batches.json").read_text())
CASES = {c["name"]: c for c in GOLDEN["cases"]}


def _case(name):
    import sys

    from leo_b200.configs import WORKLOADS

    sys.path.insert(0, str(HERE / "golden"))
    from make_golden import case_stories

    case = CASES[name]
    return case, WORKLOADS[case["workload"]], case_stories(case)


def test_oracle_trained_model_survives_save_and_load(oracle_lib, tmp_path):
    from leo_b200.ctypes_types import TRAINING

    case, w, batches = _case("test")
    rt = oracle_lib.OracleRuntime(oracle_lib.OracleModel.initialize(w.config, w.topology))
    path = tmp_path / "trained.pscls"
    for rec, batch in zip(case["batches"], batches):
        rt.train_story_batch(batch, TRAINING, 0)
        host = HostModel(w.config, rt.model.arrays())
        host.generation, host.parameter_revision, host.statistics = rt.model.scalars()
        ck.save_model_atomic(path, host, True)
        loaded = ck.load_model(path)
        assert loaded.generation == rec["generation"]
        assert loaded.training_state_hash().hex() == rec["state_hash"]


# ---------------------------------------------------------------- GPU: synchronize, checkpoint, resume

@pytest.mark.gpu
@pytest.mark.parametrize("name,cut", [("test", 1), ("baseline1", 1)])
def test_gpu_model_checkpoint_and_resume_keep_golden_hashes(native_lib, tmp_path, name, cut):
    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING

    case, w, batches = _case(name)
    path = tmp_path / "gpu.pscls"
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as gpu:
        for rec, batch in zip(case["batches"][:cut], batches[:cut]):
            gpu.train_story_batch(batch, TRAINING)
            assert gpu.state_digest().hex() == rec["state_hash"]
        ck.save_model_atomic(path, gpu.synchronize_model(), False)
        tick = gpu.canonical_tick
    loaded = ck.load_model(path)
    assert loaded.training_state_hash().hex() == case["batches"][cut - 1]["state_hash"]
    with GpuBackend(loaded, device=0, max_lanes=case["stories_per_batch"]) as gpu:
        gpu.canonical_tick = tick  # the run loop's own resume record carries the tick
        for rec, batch in zip(case["batches"][cut:], batches[cut:]):
            gpu.train_story_batch(batch, TRAINING)
            assert gpu.state_digest().hex() == rec["state_hash"]
            assert gpu.canonical_tick == rec["canonical_tick"]
        final = gpu.synchronize_model()
    assert final.training_state_hash().hex() == case["batches"][-1]["state_hash"]
    ck.save_model_atomic(path, final, False)
    assert ck.load_model(path).training_state_hash() == final.training_state_hash()
