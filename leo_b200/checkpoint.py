"""``PSCLS100`` model checkpoints for the host model.

Restates the artifact format of ``crates/leo-format/src/lib.rs`` so that a
model trained through :class:`leo_b200.backend.GpuBackend` and read back with
``synchronize_model()`` is written, committed, loaded and rolled back exactly
as the reference's runtime does:

* file = 128-byte header, one 128-byte descriptor per section, then the twelve
  section payloads, each starting on a 64-byte boundary (``encode_model``
  lib.rs:289-444);
* header: magic ``PSCLS100``, format version, endian marker ``0x01020304``,
  generation, section count, flags (0), CONFIG offset and length, zero
  reserved bytes, and at byte 96 the SHA-256 of the header with that field
  zeroed (lib.rs:421-440, ``validate_header`` :613-649);
* descriptor: kind, schema version 1, dtype, rank, four shape words, offset,
  length, alignment 64, compression 0, the payload's SHA-256, zero padding
  (``encode_descriptor`` :801-817);
* payload vectors are a little-endian u64 element count followed by the
  elements (``put_vec_*`` :1070-1097).

Loading checks everything the reference's ``decode_model`` (:446-611) checks
-- header digest, section count and flags, descriptor schema/dtype/rank/
alignment/compression, in-bounds non-overlapping aligned ranges, per-section
SHA-256, duplicate and missing sections, the CONFIG header pointer, the
semantics contract, trailing bytes inside each payload, the generation echo,
model validation and every section shape -- and raises
:class:`CheckpointCorrupt` or :class:`CheckpointIncompatible` the way the
reference returns ``checkpoint_corrupt`` / ``checkpoint_incompatible``.
"""

from __future__ import annotations

import hashlib
import os
import re
import shutil
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .configs import ConfigurationError, config_from_toml, config_to_toml
from .ctypes_types import LeoB200Statistics, OUTPUT_CLASSES, SYMBOL_COUNT
from .model import HostModel
from .native import LeoError

MAGIC = b"PSCLS100"
FORMAT_VERSION = 1                   # CHECKPOINT_SCHEMA_VERSION (crates/leo-core/src/semantics.rs:13)
ENDIAN_MARKER = 0x01020304
HEADER_SIZE = 128
DESCRIPTOR_SIZE = 128
ALIGNMENT = 64
HEADER_DIGEST_OFFSET = 96
MAX_CHECKPOINT_BYTES = 64 * 1024 ** 3
MAX_CONFIG_BYTES = 1024 * 1024
# SemanticsContract::CURRENT (semantics.rs:28-34): model schema, training
# policy, execution semantics, dataset schema, CUDA ABI.
SEMANTICS_CURRENT = (1, 1, 1, 1, 1)

# Section kinds (lib.rs:31-45) and payload dtypes (lib.rs:93-99).
CONFIG, NEURONS, RECURRENT_TARGETS, RECURRENT_METADATA, RECURRENT_WEIGHTS, INPUT_PROJECTION, \
    OUTPUT_WEIGHTS, OUTPUT_BIAS, CONTEXT_PROJECTION, TRAINING_STATISTICS, GENERATION, SEMANTICS = range(1, 13)
SECTION_NAMES = {
    CONFIG: "Config", NEURONS: "NeuronParameters", RECURRENT_TARGETS: "RecurrentTargets",
    RECURRENT_METADATA: "RecurrentMetadata", RECURRENT_WEIGHTS: "RecurrentWeights",
    INPUT_PROJECTION: "InputProjection", OUTPUT_WEIGHTS: "OutputWeights", OUTPUT_BIAS: "OutputBias",
    CONTEXT_PROJECTION: "ContextProjection", TRAINING_STATISTICS: "TrainingStatistics",
    GENERATION: "GenerationMetadata", SEMANTICS: "SemanticsContract",
}
DT_BYTES, DT_F32, DT_U32, DT_U64 = 1, 2, 3, 4
_EXPECTED_DTYPE = {RECURRENT_WEIGHTS: DT_F32, OUTPUT_WEIGHTS: DT_F32, OUTPUT_BIAS: DT_F32,
                   GENERATION: DT_U64, SEMANTICS: DT_U32}

_STAT_FIELDS = ("processed_bytes", "processed_stories", "training_loss_sum", "training_targets",
                "active_neurons_sum", "active_neurons_peak", "synaptic_events", "numerical_rejections",
                "persistent_ticks")


class CheckpointError(LeoError):
    """A checkpoint that cannot be loaded."""


class CheckpointCorrupt(CheckpointError):
    """LeoError::checkpoint_corrupt: damaged or inconsistent bytes."""


class CheckpointIncompatible(CheckpointError):
    """LeoError::checkpoint_incompatible: a different format or semantics."""


def sha256(data: bytes | memoryview) -> bytes:
    return hashlib.sha256(data).digest()


def _align_up(value: int) -> int:
    return (value + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT


def _rank_for_shape(shape: tuple[int, int, int, int]) -> int:
    """Leading nonzero dimensions; a nonzero after a zero is rank 5 (invalid)."""
    rank, saw_zero = 0, False
    for d in shape:
        if d == 0:
            saw_zero = True
        elif saw_zero:
            return 5
        else:
            rank += 1
    return rank


# ---------------------------------------------------------------- payload encoding

def _vec(a: np.ndarray, dtype: str) -> bytes:
    a = np.ascontiguousarray(a).astype(dtype, copy=False)
    return struct.pack("<Q", a.size) + a.tobytes()


class _Reader:
    """Bounds-checked cursor over one payload (lib.rs:1099-1183)."""

    def __init__(self, data: memoryview):
        self.data, self.pos = data, 0

    def take(self, n: int) -> memoryview:
        end = self.pos + n
        if end > len(self.data):
            raise CheckpointCorrupt("truncated checkpoint tensor")
        out = self.data[self.pos:end]
        self.pos = end
        return out

    def u64(self) -> int:
        return struct.unpack("<Q", self.take(8))[0]

    def f64(self) -> float:
        return struct.unpack("<d", self.take(8))[0]

    def vec(self, dtype: str) -> np.ndarray:
        n = self.u64()
        width = np.dtype(dtype).itemsize
        if n > (len(self.data) - self.pos) // width:
            raise CheckpointCorrupt("truncated checkpoint tensor")
        return np.frombuffer(self.take(n * width), dtype=dtype).copy()

    def finish(self) -> None:
        if self.pos != len(self.data):
            raise CheckpointCorrupt("unexpected trailing checkpoint data")


def _statistics_payload(stats: LeoB200Statistics) -> bytes:
    return b"".join(struct.pack("<d" if f == "training_loss_sum" else "<Q", getattr(stats, f))
                    for f in _STAT_FIELDS)


def _decode_statistics(data: memoryview) -> LeoB200Statistics:
    if len(data) != 8 * len(_STAT_FIELDS):
        raise CheckpointCorrupt(f"invalid training statistics length: {len(data)}")
    r = _Reader(data)
    stats = LeoB200Statistics()
    for f in _STAT_FIELDS:
        setattr(stats, f, r.f64() if f == "training_loss_sum" else r.u64())
    r.finish()
    return stats


@dataclass
class _Section:
    kind: int
    payload: bytes
    dtype: int
    shape: tuple[int, int, int, int]


def _shapes(model: HostModel) -> dict[int, tuple[int, int, int, int]]:
    """Every section's descriptor shape (lib.rs:291-397, checked by ``validate_shapes`` :702-788)."""
    cfg, a = model.config, model.arrays
    n, s = cfg.neuron_count, cfg.synapses_per_neuron
    return {
        CONFIG: (0, 0, 0, 0), NEURONS: (n, 0, 0, 0), RECURRENT_TARGETS: (n, s, 0, 0), RECURRENT_METADATA: (n, s, 0, 0),
        RECURRENT_WEIGHTS: (a["recurrent_weight"].size, 0, 0, 0), INPUT_PROJECTION: (SYMBOL_COUNT, cfg.input_fanout, 0, 0),
        OUTPUT_WEIGHTS: (OUTPUT_CLASSES, n, 0, 0), OUTPUT_BIAS: (a["output_bias"].size, 0, 0, 0),
        CONTEXT_PROJECTION: (a["context_observations"].size, cfg.context_embedding_dim, OUTPUT_CLASSES, 0),
        TRAINING_STATISTICS: (9, 0, 0, 0), GENERATION: (2, 0, 0, 0), SEMANTICS: (5, 0, 0, 0),
    }


def _payloads(model: HostModel) -> dict[int, bytes]:
    cfg, a = model.config, model.arrays
    return {
        CONFIG: config_to_toml(cfg).encode(),
        NEURONS: _vec(a["threshold"], "<f4") + _vec(a["excitability"], "<f4") + _vec(a["neuron_type"], "u1"),
        RECURRENT_TARGETS: struct.pack("<Q", cfg.synapses_per_neuron) + _vec(a["recurrent_target"], "<u4"),
        RECURRENT_METADATA: _vec(a["recurrent_branch"], "u1") + _vec(a["recurrent_delay"], "u1"),
        RECURRENT_WEIGHTS: _vec(a["recurrent_weight"], "<f4"),
        INPUT_PROJECTION: struct.pack("<Q", cfg.input_fanout) + _vec(a["input_target"], "<u4")
        + _vec(a["input_branch"], "u1") + _vec(a["input_weight"], "<f4"),
        OUTPUT_WEIGHTS: _vec(a["output_weight"], "<f4"),
        OUTPUT_BIAS: _vec(a["output_bias"], "<f4"),
        CONTEXT_PROJECTION: _vec(a["context_keys"], "<u8") + _vec(a["context_embeddings"], "<f4")
        + _vec(a["context_observations"], "<u4") + _vec(a["context_output_weight"], "<f4"),
        TRAINING_STATISTICS: _statistics_payload(model.statistics),
        GENERATION: struct.pack("<QQ", model.generation, model.parameter_revision),
        SEMANTICS: struct.pack("<5I", *SEMANTICS_CURRENT),
    }


def _sections(model: HostModel) -> list[_Section]:
    """The twelve sections in kind order (lib.rs:291-398)."""
    shapes, payloads = _shapes(model), _payloads(model)
    return [_Section(kind, payloads[kind], _EXPECTED_DTYPE.get(kind, DT_BYTES), shapes[kind]) for kind in SECTION_NAMES]


def encode_model(model: HostModel) -> bytes:
    """The checkpoint bytes of a model (lib.rs:289-444)."""
    sections = _sections(model)
    cursor = _align_up(HEADER_SIZE + DESCRIPTOR_SIZE * len(sections))
    offsets = []
    for s in sections:
        offsets.append(cursor)
        cursor = _align_up(cursor + len(s.payload))
    out = bytearray(cursor)
    config_offset, config_length = offsets[0], len(sections[0].payload)
    struct.pack_into("<8sIIQII QQ", out, 0, MAGIC, FORMAT_VERSION, ENDIAN_MARKER, model.generation, len(sections), 0,
                     config_offset, config_length)
    for i, (s, off) in enumerate(zip(sections, offsets)):
        d = HEADER_SIZE + i * DESCRIPTOR_SIZE
        struct.pack_into("<IIII4QQQII", out, d, s.kind, 1, s.dtype, _rank_for_shape(s.shape), *s.shape, off,
                         len(s.payload), ALIGNMENT, 0)
        out[d + 72:d + 104] = sha256(s.payload)
        out[off:off + len(s.payload)] = s.payload
    out[HEADER_DIGEST_OFFSET:HEADER_SIZE] = sha256(bytes(out[:HEADER_SIZE]))
    return bytes(out)


# ---------------------------------------------------------------- decoding

def validate_header(header: bytes | memoryview) -> None:
    """lib.rs:613-649."""
    if len(header) != HEADER_SIZE:
        raise CheckpointCorrupt("invalid checkpoint header size")
    if bytes(header[0:8]) != MAGIC:
        raise CheckpointIncompatible(
            "unsupported checkpoint magic; the current Leo v1 runtime accepts only PSCLS100 artifacts")
    version, marker = struct.unpack_from("<II", header, 8)
    if version != FORMAT_VERSION:
        raise CheckpointIncompatible(f"unsupported checkpoint format version {version}; expected {FORMAT_VERSION}")
    if marker != ENDIAN_MARKER:
        raise CheckpointIncompatible("unsupported checkpoint endianness")
    if any(header[48:HEADER_DIGEST_OFFSET]):
        raise CheckpointCorrupt("checkpoint header reserved bytes are nonzero")
    normalized = bytearray(header)
    normalized[HEADER_DIGEST_OFFSET:] = bytes(HEADER_SIZE - HEADER_DIGEST_OFFSET)
    if sha256(bytes(normalized)) != bytes(header[HEADER_DIGEST_OFFSET:]):
        raise CheckpointCorrupt("checkpoint header SHA-256 mismatch")


@dataclass
class _Descriptor:
    kind: int
    schema_version: int
    dtype: int
    rank: int
    shape: tuple[int, int, int, int]
    offset: int
    length: int
    alignment: int
    compression: int
    digest: bytes

    @property
    def name(self) -> str:
        return SECTION_NAMES[self.kind]


def _decode_descriptor(raw: memoryview) -> _Descriptor:
    """lib.rs:819-847."""
    if any(raw[104:128]):
        raise CheckpointCorrupt("checkpoint descriptor reserved bytes are nonzero")
    kind, schema, dtype, rank, s0, s1, s2, s3, offset, length, alignment, compression = \
        struct.unpack_from("<IIII4QQQII", raw, 0)
    if kind not in SECTION_NAMES:
        raise CheckpointCorrupt(f"unknown checkpoint section type: {kind}")
    if dtype not in (DT_BYTES, DT_F32, DT_U32, DT_U64):
        raise CheckpointCorrupt(f"unknown checkpoint dtype: {dtype}")
    return _Descriptor(kind, schema, dtype, rank, (s0, s1, s2, s3), offset, length, alignment, compression,
                       bytes(raw[72:104]))


def _validate_descriptor(d: _Descriptor, payload_start: int, file_len: int) -> None:
    """lib.rs:651-700."""
    if d.schema_version != 1:
        raise CheckpointIncompatible(f"unsupported schema version {d.schema_version} in {d.name}")
    if d.dtype != _EXPECTED_DTYPE.get(d.kind, DT_BYTES):
        raise CheckpointCorrupt(f"invalid dtype in {d.name} section")
    if d.rank != _rank_for_shape(d.shape) or d.rank > 4:
        raise CheckpointCorrupt(f"invalid rank/shape in {d.name} section")
    if d.alignment != ALIGNMENT:
        raise CheckpointCorrupt(f"invalid alignment in {d.name} section")
    if d.compression != 0:
        raise CheckpointIncompatible("compressed checkpoint sections are not supported in v1")
    end = d.offset + d.length
    if d.offset < payload_start or d.offset % ALIGNMENT != 0 or end > file_len:
        raise CheckpointCorrupt(f"invalid byte range for {d.name} section")


def decode_model(data: bytes) -> HostModel:
    """lib.rs:446-611."""
    view = memoryview(data)
    if len(view) < HEADER_SIZE:
        raise CheckpointCorrupt("checkpoint is smaller than the v1 header")
    validate_header(view[:HEADER_SIZE])
    generation, count, flags = struct.unpack_from("<QII", view, 16)
    if count != len(SECTION_NAMES):
        raise CheckpointCorrupt(f"invalid checkpoint section count {count}; expected {len(SECTION_NAMES)}")
    if flags != 0:
        raise CheckpointCorrupt("unsupported checkpoint header flags")
    table_end = HEADER_SIZE + count * DESCRIPTOR_SIZE
    if table_end > len(view):
        raise CheckpointCorrupt("truncated checkpoint descriptor table")
    payload_start = _align_up(table_end)
    descriptors = [_decode_descriptor(view[HEADER_SIZE + i * DESCRIPTOR_SIZE:HEADER_SIZE + (i + 1) * DESCRIPTOR_SIZE])
                   for i in range(count)]
    for d in descriptors:
        _validate_descriptor(d, payload_start, len(view))
    previous_end = payload_start
    for d in sorted(descriptors, key=lambda d: d.offset):
        if d.offset < previous_end:
            raise CheckpointCorrupt(f"overlapping {d.name} checkpoint section")
        previous_end = d.offset + d.length
    sections: dict[int, tuple[_Descriptor, memoryview]] = {}
    for d in descriptors:
        payload = view[d.offset:d.offset + d.length]
        if sha256(payload) != d.digest:
            raise CheckpointCorrupt(f"SHA-256 mismatch in {d.name} section")
        if d.kind in sections:
            raise CheckpointCorrupt(f"duplicate {d.name} checkpoint section")
        sections[d.kind] = (d, payload)
    for kind, name in SECTION_NAMES.items():
        if kind not in sections:
            raise CheckpointCorrupt(f"missing {name} checkpoint section")

    config_d, config_payload = sections[CONFIG]
    if len(config_payload) > MAX_CONFIG_BYTES:
        raise CheckpointCorrupt("CONFIG section exceeds 1 MiB")
    config_offset, config_length = struct.unpack_from("<QQ", view, 32)
    if config_d.offset != config_offset or config_d.length != config_length:
        raise CheckpointCorrupt("CONFIG header pointer does not match descriptor")
    contract_payload = sections[SEMANTICS][1]
    if len(contract_payload) != 20:
        raise CheckpointCorrupt("invalid semantics contract length")
    contract = struct.unpack("<5I", contract_payload)
    if contract != SEMANTICS_CURRENT:
        raise CheckpointIncompatible(
            f"checkpoint semantics {contract} do not match the current Leo v1 semantics {SEMANTICS_CURRENT}")
    try:
        config = config_from_toml(bytes(config_payload).decode("utf-8"))
    except UnicodeDecodeError as e:
        raise CheckpointCorrupt(f"invalid CONFIG UTF-8: {e}") from None

    arrays: dict[str, np.ndarray] = {}
    r = _Reader(sections[NEURONS][1])
    arrays["threshold"], arrays["excitability"], arrays["neuron_type"] = r.vec("<f4"), r.vec("<f4"), r.vec("u1")
    r.finish()
    r = _Reader(sections[RECURRENT_TARGETS][1])
    capacity = r.u64()
    arrays["recurrent_target"] = r.vec("<u4")
    r.finish()
    r = _Reader(sections[RECURRENT_METADATA][1])
    arrays["recurrent_branch"], arrays["recurrent_delay"] = r.vec("u1"), r.vec("u1")
    r.finish()
    r = _Reader(sections[RECURRENT_WEIGHTS][1])
    arrays["recurrent_weight"] = r.vec("<f4")
    r.finish()
    r = _Reader(sections[INPUT_PROJECTION][1])
    fanout = r.u64()
    arrays["input_target"], arrays["input_branch"], arrays["input_weight"] = r.vec("<u4"), r.vec("u1"), r.vec("<f4")
    r.finish()
    r = _Reader(sections[OUTPUT_WEIGHTS][1])
    arrays["output_weight"] = r.vec("<f4")
    r.finish()
    r = _Reader(sections[OUTPUT_BIAS][1])
    arrays["output_bias"] = r.vec("<f4")
    r.finish()
    r = _Reader(sections[CONTEXT_PROJECTION][1])
    arrays["context_keys"], arrays["context_embeddings"] = r.vec("<u8"), r.vec("<f4")
    arrays["context_observations"], arrays["context_output_weight"] = r.vec("<u4"), r.vec("<f4")
    r.finish()
    statistics = _decode_statistics(sections[TRAINING_STATISTICS][1])
    gen_payload = sections[GENERATION][1]
    if len(gen_payload) != 16:
        raise CheckpointCorrupt("invalid generation metadata length")
    section_generation, parameter_revision = struct.unpack("<QQ", gen_payload)
    if section_generation != generation:
        raise CheckpointCorrupt("generation metadata does not match checkpoint header")

    # Model::validate (crates/leo-core/src/model.rs:223-290): recorded
    # capacity and fan-out are the configured ones and every tensor is sized
    # by the configuration.
    if capacity != config.synapses_per_neuron or fanout != config.input_fanout:
        raise LeoError("model tensor dimensions are incompatible")
    try:
        model = HostModel(config, arrays)
    except ValueError:
        raise LeoError("model tensor dimensions are incompatible") from None
    model.generation = generation
    model.parameter_revision = parameter_revision
    model.statistics = statistics
    model.validate()
    for kind, shape in _shapes(model).items():
        if sections[kind][0].shape != shape:
            raise CheckpointCorrupt(f"shape mismatch in {SECTION_NAMES[kind]} section")
    return model


# ---------------------------------------------------------------- files

def generation_path(path: str | os.PathLike, generation: int) -> Path:
    """``<path>.gen%06d`` (lib.rs:283-285)."""
    return Path(f"{os.fspath(path)}.gen{generation:06d}")


def save_model_atomic(path: str | os.PathLike, model: HostModel, retain_previous: bool) -> None:
    """Write temp, fsync, rename, fsync the directory (lib.rs:144-176); with
    ``retain_previous`` an existing checkpoint is first kept as its generation
    file."""
    try:
        model.validate()
    except LeoError as e:
        raise ConfigurationError(str(e)) from None
    path = Path(path)
    if str(path.parent) not in ("", "."):
        path.parent.mkdir(parents=True, exist_ok=True)
    if retain_previous and path.exists():
        keep = generation_path(path, read_generation(path))
        if not keep.exists():
            shutil.copyfile(path, keep)
    data = encode_model(model)
    temporary = Path(f"{path}.tmp")
    with open(temporary, "wb") as f:
        f.write(data)
        f.flush()
        os.fsync(f.fileno())
    os.replace(temporary, path)
    try:
        fd = os.open(path.parent if str(path.parent) else ".", os.O_RDONLY)
    except OSError:
        return
    try:
        os.fsync(fd)
    except OSError:
        pass
    finally:
        os.close(fd)


def commit_model(path: str | os.PathLike, model: HostModel) -> None:
    """Advance the generation and save, keeping the previous file (lib.rs:178-186);
    on failure the generation is restored."""
    previous = model.generation
    model.generation = min(previous + 1, 2**64 - 1)
    try:
        save_model_atomic(path, model, True)
    except BaseException:
        model.generation = previous
        raise


def commit_model_rolling(path: str | os.PathLike, model: HostModel, keep_previous_generations: int) -> None:
    """commit_model, then keep only the newest ``keep_previous_generations``
    generation files (lib.rs:188-241)."""
    previous = model.generation
    model.generation = min(previous + 1, 2**64 - 1)
    try:
        save_model_atomic(path, model, keep_previous_generations > 0)
    except BaseException:
        model.generation = previous
        raise
    _prune_generations(Path(path), keep_previous_generations)


def _prune_generations(path: Path, keep: int) -> None:
    parent = path.parent if str(path.parent) else Path(".")
    prefix = f"{path.name}.gen"
    found = []
    for entry in parent.iterdir():
        if not entry.is_file() or not entry.name.startswith(prefix):
            continue
        suffix = entry.name[len(prefix):]
        if not re.fullmatch(r"[0-9]+", suffix) or int(suffix) >= 2**64:
            continue
        found.append((int(suffix), entry))
    found.sort(key=lambda t: t[0])
    for _, old in found[:max(len(found) - keep, 0)]:
        old.unlink()


def load_model(path: str | os.PathLike) -> HostModel:
    """lib.rs:243-252."""
    length = os.stat(path).st_size
    if length > MAX_CHECKPOINT_BYTES:
        raise CheckpointCorrupt(f"checkpoint is too large: {length} bytes")
    return decode_model(Path(path).read_bytes())


def rollback_model(path: str | os.PathLike, generation: int) -> HostModel:
    """Load a kept generation and make it current (lib.rs:254-266)."""
    source = generation_path(path, generation)
    if not source.exists():
        raise CheckpointCorrupt(f"generation {generation} not found at {source}")
    model = load_model(source)
    save_model_atomic(path, model, True)
    return model


def read_generation(path: str | os.PathLike) -> int:
    """The header's generation after header validation (lib.rs:268-274)."""
    with open(path, "rb") as f:
        header = f.read(HEADER_SIZE)
    if len(header) != HEADER_SIZE:
        raise CheckpointCorrupt("checkpoint is smaller than the v1 header")
    validate_header(header)
    return struct.unpack_from("<Q", header, 16)[0]


def checkpoint_hash(path: str | os.PathLike) -> bytes:
    """SHA-256 of the whole file (lib.rs:276-281)."""
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.digest()


checkpoint_digest = checkpoint_hash

__all__ = [
    "CheckpointError", "CheckpointCorrupt", "CheckpointIncompatible", "encode_model", "decode_model",
    "save_model_atomic", "commit_model", "commit_model_rolling", "load_model", "rollback_model",
    "read_generation", "checkpoint_hash", "checkpoint_digest", "generation_path", "validate_header",
]
