"""``LEODATA1`` prepared datasets and the story-batch feed of the training loop.

A prepared dataset is two files (``crates/leo-data/src/lib.rs``):

* ``.bytes``: the stories' UTF-8 bytes, concatenated;
* ``.idx``: a 192-byte header -- magic ``LEODATA1``, schema version, header
  size, record count, bytes length, SHA-256 of the bytes file, SHA-256 of the
  record table, a provenance digest, the dataset ID and the SHA-256 of the
  header with its own field zeroed -- followed by one 16-byte record per story
  (u64 offset, u32 length, u32 split flags), all little-endian.

:meth:`PreparedDataset.open` checks all of it as the reference does
(``PreparedDataset::open`` lib.rs:47-176) and reads stories by offset.  The
feed restates ``crates/leo-cli/src/training/dataset.rs``: the per-pass story
order is the identity shuffled by ``SplitMix64(seed + pass + 1)`` (:9-13),
``read_story_batch`` takes up to ``workers`` stories from a position without
splitting a story at the byte limit (:119-152), and
:class:`StoryBatchPrefetcher` reads one batch ahead on a worker thread that
owns its own file handle (:38-117), so the device never waits on disk.
"""

from __future__ import annotations

import hashlib
import os
import queue
import struct
import threading
from dataclasses import dataclass
from pathlib import Path

import numpy as np

INDEX_MAGIC = b"LEODATA1"
INDEX_HEADER_SIZE = 192
INDEX_RECORD_SIZE = 16
DATASET_SCHEMA_VERSION = 1  # crates/leo-core/src/semantics.rs:11
ZERO_DIGEST = bytes(32)


class DatasetError(OSError):
    """An invalid or unreadable prepared dataset (``io::ErrorKind::InvalidData``)."""


@dataclass(frozen=True)
class StoryIndex:
    offset: int
    length: int
    split_flags: int = 0


@dataclass(frozen=True)
class DatasetIdentity:
    schema_version: int
    record_count: int
    bytes_length: int
    bytes_digest: bytes
    records_digest: bytes
    provenance_digest: bytes
    dataset_id: bytes


def digest_file(path: str | os.PathLike) -> bytes:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.digest()


def compute_dataset_id(schema_version: int, record_count: int, bytes_length: int, bytes_digest: bytes,
                       records_digest: bytes, provenance_digest: bytes) -> bytes:
    """SHA-256 over a domain tag, the counts and the three digests (lib.rs:235-252)."""
    h = hashlib.sha256(b"LEO-DATASET-ID\0")
    h.update(struct.pack("<IQQ", schema_version, record_count, bytes_length))
    h.update(bytes_digest)
    h.update(records_digest)
    h.update(provenance_digest)
    return h.digest()


def _check_ranges(entries, bytes_length: int, writing: bool) -> None:
    previous_end = 0
    for i, e in enumerate(entries):
        if e.length == 0:
            raise DatasetError(f"dataset story {i} has zero length")
        end = e.offset + e.length
        if writing:
            if e.offset < previous_end or end > bytes_length:
                raise DatasetError(f"invalid range for dataset story {i}")
        else:
            if end > bytes_length:
                raise DatasetError(f"dataset story {i} extends past the bytes file")
            if e.offset < previous_end:
                raise DatasetError(f"dataset story {i} overlaps a previous story")
        previous_end = end


def write_index(path: str | os.PathLike, bytes_path: str | os.PathLike, entries: list[StoryIndex],
                provenance_digest: bytes = ZERO_DIGEST) -> DatasetIdentity:
    """Write the ``.idx`` file for a bytes file and its story records (lib.rs:254-322)."""
    bytes_length = os.stat(bytes_path).st_size
    bytes_digest = digest_file(bytes_path)
    for e in entries:
        if not (0 <= e.offset < 2**64 and 0 <= e.length < 2**32 and 0 <= e.split_flags < 2**32):
            raise DatasetError("dataset story range overflow")
    _check_ranges(entries, bytes_length, writing=True)
    records = b"".join(struct.pack("<QII", e.offset, e.length, e.split_flags) for e in entries)
    records_digest = hashlib.sha256(records).digest()
    dataset_id = compute_dataset_id(DATASET_SCHEMA_VERSION, len(entries), bytes_length, bytes_digest, records_digest,
                                    provenance_digest)
    header = bytearray(INDEX_HEADER_SIZE)
    struct.pack_into("<8sIIQQ", header, 0, INDEX_MAGIC, DATASET_SCHEMA_VERSION, INDEX_HEADER_SIZE, len(entries),
                     bytes_length)
    header[32:64] = bytes_digest
    header[64:96] = records_digest
    header[96:128] = provenance_digest
    header[128:160] = dataset_id
    header[160:192] = hashlib.sha256(bytes(header)).digest()
    with open(path, "wb") as f:
        f.write(header)
        f.write(records)
        f.flush()
        os.fsync(f.fileno())
    return DatasetIdentity(DATASET_SCHEMA_VERSION, len(entries), bytes_length, bytes_digest, records_digest,
                           provenance_digest, dataset_id)


def prepare_dataset(bytes_path: str | os.PathLike, index_path: str | os.PathLike, stories: list[bytes],
                    provenance_digest: bytes = ZERO_DIGEST) -> DatasetIdentity:
    """Write ``stories`` back to back and index them (the artifact a run reads)."""
    with open(bytes_path, "wb") as f:
        for s in stories:
            f.write(s)
    entries, offset = [], 0
    for s in stories:
        entries.append(StoryIndex(offset, len(s), 0))
        offset += len(s)
    return write_index(index_path, bytes_path, entries, provenance_digest)


class PreparedDataset:
    """A verified dataset: parsed record table plus an open bytes file."""

    def __init__(self, fd: int, offsets: np.ndarray, lengths: np.ndarray, flags: np.ndarray,
                 identity: DatasetIdentity):
        self._fd = fd
        self.offsets, self.lengths, self.flags = offsets, lengths, flags
        self._identity = identity

    @classmethod
    def open(cls, bytes_path: str | os.PathLike, index_path: str | os.PathLike) -> "PreparedDataset":
        fd = os.open(bytes_path, os.O_RDONLY)
        try:
            bytes_length = os.fstat(fd).st_size
            bytes_digest = digest_file(bytes_path)
            raw = Path(index_path).read_bytes()
            if len(raw) < INDEX_HEADER_SIZE:
                raise DatasetError("dataset index is smaller than the v1 header")
            if raw[0:8] != INDEX_MAGIC:
                raise DatasetError("invalid dataset index magic; regenerate data for the current Leo v1 runtime")
            schema, header_size, count, declared_length = struct.unpack_from("<IIQQ", raw, 8)
            if schema != DATASET_SCHEMA_VERSION:
                raise DatasetError(f"unsupported dataset schema version {schema}; expected {DATASET_SCHEMA_VERSION}")
            if header_size != INDEX_HEADER_SIZE:
                raise DatasetError(f"invalid dataset index header size {header_size}")
            declared_bytes_digest, records_digest = raw[32:64], raw[64:96]
            provenance, declared_id, header_digest = raw[96:128], raw[128:160], raw[160:192]
            if hashlib.sha256(raw[:160] + bytes(32)).digest() != header_digest:
                raise DatasetError("dataset index header SHA-256 mismatch")
            if declared_length != bytes_length:
                raise DatasetError(f"dataset byte length mismatch: index declares {declared_length}, "
                                   f"file has {bytes_length}")
            if declared_bytes_digest != bytes_digest:
                raise DatasetError("dataset bytes SHA-256 mismatch")
            expected = INDEX_HEADER_SIZE + count * INDEX_RECORD_SIZE
            if len(raw) != expected:
                raise DatasetError(f"dataset index length mismatch: expected {expected}, got {len(raw)}")
            table = raw[INDEX_HEADER_SIZE:]
            if hashlib.sha256(table).digest() != records_digest:
                raise DatasetError("dataset record-table SHA-256 mismatch")
            if compute_dataset_id(schema, count, bytes_length, bytes_digest, records_digest, provenance) != declared_id:
                raise DatasetError("dataset ID does not match content and provenance")
            rec = np.frombuffer(table, dtype=np.dtype([("offset", "<u8"), ("length", "<u4"), ("flags", "<u4")]))
            offsets = rec["offset"].astype(np.uint64)
            lengths = rec["length"].astype(np.uint64)
            flags = rec["flags"].astype(np.uint32)
            zero = np.flatnonzero(lengths == 0)
            ends = offsets + lengths
            wrapped = np.flatnonzero(ends < offsets)
            past = np.flatnonzero(ends > np.uint64(bytes_length))
            prev_end = np.concatenate([np.zeros(1, np.uint64), ends[:-1]]) if count else ends
            overlap = np.flatnonzero(offsets < prev_end)
            # The first failing record wins, with the reference's check order per record.
            bad = [(int(a[0]), kind) for a, kind in ((zero, 0), (wrapped, 1), (past, 2), (overlap, 3)) if a.size]
            if bad:
                i, kind = min(bad)
                raise DatasetError([f"dataset story {i} has zero length", "dataset story range overflow",
                                    f"dataset story {i} extends past the bytes file",
                                    f"dataset story {i} overlaps a previous story"][kind])
            identity = DatasetIdentity(schema, count, bytes_length, bytes_digest, records_digest, provenance,
                                       declared_id)
            return cls(fd, offsets, lengths, flags, identity)
        except BaseException:
            os.close(fd)
            raise

    def identity(self) -> DatasetIdentity:
        return self._identity

    def try_clone(self) -> "PreparedDataset":
        """Another handle on the verified bytes, sharing the parsed table (no re-hash)."""
        return PreparedDataset(os.dup(self._fd), self.offsets, self.lengths, self.flags, self._identity)

    def close(self) -> None:
        if self._fd >= 0:
            os.close(self._fd)
            self._fd = -1

    def __del__(self):
        self.close()

    def __len__(self) -> int:
        return int(self.offsets.size)

    def is_empty(self) -> bool:
        return len(self) == 0

    def entry(self, index: int) -> StoryIndex | None:
        if not 0 <= index < len(self):
            return None
        return StoryIndex(int(self.offsets[index]), int(self.lengths[index]), int(self.flags[index]))

    def story(self, index: int) -> bytes:
        e = self.entry(index)
        if e is None:
            raise DatasetError("story index out of range")
        data = os.pread(self._fd, e.length, e.offset)
        if len(data) != e.length:
            raise DatasetError("failed to fill whole buffer")
        try:
            data.decode("utf-8")
        except UnicodeDecodeError as err:
            raise DatasetError(f"story is not valid UTF-8: {err}") from None
        return data


# ---------------------------------------------------------------- story order and batches

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_MIX1 = np.uint64(0xBF58476D1CE4E5B9)
_MIX2 = np.uint64(0x94D049BB133111EB)


def splitmix64_draws(seed: int, count: int) -> np.ndarray:
    """The first ``count`` outputs of SplitMix64(seed) (crates/leo-core/src/rng.rs:13-19).

    State k is seed + (k + 1) * gamma (mod 2^64), so every draw is computed at
    once with wrapping uint64 arithmetic."""
    k = np.arange(1, count + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        v = k * _GAMMA + np.uint64(seed % 2**64)
        v = (v ^ (v >> np.uint64(30))) * _MIX1
        v = (v ^ (v >> np.uint64(27))) * _MIX2
    return v ^ (v >> np.uint64(31))


def shuffled_story_order(story_count: int, seed: int, pass_index: int) -> np.ndarray:
    """0..story_count shuffled by SplitMix64(seed + pass + 1): Fisher-Yates from
    the top, swapping index i with draw % (i + 1) (rng.rs:38-43)."""
    order = np.arange(story_count, dtype=np.int64)
    if story_count < 2:
        return order
    draws = splitmix64_draws((seed + pass_index + 1) % 2**64, story_count - 1)
    uppers = np.arange(story_count, 1, -1, dtype=np.uint64)  # i + 1 for i = n - 1 .. 1
    others = (draws % uppers).astype(np.int64)
    values = order.tolist()
    for j, i in enumerate(range(story_count - 1, 0, -1)):
        o = others[j]
        values[i], values[o] = values[o], values[i]
    return np.asarray(values, dtype=np.int64)


def read_story_batch(dataset: PreparedDataset, story_order, position: int, workers: int,
                     remaining_bytes: int | None) -> tuple[list[bytes], int, int]:
    """Up to ``workers`` stories from ``position`` in ``story_order``; a story that
    would pass ``remaining_bytes`` ends the batch unread (dataset.rs:119-152).
    Returns (stories, next position, input bytes)."""
    end = min(position + workers, len(story_order))
    stories: list[bytes] = []
    input_bytes = 0
    next_position = position
    while next_position < end:
        index = int(story_order[next_position])
        entry = dataset.entry(index)
        if entry is None:
            raise DatasetError("story index is out of range")
        if remaining_bytes is not None and input_bytes + entry.length > remaining_bytes:
            break
        stories.append(dataset.story(index))
        input_bytes += entry.length
        next_position += 1
    return stories, next_position, input_bytes


class StoryBatchPrefetcher:
    """One-batch-ahead reader on its own thread and file handle (dataset.rs:38-117).

    ``request(position, workers, remaining_bytes)`` then ``receive()``; at most
    one request is outstanding.  Errors raised by the reader come back from
    ``receive()``."""

    def __init__(self, dataset: PreparedDataset, story_order):
        self._dataset = dataset.try_clone()
        self._order = story_order
        self._requests: queue.Queue = queue.Queue(maxsize=1)
        self._results: queue.Queue = queue.Queue(maxsize=1)
        self._worker = threading.Thread(target=self._run, name="leo-dataset-prefetch", daemon=True)
        self._worker.start()

    def _run(self) -> None:
        while True:
            request = self._requests.get()
            if request is None:
                return
            try:
                result = read_story_batch(self._dataset, self._order, *request)
            except Exception as e:  # noqa: BLE001 - handed to the caller
                result = e
            self._results.put(result)

    def request(self, position: int, workers: int, remaining_bytes: int | None) -> None:
        if self._worker is None:
            raise DatasetError("dataset prefetcher is closed")
        self._requests.put((position, workers, remaining_bytes))

    def receive(self) -> tuple[list[bytes], int, int]:
        if self._worker is None:
            raise DatasetError("dataset prefetcher is closed")
        result = self._results.get()
        if isinstance(result, Exception):
            raise result
        return result

    def close(self) -> None:
        if self._worker is not None:
            self._requests.put(None)
            self._worker.join()
            self._worker = None
            self._dataset.close()

    def __enter__(self) -> "StoryBatchPrefetcher":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        if getattr(self, "_worker", None) is not None:
            self.close()


def story_batches(dataset: PreparedDataset, story_order, workers: int, max_bytes: int | None = None,
                  position: int = 0, bytes_seen: int = 0):
    """Yield (stories, next position) for one pass the way the run loop requests
    them (crates/leo-cli/src/training/lifecycle.rs:214-245): the next batch is
    requested before the current one is handed out, and the pass stops at the
    first empty batch (the byte limit)."""
    limit = len(story_order)
    if position >= limit:
        return
    with StoryBatchPrefetcher(dataset, story_order) as prefetch:
        prefetch.request(position, workers, None if max_bytes is None else max(max_bytes - bytes_seen, 0))
        while position < limit:
            stories, next_position, batch_bytes = prefetch.receive()
            if not stories:
                return
            bytes_seen += batch_bytes
            if next_position < limit:
                prefetch.request(next_position, workers,
                                 None if max_bytes is None else max(max_bytes - bytes_seen, 0))
            position = next_position
            yield stories, position
