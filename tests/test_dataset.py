"""``LEODATA1`` datasets and the story-batch feed (``leo_b200.dataset``).

CPU: the reference's dataset tests (crates/leo-data/src/lib.rs:343-400 and
crates/leo-cli/src/main.rs:1623-1743), rejection of every index check of
``PreparedDataset::open``, the story order against the oracle's SplitMix64
shuffle and the published SplitMix64 output for seed 0, and the golden "test"
case fed from a prepared dataset into the oracle.
GPU: the same dataset feeds ``GpuBackend`` and every batch keeps the golden hash.
"""

import hashlib
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from leo_b200 import dataset as ds

HERE = Path(__file__).resolve().parent


def three_stories(tmp_path):
    b, i = tmp_path / "d.bytes", tmp_path / "d.idx"
    b.write_bytes(b"onetwothree")
    ds.write_index(i, b, [ds.StoryIndex(0, 3, 0), ds.StoryIndex(3, 3, 0), ds.StoryIndex(6, 5, 0)])
    return b, i


# ---------------------------------------------------------------- reference tests

def test_reads_story_by_offset_and_verifies_identity(tmp_path):
    b, i = tmp_path / "x.bytes", tmp_path / "x.idx"
    b.write_bytes(b"onetwo")
    provenance = hashlib.sha256(b"test provenance").digest()
    identity = ds.write_index(i, b, [ds.StoryIndex(0, 3, 0), ds.StoryIndex(3, 3, 0)], provenance)
    d = ds.PreparedDataset.open(b, i)
    assert d.identity() == identity
    assert d.story(1) == b"two"
    assert len(d) == 2 and d.entry(2) is None


def test_changed_middle_bytes_are_rejected(tmp_path):
    b, i = tmp_path / "m.bytes", tmp_path / "m.idx"
    b.write_bytes(b"abcdef")
    ds.write_index(i, b, [ds.StoryIndex(0, 6, 0)], ds.ZERO_DIGEST)
    b.write_bytes(b"abcXef")
    with pytest.raises(ds.DatasetError, match="bytes SHA-256"):
        ds.PreparedDataset.open(b, i)


def test_story_batches_honor_raw_byte_limits_without_splitting_records(tmp_path):
    d = ds.PreparedDataset.open(*three_stories(tmp_path))
    order = [0, 1, 2]
    assert ds.read_story_batch(d, order, 0, 3, 6) == ([b"one", b"two"], 2, 6)
    assert ds.read_story_batch(d, order, 2, 1, 4) == ([], 2, 0)


def test_prefetched_story_batch_matches_synchronous_reader(tmp_path):
    b, i = three_stories(tmp_path)
    order = [2, 0, 1]
    expected = ds.read_story_batch(ds.PreparedDataset.open(b, i), order, 0, 3, 8)
    with ds.StoryBatchPrefetcher(ds.PreparedDataset.open(b, i), order) as p:
        p.request(0, 3, 8)
        assert p.receive() == expected
    assert expected == ([b"three", b"one"], 2, 8)


def test_shuffle_is_reproducible_and_complete():
    first = ds.shuffled_story_order(100, 1337, 0)
    assert np.array_equal(first, ds.shuffled_story_order(100, 1337, 0))
    assert sorted(first.tolist()) == list(range(100))
    assert not np.array_equal(first, ds.shuffled_story_order(100, 1337, 1))


# ---------------------------------------------------------------- story order pins

def test_splitmix64_matches_published_output():
    # SplitMix64 from state 0 (Steele, Lea and Flood 2014; the generator of rng.rs).
    assert [int(x) for x in ds.splitmix64_draws(0, 3)] == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4,
                                                           0x06C45D188009454F]


@pytest.mark.parametrize("count,seed,pass_index", [(0, 0, 0), (1, 5, 0), (2, 1337, 0), (100, 1337, 0), (997, 1337, 4),
                                                   (4096, 2**64 - 1, 0), (4096, 2**64 - 3, 7), (200_000, 1337, 2)])
def test_story_order_matches_oracle(oracle_lib, count, seed, pass_index):
    got = ds.shuffled_story_order(count, seed, pass_index)
    want = oracle_lib.shuffled_story_order(count, seed, pass_index).astype(np.int64)
    assert np.array_equal(got, want)


# ---------------------------------------------------------------- index checks

def _index_bytes(tmp_path):
    b, i = three_stories(tmp_path)
    return b, i, bytearray(i.read_bytes())


def _reseal_header(raw: bytearray, recompute_id: bool = False) -> bytearray:
    if recompute_id:
        schema, _, count, length = struct.unpack_from("<IIQQ", raw, 8)
        raw[128:160] = ds.compute_dataset_id(schema, count, length, bytes(raw[32:64]), bytes(raw[64:96]),
                                             bytes(raw[96:128]))
    raw[160:192] = hashlib.sha256(bytes(raw[:160]) + bytes(32)).digest()
    return raw


def _records(raw: bytearray, records: list[tuple[int, int, int]]) -> bytearray:
    table = b"".join(struct.pack("<QII", *r) for r in records)
    raw = raw[:ds.INDEX_HEADER_SIZE] + bytearray(table)
    struct.pack_into("<Q", raw, 16, len(records))
    raw[64:96] = hashlib.sha256(table).digest()
    return _reseal_header(raw, recompute_id=True)


@pytest.mark.parametrize("edit,match", [
    (lambda r: r[:100], "smaller than the v1 header"),
    (lambda r: bytearray(b"LEODATA0") + r[8:], "magic"),
    (lambda r: _reseal_header(r[:8] + struct.pack("<I", 2) + r[12:]), "schema version"),
    (lambda r: _reseal_header(r[:12] + struct.pack("<I", 128) + r[16:]), "header size"),
    (lambda r: r[:40] + bytearray([r[40] ^ 1]) + r[41:], "header SHA-256"),
    (lambda r: _reseal_header(r[:24] + struct.pack("<Q", 12) + r[32:]), "byte length mismatch"),
    (lambda r: r + bytes(16), "index length mismatch"),
    (lambda r: r[:-1], "index length mismatch"),
    (lambda r: r[:ds.INDEX_HEADER_SIZE + 4] + bytearray([r[ds.INDEX_HEADER_SIZE + 4] ^ 1])
     + r[ds.INDEX_HEADER_SIZE + 5:], "record-table SHA-256"),
    (lambda r: _reseal_header(r[:100] + bytearray([r[100] ^ 1]) + r[101:]), "dataset ID"),
    (lambda r: _records(r, [(0, 3, 0), (3, 0, 0), (6, 5, 0)]), "story 1 has zero length"),
    (lambda r: _records(r, [(0, 3, 0), (2, 3, 0), (6, 5, 0)]), "story 1 overlaps"),
    (lambda r: _records(r, [(0, 3, 0), (3, 3, 0), (6, 6, 0)]), "story 2 extends past"),
    (lambda r: _records(r, [(0, 3, 0), (2**64 - 1, 2, 0)]), "range overflow"),
])
def test_damaged_index_is_rejected(tmp_path, edit, match):
    b, i, raw = _index_bytes(tmp_path)
    i.write_bytes(bytes(edit(raw)))
    with pytest.raises(ds.DatasetError, match=match):
        ds.PreparedDataset.open(b, i)


def test_records_may_leave_gaps_and_carry_split_flags(tmp_path):
    b, i = tmp_path / "g.bytes", tmp_path / "g.idx"
    b.write_bytes(b"xxonexxtwo")
    ds.write_index(i, b, [ds.StoryIndex(2, 3, 1), ds.StoryIndex(7, 3, 2)])
    d = ds.PreparedDataset.open(b, i)
    assert [d.story(0), d.story(1)] == [b"one", b"two"]
    assert d.entry(1) == ds.StoryIndex(7, 3, 2)


def test_writer_rejects_invalid_records(tmp_path):
    b = tmp_path / "w.bytes"
    b.write_bytes(b"abcdef")
    for entries in ([ds.StoryIndex(0, 0)], [ds.StoryIndex(0, 4), ds.StoryIndex(3, 2)], [ds.StoryIndex(4, 3)]):
        with pytest.raises(ds.DatasetError):
            ds.write_index(tmp_path / "w.idx", b, entries)


def test_invalid_utf8_story_is_rejected(tmp_path):
    b, i = tmp_path / "u.bytes", tmp_path / "u.idx"
    ds.prepare_dataset(b, i, [b"fine", b"\xff\xfe"])
    d = ds.PreparedDataset.open(b, i)
    assert d.story(0) == b"fine"
    with pytest.raises(ds.DatasetError, match="UTF-8"):
        d.story(1)
    with pytest.raises(ds.DatasetError, match="out of range"):
        d.story(2)


def test_clone_shares_the_table_and_reads_independently(tmp_path):
    d = ds.PreparedDataset.open(*three_stories(tmp_path))
    c = d.try_clone()
    d.close()
    assert c.story(2) == b"three" and c.identity().record_count == 3


def test_prefetcher_reports_reader_errors(tmp_path):
    d = ds.PreparedDataset.open(*three_stories(tmp_path))
    with ds.StoryBatchPrefetcher(d, [0, 7]) as p:
        p.request(0, 2, None)
        with pytest.raises(ds.DatasetError, match="out of range"):
            p.receive()


def test_pass_feed_stops_at_the_byte_limit(tmp_path):
    d = ds.PreparedDataset.open(*three_stories(tmp_path))
    assert list(ds.story_batches(d, [0, 1, 2], 2)) == [([b"one", b"two"], 2), ([b"three"], 3)]
    assert list(ds.story_batches(d, [0, 1, 2], 2, max_bytes=8)) == [([b"one", b"two"], 2)]
    assert list(ds.story_batches(d, [2, 1, 0], 1, max_bytes=100, position=1, bytes_seen=97)) == [([b"two"], 2)]
    assert list(ds.story_batches(d, [0, 1, 2], 2, position=3)) == []


# ---------------------------------------------------------------- golden case through the feed

GOLDEN = json.loads((HERE / "golden" / "story_batches.json").read_text())
CASES = {c["name"]: c for c in GOLDEN["cases"]}


def _golden_dataset(tmp_path, name):
    import sys

    from leo_b200.configs import WORKLOADS

    sys.path.insert(0, str(HERE / "golden"))
    from make_golden import case_stories

    case = CASES[name]
    batches = case_stories(case)
    stories = [s for batch in batches for s in batch]
    # Empty stories cannot be dataset records; the golden cases have none.
    assert all(stories)
    b, i = tmp_path / f"{name}.bytes", tmp_path / f"{name}.idx"
    ds.prepare_dataset(b, i, stories)
    return case, WORKLOADS[case["workload"]], ds.PreparedDataset.open(b, i), len(stories)


def test_golden_case_through_the_feed_on_the_oracle(oracle_lib, tmp_path):
    from leo_b200.ctypes_types import TRAINING

    case, w, d, n = _golden_dataset(tmp_path, "test")
    rt = oracle_lib.OracleRuntime(oracle_lib.OracleModel.initialize(w.config, w.topology))
    batches = list(ds.story_batches(d, np.arange(n), case["stories_per_batch"]))
    assert len(batches) == len(case["batches"])
    for rec, (stories, _) in zip(case["batches"], batches):
        assert hashlib.sha256(b"".join(stories)).hexdigest() == rec["stories_sha256"]
        rt.train_story_batch(stories, TRAINING, 0)
        assert rt.model.training_state_hash().hex() == rec["state_hash"]


@pytest.mark.gpu
def test_golden_case_through_the_feed_on_the_gpu(native_lib, tmp_path):
    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    case, w, d, n = _golden_dataset(tmp_path, "baseline1")
    model = HostModel.initialize(w.config, w.topology)
    with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as gpu:
        fed = 0
        for rec, (stories, _) in zip(case["batches"], ds.story_batches(d, np.arange(n), case["stories_per_batch"])):
            gpu.train_story_batch(stories, TRAINING)
            assert gpu.state_digest().hex() == rec["state_hash"]
            fed += 1
        assert fed == len(case["batches"])
