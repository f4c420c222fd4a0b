"""Exact logical-batch data parallelism (``leo_b200.parallel``).

CPU: the story partition against the reference's own tests
(crates/leo-cli/src/training.rs:1990-2060), and the fixed-tensor exchange run
by two gloo processes with a stand-in backend, checked bit for bit against the
oracle's single-process ``apply_sparse_scaled`` (parallel.rs:975-1022).
GPU: two and three ranks run as threads on one GPU through the real device
steps and must reproduce the single-GPU golden state hashes.
"""

import os
import socket

import numpy as np
import pytest

from leo_b200.parallel import story_work, work_balanced_story_ranges


def test_ranges_cover_batch_and_reduce_straggler_work():
    stories = [b"a" * 100] + [b"x"] * 5
    ranges = work_balanced_story_ranges(stories, 2)
    assert ranges[0][0] == 0 and ranges[-1][1] == len(stories)
    assert ranges[0][1] == ranges[1][0]
    work = [sum(story_work(s) for s in stories[a:b]) for a, b in ranges]
    count_ranges = [(0, 3), (3, 6)]
    count_work = [sum(story_work(s) for s in stories[a:b]) for a, b in count_ranges]
    assert max(work) <= max(count_work)


def test_sixteen_devices_can_own_one_story_each():
    stories = [bytes([65 + i]) * (i + 1) for i in range(16)]
    ranges = work_balanced_story_ranges(stories, 16)
    assert ranges == [(i, i + 1) for i in range(16)]


@pytest.mark.parametrize("seed", range(6))
def test_ranges_are_contiguous_nonempty_and_ordered(seed):
    rng = np.random.default_rng(seed)
    stories = [b"s" * int(n) for n in rng.integers(0, 300, size=int(rng.integers(1, 40)))]
    for shards in (1, 2, 3, 8, 64):
        ranges = work_balanced_story_ranges(stories, shards)
        assert len(ranges) == min(shards, len(stories))
        assert ranges[0][0] == 0 and ranges[-1][1] == len(stories)
        for (a, b), (c, d) in zip(ranges, ranges[1:]):
            assert b == c
        assert all(b > a for a, b in ranges)


# ---------------------------------------------------------------- gloo exchange with a stand-in backend

TENSOR_LENGTHS = [50, 400, 30, 780, 257, 514]
STORIES = 7


def story_lengths():
    return [b"x" * n for n in (40, 3, 70, 12, 0, 33, 51)]


def lane_tensors(tensor: int):
    """Base tensor and every story's lane copy (sparse random changes)."""
    rng = np.random.default_rng(100 + tensor)
    n = TENSOR_LENGTHS[tensor]
    base = rng.uniform(-0.9, 0.9, size=n).astype(np.float32)
    lanes = []
    for s in range(STORIES):
        lane = base.copy()
        pick = rng.random(n) < 0.2
        lane[pick] = (lane[pick] + rng.normal(0, 0.05, size=int(pick.sum()))).astype(np.float32)
        if s == 2 and tensor == 1:
            lane[:5] = np.float32(1.7)  # pushed past the clamp
        lanes.append(lane)
    return base, lanes


class FakeTensorBackend:
    """The rank-local merge steps on numpy, with torch CPU tensors as buffers."""

    def __init__(self, first: int, count: int, poison: bool = False):
        import torch

        self.torch = torch
        self.first, self.count = first, count
        self.base = {}
        self.lanes = {}
        for t in range(len(TENSOR_LENGTHS)):
            base, lanes = lane_tensors(t)
            self.base[t] = base
            self.lanes[t] = lanes[first:first + count]
            if poison and t == 1 and count:
                self.lanes[t][0] = self.lanes[t][0].copy()
                self.lanes[t][0][7] = np.float32("nan")
        self.lists = {}

    def tensor_elements(self, t):
        return TENSOR_LENGTHS[t]

    def empty(self, count, dtype):
        return self.torch.empty(max(count, 1), dtype=getattr(self.torch, dtype))

    def marks(self, t, out):
        m = np.zeros(TENSOR_LENGTHS[t], dtype=np.uint8)
        for lane in self.lanes[t]:
            m |= (lane - self.base[t] != 0).astype(np.uint8)
        out.numpy()[:] = m

    def plan(self, t, marks):
        self.lists[t] = np.flatnonzero(marks.numpy())
        return int(self.lists[t].size)

    def accumulate(self, t, partial, first):
        p = partial.numpy()
        idx = self.lists[t]
        if first:
            p[: idx.size] = 0.0
        for lane in self.lanes[t]:
            d = (lane[idx] - self.base[t][idx]).astype(np.float32)
            if not np.all(np.isfinite(d)):
                raise RuntimeError("invalid sparse worker parameter delta")
            nz = d != 0
            p[: idx.size][nz] = p[: idx.size][nz] + d[nz].astype(np.float64)

    def finalize(self, t, partial, values):
        idx = self.lists[t]
        v = (self.base[t][idx] + (partial.numpy()[: idx.size] / STORIES).astype(np.float32)).astype(np.float32)
        values.numpy()[: idx.size] = np.clip(v, np.float32(-1.0), np.float32(1.0))

    def commit(self, t, values):
        idx = self.lists[t]
        self.base[t][idx] = values.numpy()[: idx.size]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, poison, queue):
    import torch.distributed as dist

    from leo_b200.parallel import TorchExchange, exchange_fixed_tensors, work_balanced_story_ranges

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ranges = work_balanced_story_ranges(story_lengths(), world)
        first, end = ranges[rank]
        backend = FakeTensorBackend(first, end - first, poison=poison and rank == 1)
        ex = TorchExchange()
        try:
            updates = exchange_fixed_tensors(backend, ex)
            queue.put((rank, "ok", updates, {t: backend.base[t].tobytes() for t in backend.base}))
        except Exception as e:  # noqa: BLE001 - reported to the test
            queue.put((rank, "error", str(e), None))
    finally:
        dist.destroy_process_group()


def _run_gloo(world, poison=False):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, poison, queue)) for r in range(world)]
    for p in procs:
        p.start()
    out = [queue.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return sorted(out)


def test_gloo_exchange_matches_single_process_mean(oracle_lib):
    out = _run_gloo(2)
    assert all(status == "ok" for _, status, _, _ in out)
    assert out[0][2] == out[1][2]
    assert out[0][3] == out[1][3], "ranks disagree after the exchange"
    total_updates = 0
    for t in range(len(TENSOR_LENGTHS)):
        base, lanes = lane_tensors(t)
        idx_parts, val_parts, offsets = [], [], [0]
        for lane in lanes:
            d = (lane - base).astype(np.float32)
            nz = np.flatnonzero(d != 0)
            idx_parts.append(nz.astype(np.uint32))
            val_parts.append(d[nz])
            offsets.append(offsets[-1] + nz.size)
        want = base.copy()
        total_updates += oracle_lib.sparse_mean_apply(want, np.concatenate(idx_parts), np.concatenate(val_parts),
                                                      np.array(offsets, dtype=np.uint64), -1.0, 1.0)
        got = np.frombuffer(out[0][3][t], dtype=np.float32)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"tensor {t}"
    assert out[0][2] == total_updates


def test_gloo_exchange_error_reaches_every_rank():
    out = _run_gloo(2, poison=True)
    assert all(status == "error" for _, status, _, _ in out)


# ---------------------------------------------------------------- GPU: ranks as threads on one device

@pytest.mark.gpu
@pytest.mark.parametrize("world,case_name", [(2, "baseline1"), (3, "test-8"), (2, "baseline2-short")])
def test_sharded_batch_matches_single_gpu_golden(native_lib, world, case_name):
    import json
    from pathlib import Path

    from parallel_helpers import run_ranks

    from leo_b200.backend import GpuBackend
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel
    from leo_b200.parallel import sharded_story_batch

    golden = json.loads((Path(__file__).resolve().parent / "golden" / "story_batches.json").read_text())
    case = {c["name"]: c for c in golden["cases"]}[case_name]
    import sys

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    from make_golden import case_stories

    w = WORKLOADS[case["workload"]]
    batches = case_stories(case)
    model = HostModel.initialize(w.config, w.topology)

    def rank_fn(rank, ex):
        digests = []
        with GpuBackend(model, device=0, max_lanes=case["stories_per_batch"]) as gpu:
            for batch in batches:
                result = sharded_story_batch(gpu, ex, batch, TRAINING)
                digests.append((gpu.state_digest().hex(), gpu.canonical_tick,
                                int(result.report.fixed_parameter_updates), int(result.report.replay_steps)))
        return digests

    results = run_ranks(world, rank_fn)
    for rank_digests in results:
        for b, (digest, tick, updates, replay_steps) in enumerate(rank_digests):
            rec = case["batches"][b]
            assert digest == rec["state_hash"], f"batch {b}"
            assert tick == rec["canonical_tick"]
            assert updates == rec["report"]["fixed_parameter_updates"]
            assert replay_steps == rec["report"]["replay_steps"]
