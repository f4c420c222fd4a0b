"""Benchmark: training bytes/s of Leo's per-byte story-batch step on B200.

One benchmark step is one logical story batch of the chosen workload (default
``baseline2``: 65,536 units, fan-in 64, 32 story workers, stories of 256-1024
bytes, 30 % bounded-surprise replay): the per-story pass over every lane, the
batch-end FP64 mean merge and lane sync, and serial canonical replay.  The
metric is input story bytes per second (``input_bytes`` of the reference's
``benchmark --train``, crates/leo-cli/src/main.rs:716,737,768).

* ``value``: story bytes of the K timed batches (all ranks) / the max over
  ranks of the batch time measured with CUDA events on the backend's stream.
* ``e2e``: the same bytes / the max over ranks of the wall time of the public
  call ``train_story_batch`` with host buffers (story bytes in, per-target
  losses and summaries out).
* ``roofline``: the wavefront kernel's algorithmic bytes per launch (per-unit
  figures below, units counted on the device) over its CUDA-event launch time,
  against the measured HBM copy bandwidth.
* ``cpu_baseline``: the CPU restatement of the reference backend (oracle/)
  started from the GPU model's state at the first timed batch and run on that
  batch's first stories, timed on this box's host cores.
* ``config3`` (one GPU): the same measurement on the 262,144-unit Zipf
  configuration (``baseline3``: 64 story workers of 512-2048 bytes) over a few
  batches -- a full 25-batch run of it does not fit the driver's time limit.

``--impl reference`` times the CPU implementation alone on the same workload
configuration, one bounded sample of stories per step, its model built by the
oracle's own initializer.  Under torchrun (N GPUs) one logical batch holds
``workers`` x N stories, sharded over the ranks with the exact batch-end merge
exchanged over NCCL and the serial replay run on every rank
(``leo_b200.parallel``; weak scaling: the lanes per GPU stay fixed); rank 0
prints one JSON line with the max-over-ranks batch time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train bytes/sec (box) at 1/2/4/8 B200; wavefront HBM GB/s vs peak"
UNIT = "bytes/s"

# Algorithmic bytes per unit of work (per-phase minimal traffic, FP32 = 4 B,
# index = 4 B, branch/delay = 1 B, tick = 4 B).
BYTES_PER_EVENT = 17 + 64          # target, branch, snapshot, branch r/w + trace record r/w
BYTES_PER_INPUT_SLOT = 9 + 8 + 64
BYTES_PER_TOUCHED_SETTLE = 130
BYTES_PER_TOUCHED_SURROGATE = 16
BYTES_PER_TOUCHED_HOMEOSTASIS = 12
BYTES_PER_ELIGIBLE = 101
BYTES_PER_DESTINATION = 1032
BYTES_PER_PLASTIC = 20
BYTES_PER_INHIBIT_SLOT = 16
BYTES_PER_SELECTION_RECORD = 8


def phase_algorithmic_bytes(p, cfg) -> dict[str, float]:
    """Algorithmic bytes moved by each phase over the counters' window (every
    unit counted on the device)."""
    S, D, K = cfg.synapses_per_neuron, cfg.context_embedding_dim, cfg.context_max_order
    events = p.work_active * S  # every emitted event is delivered once
    steps = p.work_steps
    return {
        "deliver": events * BYTES_PER_EVENT + steps * cfg.input_fanout * BYTES_PER_INPUT_SLOT,
        "settle": p.work_touched * BYTES_PER_TOUCHED_SETTLE,
        "blocks": p.work_winners * BYTES_PER_SELECTION_RECORD,
        "assemble": p.work_winners * BYTES_PER_SELECTION_RECORD,
        "surrogate": p.work_touched * BYTES_PER_TOUCHED_SURROGATE,
        "eligible": p.work_eligible * BYTES_PER_ELIGIBLE,
        "emit_forward": p.work_active * (50 + 8 * S + 1028) + steps * (257 * D * 4 + K * D * 4),
        "learn": p.work_destinations * BYTES_PER_DESTINATION + p.work_active * 2056
        + p.work_touched * BYTES_PER_TOUCHED_HOMEOSTASIS,
        "plasticity": p.work_plastic * BYTES_PER_PLASTIC,
        "inhibit": p.work_inhibit * BYTES_PER_INHIBIT_SLOT,
    }


def dram_traffic(workload: str, algorithmic_bytes_per_launch: float):
    """DRAM bytes per launch of the wavefront kernel: the ratio of DRAM traffic to
    algorithmic bytes measured by the committed one-pass ncu capture that stands
    in for this workload (a small case of the same model: its timed launches'
    dram__bytes_read.sum + dram__bytes_write.sum over the algorithmic bytes the
    same run counted), applied to this run's algorithmic bytes per launch; None
    without a capture."""
    path = ROOT / "profiles" / f"leo_wavefront_kernel-dram-{workload}.json"
    if not path.exists():
        return None, None
    data = json.loads(path.read_text())
    return round(data["dram_per_algorithmic_byte"] * algorithmic_bytes_per_launch, 1), path.name


def measured_peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"leo_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


def workload_config(workload, world: int) -> dict:
    """The ``config`` object of both arms' lines."""
    cfg = workload.config
    per_batch = workload.workers * world
    return {"workload": workload.name, "neurons": cfg.neuron_count, "synapses_per_neuron": cfg.synapses_per_neuron,
            "topology": "zipf(1.1) targets" if workload.topology == 2 else "uniform targets",
            "workers": workload.workers, "story_bytes": [workload.min_story_bytes, workload.max_story_bytes],
            "replay_fraction": cfg.replay_fraction,
            "parallelism": f"dp{world}: one logical batch of {per_batch} stories sharded over {world} GPU(s)"
                           f" ({workload.workers} lanes each), exact merge over NCCL, serial replay",
            "global_batch": per_batch, "l2": "per-batch working set (lanes x 0.3-2.2 GB) exceeds L2"}


def workload_batches(workload, per_batch: int, count: int) -> list[list[bytes]]:
    """The story stream both arms read: batch i is stories [i * per_batch, (i + 1) * per_batch)."""
    from leo_b200.synthetic import story_stream

    stories = story_stream(workload.story_seed, per_batch * count, workload.min_story_bytes, workload.max_story_bytes)
    return [stories[i * per_batch:(i + 1) * per_batch] for i in range(count)]


def oracle_batch(cfg, runtime, stories: list[bytes], threads: int) -> tuple[float, int]:
    """One story batch of the CPU restatement (one thread per story, merge and
    replay included); returns (seconds, story bytes)."""
    from leo_b200.ctypes_types import TRAINING

    t0 = time.perf_counter()
    runtime.train_story_batch(stories, TRAINING, threads)
    return time.perf_counter() - t0, sum(len(x) for x in stories)


def run_reference(args, workload) -> None:
    """The reference arm: the CPU restatement of the reference backend
    (oracle/, its own model initializer; no GPU library is loaded), each step a
    bounded sample -- the first ``--cpu-stories`` stories of the GPU arm's batch
    of the same index -- trained continuously like the GPU arm's batches."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle.oracle_py import OracleModel, OracleRuntime

    world = int(os.environ.get("WORLD_SIZE", "1"))
    cfg = workload.config
    n = min(args.cpu_stories, workload.workers * world)
    threads = min(n, os.cpu_count() or 1)
    runtime = OracleRuntime(OracleModel.initialize(cfg, workload.topology))
    batches = workload_batches(workload, workload.workers * world, args.warmup + args.steps)
    for b in range(args.warmup):
        oracle_batch(cfg, runtime, batches[b][:n], threads)
    seconds, nbytes = 0.0, 0
    for b in range(args.warmup, args.warmup + args.steps):
        dt, nb = oracle_batch(cfg, runtime, batches[b][:n], threads)
        seconds += dt
        nbytes += nb
    value = nbytes / seconds
    sample = (f"{args.steps} timed batch(es) after {args.warmup} warm-up, each the first {n} of the GPU arm's "
              f"{workload.workers * world} stories of that batch ({nbytes} bytes timed), one thread per story, "
              f"merge and replay included, trained continuously from the oracle's own initial model")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": seconds * 1000 / max(args.steps, 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded order-2 Markov printable-ASCII stories), random-init model",
            "config": workload_config(workload, world), "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_sparse_apply_micro(args) -> None:
    """Config 5: the batch-end sparse delta apply + replica sync of one 2^24-entry
    FP32 tensor at several densities.  Stories' sorted delta lists are generated
    on the device (each rank its contiguous share), all-gathered over NCCL when
    N > 1, and every rank applies all of them in story order with
    ``leo_b200_sparse_mean_apply`` (identical results on every rank).  Prints
    one JSON line per density: the apply's HBM GB/s (algorithmic bytes / CUDA
    event time) and the all-gather's NVLink GB/s (bytes received per GPU)."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from leo_b200.sparse_apply import sparse_mean_apply

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    n = 1 << 24
    stories, replicas = args.micro_stories, args.micro_replicas
    per = [stories // world + (1 if r < stories % world else 0) for r in range(world)]
    first = sum(per[:rank])
    peak, peak_kind = measured_peaks()
    for density in [float(x) for x in args.densities.split(",")]:
        idx_parts, val_parts, counts = [], [], []
        for sid in range(first, first + per[rank]):
            g = torch.Generator(device=dev)
            g.manual_seed(7000 + sid)
            idx = torch.nonzero(torch.rand(n, generator=g, device=dev) < density).flatten().to(torch.int32)
            val = torch.randn(idx.numel(), generator=g, device=dev) * 1e-3
            idx_parts.append(idx)
            val_parts.append(val)
            counts.append(idx.numel())
        local_idx = torch.cat(idx_parts) if idx_parts else torch.zeros(0, dtype=torch.int32, device=dev)
        local_val = torch.cat(val_parts) if val_parts else torch.zeros(0, device=dev)
        gather_ms, nvlink_bytes = 0.0, 0
        if world > 1:
            sizes = [None] * world
            dist.all_gather_object(sizes, counts)
            longest = max(sum(c) for c in sizes)
            pad_idx = torch.zeros(longest, dtype=torch.int32, device=dev)
            pad_val = torch.zeros(longest, device=dev)
            pad_idx[: local_idx.numel()] = local_idx
            pad_val[: local_val.numel()] = local_val
            all_idx = torch.empty(world * longest, dtype=torch.int32, device=dev)
            all_val = torch.empty(world * longest, device=dev)
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            dist.all_gather_into_tensor(all_idx, pad_idx)
            dist.all_gather_into_tensor(all_val, pad_val)
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            gather_ms = float(t[0])
            nvlink_bytes = (world - 1) * longest * 8
            flat_counts = [c for rc in sizes for c in rc]
            keep = []
            for r in range(world):
                total_r = sum(sizes[r])
                keep.append((r * longest, r * longest + total_r))
            indices = torch.cat([all_idx[a:b] for a, b in keep])
            deltas = torch.cat([all_val[a:b] for a, b in keep])
        else:
            flat_counts = counts
            indices, deltas = local_idx, local_val
        offsets = np.zeros(len(flat_counts) + 1, dtype=np.uint64)
        offsets[1:] = np.cumsum(flat_counts)
        g = torch.Generator(device=dev)
        g.manual_seed(4242)
        base = torch.rand(n, generator=g, device=dev) * 2.0 - 1.0
        target = base.clone()
        reps = [base.clone() for _ in range(replicas)]
        updates = 0
        for _ in range(args.warmup):
            updates = sparse_mean_apply(target, indices, deltas, offsets, -1.0, 1.0, reps)
        times = []
        for _ in range(args.steps):
            target.copy_(base)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            updates = sparse_mean_apply(target, indices, deltas, offsets, -1.0, 1.0, reps)
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = float(np.mean(times))
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t[0])
        entries = int(offsets[-1])
        alg = 8.0 * entries + (8.0 + 4.0 * replicas) * updates
        hbm = alg / (ms / 1000.0) / 1e9
        if rank == 0:
            line = {"metric": "sparse delta apply + replica sync (config 5)", "density": density, "n_gpus": world,
                    "stories": stories, "replicas": replicas, "elements": n, "entries": entries,
                    "merged": updates, "apply_ms": round(ms, 4), "steps": args.steps, "warmup": args.warmup,
                    "roofline": {"bound": "hbm", "achieved": round(hbm, 1), "peak": peak, "unit": "GB/s",
                                 "frac": round(hbm / peak, 4), "peak_source": peak_kind,
                                 "algorithmic_bytes": alg},
                    "nvlink": {"gather_ms": round(gather_ms, 4), "bytes_received_per_gpu": nvlink_bytes,
                               "GB_per_s": round(nvlink_bytes / (gather_ms / 1000.0) / 1e9, 1) if gather_ms else None},
                    "l2": "target + replicas exceed L2"}
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_sparse_apply_reference(args) -> None:
    """Config 5's reference arm: the reference's own CUDA path for the same job,
    built from its unmodified cuda_kernels.cu (oracle/ref_cuda/Makefile ->
    oracle/_ref/libleo_ref_kernels.so).  The same 32 stories' lists are merged
    (FP64 sum in story order over the union, divided by the stories: what the
    reference's host merge packs) outside the timed region; timed are the
    reference's apply kernel over the dense delta + index list
    (leo_apply_shared_wavefront_deltas) and the replica sync, one
    leo_scatter_f32 launch per replica.  One JSON line per density on rank 0;
    other ranks exit without work."""
    import ctypes as C

    import numpy as np
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    lib_path = ROOT / "oracle" / "_ref" / "libleo_ref_kernels.so"
    if not lib_path.exists():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libleo_ref_kernels.so was not built "
                          "(needs the reference checkout at build time)"}), flush=True)
        return
    lib = C.CDLL(str(lib_path))
    lib.leo_ref_last_error.restype = C.c_char_p
    vp, u32 = C.c_void_p, C.c_uint32
    lib.leo_ref_apply_sync.argtypes = [C.c_int, vp, vp, u32, u32, vp, vp, vp, u32, vp, u32, C.c_float, C.c_float,
                                       u32, C.POINTER(C.c_float), C.POINTER(C.c_float)]
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    n, S = 1 << 24, 64
    stories, replicas = args.micro_stories, args.micro_replicas
    peak, peak_kind = measured_peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    neuron_type = (torch.rand(n // S, generator=g, device=dev) < 0.2).to(torch.uint8)
    for density in [float(x) for x in args.densities.split(",")]:
        sums = torch.zeros(n, dtype=torch.float64, device=dev)
        touched = torch.zeros(n, dtype=torch.bool, device=dev)
        entries = 0
        for sid in range(stories):
            gs = torch.Generator(device=dev)
            gs.manual_seed(7000 + sid)
            idx = torch.nonzero(torch.rand(n, generator=gs, device=dev) < density).flatten()
            val = torch.randn(idx.numel(), generator=gs, device=dev) * 1e-3
            sums[idx] += val.to(torch.float64)
            touched[idx] = True
            entries += idx.numel()
        union = torch.nonzero(touched).flatten().to(torch.int32)
        merged = (sums[union.long()] / stories).to(torch.float32)
        gb = torch.Generator(device=dev)
        gb.manual_seed(4242)
        base = torch.rand(n, generator=gb, device=dev) * 2.0 - 1.0
        target = torch.empty_like(base)
        reps = [base.clone() for _ in range(replicas)]
        ptrs = (C.c_void_p * max(replicas, 1))(*[r.data_ptr() for r in reps])
        apply_ms, sync_ms = C.c_float(), C.c_float()
        torch.cuda.synchronize()

        def run(iters):
            rc = lib.leo_ref_apply_sync(0, base.data_ptr(), target.data_ptr(), n, S, neuron_type.data_ptr(),
                                        union.data_ptr(), merged.data_ptr(), union.numel(), ptrs, replicas, -1.0, 1.0,
                                        iters, C.byref(apply_ms), C.byref(sync_ms))
            if rc != 0:
                raise RuntimeError(lib.leo_ref_last_error().decode())

        run(args.warmup)
        run(args.steps)
        a_ms, s_ms = apply_ms.value / args.steps, sync_ms.value / args.steps
        m = union.numel()
        # apply: list, dense delta, weight read + write, dense + mark clears, changed mark and list;
        # sync: per replica index + value read and the weight write.
        alg = 32.0 * m + 12.0 * m * replicas
        ms = a_ms + s_ms
        hbm = alg / (ms / 1000.0) / 1e9
        print(json.dumps({
            "impl": "reference", "metric": "sparse delta apply + replica sync (config 5)", "density": density,
            "n_gpus": 1, "stories": stories, "replicas": replicas, "elements": n, "entries": entries, "merged": m,
            "apply_ms": round(a_ms, 4), "sync_ms": round(s_ms, 4), "ms": round(ms, 4), "steps": args.steps,
            "warmup": args.warmup,
            "roofline": {"bound": "hbm", "achieved": round(hbm, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(hbm / peak, 4), "peak_source": peak_kind, "algorithmic_bytes": alg},
            "path": "reference cuda_kernels.cu: leo_apply_shared_wavefront_deltas + leo_scatter_f32 per replica; "
                    "the 32-story merge itself is host work in the reference and is not timed"}), flush=True)


def measure_replay_off(backend, workload, args, device: int) -> dict:
    """The same model with replay fraction 0 (the reference's replay-off
    figure): one warm-up and `--steps` timed batches of fresh stories, CUDA-event
    batch time.  The main backend is closed first so both never hold the device."""
    from dataclasses import replace

    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel
    from leo_b200.synthetic import story_stream

    trained = backend.synchronize_model()
    model = HostModel(replace(workload.config, replay_fraction=0.0), trained.arrays)
    model.generation, model.parameter_revision, model.statistics = (trained.generation, trained.parameter_revision,
                                                                    trained.statistics)
    backend.close()
    n = workload.workers
    stories = story_stream(workload.story_seed + 1, n * (args.steps + 1), workload.min_story_bytes,
                           workload.max_story_bytes)
    with GpuBackend(model, device=device, max_lanes=2 * n) as off:
        off.train_story_batch(stories[:n], TRAINING)
        off.reset_perf_stats()
        nbytes = 0
        for b in range(1, args.steps + 1):
            batch = stories[b * n:(b + 1) * n]
            off.train_story_batch(batch, TRAINING)
            nbytes += sum(len(s) for s in batch)
        ms = off.perf_stats().batch_ms
    return {"value": round(nbytes / (ms / 1000.0), 3), "unit": UNIT, "ms_per_step": round(ms / args.steps, 3),
            "batches": args.steps, "note": "same model, replay fraction 0, fresh stories"}


def roofline_of(perf, cfg, workload_name: str) -> dict:
    """The wavefront kernel's roofline over the counters' window."""
    peak, peak_kind = measured_peaks()
    alg = phase_algorithmic_bytes(perf, cfg)
    launches = max(perf.wavefront_launches, 1)
    per_launch_ms = perf.wavefront_ms / launches
    per_launch_bytes = sum(alg.values()) / launches
    achieved = per_launch_bytes / (per_launch_ms / 1000.0) / 1e9 if per_launch_ms > 0 else 0.0
    cycles = np.array(list(perf.phase_cycles)[:10], dtype=np.float64)
    from leo_b200.ctypes_types import PHASES

    shares = {PHASES[i]: round(float(cycles[i] / max(cycles.sum(), 1.0)), 4) for i in range(10)}
    traffic, traffic_source = dram_traffic(workload_name, per_launch_bytes)
    return {"bound": "hbm", "kernel": "leo_wavefront_kernel", "achieved": round(achieved, 3), "peak": peak,
            "unit": "GB/s", "frac": round(achieved / peak, 6), "peak_source": peak_kind, "traffic": traffic,
            "traffic_source": traffic_source, "algorithmic_bytes_per_launch": round(per_launch_bytes, 1),
            "algorithmic_bytes_by_phase": {k: round(v / launches, 1) for k, v in alg.items()},
            "frac_of_nominal_8tbs": round(achieved / 8000.0, 6), "launch_ms": round(per_launch_ms, 4),
            "launches": int(perf.wavefront_launches),
            "share_of_step_time": round(perf.wavefront_ms / max(perf.batch_ms, 1e-9), 4),
            "phase_cycle_shares": shares,
            "clusters": {"story": perf.story_cluster, "replay": perf.replay_cluster}}


def replay_step_us(perf) -> dict:
    """Replay lane: wall microseconds per step by phase (first CTA's clock)."""
    from leo_b200.ctypes_types import PHASES

    steps = max(int(perf.replay_work_steps), 1)
    mhz = 1965.0
    return {PHASES[i]: round(perf.replay_phase_cycles[i] / mhz / steps, 2) for i in range(len(PHASES))}


def measure_big(args, device: int) -> dict:
    """The 262,144-unit configuration over a few batches on one GPU (a 25-batch
    run of it does not fit the driver's limit): CUDA-event batch time after
    one warm-up batch, its roofline and its replay step breakdown."""
    from leo_b200.backend import GpuBackend
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    workload = WORKLOADS[args.big_workload]
    cfg = workload.config
    model = HostModel.initialize(cfg, workload.topology)
    batches = workload_batches(workload, workload.workers, 1 + args.big_batches)
    with GpuBackend(model, device=device, max_lanes=workload.workers) as big:
        big.train_story_batch(batches[0], TRAINING)
        big.reset_perf_stats()
        wall, nbytes, batch_ms = 0.0, 0, []
        for b in range(1, 1 + args.big_batches):
            before = big.perf_stats().batch_ms
            t0 = time.perf_counter()
            big.train_story_batch(batches[b], TRAINING)
            wall += time.perf_counter() - t0
            batch_ms.append(round(big.perf_stats().batch_ms - before, 1))
            nbytes += sum(len(x) for x in batches[b])
        perf = big.perf_stats()
        device_gb = round(big.device_bytes() / 1e9, 3)
    device_s = perf.batch_ms / 1000.0
    return {"config": workload_config(workload, 1), "value": round(nbytes / device_s, 3), "unit": UNIT,
            "e2e_value": round(nbytes / wall, 3), "timed_batches": args.big_batches, "warmup_batches": 1,
            "ms_per_step": round(device_s * 1000 / args.big_batches, 1), "batch_ms": batch_ms,
            "story_pass_ms_per_step": round(perf.story_wavefront_ms / args.big_batches, 1),
            "replay_ms_per_step": round(perf.replay_ms / args.big_batches, 1),
            "replay_steps_per_batch": round(perf.replay_work_steps / args.big_batches, 1),
            "replay_us_per_step_by_phase": replay_step_us(perf),
            "roofline": roofline_of(perf, cfg, workload.name), "device_gb": device_gb,
            "note": "not the headline: the driver's 25-batch run of this configuration would exceed its time limit"}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default="baseline2")
    ap.add_argument("--cpu-stories", type=int, default=16,
                    help="stories of the CPU samples (state-matched cpu_baseline, reference arm steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-replay-off", action="store_true",
                    help="skip the replay-off figure (same model, replay fraction 0) that follows the timed batches")
    ap.add_argument("--big-workload", default="baseline3")
    ap.add_argument("--big-batches", type=int, default=3,
                    help="timed batches of the 262,144-unit configuration reported as `config3` (0: skip)")
    ap.add_argument("--micro", choices=["sparse-apply"], default=None,
                    help="run a microbenchmark instead of the training step (config 5)")
    ap.add_argument("--densities", default="0.001,0.01,0.1")
    ap.add_argument("--micro-stories", type=int, default=32)
    ap.add_argument("--micro-replicas", type=int, default=8)
    args = ap.parse_args()
    if args.micro == "sparse-apply":
        if args.impl == "reference":
            run_sparse_apply_reference(args)
        else:
            run_sparse_apply_micro(args)
        return

    from leo_b200.configs import WORKLOADS

    workload = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, workload)
        return

    from leo_b200.backend import GpuBackend
    from leo_b200.ctypes_types import TRAINING
    from leo_b200.model import HostModel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    ex = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        from leo_b200.parallel import TorchExchange

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
        host_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=300))
        ex = TorchExchange(None, host_group)

    from leo_b200.parallel import sharded_story_batch

    cfg = workload.config
    model = HostModel.initialize(cfg, workload.topology)
    # Weak scaling: every GPU runs `workers` story lanes of one logical batch of workers x N stories.
    per_batch = workload.workers * world
    backend = GpuBackend(model, device=local, max_lanes=2 * workload.workers)
    total_batches = args.warmup + args.steps
    batches = workload_batches(workload, per_batch, total_batches)

    def run_batch(batch):
        if ex is None:
            return backend.train_story_batch(batch, TRAINING)
        return sharded_story_batch(backend, ex, batch, TRAINING)

    for b in range(args.warmup):
        run_batch(batches[b])
    # The state the first timed batch starts from, for the state-matched CPU baseline.
    snapshot = None
    if rank == 0 and not args.no_cpu_baseline:
        trained = backend.synchronize_model().copy()
        snapshot = (trained, backend.canonical_tick)
    backend.reset_perf_stats()

    if dist is not None:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    wall = 0.0
    nbytes = 0
    h2d = d2h = 0
    story_steps = replay_steps = 0
    for b in range(args.warmup, total_batches):
        batch = batches[b]
        t0 = time.perf_counter()
        result = run_batch(batch)
        wall += time.perf_counter() - t0
        nbytes += sum(len(s) for s in batch)
        h2d += sum(len(s) for s in batch) + 8 * (len(batch) + 1)
        d2h += 4 * sum(len(x) for x in result.losses) + 48 * len(batch) + 80
        story_steps += sum(len(s) + 1 for s in batch if s)
        replay_steps += int(result.report.replay_steps) + int(result.report.replay_prefix_steps)
    perf = backend.perf_stats()
    clk = clocks.stop()
    device_s = perf.batch_ms / 1000.0
    device_gb = round(backend.device_bytes() / 1e9, 3)
    replay_off = None
    if world == 1 and cfg.replay_fraction > 0 and not args.no_replay_off:
        replay_off = measure_replay_off(backend, workload, args, local)
    backend.close()
    times = np.array([device_s, wall], dtype=np.float64)
    if dist is not None:
        import torch

        t = torch.tensor(times, dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        device_s, wall = float(t[0]), float(t[1])
    total_bytes = float(nbytes)  # every rank passes the whole logical batch

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(total_bytes / device_s, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(device_s * 1000 / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded order-2 Markov printable-ASCII stories), random-init model",
            "config": workload_config(workload, world),
            "e2e": {"value": round(total_bytes / wall, 3), "unit": UNIT, "h2d_bytes_per_step": h2d // args.steps,
                    "d2h_bytes_per_step": d2h // args.steps},
            "roofline": roofline_of(perf, cfg, workload.name), "clocks": clk, "gpu_launches": int(perf.launches),
            "steps_per_second": round(story_steps / device_s, 1),
            "execution_steps_per_second": round((story_steps + replay_steps) / device_s, 1),
            "replay_off": replay_off,
            "batch_end_ms_per_step": {k: round(getattr(perf, k) / args.steps, 2)
                                      for k in ("collect_ms", "merge_fixed_ms", "merge_context_ms", "replay_ms",
                                                "replay_sync_ms")},
            "replay_us_per_step_by_phase": replay_step_us(perf),
            "device_gb": device_gb,
        }
        if snapshot is not None:
            from oracle.oracle_py import OracleModel, OracleRuntime

            trained, tick = snapshot
            gen, rev, stats = trained.generation, trained.parameter_revision, trained.statistics
            n = min(args.cpu_stories, per_batch)
            threads = min(n, os.cpu_count() or 1)
            runtime = OracleRuntime(OracleModel.from_arrays(cfg, trained.arrays, gen, rev, stats))
            runtime.tick = tick
            seconds, sample_bytes = oracle_batch(cfg, runtime, batches[args.warmup][:n], threads)
            line["cpu_baseline"] = {
                "value": sample_bytes / seconds, "unit": UNIT, "cores": threads, "kind": "port",
                "sample": f"the first {n} stories ({sample_bytes} bytes) of the first timed batch, started from the "
                          f"GPU model's state at that batch (same weights, statistics and tick), one thread per "
                          f"story, merge and replay included; {seconds:.1f} s of CPU work"}
        if world == 1 and args.big_batches > 0:
            line["config3"] = measure_big(args, local)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
