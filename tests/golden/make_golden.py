"""Generate the golden story-batch fixtures from the CPU oracle.

Usage: ``python tests/golden/make_golden.py [case ...]`` (writes
``story_batches.json`` beside this file; with case names, only those cases are
regenerated and the others kept).  The ``-full`` cases reach the regime the
benchmark times (hundreds of actives and up to 10^6 eligible slots per step,
whole-GPU replay segments, natural hub tiers) and take the oracle tens of
minutes.

The reference holds no value-level golden vectors for the story batch (its
historical digests need a corpus that is not available), so these fixtures
record what the oracle -- the restatement of the reference CPU backend, itself
pinned by the reference's known-answer tests -- produces on seeded synthetic
stories: the SHA-256 of the story bytes, and after each logical batch the
``training_state_hash`` (crates/leo-cli/src/main.rs:1151-1202), the SHA-256 of
the per-target losses (f32 little-endian), the batch report, the replay ranges
(crates/leo-cli/src/training.rs:1782-1830), the parameter revision and the
training statistics.  Both the oracle (on CPU) and the GPU path (on a B200) are
checked against them.
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

# (case name, workload, batches, stories per batch, min / max story bytes, story seed)
CASES = [
    ("test", "test", 3, 4, 8, 48, 0),
    ("test-8", "test", 2, 8, 8, 64, 17),
    ("probe", "probe", 1, 4, 256, 1024, 0),
    ("baseline1", "baseline1", 2, 4, 256, 1024, 0),
    ("baseline2-short", "baseline2", 2, 4, 48, 96, 5),
    ("baseline3-short", "baseline3", 1, 4, 24, 48, 9),
    ("baseline2-full", "baseline2", 3, 32, 256, 1024, 11),
    ("baseline3-full", "baseline3", 1, 8, 512, 2048, 13),
]


def case_stories(case: dict) -> list[list[bytes]]:
    """The case's stories, split into its batches."""
    from leo_b200.synthetic import story_stream

    n = case["stories_per_batch"]
    stories = story_stream(case["story_seed"], n * case["batch_count"], case["min_story_bytes"],
                           case["max_story_bytes"])
    return [stories[i * n:(i + 1) * n] for i in range(case["batch_count"])]


def record_batches(name: str, workload_name: str, batches: int, per_batch: int, min_bytes: int, max_bytes: int,
                   seed: int) -> dict:
    from leo_b200.configs import WORKLOADS
    from leo_b200.ctypes_types import TRAINING
    from oracle.oracle_py import OracleModel, OracleRuntime

    w = WORKLOADS[workload_name]
    out = {"name": name, "workload": workload_name, "stories_per_batch": per_batch, "batch_count": batches,
           "min_story_bytes": min_bytes, "max_story_bytes": max_bytes, "story_seed": seed, "batches": []}
    model = OracleModel.initialize(w.config, w.topology)
    rt = OracleRuntime(model)
    out["initial_state_hash"] = rt.model.training_state_hash().hex()
    for batch in case_stories(out):
        report, losses, ranges = rt.train_story_batch(batch, TRAINING, 0)
        gen, rev, stats = rt.model.scalars()
        out["batches"].append({
            "stories_sha256": hashlib.sha256(b"".join(batch)).hexdigest(),
            "story_lengths": [len(s) for s in batch],
            "state_hash": rt.model.training_state_hash().hex(),
            "losses_sha256": hashlib.sha256(losses.astype("<f4").tobytes()).hexdigest(),
            "mean_loss": report.mean_loss,
            "report": {k: int(getattr(report, k)) for k, _ in report._fields_ if k != "mean_loss"},
            "replay_ranges": ranges,
            "generation": int(gen),
            "parameter_revision": int(rev),
            "statistics": {k: (float(getattr(stats, k)) if k == "training_loss_sum" else int(getattr(stats, k)))
                           for k, _ in stats._fields_},
            "canonical_tick": int(rt.tick),
        })
    return out


def main() -> None:
    from oracle import oracle_py

    oracle_py.build()
    path = HERE / "story_batches.json"
    wanted = set(sys.argv[1:])
    unknown = wanted - {c[0] for c in CASES}
    if unknown:
        raise SystemExit(f"unknown case(s): {sorted(unknown)}")
    old = {c["name"]: c for c in json.loads(path.read_text())["cases"]} if wanted and path.exists() else {}
    cases = []
    for c in CASES:
        if wanted and c[0] not in wanted and c[0] in old:
            cases.append(old[c[0]])
        else:
            cases.append(record_batches(*c))
            print(f"recorded {c[0]}", flush=True)
    data = {"generator": "tests/golden/make_golden.py", "cases": cases}
    path.write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
