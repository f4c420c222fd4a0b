"""Helpers comparing a GPU lane with an oracle runtime field by field.

Tolerance: the kernels reproduce the reference's FP32 operation order, so
every field is compared for exact (bitwise) equality -- max-abs error 0 and
relative error 0 after N steps.  Worklists are compared as sets (the GPU
appends with atomics, the CPU with swap_remove), active lists in order.
"""

from __future__ import annotations

import numpy as np

from leo_b200.ctypes_types import BEGIN_DOCUMENT, END_DOCUMENT

NEURON_FLOATS = ["membrane", "fatigue", "adaptation_fast", "adaptation_medium", "adaptation_slow", "activation",
                 "branches", "selection_surrogate"]
NEURON_TICKS = ["refractory_until"]
TRACE_FIELDS = ["branch_sensitivity", "membrane_sensitivity", "fatigue_sensitivity", "adaptation_fast_sensitivity",
                "adaptation_medium_sensitivity", "adaptation_slow_sensitivity", "eligibility"]
PARAMS = ["threshold", "recurrent_weight", "input_weight", "output_weight", "output_bias", "context_keys",
          "context_embeddings", "context_observations", "context_output_weight"]


def story_steps(story: bytes) -> list[tuple[int, int]]:
    """train_document_pass's (input, target) schedule (training.rs:1747-1757)."""
    steps = [(BEGIN_DOCUMENT, story[0])]
    steps += [(story[i], story[i + 1]) for i in range(len(story) - 1)]
    steps.append((story[-1], END_DOCUMENT))
    return steps


def _diff(name, a, b, out):
    a = np.asarray(a)
    b = np.asarray(b)
    if a.shape != b.shape:
        out.append(f"{name}: shape {a.shape} vs {b.shape}")
        return
    if a.dtype.kind == "f":
        same = a.view(np.uint32 if a.dtype == np.float32 else np.uint64) == b.astype(a.dtype).view(
            np.uint32 if a.dtype == np.float32 else np.uint64)
        if not same.all():
            idx = np.flatnonzero(~same)
            err = float(np.max(np.abs(a.astype(np.float64) - b.astype(np.float64))))
            out.append(f"{name}: {idx.size} differ, first {idx[:5].tolist()} gpu {a.flat[idx[0]]!r} "
                       f"cpu {b.flat[idx[0]]!r} max_abs {err:.3g}")
    elif not np.array_equal(a, b):
        idx = np.flatnonzero(a != b)
        out.append(f"{name}: {idx.size} differ, first {idx[:5].tolist()} gpu {a.flat[idx[0]]} cpu {b.flat[idx[0]]}")


def compare_lane(backend, lane: int, rt, *, params: bool = True) -> list[str]:
    """Every transient and learned field of `lane` against oracle runtime `rt`."""
    out: list[str] = []
    for name in NEURON_FLOATS:
        _diff(name, backend.lane_array(lane, name, np.float32), rt.array(name).astype(np.float32), out)
    for name in NEURON_TICKS:
        _diff(name, backend.lane_array(lane, name, np.uint64), rt.array(name), out)
    _diff("active", backend.lane_array(lane, "active", np.uint64), rt.array("active"), out)
    g_elig = np.sort(backend.lane_array(lane, "eligible_recurrent_slots", np.uint64))
    c_elig = np.sort(rt.array("eligible_recurrent_slots"))
    _diff("eligible_recurrent_slots", g_elig, c_elig, out)
    g_in = np.sort(backend.lane_array(lane, "eligible_input_slots", np.uint64))
    c_in = np.sort(rt.array("eligible_input_slots"))
    _diff("eligible_input_slots", g_in, c_in, out)
    for field in TRACE_FIELDS:
        for kind, slots in (("rec_", c_elig), ("input_", c_in)):
            g = backend.lane_array(lane, kind + field, np.float32)
            c = rt.array(kind + field)
            _diff(kind + field, g, c, out)
    _diff("population_inhibition", backend.lane_array(lane, "population_inhibition", np.float32),
          rt.array("population_inhibition"), out)
    if params:
        gm = backend.lane_model(lane).arrays
        cm = rt.model.arrays()
        for name in PARAMS:
            _diff(name, gm[name], cm[name], out)
    return out
