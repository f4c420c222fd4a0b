"""Loads ``libleo_b200.so`` (built in-tree by ``leo_b200.build``) and declares
the C ABI of ``include/leo_b200.h``.  There is no fallback: a missing library
is an error."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

from .ctypes_types import (
    LeoB200BatchReport,
    LeoB200Config,
    LeoB200HostModel,
    LeoB200PackedUpdate,
    LeoB200ParameterChanges,
    LeoB200ParameterChangeSizes,
    LeoB200PerfStats,
    LeoB200ShardStory,
    LeoB200StoryDeltas,
    LeoB200StoryDeltaSizes,
    LeoB200StorySummary,
)

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libleo_b200.so"
HEADER = PKG.parent / "include" / "leo_b200.h"

_lib: C.CDLL | None = None


class LeoError(RuntimeError):
    """A failed leo_b200 call (LeoError, crates/leo-core/src/lib.rs:43-55)."""


def exported_symbols() -> list[str]:
    """Function names declared by include/leo_b200.h."""
    text = HEADER.read_text(encoding="utf-8")
    return sorted(set(re.findall(r"\b(leo_b200_[a-z0-9_]+)\s*\(", text)))


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise LeoError(f"{LIB_PATH} is missing: run `python -m leo_b200.build` (no CPU fallback exists)")
    L = C.CDLL(str(LIB_PATH))
    vp, u32, u64, sz = C.c_void_p, C.c_uint32, C.c_uint64, C.c_size_t
    P = C.POINTER
    L.leo_b200_last_error.restype = C.c_char_p
    L.leo_b200_abi_version.restype = u32
    L.leo_b200_config_validate.argtypes = [P(LeoB200Config)]
    L.leo_b200_model_initialize.argtypes = [P(LeoB200Config), C.c_int, P(LeoB200HostModel)]
    L.leo_b200_model_validate.argtypes = [P(LeoB200HostModel)]
    L.leo_b200_training_state_hash.argtypes = [P(LeoB200HostModel), vp]
    L.leo_b200_open.argtypes = [C.c_int, P(LeoB200HostModel), u32, P(vp)]
    L.leo_b200_close.argtypes = [vp]
    L.leo_b200_close.restype = None
    L.leo_b200_upload_canonical.argtypes = [vp, P(LeoB200HostModel)]
    L.leo_b200_download_model.argtypes = [vp, P(LeoB200HostModel)]
    L.leo_b200_canonical_tick.argtypes = [vp]
    L.leo_b200_canonical_tick.restype = u64
    L.leo_b200_set_canonical_tick.argtypes = [vp, u64]
    L.leo_b200_set_story_chunk.argtypes = [vp, u32]
    L.leo_b200_set_device_context_merge.argtypes = [vp, C.c_int]
    L.leo_b200_shard_begin.argtypes = [vp, vp, vp, u32, u32, u32, C.c_int]
    L.leo_b200_shard_local.argtypes = [vp, P(LeoB200ShardStory), vp, P(sz)]
    L.leo_b200_shard_context.argtypes = [vp, vp, sz]
    L.leo_b200_shard_tensor_elements.argtypes = [vp, u32, P(sz)]
    L.leo_b200_shard_marks.argtypes = [vp, u32, vp]
    L.leo_b200_shard_plan.argtypes = [vp, u32, vp, P(u32)]
    L.leo_b200_shard_accumulate.argtypes = [vp, u32, vp, C.c_int]
    L.leo_b200_shard_finalize.argtypes = [vp, u32, vp, vp]
    L.leo_b200_shard_commit.argtypes = [vp, u32, vp]
    L.leo_b200_shard_finish.argtypes = [vp, P(LeoB200ShardStory), vp, vp, vp, u64, P(LeoB200BatchReport),
                                        P(LeoB200StorySummary), vp]
    L.leo_b200_set_hub_threshold.argtypes = [vp, u32, u32, u32]
    L.leo_b200_hub_count.argtypes = [vp, P(u32), P(u64)]
    L.leo_b200_set_segment_capacity_limit.argtypes = [vp, u32]
    L.leo_b200_sparse_mean_apply.argtypes = [C.c_int, vp, u32, vp, vp, vp, u32, C.c_float, C.c_float, vp, u32, vp,
                                             P(u32)]
    L.leo_b200_sparse_mean_apply_static.argtypes = L.leo_b200_sparse_mean_apply.argtypes
    L.leo_b200_sparse_apply_scratch_bytes.argtypes = [C.c_int]
    L.leo_b200_sparse_apply_scratch_bytes.restype = sz
    L.leo_b200_train_story_batch.argtypes = [vp, vp, vp, u32, C.c_int, P(LeoB200BatchReport),
                                             P(LeoB200StorySummary), vp]
    L.leo_b200_batch_begin.argtypes = [vp, vp, vp, u32, C.c_int]
    L.leo_b200_batch_steps.argtypes = [vp, u32, P(u32)]
    L.leo_b200_batch_finish.argtypes = [vp, P(LeoB200BatchReport), P(LeoB200StorySummary), vp]
    L.leo_b200_state_digest.argtypes = [vp, vp]
    L.leo_b200_lane_model.argtypes = [vp, u32, P(LeoB200HostModel)]
    L.leo_b200_lane_array.argtypes = [vp, u32, C.c_char_p, vp, sz, P(sz)]
    L.leo_b200_set_cluster_sizes.argtypes = [vp, u32, u32]
    L.leo_b200_perf_stats.argtypes = [vp, P(LeoB200PerfStats)]
    L.leo_b200_reset_perf_stats.argtypes = [vp]
    L.leo_b200_device_bytes.argtypes = [vp]
    L.leo_b200_device_bytes.restype = sz
    L.leo_b200_training_story_batch.argtypes = [vp, vp, vp, u32, C.c_int, P(LeoB200BatchReport),
                                                P(LeoB200StorySummary), vp, vp, vp]
    L.leo_b200_training_story_batch_deltas.argtypes = [vp, vp, vp, u32, C.c_int, P(LeoB200BatchReport),
                                                       P(LeoB200StorySummary), vp, vp, vp, P(LeoB200StoryDeltaSizes)]
    L.leo_b200_story_deltas.argtypes = [vp, P(LeoB200StoryDeltas)]
    L.leo_b200_begin_document.argtypes = [vp]
    L.leo_b200_reset_transient_state.argtypes = [vp]
    L.leo_b200_training_step_batch.argtypes = [vp, vp, vp, u32, C.c_int, vp, vp]
    L.leo_b200_advance_frozen_batch.argtypes = [vp, vp, vp, u32]
    L.leo_b200_enable_parameter_tracking.argtypes = [vp]
    L.leo_b200_parameter_changes.argtypes = [vp, P(LeoB200ParameterChangeSizes), P(LeoB200ParameterChanges)]
    L.leo_b200_synchronize_packed_model.argtypes = [vp, P(LeoB200PackedUpdate)]
    L.leo_b200_commit_packed_host_model.argtypes = [vp, P(LeoB200PackedUpdate)]
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != 0:
        raise LeoError(lib().leo_b200_last_error().decode())
