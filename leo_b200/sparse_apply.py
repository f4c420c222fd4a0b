"""Batch-end sparse mean apply of one tensor (``leo_b200_sparse_mean_apply``).

``sparse_mean_apply`` restates ``apply_sparse_scaled``
(crates/leo-core/src/parallel.rs:975-1022) with divisor = number of stories,
the clamp projection of parallel.rs:1226-1233 and the replica sync of the
packed-update scatter (crates/leo-core/src/cuda.rs:2869-3080) on CUDA tensors.
PyTorch only owns the device memory and the stream here; the work is the
in-tree sm_100a kernels behind the C ABI.
"""

from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import native


def _stream_handle(stream) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def sparse_mean_apply(target, indices, deltas, story_offsets: Sequence[int], lo: float = float("-inf"),
                      hi: float = float("inf"), replicas: Sequence = (), stream=None) -> int:
    """Applies the stories' sorted sparse deltas to ``target`` in place and
    writes the merged values into every tensor of ``replicas``; returns the
    number of merged indices.

    ``target`` and each replica: contiguous float32 CUDA tensors of one length;
    ``indices`` (int32 / uint32) and ``deltas`` (float32): CUDA tensors holding
    the stories' lists back to back; ``story_offsets``: ``stories + 1`` host
    integers delimiting them.
    """
    import torch

    for t in (target, deltas, *replicas):
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("target, deltas and replicas must be contiguous float32 CUDA tensors")
    if indices.dtype not in (torch.int32, torch.uint32) or not indices.is_cuda or not indices.is_contiguous():
        raise ValueError("indices must be a contiguous int32 CUDA tensor")
    if any(r.numel() != target.numel() for r in replicas):
        raise ValueError("replicas must have the target's length")
    offsets = np.ascontiguousarray(np.asarray(story_offsets, dtype=np.uint64))
    table = (C.c_void_p * max(len(replicas), 1))(*[r.data_ptr() for r in replicas])
    updates = C.c_uint32()
    native.check(native.lib().leo_b200_sparse_mean_apply(
        target.device.index, target.data_ptr(), target.numel(), indices.data_ptr(), deltas.data_ptr(),
        offsets.ctypes.data, len(offsets) - 1, lo, hi, table, len(replicas), _stream_handle(stream),
        C.byref(updates)))
    return updates.value
