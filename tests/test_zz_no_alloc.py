"""The allocation-free sparse apply (``leo_b200_sparse_mean_apply_static``).

Called through the C ABI with ctypes on device memory the test owns; its
output must equal the allocating entry point ``leo_b200_sparse_mean_apply`` on
the same inputs (tolerance: bitwise equality) on two calls in a row, which
also shows the fixed scratch's counters are re-zeroed by each call.  This file
is collected last so that it also runs after every other GPU test in one
process; it passes alone as well.
"""

import ctypes as C

import numpy as np
import pytest

from test_sparse_apply import make_case


def _call(fn, target, idx, dl, offsets, replicas, lo=-1.0, hi=1.0):
    import torch

    table = (C.c_void_p * max(len(replicas), 1))(*[r.data_ptr() for r in replicas])
    updates = C.c_uint32()
    rc = fn(0, target.data_ptr(), target.numel(), idx.data_ptr(), dl.data_ptr(), offsets.ctypes.data,
            len(offsets) - 1, lo, hi, table, len(replicas), C.c_void_p(torch.cuda.current_stream().cuda_stream),
            C.byref(updates))
    return rc, updates.value


def test_static_variant_rejects_oversize_input_before_device_work(native_lib):
    """stories * (ceil(length / 4096) + 1) above 262080 is an error; the check
    happens on the host before any CUDA call (runs without a GPU)."""
    offsets = np.zeros(65, dtype=np.uint64)
    dummy = C.c_void_p(256)
    updates = C.c_uint32()
    rc = native_lib.leo_b200_sparse_mean_apply_static(0, dummy, 1 << 24, dummy, dummy, offsets.ctypes.data, 64,
                                                      -1.0, 1.0, None, 0, None, C.byref(updates))
    assert rc != 0
    assert b"too large" in native_lib.leo_b200_last_error()


@pytest.mark.gpu
def test_static_variant_matches_allocating_entry_point_twice(native_lib):
    import torch

    dev = torch.device("cuda:0")
    cases = [make_case(21, (1 << 20) + 5, 32, 0.01), make_case(22, 70_000, 7, 0.2, empty=(3,))]
    for target, indices, deltas, offsets in cases:
        idx = torch.from_numpy(indices.view(np.int32).copy()).to(dev)
        dl = torch.from_numpy(deltas).to(dev)
        a = torch.from_numpy(target.copy()).to(dev)
        b = torch.from_numpy(target.copy()).to(dev)
        reps_a = [torch.from_numpy(target.copy()).to(dev) for _ in range(2)]
        reps_b = [torch.from_numpy(target.copy()).to(dev) for _ in range(2)]
        rc_a, n_a = _call(native_lib.leo_b200_sparse_mean_apply, a, idx, dl, offsets, reps_a)
        rc_b, n_b = _call(native_lib.leo_b200_sparse_mean_apply_static, b, idx, dl, offsets, reps_b)
        torch.cuda.synchronize()
        assert rc_a == 0 and rc_b == 0, native_lib.leo_b200_last_error()
        assert n_a == n_b > 0
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
        for ra, rb in zip(reps_a, reps_b):
            assert torch.equal(ra.view(torch.int32), rb.view(torch.int32))
            assert torch.equal(rb.view(torch.int32), b.view(torch.int32))


_FRESH_PROCESS = r'''
import ctypes as C, sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
from leo_b200 import native
from test_sparse_apply import make_case
lib = native.lib()
dev = torch.device("cuda:0")
target, indices, deltas, offsets = make_case(31, (1 << 20) + 3, 32, 0.01)
assert 32 * (((1 << 20) + 3 + 4095) // 4096 + 1) > 64  # the table needs more than the counter words
idx = torch.from_numpy(indices.view(np.int32).copy()).to(dev)
dl = torch.from_numpy(deltas).to(dev)
a = torch.from_numpy(target.copy()).to(dev)
b = torch.from_numpy(target.copy()).to(dev)
updates = C.c_uint32()
stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
# A first small static call loads the library's kernels and its fixed scratch
# (module loading is lazy), so the free-memory check below sees only the call.
t0 = torch.zeros(8, device=dev)
i0 = torch.zeros(1, dtype=torch.int32, device=dev)
d0 = torch.zeros(1, device=dev)
o0 = np.array([0, 1], dtype=np.uint64)
rc = lib.leo_b200_sparse_mean_apply_static(0, t0.data_ptr(), 8, i0.data_ptr(), d0.data_ptr(), o0.ctypes.data, 1,
                                           -1.0, 1.0, None, 0, stream, C.byref(updates))
assert rc == 0, lib.leo_b200_last_error()
torch.cuda.synchronize()
free0, _ = torch.cuda.mem_get_info()
rc = lib.leo_b200_sparse_mean_apply_static(0, b.data_ptr(), b.numel(), idx.data_ptr(), dl.data_ptr(),
                                           offsets.ctypes.data, len(offsets) - 1, -1.0, 1.0, None, 0, stream,
                                           C.byref(updates))
torch.cuda.synchronize()
assert rc == 0, lib.leo_b200_last_error()
free1, _ = torch.cuda.mem_get_info()
assert lib.leo_b200_sparse_apply_scratch_bytes(0) == 0, "the static entry point allocated scratch"
assert free1 == free0, (free0, free1)
rc = lib.leo_b200_sparse_mean_apply(0, a.data_ptr(), a.numel(), idx.data_ptr(), dl.data_ptr(),
                                    offsets.ctypes.data, len(offsets) - 1, -1.0, 1.0, None, 0, stream,
                                    C.byref(updates))
torch.cuda.synchronize()
assert rc == 0, lib.leo_b200_last_error()
assert lib.leo_b200_sparse_apply_scratch_bytes(0) > 0
assert torch.equal(a.view(torch.int32), b.view(torch.int32))
print("ok")
'''


@pytest.mark.gpu
def test_static_variant_allocates_nothing_in_a_fresh_process(native_lib):
    """The static entry point called first in a fresh process: afterwards the
    allocating entry point's per-device scratch is still empty and the device's
    free memory is unchanged; the allocating call that follows allocates its
    scratch and gives the same result."""
    import subprocess
    import sys
    from pathlib import Path

    here = Path(__file__).resolve().parent
    proc = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, str(here.parent), str(here)], capture_output=True,
                          text=True, timeout=300)
    assert proc.returncode == 0 and proc.stdout.strip().endswith("ok"), proc.stdout[-2000:] + proc.stderr[-2000:]
