"""Batch-end sparse mean apply of one tensor (BASELINE config 5 semantics).

The GPU entry point ``leo_b200_sparse_mean_apply`` must equal the oracle's
restatement of ``apply_sparse_scaled`` (crates/leo-core/src/parallel.rs:975-1022,
divisor = stories) plus the clamp projection (parallel.rs:1226-1233) bit for
bit, write the same values into every replica, and reject invalid input before
writing anything.
"""

import ctypes as C

import numpy as np
import pytest


def make_case(seed: int, length: int, stories: int, density: float, empty: tuple = ()):
    rng = np.random.default_rng(seed)
    target = rng.uniform(-0.999, 0.999, size=length).astype(np.float32)
    idx_parts, val_parts, offsets = [], [], [0]
    for s in range(stories):
        if s in empty or density == 0.0:
            picked = np.zeros(0, dtype=np.uint32)
        elif density >= 1.0:
            picked = np.arange(length, dtype=np.uint32)
        else:
            picked = np.flatnonzero(rng.random(length) < density).astype(np.uint32)
        vals = rng.normal(0.0, 1e-3, size=picked.size).astype(np.float32)
        # a few large steps so that the clamp projection engages
        if picked.size:
            big = rng.random(picked.size) < 0.01
            vals[big] = rng.choice([-3.0, 3.0], size=int(big.sum())).astype(np.float32)
        idx_parts.append(picked)
        val_parts.append(vals)
        offsets.append(offsets[-1] + picked.size)
    indices = np.concatenate(idx_parts) if idx_parts else np.zeros(0, np.uint32)
    deltas = np.concatenate(val_parts) if val_parts else np.zeros(0, np.float32)
    return target, indices, deltas, np.array(offsets, dtype=np.uint64)


def reference(oracle_lib, target, indices, deltas, offsets, lo, hi):
    out = target.copy()
    updates = oracle_lib.sparse_mean_apply(out, indices, deltas, offsets, lo, hi)
    return out, updates


def test_oracle_matches_ordered_fp64_sum(oracle_lib):
    """The oracle's apply equals a direct restatement: per index, FP64 sum of
    the stories' deltas in story order, mean, f32 add, clamp."""
    target, indices, deltas, offsets = make_case(1, 5000, 5, 0.05)
    got, updates = reference(oracle_lib, target, indices, deltas, offsets, -1.0, 1.0)
    want = target.copy()
    sums: dict[int, float] = {}
    for s in range(len(offsets) - 1):
        for j in range(int(offsets[s]), int(offsets[s + 1])):
            i = int(indices[j])
            sums[i] = sums.get(i, 0.0) + float(np.float64(deltas[j]))
    for i, v in sums.items():
        x = np.float32(want[i] + np.float32(v / 5.0))
        want[i] = np.float32(min(max(x, np.float32(-1.0)), np.float32(1.0)))
    assert updates == len(sums)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("bad", ["empty", "too_many", "decreasing"])
def test_host_side_argument_checks(native_lib, bad):
    """Argument errors are reported before any device work (no GPU needed)."""
    from leo_b200.native import LeoError, check

    dummy = C.c_void_p(16)
    if bad == "empty":
        offsets = np.zeros(1, dtype=np.uint64)
        stories = 0
    elif bad == "too_many":
        offsets = np.zeros(300, dtype=np.uint64)
        stories = 299
    else:
        offsets = np.array([0, 5, 3], dtype=np.uint64)
        stories = 2
    updates = C.c_uint32()
    with pytest.raises(LeoError):
        check(native_lib.leo_b200_sparse_mean_apply(0, dummy, 10, dummy, dummy, offsets.ctypes.data, stories, -1.0,
                                                    1.0, None, 0, None, C.byref(updates)))


CASES = [
    # (seed, length, stories, density, replicas, empty stories)
    (1, 10_000, 4, 0.01, 0, ()),
    (2, 4096 * 3 + 17, 8, 0.1, 3, (2,)),
    (3, 1 << 20, 32, 0.001, 1, ()),
    (4, 1 << 20, 32, 0.01, 2, (0, 31)),
    (5, (1 << 20) + 37, 16, 0.1, 0, ()),
    (6, 5000, 3, 1.0, 2, ()),
    (7, 1, 2, 1.0, 1, ()),
    (8, 9000, 5, 0.0, 1, ()),
    (9, 300_000, 256, 0.002, 4, (7, 100)),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[f"n{c[1]}-s{c[2]}-d{c[3]}-r{c[4]}" for c in CASES])
def test_gpu_matches_oracle(native_lib, oracle_lib, case):
    import torch

    from leo_b200.sparse_apply import sparse_mean_apply

    seed, length, stories, density, n_rep, empty = case
    target, indices, deltas, offsets = make_case(seed, length, stories, density, empty)
    lo, hi = -1.0, 1.0
    want, want_updates = reference(oracle_lib, target, indices, deltas, offsets, lo, hi)
    dev = torch.device("cuda:0")
    t = torch.from_numpy(target.copy()).to(dev)
    reps = [torch.from_numpy(target.copy()).to(dev) for _ in range(n_rep)]
    idx = torch.from_numpy(indices.view(np.int32).copy()).to(dev)
    dl = torch.from_numpy(deltas.copy()).to(dev)
    updates = sparse_mean_apply(t, idx, dl, offsets, lo, hi, reps)
    torch.cuda.synchronize()
    assert updates == want_updates
    got = t.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    for r in reps:
        assert np.array_equal(r.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("bad", ["range", "unsorted", "duplicate", "nonfinite"])
def test_gpu_rejects_invalid_deltas_without_writing(native_lib, bad):
    """The kernels' own checks (index < length, strictly increasing, finite)
    turn bad lists into an error; no element is read out of bounds and the
    target is left unchanged."""
    import torch

    from leo_b200.native import LeoError
    from leo_b200.sparse_apply import sparse_mean_apply

    target, indices, deltas, offsets = make_case(11, 20_000, 3, 0.01)
    indices = indices.copy()
    deltas = deltas.copy()
    k = int(offsets[1]) + 2
    if bad == "range":
        indices[k] = 20_000
    elif bad == "unsorted":
        indices[k], indices[k + 1] = indices[k + 1], indices[k]
    elif bad == "duplicate":
        indices[k + 1] = indices[k]
    else:
        deltas[k] = np.float32("nan")
    dev = torch.device("cuda:0")
    t = torch.from_numpy(target.copy()).to(dev)
    idx = torch.from_numpy(indices.view(np.int32).copy()).to(dev)
    dl = torch.from_numpy(deltas).to(dev)
    with pytest.raises(LeoError):
        sparse_mean_apply(t, idx, dl, offsets, -1.0, 1.0)
    assert np.array_equal(t.cpu().numpy().view(np.uint32), target.view(np.uint32))
    # the device stays usable: a valid call afterwards succeeds
    _, good_idx, good_dl, good_off = make_case(12, 20_000, 3, 0.01)
    sparse_mean_apply(t, torch.from_numpy(good_idx.view(np.int32).copy()).to(dev),
                      torch.from_numpy(good_dl).to(dev), good_off, -1.0, 1.0)


@pytest.mark.gpu
@pytest.mark.parametrize("density", [0.001, 0.01, 0.1])
def test_reference_cuda_kernels_agree(native_lib, density):
    """The reference's own kernels (leo_apply_shared_wavefront_deltas +
    leo_scatter_f32, built unmodified by oracle/ref_cuda/Makefile) on the same
    merged deltas give this build's values bit for bit, after the sign rule the
    reference's apply adds for recurrent weights (excitatory sources >= 0,
    inhibitory <= 0; and it leaves an index whose merged delta is exactly 0
    alone), in the target and in every replica."""
    import torch
    from pathlib import Path

    from leo_b200.sparse_apply import sparse_mean_apply

    lib_path = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libleo_ref_kernels.so"
    if not lib_path.exists():
        pytest.skip("the reference kernels were not built (needs the reference checkout at build time)")
    ref = C.CDLL(str(lib_path))
    ref.leo_ref_last_error.restype = C.c_char_p
    vp, u32 = C.c_void_p, C.c_uint32
    ref.leo_ref_apply_sync.argtypes = [C.c_int, vp, vp, u32, u32, vp, vp, vp, u32, vp, u32, C.c_float, C.c_float,
                                       u32, C.POINTER(C.c_float), C.POINTER(C.c_float)]
    length, stories, S, n_rep = 1 << 20, 16, 64, 3
    target, indices, deltas, offsets = make_case(41, length, stories, density)
    dev = torch.device("cuda:0")
    base = torch.from_numpy(target.copy()).to(dev)
    ours = base.clone()
    idx = torch.from_numpy(indices.view(np.int32).copy()).to(dev)
    dl = torch.from_numpy(deltas.copy()).to(dev)
    sparse_mean_apply(ours, idx, dl, offsets, -1.0, 1.0, [])
    # the reference's input: the union and its merged deltas (FP64 sums in story order / stories)
    sums = np.zeros(length, np.float64)
    touched = np.zeros(length, bool)
    for s in range(stories):
        a, b = int(offsets[s]), int(offsets[s + 1])
        sums[indices[a:b]] += deltas[a:b].astype(np.float64)
        touched[indices[a:b]] = True
    union = np.flatnonzero(touched).astype(np.uint32)
    merged = (sums[union] / stories).astype(np.float32)
    rng = np.random.default_rng(42)
    types = (rng.random(length // S) < 0.2).astype(np.uint8)
    d_types = torch.from_numpy(types).to(dev)
    d_union = torch.from_numpy(union.view(np.int32).copy()).to(dev)
    d_merged = torch.from_numpy(merged).to(dev)
    theirs = torch.empty_like(base)
    reps = [base.clone() for _ in range(n_rep)]
    table = (C.c_void_p * n_rep)(*[r.data_ptr() for r in reps])
    apply_ms, sync_ms = C.c_float(), C.c_float()
    torch.cuda.synchronize()
    rc = ref.leo_ref_apply_sync(0, base.data_ptr(), theirs.data_ptr(), length, S, d_types.data_ptr(),
                                d_union.data_ptr(), d_merged.data_ptr(), union.size, table, n_rep, -1.0, 1.0, 1,
                                C.byref(apply_ms), C.byref(sync_ms))
    torch.cuda.synchronize()
    assert rc == 0, ref.leo_ref_last_error()
    got = ours.cpu().numpy()
    source_type = np.repeat(types, S)
    # The reference's apply skips an index whose merged delta is exactly 0 (no clamp, no sign rule).
    moved = np.zeros(length, bool)
    moved[union] = merged != 0.0
    want = np.where(moved, np.where(source_type == 0, np.maximum(got, 0.0), np.minimum(got, 0.0)), target)
    theirs_h = theirs.cpu().numpy()
    assert np.array_equal(theirs_h, want)  # +0.0 and -0.0 compare equal
    for r in reps:
        assert np.array_equal(r.cpu().numpy()[touched], theirs_h[touched])
