"""The drop-in boundary on CPU: the generated kernel ABI header, the C-ABI
library's exports, and the no-fallback rule.

The header checks restate the reference's ABI checker and build script
(``crates/leo-core/build.rs:18-126``: one ``.def`` source of truth,
``static_assert(sizeof(LeoConfig) == 160)``) and the version pin
``CUDA_ABI_VERSION = 1`` (``crates/leo-core/src/semantics.rs:12``).  The
no-fallback test follows ``backend.rs:1028-1037`` (an explicit GPU selection
never silently runs on the CPU).
"""

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "leo_b200" / "csrc"


def test_generated_header_is_current():
    from leo_b200.abi.generate import DEFAULT_HEADER, DEFAULT_SPEC, parse_spec, render_header

    spec = parse_spec(DEFAULT_SPEC.read_text(encoding="utf-8"))
    assert render_header(spec) == DEFAULT_HEADER.read_text(encoding="utf-8")


def test_abi_layout_and_version():
    from leo_b200.abi.generate import DEFAULT_SPEC, parse_spec
    from leo_b200.ctypes_types import LeoConfig

    spec = parse_spec(DEFAULT_SPEC.read_text(encoding="utf-8"))
    assert spec.version == 1
    assert len(spec.config) == 40
    assert [t for t, _ in spec.config[:14]] == ["u32"] * 14
    assert [t for t, _ in spec.config[14:]] == ["f32"] * 26
    assert C.sizeof(LeoConfig) == 160
    assert len(spec.persistent) == 105 and len(set(spec.persistent)) == 105
    assert len(spec.delta) == 23 and len(set(spec.delta)) == 23


def test_abi_parser_rejects_malformed_specs():
    from leo_b200.abi.generate import parse_spec

    with pytest.raises(ValueError):
        parse_spec("[config]\nu32 neuron_count\n")  # no abi_version
    with pytest.raises(ValueError):
        parse_spec("abi_version = 1\n[config]\n[persistent]\nA\n[delta]\nB\n")  # empty config


def test_kernels_do_not_redefine_the_abi():
    """No kernel source declares its own LeoConfig or pointer-index enums."""
    for path in list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")):
        text = path.read_text(encoding="utf-8")
        assert not re.search(r"struct\s+LeoConfig\s*\{", text), path.name
        assert not re.search(r"\bLEO_[PD]_[A-Z0-9_]+\s*=", text), path.name


def test_library_exports_every_declared_symbol(native_lib):
    from leo_b200 import native

    declared = native.exported_symbols()
    assert len(declared) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", str(native.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT\s+(leo_b200_[a-z0-9_]+)$", out, flags=re.M))
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for name in declared:
        assert getattr(native_lib, name) is not None


def test_library_reports_abi_version(native_lib):
    assert native_lib.leo_b200_abi_version() == 1


def test_open_without_gpu_fails_loudly(native_lib):
    """No CUDA device here: opening a backend is an error, never a CPU fallback."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from leo_b200.backend import GpuBackend
    from leo_b200.configs import TEST
    from leo_b200.ctypes_types import TOPOLOGY_REFERENCE
    from leo_b200.model import HostModel
    from leo_b200.native import LeoError

    model = HostModel.initialize(TEST, TOPOLOGY_REFERENCE)
    with pytest.raises(LeoError):
        GpuBackend(model, device=0, max_lanes=2)


def test_missing_library_is_an_error(monkeypatch, tmp_path):
    from leo_b200 import native

    monkeypatch.setattr(native, "_lib", None)
    monkeypatch.setattr(native, "LIB_PATH", tmp_path / "libleo_b200.so")
    with pytest.raises(native.LeoError, match="no CPU fallback"):
        native.lib()


def test_product_package_never_imports_the_oracle():
    for path in (ROOT / "leo_b200").rglob("*.py"):
        text = path.read_text(encoding="utf-8")
        assert not re.search(r"^\s*(from|import)\s+oracle\b", text, flags=re.M), path
    for path in list(CSRC.glob("*")):
        if path.suffix in (".cu", ".cuh", ".h", ".cpp"):
            assert "leo_oracle" not in path.read_text(encoding="utf-8"), path
