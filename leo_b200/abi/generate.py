"""Generate the C header for the kernel ABI from ``cuda_abi.def``.

The reference keeps one source of truth for the kernel configuration struct and
the pointer-table indices (``crates/leo-core/cuda_abi.def``) and its build
script emits ``leo_cuda_abi.h`` from it (``crates/leo-core/build.rs:18-126``,
header text at ``build.rs:97-121``).  This module reads the same definition
format and writes a byte-identical header, so kernels built here see exactly
the ``LeoConfig`` layout and ``LEO_P_*`` / ``LEO_D_*`` indices a Rust host
generated from the same file would pass.

Run as ``python -m leo_b200.abi.generate`` (or call :func:`write_header`).
"""

from __future__ import annotations

import sys
from dataclasses import dataclass, field
from pathlib import Path

ABI_DIR = Path(__file__).resolve().parent
DEFAULT_SPEC = ABI_DIR / "cuda_abi.def"
DEFAULT_HEADER = ABI_DIR.parents[1] / "include" / "leo_cuda_abi.h"


@dataclass
class AbiSpec:
    version: int
    config: list[tuple[str, str]] = field(default_factory=list)
    persistent: list[str] = field(default_factory=list)
    delta: list[str] = field(default_factory=list)


def parse_spec(text: str) -> AbiSpec:
    """Parse the ``.def`` format with the same rules as ``build.rs:27-59``."""
    section = ""
    version: int | None = None
    config: list[tuple[str, str]] = []
    persistent: list[str] = []
    delta: list[str] = []
    for raw in text.splitlines():
        line = raw.strip()
        if not line or line.startswith("#"):
            continue
        if line.startswith("abi_version "):
            if section:
                raise ValueError("abi_version must precede ABI sections")
            if version is not None:
                raise ValueError("duplicate abi_version")
            version = int(line[len("abi_version "):])
            continue
        if line.startswith("[") and line.endswith("]"):
            section = line[1:-1]
            continue
        if section == "config":
            parts = line.split()
            if len(parts) != 2:
                raise ValueError(f"invalid config ABI line: {line}")
            ty, name = parts
            if ty not in ("u32", "f32"):
                raise ValueError(f"unsupported ABI type: {ty}")
            config.append((ty, name))
        elif section == "persistent":
            persistent.append(line)
        elif section == "delta":
            delta.append(line)
        else:
            raise ValueError(f"ABI entry outside a section: {line}")
    if version is None:
        raise ValueError("cuda_abi.def must declare abi_version")
    if not config or not persistent or not delta:
        raise ValueError("cuda_abi.def sections must be non-empty")
    return AbiSpec(version, config, persistent, delta)


def render_header(spec: AbiSpec) -> str:
    """Header text in the order and spelling of ``build.rs:97-121``."""
    out = [f"#define LEO_CUDA_ABI_VERSION {spec.version}\n", "struct LeoConfig {\n"]
    for ty, name in spec.config:
        c_ty = "unsigned int" if ty == "u32" else "float"
        out.append(f"    {c_ty} {name};\n")
    out.append("};\n")
    out.append("enum LeoPersistentPointerIndex {\n")
    for i, name in enumerate(spec.persistent):
        out.append(f"    LEO_P_{name} = {i},\n")
    out.append(f"    LEO_P_POINTER_COUNT = {len(spec.persistent)}\n}};\n")
    out.append("enum LeoBatchDeltaPointerIndex {\n")
    for i, name in enumerate(spec.delta):
        out.append(f"    LEO_D_{name} = {i},\n")
    out.append(f"    LEO_D_POINTER_COUNT = {len(spec.delta)}\n}};\n")
    out.append(
        f'static_assert(sizeof(LeoConfig) == {len(spec.config) * 4}, "LeoConfig ABI size mismatch");\n'
    )
    return "".join(out)


def write_header(spec_path: Path = DEFAULT_SPEC, header_path: Path = DEFAULT_HEADER) -> Path:
    spec = parse_spec(spec_path.read_text(encoding="utf-8"))
    text = render_header(spec)
    header_path.parent.mkdir(parents=True, exist_ok=True)
    if not header_path.exists() or header_path.read_text(encoding="utf-8") != text:
        header_path.write_text(text, encoding="utf-8")
    return header_path


if __name__ == "__main__":
    path = write_header()
    print(f"wrote {path}", file=sys.stderr)
