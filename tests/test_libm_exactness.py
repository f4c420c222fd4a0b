"""The kernels' exp / ln / powi reproduce the reference's f32 arithmetic.

The reference computes ``f32::exp`` and ``f32::ln`` through the platform libm
(glibc ``expf`` / ``logf``) in the softmax and loss
(``crates/leo-core/src/runtime.rs:1108-1188``) and decays with ``f32::powi``
(``runtime.rs:78-85``).  The kernels evaluate exp / ln in double, round once,
and patch the inputs where libm's result differs from a correct rounding with
a generated exception table; ``powi`` is right-to-left binary exponentiation
with no fused multiply-add.  These checks run the same header code on the CPU.
"""

import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "leo_b200" / "csrc"


@pytest.fixture(scope="module")
def libm_check(tmp_path_factory):
    from leo_b200.build import generate_tables

    generate_tables()
    out = tmp_path_factory.mktemp("libm") / "libm_check"
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-I", str(CSRC),
                    "-o", str(out), str(ROOT / "tests" / "native" / "libm_check.cpp")], check=True)
    return out


@pytest.mark.parametrize("seed", [1, 2])
def test_exp_and_log_match_libm_bitwise(libm_check, seed):
    proc = subprocess.run([str(libm_check), "500000", str(seed)], capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "mismatches=0" in proc.stdout


def test_exception_tables_are_sorted_and_small():
    import re

    text = (CSRC / "libm_tables.inc").read_text()
    n_exp = int(re.search(r"LEO_EXP_EXCEPTIONS (\d+)", text).group(1))
    n_log = int(re.search(r"LEO_LOG_EXCEPTIONS (\d+)", text).group(1))
    # glibc misrounds a small fraction of the scanned domains; a table that
    # grew large would mean the double evaluation itself is wrong.
    assert n_exp < 200_000 and n_log < 200_000
    for name in ("leo_exp_exception_keys", "leo_log_exception_keys"):
        body = re.search(name + r"\[\d+\] = \{([^}]*)\}", text).group(1)
        keys = [int(v.strip().rstrip("u"), 16) for v in body.split(",") if v.strip()]
        assert keys == sorted(set(keys))


def _powi_rtl(base: np.float32, e: int) -> np.float32:
    """Right-to-left binary exponentiation in f32, one rounding per product."""
    result, a = np.float32(1.0), np.float32(base)
    while True:
        if e & 1:
            result = np.float32(result * a)
        e >>= 1
        if e == 0:
            return result
        a = np.float32(a * a)


def test_powi_sequence_matches_restatement(tmp_path):
    src = tmp_path / "powi.cpp"
    src.write_text(
        '#include <cstdio>\n#include "leo_math.cuh"\n'
        "int main(){const float b[]={0.9f,0.95f,0.85f,0.97f,0.999f,0.5f};"
        "for(float x: b) for(int e=0;e<70;++e){float r=leo_math::decay_for_elapsed(x,(unsigned)e);"
        "unsigned u; __builtin_memcpy(&u,&r,4); std::printf(\"%u\\n\",u);} return 0;}\n")
    exe = tmp_path / "powi"
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-I", str(CSRC), "-o", str(exe), str(src)],
                   check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = []
    for x in (0.9, 0.95, 0.85, 0.97, 0.999, 0.5):
        for e in range(70):
            v = np.float32(1.0) if e == 0 else (np.float32(x) if e == 1 else _powi_rtl(np.float32(x), e))
            want.append(int(np.array([v], dtype=np.float32).view(np.uint32)[0]))
    assert got == want
