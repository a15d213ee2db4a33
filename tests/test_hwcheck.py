"""The hardware cross-check: its tcgen05 instruction descriptors equal the
ones CUTLASS's own descriptor code builds (compiled here for the host from
the CUTLASS headers in the image), its arguments are validated, and -- on a
B200 -- real tcgen05.mma words equal the emulator's for every kind it
issues."""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from tcgen05_b200 import hwcheck


def _cutlass_include():
    try:
        import flashinfer
    except Exception:
        return None
    p = Path(flashinfer.__file__).resolve().parent / "data" / "cutlass" / "include"
    return p if (p / "cute" / "arch" / "mma_sm100_desc.hpp").exists() else None


CASES = [("tf32", "tf32", False, "tfloat32_t", "tfloat32_t", "float"),
         ("bf16", "bf16", False, "bfloat16_t", "bfloat16_t", "float"),
         ("f16", "f16", False, "half_t", "half_t", "float"),
         ("e4m3", "e5m2", False, "float_e4m3_t", "float_e5m2_t", "float"),
         ("e5m2", "e5m2", False, "float_e5m2_t", "float_e5m2_t", "float"),
         ("u8", "s8", False, "uint8_t", "int8_t", "int32_t"),
         ("s8", "s8", True, "int8_t", "int8_t", "int32_t")]


def test_instruction_descriptors_match_cutlass(tmp_path):
    inc = _cutlass_include()
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if inc is None or not os.path.exists(nvcc):
        pytest.skip("CUTLASS headers or nvcc not available")
    lines = ["#include <cstdio>", "#include <cute/arch/mma_sm100_desc.hpp>",
             "#include <cute/numeric/numeric_types.hpp>", "using namespace cute;", "int main() {"]
    for _, _, sat, ta, tb, tc in CASES:
        s = "UMMA::ScaleIn::One, UMMA::ScaleIn::One, UMMA::Saturate::True" if sat else ""
        extra = (", " + s) if s else ""
        lines.append(f'  printf("%u\\n", uint32_t(UMMA::make_instr_desc<{ta}, {tb}, {tc}, 128, 16, '
                     f'UMMA::Major::K, UMMA::Major::K{extra}>()));')
    lines.append("  return 0; }")
    src = tmp_path / "d.cu"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "d"
    subprocess.run([nvcc, "-std=c++17", "-I", str(inc), "-o", str(exe), str(src)], check=True,
                   capture_output=True, timeout=600)
    want = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    got = [hwcheck.instr_desc(fa, fb, saturate=sat)[1] for fa, fb, sat, *_ in CASES]
    assert got == want


def test_descriptor_and_shape_validation():
    assert hwcheck.instr_desc("tf32") == (0, 0x08040910)
    with pytest.raises(ValueError):
        hwcheck.instr_desc("e2m1")
    with pytest.raises(ValueError):
        hwcheck.instr_desc("tf32", "bf16")
    with pytest.raises(ValueError):
        hwcheck.instr_desc("bf16", saturate=True)
    a, b, c = hwcheck.random_tiles("bf16", None, 2, 0)
    assert a.shape == (2, 128, 16) and b.shape == (2, 16, 16) and c.shape == (2, 128, 16)


@pytest.mark.gpu
@pytest.mark.parametrize("fa,fb,sat", [(p[0], p[1], p[2]) for p in hwcheck.PAIRS],
                         ids=[f"{p[0]}x{p[1]}{'-sat' if p[2] else ''}" for p in hwcheck.PAIRS])
def test_tcgen05_hardware_equals_emulator(fa, fb, sat):
    a, b, c = hwcheck.random_tiles(fa, fb, 48, 17)
    r = hwcheck.cross_check(a, b, c, fa, fb, saturate=sat)
    assert r["mismatches"] == 0, (f"{r['mismatches']} of {r['cases']} words differ; first cases {r['first']}: "
                                  f"hardware {[hex(int(x)) for x in r['hardware'].reshape(-1)[r['first']]]} "
                                  f"emulator {[hex(int(x)) for x in r['emulator'].reshape(-1)[r['first']]]}")
