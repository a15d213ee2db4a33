"""The hardware cross-check: its tcgen05 instruction descriptors equal the
ones CUTLASS's own descriptor code builds (compiled here for the host from
the CUTLASS headers in the image), the C ABI rejects every descriptor
outside the documented encodings before launching anything, the sub-byte
operand rows have the f8f6f4 shared-memory form, and -- on a B200 -- real
tcgen05.mma words equal the emulator's for every kind, operand pair and
accumulator it issues."""

from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from tcgen05_b200 import _native as nat
from tcgen05_b200 import hwcheck


def _cutlass_include():
    try:
        import flashinfer
    except Exception:
        return None
    p = Path(flashinfer.__file__).resolve().parent / "data" / "cutlass" / "include"
    return p if (p / "cute" / "arch" / "mma_sm100_desc.hpp").exists() else None


_E2M3 = "cutlass::detail::float_e2m3_unpacksmem_t"
_E3M2 = "cutlass::detail::float_e3m2_unpacksmem_t"
_E2M1 = "cutlass::detail::float_e2m1_unpacksmem_t"

# (A, B, saturate, accumulator, CUTLASS A type, B type, C type)
CASES = [("tf32", "tf32", False, "f32", "tfloat32_t", "tfloat32_t", "float"),
         ("bf16", "bf16", False, "f32", "bfloat16_t", "bfloat16_t", "float"),
         ("f16", "f16", False, "f32", "half_t", "half_t", "float"),
         ("f16", "f16", False, "f16", "half_t", "half_t", "half_t"),
         ("e4m3", "e5m2", False, "f32", "float_e4m3_t", "float_e5m2_t", "float"),
         ("e5m2", "e5m2", False, "f16", "float_e5m2_t", "float_e5m2_t", "half_t"),
         ("e2m3", "e2m1", False, "f32", _E2M3, _E2M1, "float"),
         ("e3m2", "e4m3", False, "f16", _E3M2, "float_e4m3_t", "half_t"),
         ("e2m1", "e3m2", False, "f32", _E2M1, _E3M2, "float"),
         ("u8", "s8", False, "s32", "uint8_t", "int8_t", "int32_t"),
         ("s8", "s8", True, "s32", "int8_t", "int8_t", "int32_t")]


def test_instruction_descriptors_match_cutlass(tmp_path):
    inc = _cutlass_include()
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if inc is None or not os.path.exists(nvcc):
        pytest.skip("CUTLASS headers or nvcc not available")
    lines = ["#include <cstdio>", "#include <cute/arch/mma_sm100_desc.hpp>",
             "#include <cute/numeric/numeric_types.hpp>", "using namespace cute;", "int main() {"]
    for _, _, sat, _, ta, tb, tc in CASES:
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
    got = [hwcheck.instr_desc(fa, fb, saturate=sat, d_type=d)[1] for fa, fb, sat, d, *_ in CASES]
    assert got == want


def test_descriptor_and_shape_validation():
    assert hwcheck.instr_desc("tf32") == (0, 0x08040910)
    with pytest.raises(ValueError):
        hwcheck.instr_desc("e8m0")
    with pytest.raises(ValueError):
        hwcheck.instr_desc("tf32", "bf16")
    with pytest.raises(ValueError):
        hwcheck.instr_desc("f16", "bf16")
    with pytest.raises(ValueError):
        hwcheck.instr_desc("bf16", saturate=True)
    with pytest.raises(ValueError):
        hwcheck.instr_desc("bf16", d_type="f16")
    with pytest.raises(ValueError):
        hwcheck.instr_desc("tf32", d_type="f16")
    with pytest.raises(ValueError):
        hwcheck.instr_desc("u8", d_type="f32")
    a, b, c = hwcheck.random_tiles("bf16", None, 2, 0)
    assert a.shape == (2, 128, 16) and b.shape == (2, 16, 16) and c.shape == (2, 128, 16)
    a, b, c = hwcheck.random_tiles("e2m1", "e3m2", 2, 0, "f16")
    assert a.shape == (2, 128, 32) and b.shape == (2, 32, 16) and int(c.max()) <= 0xFFFF


def test_expired_wait_refuses_later_launches(monkeypatch):
    """After a launch reports an expired wait, the process launches no further
    hardware tiles: both entry points raise before touching the device."""

    class _Flag:
        def __init__(self, v):
            self.v = v

        def item(self):
            return self.v

    monkeypatch.setattr(hwcheck, "_WAIT_EXPIRED", False)
    hwcheck._check_wait(_Flag(0))
    assert not hwcheck._WAIT_EXPIRED
    with pytest.raises(RuntimeError, match="untrusted"):
        hwcheck._check_wait(_Flag(1))
    assert hwcheck._WAIT_EXPIRED
    a, b, c = hwcheck.random_tiles("bf16", None, 1, 0)
    with pytest.raises(RuntimeError, match="no further hardware tiles"):
        hwcheck.hardware_tiles(a, b, c, "bf16")
    with pytest.raises(RuntimeError, match="no further hardware tiles"):
        hwcheck.hardware_block_scaled_tiles(None, None, None, None, None, "mxf4", "e2m1")


def test_sub_byte_rows_have_the_f8f6f4_shared_memory_form():
    rng = np.random.default_rng(3)
    for fmt, bits in (("e2m1", 4), ("e2m3", 6), ("e3m2", 6)):
        words = rng.integers(0, 1 << bits, size=(5, 32), dtype=np.uint32)
        rows = hwcheck.smem_rows(words, fmt)
        assert rows.shape == (5, 32)
        used = 16 * bits // 8
        for r in range(5):
            for chunk in range(2):
                body = rows[r, 16 * chunk:16 * chunk + used]
                assert not rows[r, 16 * chunk + used:16 * (chunk + 1)].any()
                bitstream = int.from_bytes(body.tobytes(), "little")
                got = [(bitstream >> (bits * e)) & ((1 << bits) - 1) for e in range(16)]
                assert got == list(words[r, 16 * chunk:16 * chunk + 16])
    words = rng.integers(0, 256, size=(3, 32), dtype=np.uint32)
    assert np.array_equal(hwcheck.smem_rows(words, "e4m3"), words.astype(np.uint8))


def test_abi_rejects_descriptors_outside_the_documented_encodings():
    """Every descriptor here is refused with T5E_ERR_INVALID by the host-side
    check, before any CUDA call, so the test needs no GPU (the pointers are
    aligned placeholders that are never dereferenced)."""
    lib = nat.load()
    fake = ctypes.c_void_p(1 << 20)
    k_f16, d_f32 = hwcheck.instr_desc("f16")
    k_f8, d_f8 = hwcheck.instr_desc("e4m3", "e2m1")
    k_i8, d_i8 = hwcheck.instr_desc("s8", "u8")
    k_tf, d_tf = hwcheck.instr_desc("tf32")
    bad = [
        (k_f16, d_f32 | (1 << 2)),                        # sparse
        (k_f16, d_f32 | (1 << 15)),                       # A MN-major
        (k_f16, d_f32 | (1 << 16)),                       # B MN-major
        (k_f16, d_f32 | (1 << 13)),                       # negate A
        (k_f16, d_f32 | (1 << 6)),                        # reserved bit
        (k_f16, d_f32 | (1 << 30)),                       # max shift
        (k_f16, (d_f32 & ~(0x3F << 17)) | (1 << 17)),     # N = 8
        (k_f16, (d_f32 & ~(0x1F << 24)) | (4 << 24)),     # M = 64
        (k_f16, d_f32 | (1 << 10)),                       # F16 A with BF16 B
        (k_f16, d_f32 | (1 << 3)),                        # saturation on kind::f16
        (k_f16, (d_f32 & ~(3 << 4)) | (2 << 4)),          # S32 accumulator on kind::f16
        (k_f16, (d_f32 & ~(3 << 4)) | (1 << 7) | (1 << 10)),  # BF16 into an F16 accumulator
        (k_f8, (d_f8 & ~(7 << 7)) | (2 << 7)),            # format code 2 on kind::f8f6f4
        (k_f8, (d_f8 & ~(7 << 10)) | (6 << 10)),          # format code 6 on kind::f8f6f4
        (k_tf, d_tf & ~(3 << 4)),                         # F16 accumulator on kind::tf32
        (k_i8, (d_i8 & ~(3 << 4)) | (1 << 4)),            # F32 accumulator on kind::i8
        (k_i8, d_i8 | (2 << 7)),                          # format code 3 on kind::i8
        (7, d_f32),                                       # unknown kind
        (k_f8, d_i8),                                     # i8 descriptor under kind::f8f6f4
    ]
    for kind, desc in bad:
        rc = lib.t5e_tcgen05_tiles(kind, desc, fake, fake, fake, fake, 1, fake, None)
        assert rc == nat.ERR_INVALID, (kind, hex(desc), rc)


@pytest.mark.gpu
@pytest.mark.parametrize("fa,fb,sat,d", hwcheck.PAIRS,
                         ids=[f"{p[0]}x{p[1]}-{p[3]}{'-sat' if p[2] else ''}" for p in hwcheck.PAIRS])
def test_tcgen05_hardware_equals_emulator(fa, fb, sat, d):
    a, b, c = hwcheck.random_tiles(fa, fb, 48, 17, d)
    r = hwcheck.cross_check(a, b, c, fa, fb, saturate=sat, d_type=d)
    if fa == fb == d == "f16":
        # the raw half has NaN and infinite results: the hardware writes F16
        # special words there, the reference its F32 ones; nothing else differs
        assert r["reference_f32_special_words"] > 0
        hw = r["hardware"].reshape(-1)
        emu = r["emulator"].reshape(-1)
        special = np.isin(emu, list(hwcheck.REFERENCE_F32_SPECIAL_FOR_F16.values()))
        assert np.isin(hw[special], list(hwcheck.REFERENCE_F32_SPECIAL_FOR_F16)).all()
    else:
        assert r["reference_f32_special_words"] == 0
    assert r["mismatches"] == 0, (f"{r['mismatches']} of {r['cases']} words differ; first cases {r['first']}: "
                                  f"hardware {[hex(int(x)) for x in r['hardware'].reshape(-1)[r['first']]]} "
                                  f"emulator {[hex(int(x)) for x in r['emulator'].reshape(-1)[r['first']]]}")


# ---- block-scaled kinds

# (kind, A, B, scale, CUTLASS A type, B type, scale type)
BS_CASES = [("mxf8f6f4", "e4m3", "e5m2", "ue8m0", "float_e4m3_t", "float_e5m2_t", "float_ue8m0_t"),
            ("mxf8f6f4", "e2m3", "e2m1", "ue8m0", _E2M3, _E2M1, "float_ue8m0_t"),
            ("mxf8f6f4", "e3m2", "e4m3", "ue8m0", _E3M2, "float_e4m3_t", "float_ue8m0_t"),
            ("mxf4", "e2m1", "e2m1", "ue8m0", "float_e2m1_t", "float_e2m1_t", "float_ue8m0_t"),
            ("mxf4nvf4-4x", "e2m1", "e2m1", "ue4m3", "float_e2m1_t", "float_e2m1_t", "float_ue4m3_t")]


def test_block_scaled_descriptors_match_cutlass(tmp_path):
    inc = _cutlass_include()
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if inc is None or not os.path.exists(nvcc):
        pytest.skip("CUTLASS headers or nvcc not available")
    lines = ["#include <cstdio>", "#include <cute/arch/mma_sm100_desc.hpp>",
             "#include <cute/numeric/numeric_types.hpp>", "using namespace cute;", "int main() {"]
    for *_, ta, tb, tsf in BS_CASES:
        lines.append(f'  printf("%u\\n", uint32_t(UMMA::make_instr_desc_block_scaled<{ta}, {tb}, float, {tsf}, '
                     f'128, 128, UMMA::Major::K, UMMA::Major::K>()));')
    lines.append("  return 0; }")
    src = tmp_path / "bs.cu"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "bs"
    subprocess.run([nvcc, "-std=c++17", "-I", str(inc), "-o", str(exe), str(src)], check=True,
                   capture_output=True, timeout=600)
    want = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    got = [hwcheck.block_scaled_desc(kind, fa, fb, scale)[1] for kind, fa, fb, scale, *_ in BS_CASES]
    assert got == want


def test_block_scaled_shapes_and_validation():
    with pytest.raises(ValueError):
        hwcheck.block_scaled_desc("mxf4", "e4m3")
    with pytest.raises(ValueError):
        hwcheck.block_scaled_desc("mxf8f6f4", "e4m3", scale="ue4m3")
    with pytest.raises(ValueError):
        hwcheck.block_scaled_desc("mxf4nvf4-2x", "e2m1", scale="ue4m3")
    a, b, c, sa, sb = hwcheck.random_block_scaled_tiles("mxf4nvf4-4x", "e2m1", None, 2, 0, "ue4m3")
    assert (a.shape, b.shape, c.shape, sa.shape, sb.shape) == ((2, 128, 64), (2, 64, 128), (2, 128, 128),
                                                               (2, 128, 4), (2, 128, 4))
    assert int(sa.max()) <= 0x7F
    assert hwcheck.block_scaled_rows(a.reshape(-1, 64), "e2m1", "mxf4").shape == (256, 32)
    assert list(hwcheck.scale_words(np.array([[1, 2, 3, 4]]))) == [0x04030201]


def test_abi_rejects_block_scaled_descriptors_outside_the_documented_encodings():
    lib = nat.load()
    fake = ctypes.c_void_p(1 << 20)
    k8, d8 = hwcheck.block_scaled_desc("mxf8f6f4", "e4m3", "e2m1")
    k4, d4 = hwcheck.block_scaled_desc("mxf4", "e2m1")
    kn, dn = hwcheck.block_scaled_desc("mxf4nvf4-2x", "e2m1")
    bad = [
        (k8, d8 | (1 << 2)),                      # sparse
        (k8, d8 | (1 << 4)),                      # B scale factor id 1
        (k8, d8 | (1 << 29)),                     # A scale factor id 1
        (k8, d8 | (1 << 31)),                     # K size bit
        (k8, d8 | (1 << 15)),                     # A MN-major
        (k8, d8 | (1 << 13)),                     # negate A
        (k8, d8 & ~(1 << 23)),                    # UE4M3 scales on mxf8f6f4
        (k8, (d8 & ~(0x3F << 17)) | (2 << 17)),   # N = 16
        (k8, (d8 & ~(7 << 7)) | (2 << 7)),        # format code 2
        (k4, (d4 & ~(7 << 7)) | (5 << 7)),        # f8f6f4 E2M1 code on mxf4
        (k4, d4 & ~(1 << 23)),                    # UE4M3 on mxf4
        (kn, dn & ~(1 << 23)),                    # UE4M3 on the two-scale mxf4nvf4
        (9, d4),                                  # unknown kind
    ]
    for kind, desc in bad:
        rc = lib.t5e_tcgen05_block_scaled_tiles(kind, desc, fake, fake, fake, fake, fake, fake, 1, fake, None)
        assert rc == nat.ERR_INVALID, (kind, hex(desc), rc)


@pytest.mark.gpu
@pytest.mark.parametrize("kind,fa,fb,scale", hwcheck.BS_PAIRS,
                         ids=[f"{p[0]}-{p[1]}x{p[2]}-{p[3]}" for p in hwcheck.BS_PAIRS])
def test_tcgen05_block_scaled_hardware_equals_emulator(kind, fa, fb, scale):
    a, b, c, sa, sb = hwcheck.random_block_scaled_tiles(kind, fa, fb, 4, 23, scale)
    r = hwcheck.cross_check_block_scaled(a, b, c, sa, sb, kind, fa, fb, scale)
    assert r["mismatches"] == 0, (f"{r['mismatches']} of {r['cases']} words differ; first cases {r['first']}: "
                                  f"hardware {[hex(int(x)) for x in r['hardware'].reshape(-1)[r['first']]]} "
                                  f"emulator {[hex(int(x)) for x in r['emulator'].reshape(-1)[r['first']]]}")


# ---- sparse kinds ------------------------------------------------------

# (kind, operand format, scale format, CUTLASS operand type, scale type or None)
SP_CASES = [("tf32", "tf32", None, "tfloat32_t", None),
            ("f16", "bf16", None, "bfloat16_t", None),
            ("f16", "f16", None, "half_t", None),
            ("f8f6f4", "e4m3", None, "float_e4m3_t", None),
            ("f8f6f4", "e3m2", None, _E3M2, None),
            ("f8f6f4", "e2m1", None, _E2M1, None),
            ("mxf8f6f4", "e5m2", "ue8m0", "float_e5m2_t", "float_ue8m0_t"),
            ("mxf8f6f4", "e2m3", "ue8m0", _E2M3, "float_ue8m0_t"),
            ("mxf4", "e2m1", "ue8m0", "float_e2m1_t", "float_ue8m0_t"),
            ("mxf4nvf4-4x", "e2m1", "ue4m3", "float_e2m1_t", "float_ue4m3_t")]


def test_sparse_descriptors_match_cutlass(tmp_path):
    inc = _cutlass_include()
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if inc is None or not os.path.exists(nvcc):
        pytest.skip("CUTLASS headers or nvcc not available")
    lines = ["#include <cstdio>", "#include <cute/arch/mma_sm100_desc.hpp>",
             "#include <cute/numeric/numeric_types.hpp>", "using namespace cute;", "int main() {"]
    for kind, _, _, t, tsf in SP_CASES:
        if tsf is None:
            lines.append(f'  printf("%u\\n", uint32_t(UMMA::make_instr_desc<{t}, {t}, float, 64, 8, UMMA::Major::K, '
                         f'UMMA::Major::K, UMMA::ScaleIn::One, UMMA::ScaleIn::One, UMMA::Saturate::False, true>()));')
        else:
            lines.append(f'  printf("%u\\n", uint32_t(UMMA::make_instr_desc_block_scaled<{t}, {t}, float, {tsf}, '
                         f'128, 8, UMMA::Major::K, UMMA::Major::K, UMMA::ScaleIn::One, UMMA::ScaleIn::One, true>()));')
    lines.append("  return 0; }")
    src = tmp_path / "sp.cu"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "sp"
    subprocess.run([nvcc, "-std=c++17", "-I", str(inc), "-o", str(exe), str(src)], check=True,
                   capture_output=True, timeout=600)
    want = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    got = [hwcheck.sparse_desc(kind, fmt, scale) for kind, fmt, scale, *_ in SP_CASES]
    assert got == want


def test_sparse_paths_map_onto_the_sparse_kinds():
    paths = hwcheck.sparse_paths()
    assert len(paths) == 18
    kinds = {p.name: hwcheck.sparse_kind(p) for p in paths}
    assert kinds["sparse-tf32"] == ("tf32", None)
    assert kinds["sparse-bf16"] == kinds["sparse-f16"] == ("f16", None)
    assert kinds["sparse-e2m1"] == ("f8f6f4", None)
    assert kinds["sparse-mx-e2m1"] == ("mxf8f6f4", "ue8m0")
    assert kinds["sparse-nvfp4"] == kinds["sparse-mxf4nvf4-4x-ue4m3"] == ("mxf4nvf4-4x", "ue4m3")
    assert kinds["sparse-mxf4nvf4-4x"] == ("mxf4nvf4-4x", "ue8m0")
    assert kinds["sparse-mxf4"] == ("mxf4", "ue8m0")
    with pytest.raises(ValueError):
        hwcheck.sparse_desc("i8", "s8")


def test_sparse_compression_follows_the_selector_order():
    """Each compressed row holds exactly the elements its metadata selects
    (every sparse path), in the order of the selector's indices: a 2:4
    selector 0x6 names index 2 first, so the compressed pair is (a[2], a[1])."""
    from tcgen05_b200 import sweep

    for spec in hwcheck.sparse_paths():
        cases = sweep.host_cases(spec, 0, 64, 64)
        mode = sweep.sparse_mode(spec)
        k = cases.a.shape[1]
        comp = hwcheck.compress_a(cases.a, cases.meta, k, mode)
        act = sweep._active(np, cases.meta.astype(np.int64), k, mode)
        assert comp.shape == (64, k // 2)
        assert (np.sort(comp, 1) == np.sort(cases.a[act].reshape(64, -1), 1)).all(), spec.name
        kind, _ = hwcheck.sparse_kind(spec)
        rows_a = hwcheck.operand_bytes(comp, spec.descriptor["a_format"], kind)
        rows_b = hwcheck.operand_bytes(cases.b, spec.descriptor["a_format"], kind)
        assert rows_a.shape == (64, 32) and rows_b.shape == (64, 64), spec.name
    a = np.arange(16, dtype=np.uint32).reshape(1, 16) + 100
    meta = np.array([[0x6666_6666 & 0xFFFF_FFFF, 0]], dtype=np.uint32)
    assert list(hwcheck.compress_a(a, meta, 16, "2of4")[0, :2]) == [102, 101]
    assert list(hwcheck.compress_a(a, np.array([[0x4E4E_4E4E, 0]], dtype=np.uint32), 16, "1of2")[0, :2]) == [101, 102]
    assert list(hwcheck.compress_a(a, np.array([[0x0000_0009, 0]], dtype=np.uint32), 16, "4of8")[0, :4]) == \
        [102, 103, 104, 105]


def test_abi_rejects_sparse_descriptors_outside_the_documented_encodings():
    lib = nat.load()
    fake = ctypes.c_void_p(1 << 20)
    kf = hwcheck.SP_KINDS["f16"]
    df = hwcheck.sparse_desc("f16", "bf16")
    km = hwcheck.SP_KINDS["mxf8f6f4"]
    dm = hwcheck.sparse_desc("mxf8f6f4", "e4m3", "ue8m0")
    k4 = hwcheck.SP_KINDS["mxf4nvf4-2x"]
    d4 = hwcheck.sparse_desc("mxf4nvf4-2x", "e2m1", "ue8m0")
    bad = [
        (kf, df & ~(1 << 2), 0),                         # dense
        (kf, df | 1, 0),                                 # sparsity selector 1
        (kf, (df & ~(0x3F << 17)) | (2 << 17), 0),       # N = 16
        (kf, (df & ~(0x1F << 24)) | (8 << 24), 0),       # M = 128 on an unscaled kind
        (kf, df & ~(3 << 4), 0),                         # F16 accumulator
        (kf, df & ~(1 << 10), 0),                        # F16 B with BF16 A
        (kf, df | (1 << 15), 0),                         # A MN-major
        (km, (dm & ~(0x1F << 24)) | (4 << 24), 0),       # M = 64 on a block-scaled kind
        (km, dm & ~(1 << 23), 0),                        # UE4M3 on mxf8f6f4
        (k4, d4 & ~(1 << 23), 0),                        # UE4M3 on the two-scale mxf4nvf4
        (kf, df, 3),                                     # unknown metadata layout
        (15, df, 0),                                     # unknown kind
    ]
    for kind, desc, layout in bad:
        rc = lib.t5e_tcgen05_sparse_cases(kind, desc, layout, fake, fake, fake, fake, fake, fake, fake, None, 1,
                                          fake, None)
        assert rc == nat.ERR_INVALID, (kind, hex(desc), layout, rc)
    rc = lib.t5e_tcgen05_sparse_cases(km, dm, 0, fake, fake, fake, fake, None, fake, fake, None, 1, fake, None)
    assert rc == nat.ERR_INVALID  # block-scaled kinds need their scale words


@pytest.mark.gpu
@pytest.mark.parametrize("spec", hwcheck.sparse_paths(), ids=[p.name for p in hwcheck.sparse_paths()])
def test_tcgen05_sparse_hardware_equals_emulator(spec):
    r = hwcheck.cross_check_sparse(spec, 512)
    assert r["nonuniform_tiles"] == 0, f"{r['nonuniform_tiles']} tiles hold more than one D value"
    assert r["mismatches"] == 0, (f"{r['mismatches']} of {r['cases']} words differ; first cases {r['first']}: "
                                  f"hardware {[hex(int(x)) for x in r['hardware'][r['first']]]} "
                                  f"emulator {[hex(int(x)) for x in r['emulator'][r['first']]]}")


@pytest.mark.gpu
def test_sparse_metadata_pattern_is_what_the_hardware_reads():
    """The same cases with the kind::f16 metadata pattern on a kind::f8f6f4
    path give other words: the cross-check sees the metadata it is fed."""
    spec = next(p for p in hwcheck.sparse_paths() if p.name == "sparse-fp8")
    r = hwcheck.cross_check_sparse(spec, 128, layout=1)
    assert r["mismatches"] > 0
