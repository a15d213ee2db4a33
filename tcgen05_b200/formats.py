"""Raw-bit constants and container conversions (the reference's
tcgen05_model/formats.py:7-37 API).  These run on the host: they only build
and inspect raw words at the API boundary and never compute an MMA result."""

from __future__ import annotations

import struct

F32_SIGN_MASK = 0x8000_0000
F32_EXP_MASK = 0x7F80_0000
F32_FRAC_MASK = 0x007F_FFFF
F32_EXP_BIAS = 127
F32_POS_ZERO = 0x0000_0000
F32_POS_INF = 0x7F80_0000
F32_NEG_INF = 0xFF80_0000


def f32_to_bits(value: float) -> int:
    """IEEE F32 word of a Python float (rounded to F32 by the host)."""
    return struct.unpack("<I", struct.pack("<f", value))[0]


def bits_to_f32(bits: int) -> float:
    """The F32 value held in the low 32 bits of an integer."""
    return struct.unpack("<f", struct.pack("<I", bits & 0xFFFF_FFFF))[0]


def tf32_truncate_bits(bits: int) -> int:
    """Sign, exponent and the top ten fraction bits of an F32 word."""
    return bits & 0xFFFF_E000


def bf16_truncate_bits(bits: int) -> int:
    """Sign, exponent and the top seven fraction bits of an F32 word."""
    return bits & 0xFFFF_0000
