// t5e_select.cuh -- sparse metadata selection by byte permutes, shared by
// the kernels that evaluate sparse cases (simulator.py:26-77, :104-140).
//
// Both sparse forms these kernels take keep two units of each chunk of four:
// 2:4 on 8-bit element codes, and pairwise 4:8 on E2M1 (a unit is then a
// byte holding two adjacent nibbles).  With the chunk as one 32-bit word,
// the selection of two chunks is one byte permute of two words.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace t5e {
namespace select {

// PTX byte permute in its default mode: a selector nibble with bit 3 set
// yields the sign (bit 7) of the selected byte replicated, so 0x00 from a
// word whose bytes are all below 0x80 (the E2M1 magnitude tables use this).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Metadata word (eight chunk selectors) -> byte-permute selectors for the
// four physical words it produces (two chunks each), or false when a
// selector is illegal.  A chunk is one 32-bit word of the logical row whose
// bytes are the selectable units: four 8-bit element codes (2:4 selection
// on rows expanded to one code per byte) or four pairs of E2M1 nibbles
// (pairwise 4:8 selection on packed E2M1 rows); a selector keeps two of
// them.  Selector 6 picks the same units as 9 and is rewritten to it;
// afterwards a legal selector has its first unit index below its second
// (simulator.py:9-10, :66-67), so the kept units stay in logical order.
__device__ __forceinline__ bool chunk_selectors(uint32_t m, uint32_t& sel_lo, uint32_t& sel_hi) {
  const uint32_t x = m ^ 0x66666666u;
  const uint32_t zero = ~(((x & 0x77777777u) + 0x77777777u) | x) & 0x88888888u;
  m ^= (zero >> 3) * 0xFu;
  const uint32_t f = m & 0x33333333u, g = (m >> 2) & 0x33333333u;
  const uint32_t t = (g | 0x44444444u) - f;  // 4 + g - f per nibble, in [1, 7]
  if (((t + 0x33333333u) & 0x88888888u) != 0x88888888u) return false;
  // spread the 2-bit unit indices into selector nibbles; the second chunk of
  // each physical word reads the second source word (byte indices 4-7)
  auto spread = [](uint32_t v) {
    v = (v | (v << 8)) & 0x00FF00FFu;
    v = (v | (v << 4)) & 0x0F0F0F0Fu;
    v = (v | (v << 2)) & 0x33333333u;
    return v | 0x44004400u;
  };
  sel_lo = spread(m & 0xFFFFu);
  sel_hi = spread(m >> 16);
  return true;
}

// Eight physical words from sixteen logical words of a row.
__device__ __forceinline__ void select_row(const uint32_t (&lw)[16], uint32_t s0, uint32_t s1, uint32_t s2,
                                           uint32_t s3, uint32_t (&pw)[8]) {
  pw[0] = prmt(lw[0], lw[1], s0);
  pw[1] = prmt(lw[2], lw[3], s0 >> 16);
  pw[2] = prmt(lw[4], lw[5], s1);
  pw[3] = prmt(lw[6], lw[7], s1 >> 16);
  pw[4] = prmt(lw[8], lw[9], s2);
  pw[5] = prmt(lw[10], lw[11], s2 >> 16);
  pw[6] = prmt(lw[12], lw[13], s3);
  pw[7] = prmt(lw[14], lw[15], s3 >> 16);
}

// Four physical words from eight logical words (one metadata word's chunks).
__device__ __forceinline__ void select_half(const uint32_t (&lw)[8], uint32_t s_lo, uint32_t s_hi,
                                            uint32_t (&pw)[4]) {
  pw[0] = prmt(lw[0], lw[1], s_lo);
  pw[1] = prmt(lw[2], lw[3], s_lo >> 16);
  pw[2] = prmt(lw[4], lw[5], s_hi);
  pw[3] = prmt(lw[6], lw[7], s_hi >> 16);
}

}  // namespace select
}  // namespace t5e
