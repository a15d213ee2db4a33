// t5e_e2m1.cuh -- integer SIMD helpers shared by the E2M1 kernels (NVFP4 with
// UE4M3 scales, t5e_nvfp4.cu; the UE8M0 MXF4 family, t5e_mxf4.cu).
//
// An E2M1 element is n * 2**-1 with |n| in {0,1,2,3,4,6,8,12}
// (tcgen05_model/model.py:210-222): byte permutes over two constant words
// turn eight 4-bit codes into byte magnitudes, and dp4a forms four-element
// dot products of them.  Pairwise 4:8 sparse metadata (simulator.py:26-77)
// selects two bytes of each 32-bit word of a packed row.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "t5e_select.cuh"

namespace t5e {
namespace e2m1 {

using namespace select;

constexpr uint32_t kMag0 = 0x03020100u;  // |n| of magnitude codes 0-3 (units of 2**-1)
constexpr uint32_t kMag1 = 0x0C080604u;  // |n| of magnitude codes 4-7
constexpr uint32_t kRaw0 = 0x04040400u;  // 0 for code 0, else raw exponent + 4 (codes 0-3)
constexpr uint32_t kRaw1 = 0x06060505u;  // codes 4-7

// x >> 16 on the multiply pipe (the ALU pipe is this kernel's bottleneck).
__device__ __forceinline__ uint32_t hi16(uint32_t x) {
  uint32_t r;
  asm("mul.hi.u32 %0, %1, 65536;" : "=r"(r) : "r"(x));
  return r;
}

// Four products: am holds the A magnitude codes (sign bits clear), bx the B
// codes with the product sign in bit 3 and bn the same with that bit
// inverted.  pos / neg accumulate |a*b| of the positive / negative products.
__device__ __forceinline__ void quad(uint32_t am, uint32_t bx, uint32_t bn, uint32_t& pos, uint32_t& neg) {
  const uint32_t ma = prmt(kMag0, kMag1, am);
  pos = __dp4a(ma, prmt(kMag0, kMag1, bx), pos);
  neg = __dp4a(ma, prmt(kMag0, kMag1, bn), neg);
}

// Eight products of one packed word of A and B.
__device__ __forceinline__ void octet(uint32_t wa, uint32_t wb, uint32_t& pos, uint32_t& neg) {
  const uint32_t am = wa & 0x77777777u;
  const uint32_t bx = wb ^ (wa & 0x88888888u);
  const uint32_t bn = wb ^ (~wa & 0x88888888u);
  quad(am, bx, bn, pos, neg);
  quad(hi16(am), hi16(bx), hi16(bn), pos, neg);
}

// Signed units of m * 2**d: exact for 0 <= d <= 55, truncated toward zero
// for d < 0 (ones' complement: an arithmetic shift of m - 1 = ~|m| is
// ~(|m| >> r) for negative m).  Both forms are computed and selected, so
// lanes never diverge on the sign of d.
__device__ __forceinline__ int64_t shift_trunc(int32_t m, int d) {
  const int64_t left = (int64_t)m << (d > 0 ? d : 0);
  const int r = d < 0 ? (d < -31 ? 31 : -d) : 0;
  const int32_t s = m >> 31;
  const int32_t right = ((m + s) >> r) - s;
  return d >= 0 ? left : (int64_t)right;
}

// Whether some nonzero product among the 16 elements of (wa[0..1], wb[0..1])
// has a_raw + b_raw > t, for 0 <= t <= 3.  Byte sums of the kRaw tables are
// 8 + a_raw + b_raw when both elements are nonzero and at most 6 otherwise.
__device__ __forceinline__ bool block_exceeds(uint32_t wa0, uint32_t wa1, uint32_t wb0, uint32_t wb1, int t) {
  const uint32_t bias = (uint32_t)(128 - (t + 9)) * 0x01010101u;
  const uint32_t a0 = wa0 & 0x77777777u, a1 = wa1 & 0x77777777u;
  const uint32_t b0 = wb0 & 0x77777777u, b1 = wb1 & 0x77777777u;
  uint32_t acc = (prmt(kRaw0, kRaw1, a0) + prmt(kRaw0, kRaw1, b0) + bias);
  acc |= (prmt(kRaw0, kRaw1, a0 >> 16) + prmt(kRaw0, kRaw1, b0 >> 16) + bias);
  acc |= (prmt(kRaw0, kRaw1, a1) + prmt(kRaw0, kRaw1, b1) + bias);
  acc |= (prmt(kRaw0, kRaw1, a1 >> 16) + prmt(kRaw0, kRaw1, b1 >> 16) + bias);
  return (acc & 0x80808080u) != 0u;
}

template <int WORDS>
__device__ __forceinline__ void load_row(const uint8_t* __restrict__ row, uint32_t (&w)[WORDS]) {
  const uint4* p = reinterpret_cast<const uint4*>(row);
#pragma unroll
  for (int i = 0; i < WORDS / 4; ++i) {
    const uint4 v = __ldg(p + i);
    w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
  }
}

}  // namespace e2m1
}  // namespace t5e
