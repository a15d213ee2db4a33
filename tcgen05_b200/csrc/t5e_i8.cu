// t5e_i8.cu -- specialised kernel for kind::i8: U8/S8 x U8/S8 with S32 C/D,
// wrapping or saturating (tcgen05_model/model.py:1120-1152).
//
// The reference sums the exact products into C and then clamps (saturate)
// or keeps the low 32 bits (wrap).  Four products at a time are one dp4a in
// the operands' signedness; the dot product of K <= 4096 elements fits in
// 32 bits (|a*b| <= 255*255), and C plus the dot product is formed in 64.
#include <cuda_runtime.h>

#include "t5e_arith.cuh"
#include "t5e_dispatch.h"

namespace t5e {
namespace i8 {

constexpr int kThreads = 256;
constexpr int kMaxK = 4096;

// dp4a of four byte pairs with A and B signed or unsigned.
template <bool AS, bool BS>
__device__ __forceinline__ int32_t dot4(uint32_t a, uint32_t b, int32_t c) {
  int32_t r;
  if constexpr (AS && BS) {
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  } else if constexpr (AS) {
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  } else if constexpr (BS) {
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  } else {
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  }
  return r;
}

template <bool AS, bool BS, bool SAT>
__global__ void __launch_bounds__(kThreads) i8_kernel(const t5e_batch B) {
  // programmatic dependent launch: no prologue, so wait for the previous grid at once
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t n = (uint32_t)B.n;
  const uint32_t stride = gridDim.x * blockDim.x;
  const int chunks = B.k / 16;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint4* pa = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(B.a) + (size_t)i * B.a_stride);
    const uint4* pb = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(B.b) + (size_t)i * B.b_stride);
    int32_t dot = 0;
#pragma unroll 4
    for (int j = 0; j < chunks; ++j) {
      const uint4 a = __ldg(pa + j), b = __ldg(pb + j);
      dot = dot4<AS, BS>(a.x, b.x, dot);
      dot = dot4<AS, BS>(a.y, b.y, dot);
      dot = dot4<AS, BS>(a.z, b.z, dot);
      dot = dot4<AS, BS>(a.w, b.w, dot);
    }
    const int64_t total = (int64_t)(int32_t)__ldg(static_cast<const uint32_t*>(B.c) + i) + dot;
    int64_t r = total;
    if constexpr (SAT) r = total < -2147483648ll ? -2147483648ll : (total > 2147483647ll ? 2147483647ll : total);
    B.d[i] = (uint32_t)r;
    if (B.status) B.status[i] = (uint8_t)T5E_CASE_OK;
  }
}

template <bool AS, bool BS, bool SAT>
int launch(const t5e_batch& B, cudaStream_t stream) {
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, i8_kernel<AS, BS, SAT>, kThreads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const uint64_t need = (B.n + kThreads - 1) / kThreads;
  const uint64_t cap = (uint64_t)sms * (uint64_t)per_sm;
  const int grid = (int)(need < cap ? (need ? need : 1) : cap);
  const cudaError_t e = launch_dependent(i8_kernel<AS, BS, SAT>, (unsigned)grid, kThreads, 0, stream, B);
  if (e != cudaSuccess) {
    set_cuda_error("i8_kernel launch", e);
    return T5E_ERR_CUDA;
  }
  return kernel_status("i8_kernel launch");
}

template <bool AS, bool BS>
int launch_sat(bool sat, const t5e_batch& B, cudaStream_t s) {
  return sat ? launch<AS, BS, true>(B, s) : launch<AS, BS, false>(B, s);
}

}  // namespace i8

int launch_i8(const t5e_model& M, const t5e_batch& B, cudaStream_t stream) {
  using namespace i8;
  if (M.family != T5E_FAMILY_I8 || B.sparse != 0 || B.tile_m != 1 || B.tile_n != 1) return T5E_ERR_UNSUPPORTED;
  if (B.n >= (1ull << 31) || B.k % 16 != 0 || B.k > kMaxK || B.c_bytes != 4) return T5E_ERR_UNSUPPORTED;
  if (B.a_stride % 16 != 0 || B.b_stride % 16 != 0) return T5E_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(B.a) | reinterpret_cast<uintptr_t>(B.b)) % 16 != 0) return T5E_ERR_UNSUPPORTED;
  const bool as = M.a_format == T5E_FMT_S8, bs = M.b_format == T5E_FMT_S8;
  const bool sat = M.saturate != 0;
  if (as) return bs ? launch_sat<true, true>(sat, B, stream) : launch_sat<true, false>(sat, B, stream);
  return bs ? launch_sat<false, true>(sat, B, stream) : launch_sat<false, false>(sat, B, stream);
}

}  // namespace t5e
