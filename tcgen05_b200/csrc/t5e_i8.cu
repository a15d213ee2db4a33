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

// One case's result word from its dot product and C.
template <bool SAT>
__device__ __forceinline__ uint32_t i8_word(int32_t dot, uint32_t cword) {
  const int64_t total = (int64_t)(int32_t)cword + dot;
  int64_t r = total;
  if constexpr (SAT) r = total < -2147483648ll ? -2147483648ll : (total > 2147483647ll ? 2147483647ll : total);
  return (uint32_t)r;
}

// The dot product of `chunks` 16-byte chunks of two rows (CHUNKS > 0: that
// many, unrolled; 0: `chunks` at run time).
template <bool AS, bool BS, int CHUNKS>
__device__ __forceinline__ int32_t i8_dot(const uint4* pa, const uint4* pb, int chunks) {
  int32_t dot = 0;
  if constexpr (CHUNKS > 0) {
    uint4 a[CHUNKS], b[CHUNKS];
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) a[j] = __ldg(pa + j), b[j] = __ldg(pb + j);
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
      dot = dot4<AS, BS>(a[j].x, b[j].x, dot);
      dot = dot4<AS, BS>(a[j].y, b[j].y, dot);
      dot = dot4<AS, BS>(a[j].z, b[j].z, dot);
      dot = dot4<AS, BS>(a[j].w, b[j].w, dot);
    }
  } else {
#pragma unroll 4
    for (int j = 0; j < chunks; ++j) {
      const uint4 a = __ldg(pa + j), b = __ldg(pb + j);
      dot = dot4<AS, BS>(a.x, b.x, dot);
      dot = dot4<AS, BS>(a.y, b.y, dot);
      dot = dot4<AS, BS>(a.z, b.z, dot);
      dot = dot4<AS, BS>(a.w, b.w, dot);
    }
  }
  return dot;
}

// Two cases a stride apart per step: both cases' rows and C words are
// requested before either is summed, so twice the bytes are in flight.
template <bool AS, bool BS, bool SAT, int CHUNKS>
__global__ void __launch_bounds__(kThreads) i8_kernel(const t5e_batch B) {
  // programmatic dependent launch: no prologue, so wait for the previous grid at once
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t n = (uint32_t)B.n;
  const uint32_t stride = gridDim.x * blockDim.x;
  const int chunks = B.k / 16;
  const uint8_t* A = static_cast<const uint8_t*>(B.a);
  const uint8_t* Bm = static_cast<const uint8_t*>(B.b);
  const uint32_t* C = static_cast<const uint32_t*>(B.c);
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += 2 * stride) {
    const uint32_t i2 = i + stride;
    const bool two = i2 < n;
    const uint32_t c1 = __ldg(C + i), c2 = two ? __ldg(C + i2) : 0u;
    const int32_t d1 = i8_dot<AS, BS, CHUNKS>(reinterpret_cast<const uint4*>(A + (size_t)i * B.a_stride),
                                              reinterpret_cast<const uint4*>(Bm + (size_t)i * B.b_stride), chunks);
    int32_t d2 = 0;
    if (two)
      d2 = i8_dot<AS, BS, CHUNKS>(reinterpret_cast<const uint4*>(A + (size_t)i2 * B.a_stride),
                                  reinterpret_cast<const uint4*>(Bm + (size_t)i2 * B.b_stride), chunks);
    B.d[i] = i8_word<SAT>(d1, c1);
    if (B.status) B.status[i] = (uint8_t)T5E_CASE_OK;
    if (two) {
      B.d[i2] = i8_word<SAT>(d2, c2);
      if (B.status) B.status[i2] = (uint8_t)T5E_CASE_OK;
    }
  }
}

template <bool AS, bool BS, bool SAT, int CHUNKS>
int launch_chunks(const t5e_batch& B, cudaStream_t stream) {
  auto kernel = i8_kernel<AS, BS, SAT, CHUNKS>;
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const uint64_t need = (B.n + kThreads - 1) / kThreads;
  const uint64_t cap = (uint64_t)sms * (uint64_t)per_sm;
  const int grid = (int)(need < cap ? (need ? need : 1) : cap);
  const cudaError_t e = launch_dependent(kernel, (unsigned)grid, kThreads, 0, stream, B);
  if (e != cudaSuccess) {
    set_cuda_error("i8_kernel launch", e);
    return T5E_ERR_CUDA;
  }
  return kernel_status("i8_kernel launch");
}

template <bool AS, bool BS, bool SAT>
int launch(const t5e_batch& B, cudaStream_t stream) {
  // K = 32, one instruction's K and the sweep's, unrolled; any other K in a loop
  return B.k == 32 ? launch_chunks<AS, BS, SAT, 2>(B, stream) : launch_chunks<AS, BS, SAT, 0>(B, stream);
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
