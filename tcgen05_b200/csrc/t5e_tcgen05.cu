// t5e_tcgen05.cu -- the hardware side of the cross-check: real tcgen05.mma
// instructions on the B200's tensor cores, for comparing the emulator's words
// with the hardware's (the role of the reference harness's probe runners,
// hardware_validation/src/tcgen05_*_probe.cu, written anew).
//
// One CTA of 128 threads per tile D = A B + C with M = 128, N = 16 and one
// instruction's K (8 TF32, 16 F16/BF16, 32 FP8 or 8-bit integers: 32-byte
// K-major rows in every case):
//
//  * A (128 rows) and B (16 rows) are staged in shared memory in the
//    non-swizzled K-major layout: 8-row x 16-byte core matrices, the two
//    16-byte halves of a row 128 bytes apart (leading byte offset) and groups
//    of 8 rows 256 bytes apart (stride byte offset);
//  * C is written into tensor memory (TMEM lane = row, column = n) with
//    tcgen05.st, one tcgen05.mma.cta_group::1 accumulates onto it, and
//    tcgen05.commit arrives on an mbarrier when the product is complete;
//  * every thread waits on that mbarrier with a bounded number of polls; a
//    wait that runs out sets the error word and the CTA stops (freeing its
//    tensor memory) instead of hanging;
//  * each thread reads its row of D back with tcgen05.ld.
//
// Accumulators take one 32-bit TMEM column per n: F32, S32, or F16 in the low
// half of the column.  FP6 and FP4 operands of kind::f8f6f4 sit in shared
// memory as 16-byte chunks of 16 packed elements followed by zero padding, so
// their 32-element rows are 32 bytes like the 8-bit ones.  No TMA, no
// clusters, no multicast.
#include <cuda_runtime.h>

#include "t5e.h"
#include "t5e_dispatch.h"

namespace t5e {
namespace hw {

constexpr int kRows = 128, kCols = 16, kRowBytes = 32, kTmemCols = 32;
constexpr uint32_t kWaitPolls = 1u << 20;  // bounded mbarrier polls per tile

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory matrix descriptor: start address, leading byte offset 128,
// stride byte offset 256 (all in 16-byte units), descriptor version 1, no
// swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
         (1ull << 46);
}

template <int KIND>
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc) {
  const uint32_t zero = 0, accumulate = 1;
  if constexpr (KIND == T5E_HW_TF32) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(zero));
  } else if constexpr (KIND == T5E_HW_F16) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(zero));
  } else if constexpr (KIND == T5E_HW_F8F6F4) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(zero));
  } else {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(zero));
  }
}

__device__ __forceinline__ bool wait_phase(uint32_t mbar, uint32_t phase) {
  for (uint32_t poll = 0; poll < kWaitPolls; ++poll) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, P1;\n\t}\n"
                 : "=r"(done) : "r"(mbar), "r"(phase) : "memory");
    if (done) return true;
  }
  return false;
}

template <int KIND>
__global__ void __launch_bounds__(kRows) tcgen05_tile_kernel(const uint8_t* __restrict__ A, const uint8_t* __restrict__ B,
                                                             const uint32_t* __restrict__ C, uint32_t* __restrict__ D,
                                                             uint32_t idesc, uint32_t tiles, int* error) {
  __shared__ __align__(128) uint8_t sA[kRows * kRowBytes];
  __shared__ __align__(128) uint8_t sB[kCols * kRowBytes];
  __shared__ __align__(8) uint64_t mbar;
  __shared__ uint32_t tmem_slot;
  const int t = threadIdx.x, warp = t >> 5;
  const uint32_t bar = smem_u32(&mbar);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(&tmem_slot)), "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (t == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(1));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  uint32_t phase = 0;
  for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    // stage row t of A and, for t < 16, row t of B in the core-matrix layout
    const uint4* ga = reinterpret_cast<const uint4*>(A + ((size_t)tile * kRows + t) * kRowBytes);
    const uint4 a0 = __ldg(ga), a1 = __ldg(ga + 1);
    *reinterpret_cast<uint4*>(sA + (t >> 3) * 256 + (t & 7) * 16) = a0;
    *reinterpret_cast<uint4*>(sA + (t >> 3) * 256 + 128 + (t & 7) * 16) = a1;
    if (t < kCols) {
      const uint4* gb = reinterpret_cast<const uint4*>(B + ((size_t)tile * kCols + t) * kRowBytes);
      const uint4 b0 = __ldg(gb), b1 = __ldg(gb + 1);
      *reinterpret_cast<uint4*>(sB + (t >> 3) * 256 + (t & 7) * 16) = b0;
      *reinterpret_cast<uint4*>(sB + (t >> 3) * 256 + 128 + (t & 7) * 16) = b1;
    }
    // C row t into TMEM lane t, columns 0..15
    const uint32_t* crow = C + ((size_t)tile * kRows + t) * kCols;
    uint32_t c[kCols];
#pragma unroll
    for (int j = 0; j < kCols; ++j) c[j] = __ldg(crow + j);
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                 "%13, %14, %15, %16};"
                 :: "r"(lane_base), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3]), "r"(c[4]), "r"(c[5]), "r"(c[6]),
                    "r"(c[7]), "r"(c[8]), "r"(c[9]), "r"(c[10]), "r"(c[11]), "r"(c[12]), "r"(c[13]), "r"(c[14]),
                    "r"(c[15]) : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // smem operands visible to the tensor core
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (t == 0) {
      mma<KIND>(tmem, smem_desc(smem_u32(sA)), smem_desc(smem_u32(sB)), idesc);
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                   :: "r"(bar) : "memory");
    }
    const bool ok = wait_phase(bar, phase);
    phase ^= 1u;
    if (__syncthreads_or(!ok)) {  // the product never arrived: record it and stop
      if (t == 0) atomicExch(error, 1);
      break;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    uint32_t d[kCols];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                 "%13, %14, %15}, [%16];"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
                   "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15])
                 : "r"(lane_base) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    uint32_t* drow = D + ((size_t)tile * kRows + t) * kCols;
#pragma unroll
    for (int j = 0; j < kCols; ++j) drow[j] = d[j];
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();  // shared memory and TMEM are reused by the next tile
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(kTmemCols));
  }
}

// The instruction descriptors this kernel's layouts implement, and only
// documented encodings of them: dense, A and B K-major, no negation or shift,
// M = 128, N = 16; per kind the operand format codes the instruction defines
// (kind::f16 with one type for A and B), the accumulator format (F16 only for
// F16 x F16 or f8f6f4 operands) and saturation for kind::i8 only.
bool descriptor_ok(int32_t kind, uint32_t idesc) {
  const uint32_t fields = (1u << 3) | (3u << 4) | (7u << 7) | (7u << 10) | (0x3Fu << 17) | (0x1Fu << 24);
  if ((idesc & ~fields) != 0u) return false;
  if (((idesc >> 24) & 0x1Fu) != 8u || ((idesc >> 17) & 0x3Fu) != 2u) return false;
  const uint32_t sat = (idesc >> 3) & 1u, cfmt = (idesc >> 4) & 3u;
  const uint32_t af = (idesc >> 7) & 7u, bf = (idesc >> 10) & 7u;
  constexpr uint32_t kF16 = 0u, kF32 = 1u, kS32 = 2u;
  auto f8f6f4 = [](uint32_t f) { return f == 0u || f == 1u || f == 3u || f == 4u || f == 5u; };
  switch (kind) {
    case T5E_HW_TF32: return af == 2u && bf == 2u && cfmt == kF32 && !sat;
    case T5E_HW_F16: return af <= 1u && bf == af && (cfmt == kF32 || (cfmt == kF16 && af == 0u)) && !sat;
    case T5E_HW_F8F6F4: return f8f6f4(af) && f8f6f4(bf) && (cfmt == kF32 || cfmt == kF16) && !sat;
    case T5E_HW_I8: return af <= 1u && bf <= 1u && cfmt == kS32;
    default: return false;
  }
}

template <int KIND>
int launch(const void* a, const void* b, const uint32_t* c, uint32_t* d, uint64_t tiles, uint32_t idesc, int* error,
           cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t cap = (uint64_t)sms * 4u;
  const int grid = (int)(tiles < cap ? tiles : cap);
  tcgen05_tile_kernel<KIND><<<grid, kRows, 0, stream>>>(static_cast<const uint8_t*>(a), static_cast<const uint8_t*>(b),
                                                        c, d, idesc, (uint32_t)tiles, error);
  return kernel_status("tcgen05_tile_kernel launch");
}


// ---- block-scaled kinds ---------------------------------------------------
//
// kind::mxf8f6f4 (UE8M0, one scale per 32 K), kind::mxf4 (E2M1, UE8M0, two
// scales per 64 K) and kind::mxf4nvf4 (E2M1, two UE8M0 or four UE4M3/UE8M0
// scales per 64 K) on tiles of M = 128, N = 128 and one instruction's K (32
// elements of f8f6f4, 64 packed E2M1), 32-byte K-major operand rows in the same
// shared-memory layout as above.  The scale factors live in tensor memory in
// the layout the instruction reads for cta_group::1: the factor of row (or
// column) r sits in lane r % 32 of every 32-lane subpartition, column r / 32
// of the scale-factor area, byte = the scale block along K (scale factor
// id 0).  One CTA of 128 threads per tile allocates 256 TMEM columns (D in
// 0-127, A scale factors at 192, B scale factors at 224); its dynamic shared
// memory request keeps at most two CTAs on an SM, so an allocation never
// waits.
constexpr int kBsRows = 128, kBsCols = 128, kBsTmemCols = 256, kBsSfaCol = 192, kBsSfbCol = 224;
constexpr int kBsSmemBytes = 96 * 1024;

__device__ __forceinline__ void tmem_st32(uint32_t addr, const uint32_t (&v)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
               :: "r"(addr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31]) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t (&v)[32]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]) : "r"(addr) : "memory");
}

template <int KIND>
__device__ __forceinline__ void mma_block_scaled(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                                 uint32_t tsfa, uint32_t tsfb) {
  const uint32_t accumulate = 1;
  if constexpr (KIND == T5E_HW_MXF8F6F4) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  } else if constexpr (KIND == T5E_HW_MXF4) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  } else if constexpr (KIND == T5E_HW_MXF4NVF4_2X) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  } else {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  }
}

template <int KIND>
__global__ void __launch_bounds__(kBsRows) tcgen05_block_scaled_kernel(
    const uint8_t* __restrict__ A, const uint8_t* __restrict__ B, const uint32_t* __restrict__ C,
    uint32_t* __restrict__ D, const uint32_t* __restrict__ SFA, const uint32_t* __restrict__ SFB, uint32_t idesc,
    uint32_t tiles, int* error) {
  extern __shared__ __align__(128) uint8_t smem_bs[];
  uint8_t* sA = smem_bs;                     // 128 rows of 32 bytes, core-matrix layout
  uint8_t* sB = smem_bs + kBsRows * kRowBytes;
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem_bs + 2 * kBsRows * kRowBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mbar + 1);
  const int t = threadIdx.x, warp = t >> 5, l = t & 31;
  const uint32_t bar = smem_u32(mbar);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(kBsTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (t == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(1));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  uint32_t phase = 0;
  for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    // row t of A and of B into the core-matrix layout
    const uint4* ga = reinterpret_cast<const uint4*>(A + ((size_t)tile * kBsRows + t) * kRowBytes);
    const uint4* gb = reinterpret_cast<const uint4*>(B + ((size_t)tile * kBsCols + t) * kRowBytes);
    const uint4 a0 = __ldg(ga), a1 = __ldg(ga + 1), b0 = __ldg(gb), b1 = __ldg(gb + 1);
    *reinterpret_cast<uint4*>(sA + (t >> 3) * 256 + (t & 7) * 16) = a0;
    *reinterpret_cast<uint4*>(sA + (t >> 3) * 256 + 128 + (t & 7) * 16) = a1;
    *reinterpret_cast<uint4*>(sB + (t >> 3) * 256 + (t & 7) * 16) = b0;
    *reinterpret_cast<uint4*>(sB + (t >> 3) * 256 + 128 + (t & 7) * 16) = b1;
    // C row t into lane t, columns 0-127
    const uint4* crow = reinterpret_cast<const uint4*>(C + ((size_t)tile * kBsRows + t) * kBsCols);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      uint32_t v[32];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint4 x = __ldg(crow + ch * 8 + q);
        v[4 * q] = x.x; v[4 * q + 1] = x.y; v[4 * q + 2] = x.z; v[4 * q + 3] = x.w;
      }
      tmem_st32(lane_base + (uint32_t)(ch * 32), v);
    }
    // scale factors: column c holds the factors of rows 32 c + (lane % 32),
    // the same in every subpartition
    uint32_t fa[4], fb[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      fa[c] = __ldg(SFA + (size_t)tile * kBsRows + 32 * c + l);
      fb[c] = __ldg(SFB + (size_t)tile * kBsCols + 32 * c + l);
    }
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};"
                 :: "r"(lane_base + (uint32_t)kBsSfaCol), "r"(fa[0]), "r"(fa[1]), "r"(fa[2]), "r"(fa[3]) : "memory");
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};"
                 :: "r"(lane_base + (uint32_t)kBsSfbCol), "r"(fb[0]), "r"(fb[1]), "r"(fb[2]), "r"(fb[3]) : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (t == 0) {
      mma_block_scaled<KIND>(tmem, smem_desc(smem_u32(sA)), smem_desc(smem_u32(sB)), idesc,
                             tmem + (uint32_t)kBsSfaCol, tmem + (uint32_t)kBsSfbCol);
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                   :: "r"(bar) : "memory");
    }
    const bool ok = wait_phase(bar, phase);
    phase ^= 1u;
    if (__syncthreads_or(!ok)) {  // the product never arrived: record it and stop
      if (t == 0) atomicExch(error, 1);
      break;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    uint4* drow = reinterpret_cast<uint4*>(D + ((size_t)tile * kBsRows + t) * kBsCols);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      uint32_t v[32];
      tmem_ld32(lane_base + (uint32_t)(ch * 32), v);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int q = 0; q < 8; ++q) drow[ch * 8 + q] = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();  // shared memory and TMEM are reused by the next tile
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(kBsTmemCols));
  }
}

// Documented block-scaled encodings for M = 128, N = 128, dense K-major
// operands, scale factor ids 0 and the default K: E2M1 (code 1) for the mxf4
// kinds, the f8f6f4 codes for mxf8f6f4, UE8M0 scales (bit 23 set) except for
// the four-scale mxf4nvf4 form, which also takes UE4M3.
bool block_scaled_descriptor_ok(int32_t kind, uint32_t idesc) {
  const uint32_t fields = (7u << 7) | (7u << 10) | (0x3Fu << 17) | (1u << 23) | (0x1Fu << 24);
  if ((idesc & ~fields) != 0u) return false;
  if (((idesc >> 24) & 0x1Fu) != 8u || ((idesc >> 17) & 0x3Fu) != 16u) return false;
  const uint32_t af = (idesc >> 7) & 7u, bf = (idesc >> 10) & 7u, ue8m0 = (idesc >> 23) & 1u;
  auto f8f6f4 = [](uint32_t f) { return f == 0u || f == 1u || f == 3u || f == 4u || f == 5u; };
  switch (kind) {
    case T5E_HW_MXF8F6F4: return f8f6f4(af) && f8f6f4(bf) && ue8m0;
    case T5E_HW_MXF4: return af == 1u && bf == 1u && ue8m0;
    case T5E_HW_MXF4NVF4_2X: return af == 1u && bf == 1u && ue8m0;
    case T5E_HW_MXF4NVF4_4X: return af == 1u && bf == 1u;
    default: return false;
  }
}

template <int KIND>
int launch_block_scaled(const void* a, const void* b, const uint32_t* c, uint32_t* d, const uint32_t* sfa,
                        const uint32_t* sfb, uint64_t tiles, uint32_t idesc, int* error, cudaStream_t stream) {
  const int rc = raise_smem_limit<tcgen05_block_scaled_kernel<KIND>>(kBsSmemBytes, "tcgen05 block-scaled attribute");
  if (rc != T5E_OK) return rc;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t cap = (uint64_t)sms * 2u;
  const int grid = (int)(tiles < cap ? tiles : cap);
  tcgen05_block_scaled_kernel<KIND><<<grid, kBsRows, kBsSmemBytes, stream>>>(
      static_cast<const uint8_t*>(a), static_cast<const uint8_t*>(b), c, d, sfa, sfb, idesc, (uint32_t)tiles, error);
  return kernel_status("tcgen05_block_scaled_kernel launch");
}

// ---- sparse kinds ----------------------------------------------------------
//
// tcgen05.mma.sp with a 2:4 (1:2 for TF32, pairwise 4:8 for the mxf4 kinds)
// compressed A: kind::tf32, kind::f16 and kind::f8f6f4 on tiles of M = 64,
// N = 8, and the block-scaled kinds on tiles of M = 128, N = 8 (the shapes the
// reference harness's sparse probes run, hardware_validation/src/
// tcgen05_*_sparse_probe.cu).  Each case is one uniform tile: every row of A
// is the case's compressed row (32 bytes: half the logical K), every column
// of B its logical K row (64 bytes), every element of C its c word, every
// row's metadata (and scale word) the case's.  Every element of D is then the
// same scalar, so the result does not depend on which TMEM lane holds which
// row's metadata; the kernel reports D[0][0] and how many of the tile's
// other D elements differ from it.
//
// The metadata region (TMEM columns 128-255 of every lane) is filled
// uniformly with one of three word patterns (`layout`):
//   0  even columns the first metadata word, odd columns the second (64 bits
//      of selectors per row in two consecutive columns);
//   1  lanes 0-7 of each 16 the low 16 bits of the first word in both
//      halves, lanes 8-15 its high 16 bits (the pattern the reference's
//      kind::tf32 and kind::f16 probes store);
//   2  lanes 0-7 of each 16 the first word, lanes 8-15 the second.
// Every pattern holds only the case's legal selectors.  D sits in columns
// 0-7 (for M = 64 in lanes 0-15 of each 32-lane subpartition), the scale
// factors at columns 64 (A) and 96 (B) as for the dense block-scaled tiles.
// The 96 KB dynamic shared memory request keeps at most two CTAs (2 x 256
// TMEM columns) on an SM, so an allocation never waits.
constexpr int kSpN = 8, kSpTmemCols = 256, kSpSfaCol = 64, kSpSfbCol = 96, kSpMetaCol = 128;
constexpr int kSpARow = 32, kSpBRow = 64, kSpDump = 128 * kSpN, kSpSmemBytes = 96 * 1024;

template <int KIND>
constexpr bool sparse_scaled() {
  return KIND >= T5E_HW_SP_MXF8F6F4;
}

__device__ __forceinline__ void tmem_st8(uint32_t addr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
               :: "r"(addr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t addr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(addr) : "memory");
}

// Shared-memory matrix descriptor with explicit leading (K direction) and
// stride (8-row groups) byte offsets, version 1, no swizzle.
__device__ __forceinline__ uint64_t smem_desc_lbo_sbo(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ uint32_t metadata_word(int layout, int lane, int col, uint32_t m0, uint32_t m1) {
  if (layout == 1) {
    const uint32_t h = (lane & 15) < 8 ? (m0 & 0xFFFFu) : (m0 >> 16);
    return h | (h << 16);
  }
  if (layout == 2) return (lane & 15) < 8 ? m0 : m1;
  return (col & 1) ? m1 : m0;
}

template <int KIND>
__device__ __forceinline__ void mma_sparse(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t tmeta, uint32_t idesc,
                                           uint32_t tsfa, uint32_t tsfb) {
  const uint32_t accumulate = 1, zero = 0;
  if constexpr (KIND == T5E_HW_SP_TF32) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
                 "tcgen05.mma.sp.cta_group::1.kind::tf32 [%0], %1, %2, [%3], %4, {%6, %6, %6, %6}, p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(tmeta), "r"(idesc), "r"(accumulate), "r"(zero));
  } else if constexpr (KIND == T5E_HW_SP_F16) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
                 "tcgen05.mma.sp.cta_group::1.kind::f16 [%0], %1, %2, [%3], %4, {%6, %6, %6, %6}, p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(tmeta), "r"(idesc), "r"(accumulate), "r"(zero));
  } else if constexpr (KIND == T5E_HW_SP_F8F6F4) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
                 "tcgen05.mma.sp.cta_group::1.kind::f8f6f4 [%0], %1, %2, [%3], %4, {%6, %6, %6, %6}, p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(tmeta), "r"(idesc), "r"(accumulate), "r"(zero));
  } else if constexpr (KIND == T5E_HW_SP_MXF8F6F4) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
                 "tcgen05.mma.sp.cta_group::1.kind::mxf8f6f4.block_scale.scale_vec::1X [%0], %1, %2, [%3], %4, "
                 "[%6], [%7], p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(tmeta), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  } else if constexpr (KIND == T5E_HW_SP_MXF4) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
                 "tcgen05.mma.sp.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, [%3], %4, "
                 "[%6], [%7], p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(tmeta), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  } else if constexpr (KIND == T5E_HW_SP_MXF4NVF4_2X) {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
                 "tcgen05.mma.sp.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::2X [%0], %1, %2, [%3], %4, "
                 "[%6], [%7], p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(tmeta), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  } else {
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %5, 0;\n\t"
                 "tcgen05.mma.sp.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, [%3], %4, "
                 "[%6], [%7], p;\n\t}\n"
                 :: "r"(tmem_d), "l"(da), "l"(db), "r"(tmeta), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
  }
}

template <int KIND>
__global__ void __launch_bounds__(128) tcgen05_sparse_kernel(
    const uint8_t* __restrict__ A, const uint8_t* __restrict__ B, const uint32_t* __restrict__ C,
    const uint32_t* __restrict__ META, const uint32_t* __restrict__ SF, uint32_t* __restrict__ D,
    int32_t* __restrict__ disagree, uint32_t* __restrict__ dump, uint32_t idesc, int32_t layout, uint32_t cases,
    int* error) {
  constexpr int kM = sparse_scaled<KIND>() ? 128 : 64;
  extern __shared__ __align__(128) uint8_t smem_sp[];
  uint8_t* sA = smem_sp;                    // kM rows of 32 bytes, core-matrix layout
  uint8_t* sB = smem_sp + 128 * kSpARow;    // 8 rows of 64 bytes: four K chunks 128 bytes apart
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sB + kSpN * kSpBRow);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mbar + 1);
  uint32_t* sref = tmem_slot + 1;
  int* scount = reinterpret_cast<int*>(tmem_slot + 2);
  const int t = threadIdx.x, warp = t >> 5, l = t & 31;
  const uint32_t bar = smem_u32(mbar);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(tmem_slot)), "r"(kSpTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (t == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(1));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *scount = 0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  uint32_t phase = 0;
  for (uint32_t cs = blockIdx.x; cs < cases; cs += gridDim.x) {
    // every row of A is the case's compressed row; every column of B its K row
    const uint4* ga = reinterpret_cast<const uint4*>(A + (size_t)cs * kSpARow);
    const uint4 a0 = __ldg(ga), a1 = __ldg(ga + 1);
    if (t < kM) {
      *reinterpret_cast<uint4*>(sA + (t >> 3) * 256 + (t & 7) * 16) = a0;
      *reinterpret_cast<uint4*>(sA + (t >> 3) * 256 + 128 + (t & 7) * 16) = a1;
    }
    if (t < 4 * kSpN) {
      const int row = t & 7, chunk = t >> 3;
      const uint4 bv = __ldg(reinterpret_cast<const uint4*>(B + (size_t)cs * kSpBRow) + chunk);
      *reinterpret_cast<uint4*>(sB + chunk * 128 + row * 16) = bv;
    }
    const uint32_t c = __ldg(C + cs);
    const uint32_t cv[8] = {c, c, c, c, c, c, c, c};
    tmem_st8(lane_base, cv);
    if constexpr (sparse_scaled<KIND>()) {
      const uint32_t sa = __ldg(SF + 2 * (size_t)cs), sb = __ldg(SF + 2 * (size_t)cs + 1);
      asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %1, %1, %1};"
                   :: "r"(lane_base + (uint32_t)kSpSfaCol), "r"(sa) : "memory");
      asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %1, %1, %1};"
                   :: "r"(lane_base + (uint32_t)kSpSfbCol), "r"(sb) : "memory");
    }
    const uint32_t m0 = __ldg(META + 2 * (size_t)cs), m1 = __ldg(META + 2 * (size_t)cs + 1);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t mv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) mv[j] = metadata_word(layout, l, j, m0, m1);
      tmem_st32(lane_base + (uint32_t)(kSpMetaCol + 32 * q), mv);
    }
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (t == 0) {
      mma_sparse<KIND>(tmem, smem_desc_lbo_sbo(smem_u32(sA), 128, 256), smem_desc_lbo_sbo(smem_u32(sB), 128, 512),
                       tmem + (uint32_t)kSpMetaCol, idesc, tmem + (uint32_t)kSpSfaCol, tmem + (uint32_t)kSpSfbCol);
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                   :: "r"(bar) : "memory");
    }
    const bool ok = wait_phase(bar, phase);
    phase ^= 1u;
    if (__syncthreads_or(!ok)) {  // the product never arrived: record it and stop
      if (t == 0) atomicExch(error, 1);
      break;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    uint32_t dv[8];
    tmem_ld8(lane_base, dv);
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    if (t == 0) *sref = dv[0];
    __syncthreads();
    const uint32_t ref = *sref;
    int bad = 0;
    if (kM == 128 || l < 16) {  // the lanes that hold rows of D
#pragma unroll
      for (int j = 0; j < 8; ++j) bad += dv[j] != ref;
    }
    if (bad) atomicAdd(scount, bad);
    if (dump) {
#pragma unroll
      for (int j = 0; j < 8; ++j) dump[(size_t)cs * kSpDump + t * 8 + j] = dv[j];
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();  // shared memory and TMEM are reused by the next case
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (t == 0) {
      D[cs] = ref;
      disagree[cs] = *scount;
      *scount = 0;
    }
  }
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(kSpTmemCols));
  }
}

// Documented sparse encodings for the tiles above: the sparse flag (bit 2)
// set, sparsity selector 0, dense K-major operands, N = 8 and M = 64 (M = 128
// for the block-scaled kinds); per kind the operand formats the dense check
// takes, an F32 accumulator for the unscaled kinds, UE8M0 scales except for
// the four-scale mxf4nvf4 form, scale factor ids 0.
bool sparse_descriptor_ok(int32_t kind, uint32_t idesc) {
  const bool scaled = kind >= T5E_HW_SP_MXF8F6F4;
  uint32_t fields = (1u << 2) | (7u << 7) | (7u << 10) | (0x3Fu << 17) | (0x1Fu << 24);
  fields |= scaled ? (1u << 23) : (3u << 4);
  if ((idesc & ~fields) != 0u || ((idesc >> 2) & 1u) == 0u) return false;
  if (((idesc >> 17) & 0x3Fu) != (uint32_t)(kSpN >> 3) || ((idesc >> 24) & 0x1Fu) != (scaled ? 8u : 4u)) return false;
  const uint32_t cfmt = (idesc >> 4) & 3u, af = (idesc >> 7) & 7u, bf = (idesc >> 10) & 7u, ue8m0 = (idesc >> 23) & 1u;
  auto f8f6f4 = [](uint32_t f) { return f == 0u || f == 1u || f == 3u || f == 4u || f == 5u; };
  switch (kind) {
    case T5E_HW_SP_TF32: return af == 2u && bf == 2u && cfmt == 1u;
    case T5E_HW_SP_F16: return af <= 1u && bf == af && cfmt == 1u;
    case T5E_HW_SP_F8F6F4: return f8f6f4(af) && f8f6f4(bf) && cfmt == 1u;
    case T5E_HW_SP_MXF8F6F4: return f8f6f4(af) && f8f6f4(bf) && ue8m0;
    case T5E_HW_SP_MXF4:
    case T5E_HW_SP_MXF4NVF4_2X: return af == 1u && bf == 1u && ue8m0;
    case T5E_HW_SP_MXF4NVF4_4X: return af == 1u && bf == 1u;
    default: return false;
  }
}

template <int KIND>
int launch_sparse(const void* a, const void* b, const uint32_t* c, const uint32_t* meta, const uint32_t* scales,
                  uint32_t* d, int32_t* disagree, uint32_t* dump, uint64_t cases, uint32_t idesc, int32_t layout,
                  int* error, cudaStream_t stream) {
  const int rc = raise_smem_limit<tcgen05_sparse_kernel<KIND>>(kSpSmemBytes, "tcgen05 sparse attribute");
  if (rc != T5E_OK) return rc;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t cap = (uint64_t)sms * 2u;
  const int grid = (int)(cases < cap ? cases : cap);
  tcgen05_sparse_kernel<KIND><<<grid, 128, kSpSmemBytes, stream>>>(
      static_cast<const uint8_t*>(a), static_cast<const uint8_t*>(b), c, meta, scales, d, disagree, dump, idesc,
      layout, (uint32_t)cases, error);
  return kernel_status("tcgen05_sparse_kernel launch");
}

}  // namespace hw
}  // namespace t5e

extern "C" int t5e_tcgen05_tiles(int32_t kind, uint32_t idesc, const void* a, const void* b, const uint32_t* c,
                                 uint32_t* d, uint64_t tiles, int32_t* error, void* stream) {
  using namespace t5e::hw;
  if (tiles == 0) return T5E_OK;
  if (!a || !b || !c || !d || !error || tiles >= (1ull << 31)) return T5E_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) % 16 != 0) return T5E_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(d)) % 4 != 0) return T5E_ERR_INVALID;
  if (!descriptor_ok(kind, idesc)) return T5E_ERR_INVALID;
  int* err = reinterpret_cast<int*>(error);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (kind) {
    case T5E_HW_TF32: return launch<T5E_HW_TF32>(a, b, c, d, tiles, idesc, err, s);
    case T5E_HW_F16: return launch<T5E_HW_F16>(a, b, c, d, tiles, idesc, err, s);
    case T5E_HW_F8F6F4: return launch<T5E_HW_F8F6F4>(a, b, c, d, tiles, idesc, err, s);
    case T5E_HW_I8: return launch<T5E_HW_I8>(a, b, c, d, tiles, idesc, err, s);
    default: return T5E_ERR_INVALID;
  }
}

extern "C" int t5e_tcgen05_block_scaled_tiles(int32_t kind, uint32_t idesc, const void* a, const void* b,
                                              const uint32_t* c, uint32_t* d, const uint32_t* scale_a,
                                              const uint32_t* scale_b, uint64_t tiles, int32_t* error,
                                              void* stream) {
  using namespace t5e::hw;
  if (tiles == 0) return T5E_OK;
  if (!a || !b || !c || !d || !scale_a || !scale_b || !error || tiles >= (1ull << 31)) return T5E_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c) |
       reinterpret_cast<uintptr_t>(d)) % 16 != 0)
    return T5E_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(scale_a) | reinterpret_cast<uintptr_t>(scale_b)) % 4 != 0) return T5E_ERR_INVALID;
  if (!block_scaled_descriptor_ok(kind, idesc)) return T5E_ERR_INVALID;
  int* err = reinterpret_cast<int*>(error);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (kind) {
    case T5E_HW_MXF8F6F4: return launch_block_scaled<T5E_HW_MXF8F6F4>(a, b, c, d, scale_a, scale_b, tiles, idesc, err, s);
    case T5E_HW_MXF4: return launch_block_scaled<T5E_HW_MXF4>(a, b, c, d, scale_a, scale_b, tiles, idesc, err, s);
    case T5E_HW_MXF4NVF4_2X:
      return launch_block_scaled<T5E_HW_MXF4NVF4_2X>(a, b, c, d, scale_a, scale_b, tiles, idesc, err, s);
    case T5E_HW_MXF4NVF4_4X:
      return launch_block_scaled<T5E_HW_MXF4NVF4_4X>(a, b, c, d, scale_a, scale_b, tiles, idesc, err, s);
    default: return T5E_ERR_INVALID;
  }
}

extern "C" int t5e_tcgen05_sparse_cases(int32_t kind, uint32_t idesc, int32_t meta_layout, const void* a,
                                        const void* b, const uint32_t* c, const uint32_t* meta,
                                        const uint32_t* scales, uint32_t* d, int32_t* disagree, uint32_t* dump,
                                        uint64_t cases, int32_t* error, void* stream) {
  using namespace t5e::hw;
  if (cases == 0) return T5E_OK;
  const bool scaled = kind >= T5E_HW_SP_MXF8F6F4;
  if (!a || !b || !c || !meta || !d || !disagree || !error || (scaled && !scales) || cases >= (1ull << 31))
    return T5E_ERR_INVALID;
  if (meta_layout < 0 || meta_layout > 2) return T5E_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) % 16 != 0) return T5E_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(c) | reinterpret_cast<uintptr_t>(meta) | reinterpret_cast<uintptr_t>(scales) |
       reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(disagree) | reinterpret_cast<uintptr_t>(dump)) %
          4 != 0)
    return T5E_ERR_INVALID;
  if (!sparse_descriptor_ok(kind, idesc)) return T5E_ERR_INVALID;
  int* err = reinterpret_cast<int*>(error);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define T5E_SPARSE_CASE(K)                                                                                      \
  case K:                                                                                                       \
    return launch_sparse<K>(a, b, c, meta, scales, d, disagree, dump, cases, idesc, meta_layout, err, s);
  switch (kind) {
    T5E_SPARSE_CASE(T5E_HW_SP_TF32)
    T5E_SPARSE_CASE(T5E_HW_SP_F16)
    T5E_SPARSE_CASE(T5E_HW_SP_F8F6F4)
    T5E_SPARSE_CASE(T5E_HW_SP_MXF8F6F4)
    T5E_SPARSE_CASE(T5E_HW_SP_MXF4)
    T5E_SPARSE_CASE(T5E_HW_SP_MXF4NVF4_2X)
    T5E_SPARSE_CASE(T5E_HW_SP_MXF4NVF4_4X)
    default: return T5E_ERR_INVALID;
  }
#undef T5E_SPARSE_CASE
}
