// t5e_dispatch.h -- internal interface between the C ABI layer and the
// specialised kernels.
#pragma once

#include <cuda_runtime.h>

#include <atomic>

#include "t5e.h"

namespace t5e {

// Launches a specialised kernel when one covers (model, batch); returns
// T5E_ERR_UNSUPPORTED (and launches nothing) otherwise.
int launch_fast(const t5e_model& M, const t5e_batch& B, cudaStream_t stream);

// The NVFP4 kernel (t5e_nvfp4.cu); same contract as launch_fast.
int launch_nvfp4(const t5e_model& M, const t5e_batch& B, cudaStream_t stream);

// The UE8M0 MXF4-family kernel (t5e_mxf4.cu); same contract as launch_fast.
int launch_mxf4(const t5e_model& M, const t5e_batch& B, cudaStream_t stream);

// The kind::i8 kernel (t5e_i8.cu); same contract as launch_fast.
int launch_i8(const t5e_model& M, const t5e_batch& B, cudaStream_t stream);

// The TF32/BF16/F16 raw-window kernel (t5e_wide.cu); same contract.
int launch_wide(const t5e_model& M, const t5e_batch& B, cudaStream_t stream);

// Records the last launch error for t5e_last_error(); T5E_OK or T5E_ERR_CUDA.
int kernel_status(const char* what);

// Records a failing CUDA call for t5e_last_error().
void set_cuda_error(const char* what, cudaError_t err);

// Grid size for a grid-stride loop over n items.
int grid_for(uint64_t n, int block);

// The host-side checks of t5e_mma_dot_batch (T5E_OK or the error code it
// would return), made without any CUDA call.
int validate(const t5e_model* M, const t5e_batch* B);

// Launches `kernel` on `stream` as a programmatic dependent of the previous
// kernel there (programmatic stream serialisation): its blocks may start
// while that kernel's last blocks run, so the kernel must execute
// griddepcontrol.wait before it reads or writes global memory that earlier
// work on the stream may touch.
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kernel)(Params...), unsigned grid, unsigned block, size_t smem,
                             cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Raises Kernel's dynamic shared-memory limit to `bytes` on the current
// device, once per device and kernel (one flag array per kernel; host
// threads may race to set it, which is harmless: the attribute value is the
// same).  Returns T5E_OK or T5E_ERR_CUDA.
template <auto Kernel>
int raise_smem_limit(int bytes, const char* what) {
  static std::atomic<bool> done[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  const bool cached = dev >= 0 && dev < 64;
  if (cached && done[dev].load(std::memory_order_acquire)) return T5E_OK;
  const cudaError_t err = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err != cudaSuccess) {
    set_cuda_error(what, err);
    return T5E_ERR_CUDA;
  }
  if (cached) done[dev].store(true, std::memory_order_release);
  return T5E_OK;
}

}  // namespace t5e
