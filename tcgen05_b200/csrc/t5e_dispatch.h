// t5e_dispatch.h -- internal interface between the C ABI layer and the
// specialised kernels.
#pragma once

#include <cuda_runtime.h>

#include "t5e.h"

namespace t5e {

// Launches a specialised kernel when one covers (model, batch); returns
// T5E_ERR_UNSUPPORTED (and launches nothing) otherwise.
int launch_fast(const t5e_model& M, const t5e_batch& B, cudaStream_t stream);

// The NVFP4 kernel (t5e_nvfp4.cu); same contract as launch_fast.
int launch_nvfp4(const t5e_model& M, const t5e_batch& B, cudaStream_t stream);

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

}  // namespace t5e
