// t5e_fast.cu -- specialised emulator kernels for the hot descriptors.
#include "t5e_dispatch.h"

namespace t5e {

int launch_fast(const t5e_model&, const t5e_batch&, cudaStream_t) { return T5E_ERR_UNSUPPORTED; }

}  // namespace t5e
