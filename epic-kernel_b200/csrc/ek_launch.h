// Host-side declaration of the kernel launcher shared by ek_decode.cu and the
// C ABI in ek_capi.cu.
#pragma once

#include <cuda_runtime.h>

#include "ek_kernel.cuh"

namespace ek {

// Cooperative launch of the decode kernel: one block per instruction queue.
cudaError_t launch_decode(const KParams& p, cudaStream_t stream);

}  // namespace ek
