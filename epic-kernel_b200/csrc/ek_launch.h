// Host-side declarations of the kernel launchers. ek_decode.cu is compiled
// once per variant; each copy defines one launcher below. launch_decode picks
// the variant for the model and the prefetch options.
#pragma once

#include <cuda_runtime.h>

#include "ek_kernel.cuh"

namespace ek {

namespace llama { cudaError_t launch(const KParams& p, cudaStream_t stream); }
namespace llama_pf { cudaError_t launch(const KParams& p, cudaStream_t stream); }
namespace mixtral { cudaError_t launch(const KParams& p, cudaStream_t stream); }
namespace mixtral_pf { cudaError_t launch(const KParams& p, cudaStream_t stream); }

// Cooperative launch of the decode kernel: one block per instruction queue.
inline cudaError_t launch_decode(const KParams& p, cudaStream_t stream) {
  const bool pf = p.pf_stages > 0 || p.pf_next > 0 || (p.pf_mlp & (PF_UPGATE | PF_DOWN)) != 0;
  if (p.model == MODEL_MIXTRAL) return pf ? mixtral_pf::launch(p, stream) : mixtral::launch(p, stream);
  return pf ? llama_pf::launch(p, stream) : llama::launch(p, stream);
}

}  // namespace ek
