// tcgen05 / TMEM / TMA block-sparse attention (work in progress).
#include "common.cuh"
#include "kernels.h"

namespace vggt {

bool attn_tc05_supported(const AttnArgs&) { return false; }

cudaError_t launch_attn_tc05(const AttnArgs&, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace vggt
