// Tensor-core (tcgen05) flash-attention prefill. Placeholder entry points until
// the kernel lands; attn_tc_supported() = false routes every call to the
// CUDA-core kernel.
#include "common.cuh"
#include "kernels.h"

namespace wv {

bool attn_tc_supported(const AttnArgs&) { return false; }

cudaError_t attn_prefill_tc(const AttnArgs&, cudaStream_t) { return cudaErrorNotSupported; }

} // namespace wv
