// tcgen05 attention backward (bf16, head_dim 64/128). Placeholder.
#include "hx_internal.h"

namespace hx {

bool sm100_bwd_supported(hx_dtype, const AttnDims&) { return false; }

uint64_t sm100_bwd_workspace_bytes(const AttnDims&) { return 0; }

cudaError_t sm100_attn_bwd(cudaStream_t, int, DeviceStatus*, const AttnDims&, const void*,
                           const void*, const void*, const void*, const void*, const float*,
                           void*, void*, void*, void*, float, int) {
    return cudaErrorNotSupported;
}

}  // namespace hx
