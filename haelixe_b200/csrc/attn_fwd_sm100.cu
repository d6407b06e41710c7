// tcgen05 attention forward (bf16, head_dim 64/128). Placeholder until the
// kernel lands: reports "not supported" so the dispatcher uses SIMT.
#include "hx_internal.h"

namespace hx {

bool sm100_supported(hx_dtype, const AttnDims&) { return false; }

cudaError_t sm100_attn_fwd(cudaStream_t, int, DeviceStatus*, const AttnDims&, const void*,
                           const void*, const void*, void*, float*, float, int) {
    return cudaErrorNotSupported;
}

}  // namespace hx
