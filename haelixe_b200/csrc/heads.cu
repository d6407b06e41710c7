// Head reassembly after an all-gather of per-rank head shards: the
// [B,H,S,D] -> [B,S,H,D] merge of MultiHeadAttention::forward
// (src/nn/attention.rs:91-94) done directly from the gathered shards, so no
// intermediate [B,H,S,D] copy is made. HBM-bound copy, 16 bytes per thread
// when a head row allows it.
#include "hx_internal.h"

namespace hx {
namespace {

template <typename U>
__global__ void __launch_bounds__(256) reassemble_kernel(const U* __restrict__ src, U* __restrict__ dst,
                                                         int n, int B, int Hs, int S, int units,
                                                         int layout) {
    const int H = n * Hs;
    const int64_t total = (int64_t)n * B * Hs * S * units;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int u = (int)(idx % units);
        int64_t rest = idx / units;
        const int s = (int)(rest % S);
        rest /= S;
        const int hs = (int)(rest % Hs);
        rest /= Hs;
        const int b = (int)(rest % B);
        const int r = (int)(rest / B);
        const int h = r * Hs + hs;
        const int64_t row = layout == 0 ? ((int64_t)b * H + h) * S + s : ((int64_t)b * S + s) * H + h;
        dst[row * units + u] = src[idx];
    }
}

template <typename U>
cudaError_t launch(cudaStream_t st, const void* src, void* dst, int n, int B, int Hs, int S,
                   int units, int layout, int sm_count) {
    const int64_t total = (int64_t)n * B * Hs * S * units;
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = (int64_t)sm_count * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    reassemble_kernel<U><<<(unsigned)blocks, 256, 0, st>>>((const U*)src, (U*)dst, n, B, Hs, S,
                                                          units, layout);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t reassemble_heads(cudaStream_t st, int elem_bytes, const void* src, void* dst, int n,
                             int B, int Hs, int S, int D, int layout, int sm_count) {
    const int row = D * elem_bytes;
    const bool al16 = ((uintptr_t)src % 16 == 0) && ((uintptr_t)dst % 16 == 0);
    if (row % 16 == 0 && al16) return launch<uint4>(st, src, dst, n, B, Hs, S, row / 16, layout, sm_count);
    if (row % 4 == 0) return launch<uint32_t>(st, src, dst, n, B, Hs, S, row / 4, layout, sm_count);
    return launch<uint16_t>(st, src, dst, n, B, Hs, S, row / 2, layout, sm_count);
}

}  // namespace hx
