// Attention backward that allocates nothing.
//
// hx_flash_attention_bwd needs a workspace (the f32 dQ accumulator and the
// per-row delta) and, when the caller passes none, takes it from the
// context's arena, which may call cudaMallocAsync. Some callers cannot let a
// library allocate: runtimes that hand all device memory to their own pool at
// start-up (serving engines commonly reserve most of HBM before the first
// request), latency-critical loops that cannot risk the device-wide
// synchronisation cudaMalloc/cudaFree may cause, and plugin hosts whose
// operator callbacks must not allocate. For them this file provides
// hx_flash_attention_bwd_noalloc, which runs the same tcgen05 backward
// kernels with the workspace placed in a fixed device array compiled into
// the library.
//
// Properties a user must know:
//   * The array holds kNoAllocScratchBytes (64 MiB). Every GPU that loads this
//     library keeps that much device memory until the process exits, whether
//     or not the entry point is used.
//   * A problem whose workspace exceeds the array is rejected with
//     HX_ERR_INVALID before any GPU work; use hx_flash_attention_bwd instead.
//   * All calls on a device share the one array and it keeps whatever the
//     last call left in it. The kernels rewrite every byte they read (the
//     delta rows and the zeroed dQ accumulator) at the start of each call,
//     so stale contents never leak into a result; but two calls whose
//     kernels overlap on the GPU (different streams, or different host
//     threads) race on the array and corrupt each other. Serialize them.
//   * The first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and keeps it for the
//     life of the process. Make that first call before any stream capture
//     begins, and do not use the entry point after cudaDeviceReset (or any
//     other teardown of the device's primary context): the kept address
//     belonged to the destroyed context.
//   * It always runs the tcgen05 kernels: a context forced onto the SIMT
//     path (hx_set_force_simt) gets HX_ERR_UNSUPPORTED.
#include <mutex>

#include "hx_internal.h"

namespace hx {
namespace {

constexpr uint64_t kNoAllocScratchBytes = 64ull << 20;
constexpr int kMaxDevices = 64;

// Host code must never use this name as a pointer: on the host it is only a
// stand-in for the symbol. Its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Once per device, with that device current: resolve the array's address.
cudaError_t scratch_for_device(int device, void** out) {
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (g_scratch_ptr[device] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[device] = p;
    }
    *out = g_scratch_ptr[device];
    return cudaSuccess;
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace
}  // namespace hx

extern "C" int hx_flash_attention_bwd_noalloc(hx_ctx* c, hx_dtype dt, const void* q,
                                              const void* k, const void* v, const void* o,
                                              const void* dout, const float* lse, void* dq,
                                              void* dk, void* dv, int bh, int seq_len,
                                              int head_dim, float scale, int causal) {
    using namespace hx;
    if (c == nullptr) return HX_ERR_INVALID;
    const char* who = "hx_flash_attention_bwd_noalloc";
    if (dt != HX_BF16 || (head_dim != 64 && head_dim != 128))
        return set_error(c, HX_ERR_UNSUPPORTED,
                         "%s: only bf16 with head_dim 64 or 128 (the tcgen05 kernels) is supported",
                         who);
    if (bh < 0 || seq_len < 0 || bh > 65535)
        return set_error(c, HX_ERR_INVALID, "%s: bad shape bh=%d seq_len=%d", who, bh, seq_len);
    if (bh == 0 || seq_len == 0) return HX_OK;  // empty problem
    if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv)
        return set_error(c, HX_ERR_INVALID, "%s: NULL operand", who);
    if (!isfinite(scale)) return set_error(c, HX_ERR_INVALID, "%s: scale is not finite", who);
    if (c->force_simt)
        return set_error(c, HX_ERR_UNSUPPORTED,
                         "%s: the context is forced onto the SIMT path; this entry point runs "
                         "only the tcgen05 kernels",
                         who);
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(dout) ||
        !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
        return set_error(c, HX_ERR_INVALID, "%s: operands must be 16-byte aligned", who);
    AttnDims d{bh, 1, seq_len, head_dim, (int64_t)seq_len * head_dim,
               (int64_t)seq_len * head_dim, (int64_t)head_dim};
    const uint64_t need = sm100_bwd_workspace_bytes(d);
    if (need > kNoAllocScratchBytes)
        return set_error(c, HX_ERR_INVALID,
                         "%s: this problem needs %llu bytes of workspace but the fixed scratch "
                         "holds %llu (64 MiB); call hx_flash_attention_bwd instead",
                         who, (unsigned long long)need, (unsigned long long)kNoAllocScratchBytes);
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != c->device && cudaSetDevice(c->device) != cudaSuccess)
        return set_error(c, HX_ERR_CUDA, "%s: cannot make device %d current", who, c->device);
    void* scratch = nullptr;
    int st = check_cuda(c, scratch_for_device(c->device, &scratch), "cudaGetSymbolAddress");
    if (st == HX_OK) {
        const uint64_t t0 = launches_of_this_thread();
        st = check_cuda(c,
                        sm100_attn_bwd(c->stream, c->sm_count, c->status, d, q, k, v, o, dout,
                                       lse, dq, dk, dv, scratch, scale, causal),
                        "attention backward (tcgen05, fixed scratch)");
        c->kernel_launches += launches_of_this_thread() - t0;
        c->last_path = 2;
    }
    if (prev >= 0 && prev != c->device) cudaSetDevice(prev);
    return st;
}
