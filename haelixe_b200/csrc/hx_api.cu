// C ABI implementation: context, binning arena, transfers and dispatch of
// the attention and RoPE kernels. See include/haelixe_cuda.h for the
// reference interface each entry point replaces.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>

#include <cublas_v2.h>
#include <nvtx3/nvToolsExt.h>

#include "hx_internal.h"

namespace hx {

int set_error(const hx_ctx* ctx, int status, const char* fmt, ...) {
    if (ctx != nullptr) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        std::lock_guard<std::mutex> g(ctx->err_mu);
        const_cast<hx_ctx*>(ctx)->last_error = buf;
    }
    return status;
}

static thread_local uint64_t t_launches = 0;
void note_launch() { ++t_launches; }
uint64_t launches_of_this_thread() { return t_launches; }

int check_cuda(const hx_ctx* ctx, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return HX_OK;
    const int st = (e == cudaErrorMemoryAllocation) ? HX_ERR_OOM : HX_ERR_CUDA;
    return set_error(ctx, st, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

}  // namespace hx

using hx::check_cuda;
using hx::set_error;

namespace {

// An NVTX range named after the public call, so that profiler timelines
// (nsys, ncu's NVTX filters) show the library's calls around their kernels.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
};

// Adds the kernels launched during one public call to the context's count.
struct LaunchCount {
    hx_ctx* c;
    uint64_t t0;
    explicit LaunchCount(hx_ctx* ctx) : c(ctx), t0(hx::launches_of_this_thread()) {}
    ~LaunchCount() { c->kernel_launches += hx::launches_of_this_thread() - t0; }
};

// RAII guard that makes the context's device current for one call and
// restores the caller's device afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        // Always set it: cudaSetDevice also makes the device's primary context
        // current in this thread, which the driver calls made before any
        // runtime call (tensor-map encoding) need; a thread that has only
        // asked for the device (e.g. an autograd worker) may have none yet.
        ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// B, H or S may be 0 (an empty problem: nothing to compute, see empty_shape);
// D must be positive.
int validate_shape(const hx_ctx* ctx, const hx_attn_shape* s, const char* who) {
    if (s == nullptr) return set_error(ctx, HX_ERR_INVALID, "%s: shape is NULL", who);
    if (s->B < 0 || s->H < 0 || s->S < 0 || s->D <= 0)
        return set_error(ctx, HX_ERR_INVALID,
                         "%s: B, H, S must be >= 0 and D positive (got %d,%d,%d,%d)", who, s->B, s->H,
                         s->S, s->D);
    if (s->D > 256)
        return set_error(ctx, HX_ERR_UNSUPPORTED, "%s: head_dim %d > 256 is not supported", who,
                         s->D);
    if (s->B > 65535 || s->H > 65535)
        return set_error(ctx, HX_ERR_UNSUPPORTED, "%s: B and H must be <= 65535", who);
    if (s->stride_s < s->D || s->stride_h < 0 || s->stride_b < 0)
        return set_error(ctx, HX_ERR_INVALID,
                         "%s: strides (b=%lld, h=%lld, s=%lld) overlap rows of length D=%d", who,
                         (long long)s->stride_b, (long long)s->stride_h, (long long)s->stride_s,
                         s->D);
    return HX_OK;
}

// No rows to attend over: every entry point returns HX_OK without touching
// its operands (which may then be NULL), as an empty tensor in gives an
// empty tensor out.
inline bool empty_shape(const hx_attn_shape* s) { return s->B == 0 || s->H == 0 || s->S == 0; }

int validate_dtype(const hx_ctx* ctx, hx_dtype dt, const char* who) {
    if (dt != HX_F32 && dt != HX_BF16)
        return set_error(ctx, HX_ERR_INVALID, "%s: unknown dtype %d", who, (int)dt);
    return HX_OK;
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// The tcgen05 kernels move tiles with TMA: base addresses and every stride
// must be 16-byte multiples.
bool tma_layout_ok(const hx::AttnDims& d, std::initializer_list<const void*> ptrs) {
    const int64_t eb = 2;  // bf16
    if ((d.ss * eb) % 16 || (d.sh * eb) % 16 || (d.sb * eb) % 16) return false;
    for (const void* p : ptrs)
        if (!aligned16(p)) return false;
    return true;
}

uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

uint64_t simt_ws_bytes(const hx::AttnDims& d) {
    return align256((uint64_t)d.B * d.H * d.S * sizeof(float));
}

}  // namespace

extern "C" {

int hx_abi_version(void) { return HX_ABI_VERSION; }

const char* hx_status_string(int status) {
    switch (status) {
        case HX_OK: return "ok";
        case HX_ERR_INVALID: return "invalid argument";
        case HX_ERR_UNSUPPORTED: return "unsupported";
        case HX_ERR_CUDA: return "CUDA error";
        case HX_ERR_OOM: return "out of device memory";
        case HX_ERR_TIMEOUT: return "device wait timed out";
        case HX_ERR_NCCL: return "collective error";
        default: return "unknown status";
    }
}

int hx_ctx_create(int device, hx_ctx** out) {
    if (out == nullptr) return HX_ERR_INVALID;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return HX_ERR_INVALID;
    DeviceGuard g(device);
    if (!g.ok) return HX_ERR_CUDA;
    hx_ctx* c = new hx_ctx();
    c->device = device;
    int st = HX_OK;
    do {
        if ((st = check_cuda(c, cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount,
                                                       device),
                             "cudaDeviceGetAttribute")))
            break;
        if ((st = check_cuda(c, cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking),
                             "cudaStreamCreateWithFlags")))
            break;
        c->stream = c->own_stream;
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        if ((st = check_cuda(c, cudaMemPoolCreate(&c->arena.pool, &props), "cudaMemPoolCreate")))
            break;
        uint64_t threshold = UINT64_MAX;
        if ((st = check_cuda(c, cudaMemPoolSetAttribute(c->arena.pool,
                                                        cudaMemPoolAttrReleaseThreshold, &threshold),
                             "cudaMemPoolSetAttribute")))
            break;
        if ((st = check_cuda(c, cudaMalloc(&c->status, sizeof(hx::DeviceStatus)), "cudaMalloc")))
            break;
        if ((st = check_cuda(c, cudaMemset(c->status, 0, sizeof(hx::DeviceStatus)), "cudaMemset")))
            break;
    } while (0);
    if (st != HX_OK) {
        hx_ctx_destroy(c);
        return st;
    }
    *out = c;
    return HX_OK;
}

int hx_ctx_destroy(hx_ctx* c) {
    if (c == nullptr) return HX_OK;
    DeviceGuard g(c->device);
    if (c->own_stream) cudaStreamSynchronize(c->own_stream);
    if (c->stream != c->own_stream) cudaStreamSynchronize(c->stream);
    if (c->own_stream) {
        std::lock_guard<std::mutex> lk(c->arena.mu);
        for (auto& kv : c->arena.free_list)
            for (void* p : kv.second) cudaFreeAsync(p, c->own_stream);
        for (auto& kv : c->arena.live) cudaFreeAsync(kv.first, c->own_stream);
        c->arena.free_list.clear();
        c->arena.live.clear();
        cudaStreamSynchronize(c->own_stream);
    }
    for (auto& t : c->rope_tables) cudaFree(t.tab);
    c->rope_tables.clear();
    if (c->blas) cublasDestroy((cublasHandle_t)c->blas);
    if (c->arena.pool) cudaMemPoolDestroy(c->arena.pool);
    if (c->status) cudaFree(c->status);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    delete c;
    return HX_OK;
}

int hx_ctx_device(const hx_ctx* c, int* device) {
    if (c == nullptr || device == nullptr) return HX_ERR_INVALID;
    *device = c->device;
    return HX_OK;
}

void* hx_ctx_stream(hx_ctx* c) { return c ? (void*)c->stream : nullptr; }

int hx_ctx_set_stream(hx_ctx* c, void* stream) {
    if (c == nullptr) return HX_ERR_INVALID;
    c->stream = (cudaStream_t)stream;
    return HX_OK;
}

int hx_ctx_use_own_stream(hx_ctx* c) {
    if (c == nullptr) return HX_ERR_INVALID;
    c->stream = c->own_stream;
    return HX_OK;
}

int hx_sync(hx_ctx* c) {
    if (c == nullptr) return HX_ERR_INVALID;
    DeviceGuard g(c->device);
    int st = check_cuda(c, cudaStreamSynchronize(c->stream), "cudaStreamSynchronize");
    if (st != HX_OK) return st;
    hx::DeviceStatus s{};
    st = check_cuda(c, cudaMemcpy(&s, c->status, sizeof(s), cudaMemcpyDeviceToHost), "cudaMemcpy");
    if (st != HX_OK) return st;
    if (s.code != 0) {
        cudaMemset(c->status, 0, sizeof(hx::DeviceStatus));
        return set_error(c, HX_ERR_TIMEOUT,
                         "a device-side bounded wait expired (code %d at site %d, block %d)",
                         s.code, s.where, s.block);
    }
    return HX_OK;
}

int hx_last_error(const hx_ctx* c, char* buf, size_t len) {
    if (c == nullptr || buf == nullptr || len == 0) return HX_ERR_INVALID;
    std::lock_guard<std::mutex> g(c->err_mu);
    snprintf(buf, len, "%s", c->last_error.c_str());
    return HX_OK;
}

// ---- arena ------------------------------------------------------------------

uint64_t hx_bin_size(uint64_t requested) {
    const uint64_t kMin = 512;  // arena.rs:85
    if (requested <= kMin) return kMin;
    uint64_t b = 1;
    while (b < requested) b <<= 1;  // next_power_of_two (arena.rs:89)
    return b;
}

int hx_alloc(hx_ctx* c, uint64_t bytes, void** ptr) {
    if (c == nullptr || ptr == nullptr) return HX_ERR_INVALID;
    *ptr = nullptr;
    const uint64_t bin = hx_bin_size(bytes);
    {
        std::lock_guard<std::mutex> lk(c->arena.mu);
        auto it = c->arena.free_list.find(bin);
        if (it != c->arena.free_list.end() && !it->second.empty()) {
            void* p = it->second.back();
            it->second.pop_back();
            if (it->second.empty()) c->arena.free_list.erase(it);
            c->arena.cached_bytes -= bin;
            c->arena.live[p] = bin;
            c->arena.live_bytes += bin;
            c->arena.hits++;
            *ptr = p;
            return HX_OK;
        }
    }
    // Miss: the mutex is released before the driver call (arena.rs:45-47).
    DeviceGuard g(c->device);
    uint64_t limit, held;
    {
        std::lock_guard<std::mutex> lk(c->arena.mu);
        limit = c->arena.limit;
        held = c->arena.live_bytes + c->arena.cached_bytes;
    }
    if (limit != 0 && held + bin > limit) {
        hx_arena_reset(c);  // parked slabs count against the budget: give them back first
        std::lock_guard<std::mutex> lk(c->arena.mu);
        if (c->arena.live_bytes + bin > limit)
            return set_error(c, HX_ERR_OOM, "hx_alloc: %llu bytes (bin) over the arena limit of %llu (%llu live)",
                             (unsigned long long)bin, (unsigned long long)limit,
                             (unsigned long long)c->arena.live_bytes);
    }
    void* p = nullptr;
    cudaError_t e = cudaMallocFromPoolAsync(&p, bin, c->arena.pool, c->stream);
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        hx_arena_reset(c);  // give parked slabs back, then retry once
        e = cudaMallocFromPoolAsync(&p, bin, c->arena.pool, c->stream);
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return check_cuda(c, e, "cudaMallocFromPoolAsync");
    }
    std::lock_guard<std::mutex> lk(c->arena.mu);
    c->arena.live[p] = bin;
    c->arena.live_bytes += bin;
    c->arena.misses++;
    *ptr = p;
    return HX_OK;
}

int hx_free(hx_ctx* c, void* ptr) {
    if (c == nullptr) return HX_ERR_INVALID;
    if (ptr == nullptr) return HX_OK;
    std::lock_guard<std::mutex> lk(c->arena.mu);
    auto it = c->arena.live.find(ptr);
    if (it == c->arena.live.end())
        return set_error(c, HX_ERR_INVALID, "hx_free: %p was not allocated by this arena", ptr);
    const uint64_t bin = it->second;
    c->arena.live.erase(it);
    c->arena.live_bytes -= bin;
    c->arena.free_list[bin].push_back(ptr);
    c->arena.cached_bytes += bin;
    return HX_OK;
}

int hx_arena_reset(hx_ctx* c) {
    if (c == nullptr) return HX_ERR_INVALID;
    DeviceGuard g(c->device);
    std::lock_guard<std::mutex> lk(c->arena.mu);
    for (auto& kv : c->arena.free_list)
        for (void* p : kv.second) cudaFreeAsync(p, c->stream);
    c->arena.free_list.clear();
    c->arena.cached_bytes = 0;
    return check_cuda(c, cudaGetLastError(), "cudaFreeAsync");
}

int hx_arena_set_limit(hx_ctx* c, uint64_t bytes) {
    if (c == nullptr) return HX_ERR_INVALID;
    std::lock_guard<std::mutex> lk(c->arena.mu);
    c->arena.limit = bytes;
    return HX_OK;
}

int hx_arena_stats_get(const hx_ctx* c, hx_arena_stats* out) {
    if (c == nullptr || out == nullptr) return HX_ERR_INVALID;
    std::lock_guard<std::mutex> lk(const_cast<hx_ctx*>(c)->arena.mu);
    out->live_bytes = c->arena.live_bytes;
    out->cached_bytes = c->arena.cached_bytes;
    uint64_t slabs = 0;
    for (auto& kv : c->arena.free_list) slabs += kv.second.size();
    out->cached_slabs = slabs;
    out->cached_bins = c->arena.free_list.size();
    out->hits = c->arena.hits;
    out->misses = c->arena.misses;
    return HX_OK;
}

// ---- transfers ----------------------------------------------------------------

int hx_copy_h2d_async(hx_ctx* c, void* dst, const void* src, uint64_t bytes) {
    if (c == nullptr || (bytes && (dst == nullptr || src == nullptr))) return HX_ERR_INVALID;
    DeviceGuard g(c->device);
    return check_cuda(c, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream),
                      "cudaMemcpyAsync(H2D)");
}

int hx_copy_d2h_async(hx_ctx* c, void* dst, const void* src, uint64_t bytes) {
    if (c == nullptr || (bytes && (dst == nullptr || src == nullptr))) return HX_ERR_INVALID;
    DeviceGuard g(c->device);
    return check_cuda(c, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream),
                      "cudaMemcpyAsync(D2H)");
}

int hx_copy_h2d(hx_ctx* c, void* dst, const void* src, uint64_t bytes) {
    int st = hx_copy_h2d_async(c, dst, src, bytes);
    if (st != HX_OK) return st;
    return check_cuda(c, cudaStreamSynchronize(c->stream), "cudaStreamSynchronize");
}

int hx_copy_d2h(hx_ctx* c, void* dst, const void* src, uint64_t bytes) {
    int st = hx_copy_d2h_async(c, dst, src, bytes);
    if (st != HX_OK) return st;
    return check_cuda(c, cudaStreamSynchronize(c->stream), "cudaStreamSynchronize");
}

int hx_host_alloc_pinned(uint64_t bytes, void** ptr) {
    if (ptr == nullptr) return HX_ERR_INVALID;
    cudaError_t e = cudaMallocHost(ptr, bytes);
    return e == cudaSuccess ? HX_OK : (e == cudaErrorMemoryAllocation ? HX_ERR_OOM : HX_ERR_CUDA);
}

int hx_host_free_pinned(void* ptr) {
    return cudaFreeHost(ptr) == cudaSuccess ? HX_OK : HX_ERR_CUDA;
}

// ---- attention --------------------------------------------------------------------

int hx_attn_fwd_strided(hx_ctx* c, hx_dtype dt, const hx_attn_shape* shape, const void* q,
                        const void* k, const void* v, void* o, float* lse, float scale,
                        int causal) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, "hx_attn_fwd")) || (st = validate_shape(c, shape, "hx_attn_fwd")))
        return st;
    if (empty_shape(shape)) return HX_OK;
    if (!q || !k || !v || !o) return set_error(c, HX_ERR_INVALID, "hx_attn_fwd: NULL operand");
    if (!isfinite(scale)) return set_error(c, HX_ERR_INVALID, "hx_attn_fwd: scale is not finite");
    DeviceGuard g(c->device);
    NvtxRange nv("hx_attn_fwd_strided");
    LaunchCount lc(c);
    const hx::AttnDims d = hx::dims_of(*shape);
    const bool fast = !c->force_simt && hx::sm100_supported(dt, d) && tma_layout_ok(d, {q, k, v, o});
    // f32 at head_dim 64/128: tcgen05 on f16 hi/lo operand planes (a
    // workspace from the context's arena, released stream-ordered).
    const bool split = !c->force_simt && !fast && hx::split_supported(dt, d);
    // The tcgen05 kernels always write the log-sum-exp: without a caller
    // buffer (no backward follows) they get a temporary one from the arena.
    float* lse_tmp = nullptr;
    if ((fast || split) && lse == nullptr) {
        if ((st = hx_alloc(c, (uint64_t)d.B * d.H * d.S * sizeof(float), (void**)&lse_tmp))) return st;
        lse = lse_tmp;
    }
    cudaError_t e;
    if (fast) {
        e = hx::sm100_attn_fwd(c->stream, c->sm_count, c->status, d, q, k, v, o, lse, scale,
                               causal);
        c->last_path = 2;
    } else if (split) {
        void* ws = nullptr;
        if ((st = hx_alloc(c, hx::split_fwd_workspace_bytes(d), &ws))) {
            if (lse_tmp) hx_free(c, lse_tmp);
            return st;
        }
        e = hx::split_attn_fwd(c->stream, c->sm_count, c->status, d, q, k, v, o, lse, scale, causal, ws);
        hx_free(c, ws);
        c->last_path = 2;
    } else {
        e = hx::simt_attn_fwd(c->stream, dt, d, q, k, v, o, lse, scale, causal);
        c->last_path = 1;
    }
    if (lse_tmp) hx_free(c, lse_tmp);  // stream-ordered: the next user of the slab queues behind us
    return check_cuda(c, e, fast ? "attention forward (tcgen05)"
                                 : split ? "attention forward (tcgen05, split f32)" : "attention forward (SIMT)");
}

int hx_attn_bwd_workspace_size(hx_dtype dt, const hx_attn_shape* shape, uint64_t* bytes) {
    if (shape == nullptr || bytes == nullptr) return HX_ERR_INVALID;
    if (validate_dtype(nullptr, dt, "") || validate_shape(nullptr, shape, "")) return HX_ERR_INVALID;
    if (empty_shape(shape)) {
        *bytes = 0;
        return HX_OK;
    }
    const hx::AttnDims d = hx::dims_of(*shape);
    uint64_t n = simt_ws_bytes(d);
    if (hx::sm100_bwd_supported(dt, d)) n = std::max(n, hx::sm100_bwd_workspace_bytes(d));
    if (hx::split_supported(dt, d)) n = std::max(n, hx::split_bwd_workspace_bytes(d));
    *bytes = n;
    return HX_OK;
}

static int rope_table_for(hx_ctx* c, const hx_attn_shape* shape, float base, float2** out,
                          const char* who);
static int attn_bwd_common(hx_ctx* c, hx_dtype dt, const hx_attn_shape* shape, const void* q,
                           const void* k, const void* v, const void* o, const void* dout,
                           const float* lse, void* dq, void* dk, void* dv, void* workspace,
                           uint64_t workspace_bytes, float scale, int causal, const float* rope_base);

int hx_attn_bwd_strided(hx_ctx* c, hx_dtype dt, const hx_attn_shape* shape, const void* q,
                        const void* k, const void* v, const void* o, const void* dout,
                        const float* lse, void* dq, void* dk, void* dv, void* workspace,
                        uint64_t workspace_bytes, float scale, int causal) {
    return attn_bwd_common(c, dt, shape, q, k, v, o, dout, lse, dq, dk, dv, workspace,
                           workspace_bytes, scale, causal, nullptr);
}

int hx_attn_bwd_rope_strided(hx_ctx* c, hx_dtype dt, const hx_attn_shape* shape, const void* q,
                             const void* k, const void* v, const void* o, const void* dout,
                             const float* lse, void* dq, void* dk, void* dv, void* workspace,
                             uint64_t workspace_bytes, float scale, int causal, float rope_base) {
    return attn_bwd_common(c, dt, shape, q, k, v, o, dout, lse, dq, dk, dv, workspace,
                           workspace_bytes, scale, causal, &rope_base);
}

static int attn_bwd_common(hx_ctx* c, hx_dtype dt, const hx_attn_shape* shape, const void* q,
                           const void* k, const void* v, const void* o, const void* dout,
                           const float* lse, void* dq, void* dk, void* dv, void* workspace,
                           uint64_t workspace_bytes, float scale, int causal, const float* rope_base) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, "hx_attn_bwd")) || (st = validate_shape(c, shape, "hx_attn_bwd")))
        return st;
    if (empty_shape(shape)) return HX_OK;
    float2* tab = nullptr;
    if (rope_base != nullptr) {
        if (shape->D % 2) return set_error(c, HX_ERR_INVALID, "hx_attn_bwd_rope: head_dim must be even");
        if (!isfinite(*rope_base) || *rope_base <= 0.f)
            return set_error(c, HX_ERR_INVALID, "hx_attn_bwd_rope: base must be positive and finite");
    }
    if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv)
        return set_error(c, HX_ERR_INVALID, "hx_attn_bwd: NULL operand");
    if (!isfinite(scale)) return set_error(c, HX_ERR_INVALID, "hx_attn_bwd: scale is not finite");
    DeviceGuard g(c->device);
    NvtxRange nv(rope_base ? "hx_attn_bwd_rope" : "hx_attn_bwd");
    LaunchCount lc(c);
    if (rope_base != nullptr && (st = rope_table_for(c, shape, *rope_base, &tab, "hx_attn_bwd_rope")))
        return st;
    const hx::AttnDims d = hx::dims_of(*shape);
    const bool fast = !c->force_simt && hx::sm100_bwd_supported(dt, d) &&
                      tma_layout_ok(d, {q, k, v, o, dout, dq, dk, dv});
    const bool split = !c->force_simt && !fast && hx::split_supported(dt, d);
    const uint64_t need = fast    ? hx::sm100_bwd_workspace_bytes(d)
                          : split ? hx::split_bwd_workspace_bytes(d)
                                  : simt_ws_bytes(d);
    void* ws = workspace;
    bool owned = false;
    if (ws == nullptr) {
        if ((st = hx_alloc(c, need, &ws))) return st;
        owned = true;
    } else if (workspace_bytes < need) {
        return set_error(c, HX_ERR_INVALID, "hx_attn_bwd: workspace of %llu bytes < %llu needed",
                         (unsigned long long)workspace_bytes, (unsigned long long)need);
    } else if (((uintptr_t)ws & 255u) != 0) {
        return set_error(c, HX_ERR_INVALID, "hx_attn_bwd: workspace must be 256-byte aligned");
    }
    cudaError_t e;
    if (fast) {
        // With a rotary table the kernel's last writes of dK (main kernel) and
        // dQ (post kernel) rotate them back: no extra pass over either.
        e = hx::sm100_attn_bwd(c->stream, c->sm_count, c->status, d, q, k, v, o, dout, lse, dq, dk,
                               dv, ws, scale, causal, tab);
        c->last_path = 2;
    } else if (split) {
        e = hx::split_attn_bwd(c->stream, c->sm_count, c->status, d, q, k, v, o, dout, lse, dq, dk, dv, ws, scale,
                               causal);
        if (e == cudaSuccess && tab != nullptr) {  // dQ and dK rotated back in place after the kernel
            e = hx::rope_apply(c->stream, c->sm_count, dt, d, dq, dq, tab, -1.f);
            if (e == cudaSuccess) e = hx::rope_apply(c->stream, c->sm_count, dt, d, dk, dk, tab, -1.f);
        }
        c->last_path = 2;
    } else {
        e = hx::simt_attn_bwd(c->stream, dt, d, q, k, v, o, dout, lse, dq, dk, dv, (float*)ws,
                              scale, causal);
        if (e == cudaSuccess && tab != nullptr) {  // SIMT path: separate in-place rotations
            e = hx::rope_apply(c->stream, c->sm_count, dt, d, dq, dq, tab, -1.f);
            if (e == cudaSuccess) e = hx::rope_apply(c->stream, c->sm_count, dt, d, dk, dk, tab, -1.f);
        }
        c->last_path = 1;
    }
    st = check_cuda(c, e, fast    ? "attention backward (tcgen05)"
                          : split ? "attention backward (tcgen05, split f32)"
                                  : "attention backward (SIMT)");
    if (owned) hx_free(c, ws);  // stream-ordered: the next user of the slab queues behind us
    return st;
}

static hx_attn_shape contiguous_shape(int bh, int seq_len, int head_dim) {
    hx_attn_shape s;
    s.B = bh;
    s.H = 1;
    s.S = seq_len;
    s.D = head_dim;
    s.stride_s = head_dim;
    s.stride_h = (int64_t)seq_len * head_dim;
    s.stride_b = (int64_t)seq_len * head_dim;
    return s;
}

int hx_flash_attention_fwd(hx_ctx* c, hx_dtype dt, const void* q, const void* k, const void* v,
                           void* o, float* lse, int bh, int seq_len, int head_dim, float scale,
                           int causal) {
    const hx_attn_shape s = contiguous_shape(bh, seq_len, head_dim);
    return hx_attn_fwd_strided(c, dt, &s, q, k, v, o, lse, scale, causal);
}

int hx_flash_attention_bwd(hx_ctx* c, hx_dtype dt, const void* q, const void* k, const void* v,
                           const void* o, const void* dout, const float* lse, void* dq, void* dk,
                           void* dv, void* workspace, uint64_t workspace_bytes, int bh,
                           int seq_len, int head_dim, float scale, int causal) {
    const hx_attn_shape s = contiguous_shape(bh, seq_len, head_dim);
    return hx_attn_bwd_strided(c, dt, &s, q, k, v, o, dout, lse, dq, dk, dv, workspace,
                               workspace_bytes, scale, causal);
}

// ---- RoPE -----------------------------------------------------------------------------

// The (cos, sin) table of (S, D, base), built on first use and cached in the
// context. Caller holds a DeviceGuard.
static int rope_table_for(hx_ctx* c, const hx_attn_shape* shape, float base, float2** out,
                          const char* who) {
    int st;
    uint32_t base_bits;
    memcpy(&base_bits, &base, 4);
    float2* tab = nullptr;
    {
        std::lock_guard<std::mutex> lk(c->rope_mu);
        for (const auto& t : c->rope_tables)
            if (t.S == shape->S && t.D == shape->D && t.base_bits == base_bits) tab = t.tab;
        if (tab == nullptr) {
            // base^(-(2i)/D) in f32, the reference's expression (src/kernels/rope.rs:27-28).
            float inv_freq[128];
            for (int i = 0; i < shape->D / 2; ++i) {
                const float exponent = -((float)(2 * i)) / (float)shape->D;
                inv_freq[i] = powf(base, exponent);
            }
            if ((st = check_cuda(c, cudaMalloc(&tab, sizeof(float2) * (size_t)shape->S * (shape->D / 2)),
                                 "cudaMalloc(rope table)")))
                return st;
            if ((st = check_cuda(c, hx::rope_table(c->stream, shape->S, shape->D, inv_freq, tab), who))) {
                cudaFree(tab);
                return st;
            }
            // One-time: later calls may come on other streams.
            if ((st = check_cuda(c, cudaStreamSynchronize(c->stream), "cudaStreamSynchronize"))) {
                cudaFree(tab);
                return st;
            }
            c->rope_tables.push_back({shape->S, shape->D, base_bits, tab});
        }
    }
    *out = tab;
    return HX_OK;
}

static int rope_common(hx_ctx* c, hx_dtype dt, const hx_attn_shape* shape, const void* x,
                       void* out, float base, float sign, const char* who, const void* x2 = nullptr,
                       void* out2 = nullptr, bool pair = false) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, who)) || (st = validate_shape(c, shape, who))) return st;
    if (empty_shape(shape)) return HX_OK;
    if (!x || !out || (pair && (!x2 || !out2))) return set_error(c, HX_ERR_INVALID, "%s: NULL operand", who);
    if (shape->D % 2) return set_error(c, HX_ERR_INVALID, "%s: head_dim must be even", who);
    if (!isfinite(base) || base <= 0.f)
        return set_error(c, HX_ERR_INVALID, "%s: base must be positive and finite", who);
    DeviceGuard g(c->device);
    NvtxRange nv(who);
    LaunchCount lc(c);
    float2* tab = nullptr;
    if ((st = rope_table_for(c, shape, base, &tab, who))) return st;
    return check_cuda(c, hx::rope_apply(c->stream, c->sm_count, dt, hx::dims_of(*shape), x, out, tab, sign, x2,
                                        out2),
                      who);
}

int hx_rope_fwd_qk(hx_ctx* c, hx_dtype dt, const hx_attn_shape* shape, const void* q, const void* k,
                   void* q_out, void* k_out, float base) {
    return rope_common(c, dt, shape, q, q_out, base, 1.f, "hx_rope_fwd_qk", k, k_out, true);
}

int hx_rope_fwd(hx_ctx* c, hx_dtype dt, const hx_attn_shape* shape, const void* x, void* out,
                float base) {
    return rope_common(c, dt, shape, x, out, base, 1.f, "hx_rope_fwd");
}

int hx_rope_bwd(hx_ctx* c, hx_dtype dt, const hx_attn_shape* shape, const void* g, void* out,
                float base) {
    return rope_common(c, dt, shape, g, out, base, -1.f, "hx_rope_bwd");
}

int hx_reassemble_heads(hx_ctx* c, hx_dtype dt, const void* shards, void* out, int n_shards,
                        int B, int H_shard, int S, int D, int out_layout) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, "hx_reassemble_heads"))) return st;
    if (!shards || !out || n_shards <= 0 || B <= 0 || H_shard <= 0 || S <= 0 || D <= 0 ||
        (out_layout != 0 && out_layout != 1))
        return set_error(c, HX_ERR_INVALID, "hx_reassemble_heads: bad arguments");
    DeviceGuard g(c->device);
    NvtxRange nv("hx_reassemble_heads");
    LaunchCount lc(c);
    return check_cuda(c, hx::reassemble_heads(c->stream, dt == HX_F32 ? 4 : 2, shards, out,
                                              n_shards, B, H_shard, S, D, out_layout,
                                              c->sm_count),
                      "hx_reassemble_heads");
}

uint64_t hx_kernel_launches(const hx_ctx* c) { return c ? c->kernel_launches : 0; }

// ---- the attention block around the kernel: Linear and RMSNorm ------------

static int blas_for(hx_ctx* c, cublasHandle_t* out) {
    std::lock_guard<std::mutex> lk(c->blas_mu);
    if (c->blas == nullptr) {
        cublasHandle_t h;
        if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS)
            return set_error(c, HX_ERR_CUDA, "cublasCreate failed");
        // Default math: bf16 operands run on the tensor cores with f32
        // accumulation; f32 operands stay f32 (TF32 is used only when asked
        // for with CUBLAS_COMPUTE_32F_FAST_TF32 or CUBLAS_TF32_TENSOR_OP_MATH).
        cublasSetMathMode(h, CUBLAS_DEFAULT_MATH);
        c->blas = h;
    }
    *out = (cublasHandle_t)c->blas;
    if (cublasSetStream(*out, c->stream) != CUBLAS_STATUS_SUCCESS)
        return set_error(c, HX_ERR_CUDA, "cublasSetStream failed");
    return HX_OK;
}

// Row-major C[m, n] = op(A) op(B) with A, B, C row-major, expressed as the
// column-major product C^T = op(B)^T op(A)^T that cuBLAS computes.
static int gemm_rm(hx_ctx* c, cublasHandle_t h, hx_dtype dt, bool ta, bool tb, int m, int n, int k,
                   const void* A, int lda, const void* B, int ldb, void* C, int ldc, float beta,
                   const char* who) {
    const cudaDataType_t ty = dt == HX_BF16 ? CUDA_R_16BF : CUDA_R_32F;
    const float alpha = 1.f;
    const cublasStatus_t s = cublasGemmEx(h, tb ? CUBLAS_OP_T : CUBLAS_OP_N, ta ? CUBLAS_OP_T : CUBLAS_OP_N,
                                          n, m, k, &alpha, B, ty, ldb, A, ty, lda, &beta, C, ty, ldc,
                                          CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    if (s != CUBLAS_STATUS_SUCCESS) return set_error(c, HX_ERR_CUDA, "%s: cublasGemmEx status %d", who, (int)s);
    return HX_OK;
}

// The bf16 GEMMs of the Linear layers run on this library's tcgen05 kernel
// when its layout rules hold (16-byte aligned operands and rows); otherwise,
// and for f32 (which the reference computes in f32 and this library keeps off
// TF32), on cuBLAS. *done is set when the tcgen05 kernel took the product.
static int gemm_tc(hx_ctx* c, hx_dtype dt, bool a_mn, bool b_mn, int m, int n, int k, const void* A, int lda,
                   const void* B, int ldb, void* C, int ldc, const void* R, const void* bias, const char* who,
                   bool* done) {
    *done = false;
    if (dt != HX_BF16 || c->gemm_backend == 1 ||
        !hx::gemm_bf16_supported(a_mn, b_mn, m, n, k, A, lda, B, ldb, C, ldc, R, ldc, bias))
        return HX_OK;
    const int st = check_cuda(c, hx::gemm_bf16(c->stream, c->sm_count, c->status, a_mn, b_mn, m, n, k, A, lda, B,
                                               ldb, C, ldc, R, ldc, bias,
                                               c->gemm_backend >= 2 ? c->gemm_backend - 1 : 0),
                              who);
    if (st == HX_OK) {
        *done = true;
        c->last_gemm_path = 2;
    }
    return st;
}

static int linear_args(hx_ctx* c, hx_dtype dt, int rows, int in, int out, const char* who) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, who))) return st;
    if (rows <= 0 || in <= 0 || out <= 0)
        return set_error(c, HX_ERR_INVALID, "%s: rows, in_features, out_features must be positive", who);
    return HX_OK;
}

int hx_linear_fwd(hx_ctx* c, hx_dtype dt, const void* x, const void* w, const void* b, void* y, int rows,
                  int in_features, int out_features) {
    int st;
    if ((st = linear_args(c, dt, rows, in_features, out_features, "hx_linear_fwd"))) return st;
    if (!x || !w || !y) return set_error(c, HX_ERR_INVALID, "hx_linear_fwd: NULL operand");
    DeviceGuard g(c->device);
    NvtxRange nv("hx_linear_fwd");
    LaunchCount lc(c);
    bool done;
    if ((st = gemm_tc(c, dt, false, true, rows, out_features, in_features, x, in_features, w, out_features, y,
                      out_features, nullptr, b, "hx_linear_fwd", &done)) || done)
        return st;
    c->last_gemm_path = 1;
    cublasHandle_t h;
    if ((st = blas_for(c, &h))) return st;
    float beta = 0.f;
    if (b != nullptr) {
        if ((st = check_cuda(c, hx::rows_init(c->stream, c->sm_count, dt, y, nullptr, b, rows, out_features),
                             "bias")))
            return st;
        beta = 1.f;
    }
    // y[rows, out] = x[rows, in] w[in, out] (+ the bias rows)
    return gemm_rm(c, h, dt, false, false, rows, out_features, in_features, x, in_features, w, out_features, y,
                   out_features, beta, "hx_linear_fwd");
}

int hx_linear_bwd(hx_ctx* c, hx_dtype dt, const void* x, const void* w, const void* dy, void* dx, void* dw,
                  void* db, int rows, int in_features, int out_features) {
    int st;
    if ((st = linear_args(c, dt, rows, in_features, out_features, "hx_linear_bwd"))) return st;
    if (!dy || (dx && !w) || (dw && !x)) return set_error(c, HX_ERR_INVALID, "hx_linear_bwd: NULL operand");
    DeviceGuard g(c->device);
    NvtxRange nv("hx_linear_bwd");
    LaunchCount lc(c);
    cublasHandle_t h = nullptr;
    bool done = false;
    if (dx != nullptr) {  // dx[rows, in] = dy[rows, out] w[in, out]^T
        if ((st = gemm_tc(c, dt, false, false, rows, in_features, out_features, dy, out_features, w, out_features,
                          dx, in_features, nullptr, nullptr, "hx_linear_bwd dx", &done)))
            return st;
        if (!done) {
            c->last_gemm_path = 1;
            if ((st = blas_for(c, &h)) ||
                (st = gemm_rm(c, h, dt, false, true, rows, in_features, out_features, dy, out_features, w,
                              out_features, dx, in_features, 0.f, "hx_linear_bwd dx")))
                return st;
        }
    }
    if (dw != nullptr) {  // dw[in, out] = x[rows, in]^T dy[rows, out]
        if ((st = gemm_tc(c, dt, true, true, in_features, out_features, rows, x, in_features, dy, out_features,
                          dw, out_features, nullptr, nullptr, "hx_linear_bwd dw", &done)))
            return st;
        if (!done) {
            c->last_gemm_path = 1;
            if ((!h && (st = blas_for(c, &h))) ||
                (st = gemm_rm(c, h, dt, true, false, in_features, out_features, rows, x, in_features, dy,
                              out_features, dw, out_features, 0.f, "hx_linear_bwd dw")))
                return st;
        }
    }
    if (db != nullptr) {  // db[out] = sum over rows of dy
        void* scratch = nullptr;
        if ((st = hx_alloc(c, sizeof(float) * (uint64_t)hx::col_scratch_floats(rows, out_features), &scratch)))
            return st;
        st = check_cuda(c, hx::col_sum(c->stream, dt, dy, db, (float*)scratch, rows, out_features), "bias grad");
        hx_free(c, scratch);
    }
    return st;
}

int hx_rmsnorm_fwd(hx_ctx* c, hx_dtype dt, const void* x, const void* w, void* y, int rows, int hidden,
                   float eps) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, "hx_rmsnorm_fwd"))) return st;
    if (!x || !w || !y) return set_error(c, HX_ERR_INVALID, "hx_rmsnorm_fwd: NULL operand");
    if (rows <= 0 || hidden <= 0 || !(eps >= 0.f))
        return set_error(c, HX_ERR_INVALID, "hx_rmsnorm_fwd: rows, hidden must be positive, eps >= 0");
    DeviceGuard g(c->device);
    NvtxRange nv("hx_rmsnorm_fwd");
    LaunchCount lc(c);
    return check_cuda(c, hx::rmsnorm_fwd(c->stream, c->sm_count, dt, x, w, y, rows, hidden, eps), "hx_rmsnorm_fwd");
}

int hx_rmsnorm_bwd(hx_ctx* c, hx_dtype dt, const void* dy, const void* x, const void* w, void* dx, float* dw,
                   int rows, int hidden, float eps) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, "hx_rmsnorm_bwd"))) return st;
    if (!dy || !x || !w || !dx || !dw) return set_error(c, HX_ERR_INVALID, "hx_rmsnorm_bwd: NULL operand");
    if (rows <= 0 || hidden <= 0 || !(eps >= 0.f))
        return set_error(c, HX_ERR_INVALID, "hx_rmsnorm_bwd: rows, hidden must be positive, eps >= 0");
    DeviceGuard g(c->device);
    NvtxRange nv("hx_rmsnorm_bwd");
    LaunchCount lc(c);
    void* scratch = nullptr;
    if ((st = hx_alloc(c, sizeof(float) * (uint64_t)hx::rmsnorm_bwd_scratch_floats(rows, hidden), &scratch)))
        return st;
    st = check_cuda(c, hx::rmsnorm_bwd(c->stream, c->sm_count, dt, dy, x, w, dx, dw, (float*)scratch, rows, hidden,
                                       eps),
                    "hx_rmsnorm_bwd");
    hx_free(c, scratch);
    return st;
}

int hx_gelu_fwd(hx_ctx* c, hx_dtype dt, const void* x, void* y, uint64_t n) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, "hx_gelu_fwd"))) return st;
    if (!x || !y) return set_error(c, HX_ERR_INVALID, "hx_gelu_fwd: NULL operand");
    if (n == 0) return HX_OK;
    DeviceGuard g(c->device);
    NvtxRange nv("hx_gelu_fwd");
    LaunchCount lc(c);
    return check_cuda(c, hx::gelu_fwd(c->stream, c->sm_count, dt, x, y, (int64_t)n), "hx_gelu_fwd");
}

int hx_add(hx_ctx* c, hx_dtype dt, const void* a, const void* b, void* out, uint64_t n) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, "hx_add"))) return st;
    if (!a || !b || !out) return set_error(c, HX_ERR_INVALID, "hx_add: NULL operand");
    if (n == 0) return HX_OK;
    DeviceGuard g(c->device);
    NvtxRange nv("hx_add");
    LaunchCount lc(c);
    return check_cuda(c, hx::add(c->stream, c->sm_count, dt, a, b, out, (int64_t)n), "hx_add");
}

int hx_gelu_bwd(hx_ctx* c, hx_dtype dt, const void* dy, const void* x, void* dx, uint64_t n) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, "hx_gelu_bwd"))) return st;
    if (!dy || !x || !dx) return set_error(c, HX_ERR_INVALID, "hx_gelu_bwd: NULL operand");
    if (n == 0) return HX_OK;
    DeviceGuard g(c->device);
    NvtxRange nv("hx_gelu_bwd");
    LaunchCount lc(c);
    return check_cuda(c, hx::gelu_bwd(c->stream, c->sm_count, dt, dy, x, dx, (int64_t)n), "hx_gelu_bwd");
}

// ---- the training step around the block stack ------------------------------

int hx_linear_residual_fwd(hx_ctx* c, hx_dtype dt, const void* x, const void* w, const void* b,
                           const void* residual, void* y, int rows, int in_features, int out_features) {
    int st;
    if ((st = linear_args(c, dt, rows, in_features, out_features, "hx_linear_residual_fwd"))) return st;
    if (!x || !w || !y) return set_error(c, HX_ERR_INVALID, "hx_linear_residual_fwd: NULL operand");
    DeviceGuard g(c->device);
    NvtxRange nv("hx_linear_residual_fwd");
    LaunchCount lc(c);
    bool done;
    if ((st = gemm_tc(c, dt, false, true, rows, out_features, in_features, x, in_features, w, out_features, y,
                      out_features, residual, b, "hx_linear_residual_fwd", &done)) || done)
        return st;
    c->last_gemm_path = 1;
    cublasHandle_t h;
    if ((st = blas_for(c, &h))) return st;
    float beta = 0.f;
    if (b != nullptr || residual != nullptr) {
        if ((st = check_cuda(c, hx::rows_init(c->stream, c->sm_count, dt, y, residual, b, rows, out_features),
                             "residual rows")))
            return st;
        beta = 1.f;
    }
    return gemm_rm(c, h, dt, false, false, rows, out_features, in_features, x, in_features, w, out_features, y,
                   out_features, beta, "hx_linear_residual_fwd");
}

int hx_cross_entropy(hx_ctx* c, hx_dtype dt, const void* logits, const uint32_t* targets, float* loss,
                     void* dlogits, int rows, int classes) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, "hx_cross_entropy"))) return st;
    if (!logits || !targets || !loss) return set_error(c, HX_ERR_INVALID, "hx_cross_entropy: NULL operand");
    if (rows <= 0 || classes <= 0)
        return set_error(c, HX_ERR_INVALID, "hx_cross_entropy: rows and classes must be positive");
    DeviceGuard g(c->device);
    NvtxRange nv("hx_cross_entropy");
    LaunchCount lc(c);
    void* row_loss = nullptr;
    if ((st = hx_alloc(c, sizeof(float) * (uint64_t)rows, &row_loss))) return st;
    st = check_cuda(c, hx::cross_entropy(c->stream, dt, logits, targets, (float*)row_loss, loss, dlogits, rows,
                                         classes),
                    "hx_cross_entropy");
    hx_free(c, row_loss);
    return st;
}

// f32 a^n by binary exponentiation with one rounding per product: the
// evaluation of Rust's f32::powi for a run-time exponent (the llvm.powi
// intrinsic's square-and-multiply routine). n >= 0 here.
static float powi_f32(float a, int n) {
    float r = 1.0f;
    for (;;) {
        if (n & 1) r *= a;
        n /= 2;
        if (n == 0) break;
        a *= a;
    }
    return r;
}

int hx_adamw_step(hx_ctx* c, const hx_adamw_tensor* tensors, int count, float lr, float beta1, float beta2,
                  float eps, float weight_decay, int step) {
    if (c == nullptr) return HX_ERR_INVALID;
    if (count < 0 || (count > 0 && tensors == nullptr) || step < 1)
        return set_error(c, HX_ERR_INVALID, "hx_adamw_step: bad tensor list or step < 1");
    for (int i = 0; i < count; ++i) {
        const hx_adamw_tensor& t = tensors[i];
        if (t.n == 0) continue;
        if (!t.param || !t.grad || !t.m || !t.v || (t.grad_dtype != HX_F32 && t.grad_dtype != HX_BF16))
            return set_error(c, HX_ERR_INVALID, "hx_adamw_step: tensor %d has a NULL pointer or bad dtype", i);
    }
    if (count == 0) return HX_OK;
    DeviceGuard g(c->device);
    NvtxRange nv("hx_adamw_step");
    LaunchCount lc(c);
    const float bc1 = 1.0f - powi_f32(beta1, step);
    const float bc2 = 1.0f - powi_f32(beta2, step);
    return check_cuda(c, hx::adamw_step(c->stream, c->sm_count, tensors, count, lr, beta1, beta2, eps,
                                        weight_decay, bc1, bc2),
                      "hx_adamw_step");
}

static int embedding_args(hx_ctx* c, hx_dtype dt, const void* a, const uint32_t* ids, const void* b, int vocab,
                          int dim, const char* who) {
    if (c == nullptr) return HX_ERR_INVALID;
    int st;
    if ((st = validate_dtype(c, dt, who))) return st;
    if (!a || !ids || !b) return set_error(c, HX_ERR_INVALID, "%s: NULL operand", who);
    if (vocab <= 0 || dim <= 0) return set_error(c, HX_ERR_INVALID, "%s: vocab and dim must be positive", who);
    return HX_OK;
}

int hx_embedding_fwd(hx_ctx* c, hx_dtype dt, const void* table, const uint32_t* ids, void* out, uint64_t tokens,
                     int vocab, int dim) {
    int st;
    if ((st = embedding_args(c, dt, table, ids, out, vocab, dim, "hx_embedding_fwd"))) return st;
    if (tokens == 0) return HX_OK;
    DeviceGuard g(c->device);
    NvtxRange nv("hx_embedding_fwd");
    LaunchCount lc(c);
    return check_cuda(c, hx::embedding_fwd(c->stream, c->sm_count, dt, table, ids, out, (int64_t)tokens, vocab, dim),
                      "hx_embedding_fwd");
}

int hx_embedding_bwd(hx_ctx* c, hx_dtype dt, const void* dout, const uint32_t* ids, float* dtable, uint64_t tokens,
                     int vocab, int dim) {
    int st;
    if ((st = embedding_args(c, dt, dout, ids, dtable, vocab, dim, "hx_embedding_bwd"))) return st;
    if (tokens == 0) return HX_OK;
    DeviceGuard g(c->device);
    NvtxRange nv("hx_embedding_bwd");
    LaunchCount lc(c);
    return check_cuda(c, hx::embedding_bwd(c->stream, c->sm_count, dt, dout, ids, dtable, (int64_t)tokens, vocab,
                                           dim),
                      "hx_embedding_bwd");
}

int hx_last_path(const hx_ctx* c) { return c ? c->last_path : 0; }

int hx_selftest_wait_timeout(hx_ctx* c) {
    if (c == nullptr) return HX_ERR_INVALID;
    DeviceGuard g(c->device);
    NvtxRange nv("hx_selftest_wait_timeout");
    LaunchCount lc(c);
    return check_cuda(c, hx::selftest_wait_timeout(c->stream, c->status), "hx_selftest_wait_timeout");
}

int hx_last_gemm_path(const hx_ctx* c) { return c ? c->last_gemm_path : 0; }

int hx_set_gemm_backend(hx_ctx* c, int backend) {
    if (c == nullptr || backend < 0 || backend > 4) return HX_ERR_INVALID;
    c->gemm_backend = backend;
    return HX_OK;
}

int hx_set_force_simt(hx_ctx* c, int force) {
    if (c == nullptr) return HX_ERR_INVALID;
    c->force_simt = force ? 1 : 0;
    return HX_OK;
}

}  // extern "C"
