// Head-sharded attention's one exchange, behind the C ABI: an NCCL
// all-gather of every rank's output heads followed by the reassembly into the
// merged [B, S, H, D] layout that MultiHeadAttention::forward builds after the
// attention (src/nn/attention.rs:91-94: transpose(1, 2) then view to
// [B, S, H*D]). Heads are independent, so this is the only data exchange of a
// sharded step; dQ, dK and dV stay on their ranks.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2): the library needs NCCL
// only when a group is created, and a process that already loaded NCCL (for
// example through torch) shares that copy. Communicators are created
// non-blocking, so every NCCL call that could wait on a peer (initialisation,
// enqueueing a collective, completion) is polled against a deadline; on expiry
// the communicator is aborted (ncclCommAbort makes its kernels return) and the
// call returns HX_ERR_NCCL instead of hanging on a rank that never joins or
// has left.
#include <dlfcn.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "hx_internal.h"

namespace hx {
namespace {

// SMs' worth of blocks the reassembly kernel may use (0 = the whole GPU). It
// runs beside the backward, whose CTAs it displaces when they retire.
#ifndef HX_EXCHANGE_MERGE_SMS
#define HX_EXCHANGE_MERGE_SMS 0
#endif

// NCCL_CTA_POLICY_ZERO of NCCL 2.28 (collectives on copy engines where the
// buffers allow it); the header this file builds against may predate it.
constexpr int kCtaPolicyZero = 0x02;

struct NcclApi {
    void* so = nullptr;
    int version = 0;
    ncclResult_t (*GetVersion)(int*) = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*MemAlloc)(void**, size_t) = nullptr;
    ncclResult_t (*MemFree)(void*) = nullptr;
    ncclResult_t (*CommRegister)(ncclComm_t, void*, size_t, void**) = nullptr;
    ncclResult_t (*CommDeregister)(ncclComm_t, void*) = nullptr;
    ncclResult_t (*CommWindowRegister)(ncclComm_t, void*, size_t, ncclWindow_t*, int) = nullptr;
    ncclResult_t (*CommWindowDeregister)(ncclComm_t, ncclWindow_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    const char* (*GetLastError)(ncclComm_t) = nullptr;
};

std::once_flag g_nccl_once;
NcclApi g_nccl;
std::string g_nccl_err;

void load_nccl() {
    const char* names[] = {"libnccl.so.2", "libnccl.so"};
    for (const char* n : names) {
        g_nccl.so = dlopen(n, RTLD_NOW | RTLD_LOCAL);
        if (g_nccl.so) break;
    }
    if (!g_nccl.so) {
        const char* e = dlerror();
        g_nccl_err = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown error");
        return;
    }
    bool ok = true;
    auto sym = [&](auto& fn, const char* name, bool required) {
        fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(g_nccl.so, name));
        if (!fn && required) {
            ok = false;
            g_nccl_err = std::string("libnccl.so.2 lacks ") + name;
        }
    };
    sym(g_nccl.GetVersion, "ncclGetVersion", true);
    sym(g_nccl.GetUniqueId, "ncclGetUniqueId", true);
    sym(g_nccl.CommInitRankConfig, "ncclCommInitRankConfig", true);
    sym(g_nccl.CommGetAsyncError, "ncclCommGetAsyncError", true);
    sym(g_nccl.CommAbort, "ncclCommAbort", true);
    sym(g_nccl.CommDestroy, "ncclCommDestroy", true);
    sym(g_nccl.CommFinalize, "ncclCommFinalize", true);
    sym(g_nccl.AllGather, "ncclAllGather", true);
    sym(g_nccl.GroupStart, "ncclGroupStart", true);
    sym(g_nccl.GroupEnd, "ncclGroupEnd", true);
    sym(g_nccl.MemAlloc, "ncclMemAlloc", true);
    sym(g_nccl.MemFree, "ncclMemFree", true);
    sym(g_nccl.CommRegister, "ncclCommRegister", true);
    sym(g_nccl.CommDeregister, "ncclCommDeregister", true);
    sym(g_nccl.CommWindowRegister, "ncclCommWindowRegister", false);
    sym(g_nccl.CommWindowDeregister, "ncclCommWindowDeregister", false);
    sym(g_nccl.GetErrorString, "ncclGetErrorString", true);
    sym(g_nccl.GetLastError, "ncclGetLastError", false);
    if (ok && g_nccl.GetVersion(&g_nccl.version) != ncclSuccess) {
        ok = false;
        g_nccl_err = "ncclGetVersion failed";
    }
    if (!ok) {
        dlclose(g_nccl.so);
        g_nccl.so = nullptr;
    }
}

const NcclApi* nccl() {
    std::call_once(g_nccl_once, load_nccl);
    return g_nccl.so ? &g_nccl : nullptr;
}

using Clock = std::chrono::steady_clock;

}  // namespace
}  // namespace hx

// One rank of the communicator held by this process: its device, its
// communicator, the side stream the exchange runs on, and the gather buffer.
struct hx_group_member {
    int device = -1;
    int rank = -1;
    ncclComm_t comm = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ready = nullptr;  // recorded on the caller's stream: inputs are written
    cudaEvent_t done = nullptr;   // recorded on the side stream: gather + reassembly finished
    void* buf = nullptr;          // nranks packed slots of slot_bytes (ncclMemAlloc)
    uint64_t slot_bytes = 0;      // one rank's shard: the all-gather's chunk
    void* reg = nullptr;          // ncclCommRegister handle
    ncclWindow_t win = nullptr;   // ncclCommWindowRegister handle
    bool pending = false;         // a gather was enqueued since the last hx_group_sync
};

struct hx_group {
    int nranks = 0;
    int flags = 0;
    int timeout_ms = 0;
    bool aborted = false;
    std::mutex abort_mu;  // members driven from several threads may give up at once
    std::vector<hx_group_member> m;
    mutable std::mutex err_mu;
    std::string last_error;
};

namespace hx {
namespace {

int gfail(hx_group* g, int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (g) {
        std::lock_guard<std::mutex> lk(g->err_mu);
        g->last_error = buf;
    }
    return status;
}

const char* nstr(ncclResult_t r) {
    const NcclApi* a = nccl();
    return a ? a->GetErrorString(r) : "NCCL not loaded";
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        cudaSetDevice(dev);  // also makes the primary context current in this thread
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Aborts every communicator of the group (their kernels return, their
// resources are released) after a failure or a missed deadline.
void abort_all(hx_group* g) {
    const NcclApi* a = nccl();
    std::lock_guard<std::mutex> lk(g->abort_mu);
    if (!a || g->aborted) return;
    for (auto& m : g->m) {
        if (m.comm) {
            DeviceGuard dg(m.device);
            a->CommAbort(m.comm);
            m.comm = nullptr;
        }
        m.reg = nullptr;
        m.win = nullptr;
    }
    g->aborted = true;
}

// Polls a non-blocking communicator until its last call has left the
// in-progress state, or the deadline passes (then the group is aborted).
int settle(hx_group* g, hx_group_member& m, const char* what, Clock::time_point deadline) {
    const NcclApi* a = nccl();
    for (;;) {
        ncclResult_t st = ncclInProgress;
        const ncclResult_t r = a->CommGetAsyncError(m.comm, &st);
        if (r != ncclSuccess) {
            abort_all(g);
            return gfail(g, HX_ERR_NCCL, "%s (rank %d): ncclCommGetAsyncError: %s", what, m.rank, nstr(r));
        }
        if (st == ncclSuccess) return HX_OK;
        if (st != ncclInProgress) {
            const char* detail = a->GetLastError ? a->GetLastError(m.comm) : "";
            abort_all(g);
            return gfail(g, HX_ERR_NCCL, "%s (rank %d): %s %s; communicator aborted", what, m.rank, nstr(st),
                         detail ? detail : "");
        }
        if (Clock::now() > deadline) {
            abort_all(g);
            return gfail(g, HX_ERR_NCCL, "%s (rank %d): no progress within %d ms (a peer did not join or has "
                         "left); communicator aborted", what, m.rank, g->timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

Clock::time_point deadline_of(const hx_group* g) {
    return Clock::now() + std::chrono::milliseconds(g->timeout_ms);
}

int setup_member(hx_group* g, hx_group_member& m) {
    DeviceGuard dg(m.device);
    int least = 0, greatest = 0;
    cudaDeviceGetStreamPriorityRange(&least, &greatest);
    if (cudaStreamCreateWithPriority(&m.stream, cudaStreamNonBlocking, least) != cudaSuccess ||
        cudaEventCreateWithFlags(&m.ready, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&m.done, cudaEventDisableTiming) != cudaSuccess)
        return gfail(g, HX_ERR_CUDA, "device %d: cannot create the exchange stream or events", m.device);
    return HX_OK;
}

ncclConfig_t config_of(int flags) {
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    if (flags & HX_GROUP_COPY_ENGINE) cfg.CTAPolicy = kCtaPolicyZero;
    return cfg;
}

int check_flags(int flags) {
    const int known = HX_GROUP_REGISTER | HX_GROUP_SYMMETRIC | HX_GROUP_COPY_ENGINE;
    return (flags & ~known) ? HX_ERR_INVALID : HX_OK;
}

// Waits for the member's side stream, but never for longer than the group's
// timeout: a gather whose peer never came is aborted first (its kernel then
// returns), so tearing a group down cannot hang.
void drain_member(hx_group* g, hx_group_member& m) {
    if (!m.stream) return;
    const auto dl = deadline_of(g);
    while (cudaStreamQuery(m.stream) == cudaErrorNotReady) {
        if (Clock::now() > dl) {
            abort_all(g);
            break;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
    cudaStreamSynchronize(m.stream);
}

void release_member(const NcclApi* a, hx_group* g, hx_group_member& m) {
    DeviceGuard dg(m.device >= 0 ? m.device : 0);
    drain_member(g, m);
    if (a && m.comm && !g->aborted) {
        if (m.win && a->CommWindowDeregister) a->CommWindowDeregister(m.comm, m.win);
        if (m.reg) a->CommDeregister(m.comm, m.reg);
    }
    if (a && m.buf) a->MemFree(m.buf);
    if (a && m.comm) a->CommDestroy(m.comm);
    if (m.ready) cudaEventDestroy(m.ready);
    if (m.done) cudaEventDestroy(m.done);
    if (m.stream) cudaStreamDestroy(m.stream);
    m = hx_group_member{};
}

// Makes the member's gather buffer hold nranks packed slots of exactly `slot`
// bytes (NCCL places rank r's chunk at r * chunk bytes). The
// registration calls are collective over the communicator when the group was
// made with HX_GROUP_SYMMETRIC, so every rank must reach this with the same
// size (it does: every rank gathers the same shard shape).
int ensure_buffer(hx_group* g, hx_group_member& m, uint64_t slot) {
    if (m.buf && m.slot_bytes == slot) return HX_OK;
    const NcclApi* a = nccl();
    DeviceGuard dg(m.device);
    if (m.buf) {
        drain_member(g, m);
        if (g->aborted) return gfail(g, HX_ERR_NCCL, "the group was aborted");
        if (m.win && a->CommWindowDeregister) a->CommWindowDeregister(m.comm, m.win);
        if (m.reg) a->CommDeregister(m.comm, m.reg);
        a->MemFree(m.buf);
        m.buf = nullptr;
        m.reg = nullptr;
        m.win = nullptr;
        m.slot_bytes = 0;
    }
    // The allocation is rounded up to whole 4 KiB pages (window registration).
    const uint64_t bytes = (slot * (uint64_t)g->nranks + 4095) & ~uint64_t(4095);
    ncclResult_t r = a->MemAlloc(&m.buf, bytes);
    if (r != ncclSuccess)
        return gfail(g, HX_ERR_OOM, "ncclMemAlloc of %llu bytes on device %d: %s", (unsigned long long)bytes,
                     m.device, nstr(r));
    m.slot_bytes = slot;
    if (g->flags & HX_GROUP_SYMMETRIC) {
        if (!a->CommWindowRegister)
            return gfail(g, HX_ERR_UNSUPPORTED, "HX_GROUP_SYMMETRIC needs NCCL >= 2.27 (loaded %d)", a->version);
        r = a->CommWindowRegister(m.comm, m.buf, bytes, &m.win, NCCL_WIN_COLL_SYMMETRIC);
        if (r != ncclSuccess && r != ncclInProgress)
            return gfail(g, HX_ERR_NCCL, "ncclCommWindowRegister: %s", nstr(r));
        if (int st = settle(g, m, "ncclCommWindowRegister", deadline_of(g))) return st;
    } else if (g->flags & HX_GROUP_REGISTER) {
        r = a->CommRegister(m.comm, m.buf, bytes, &m.reg);
        if (r != ncclSuccess && r != ncclInProgress) return gfail(g, HX_ERR_NCCL, "ncclCommRegister: %s", nstr(r));
        if (int st = settle(g, m, "ncclCommRegister", deadline_of(g))) return st;
    }
    return HX_OK;
}

hx_group_member* member_of(hx_group* g, int member) {
    if (!g || member < 0 || member >= (int)g->m.size()) return nullptr;
    return &g->m[member];
}

}  // namespace
}  // namespace hx

extern "C" {

int hx_group_unique_id(void* id) {
    using namespace hx;
    if (!id) return HX_ERR_INVALID;
    const NcclApi* a = nccl();
    if (!a) return HX_ERR_UNSUPPORTED;
    ncclUniqueId u;
    if (a->GetUniqueId(&u) != ncclSuccess) return HX_ERR_NCCL;
    memcpy(id, u.internal, HX_GROUP_ID_BYTES);
    return HX_OK;
}

int hx_group_create_rank(int device, int nranks, int rank, const void* id, int flags, int timeout_ms,
                         hx_group** out) {
    using namespace hx;
    if (!out) return HX_ERR_INVALID;
    *out = nullptr;
    if (!id || nranks < 1 || rank < 0 || rank >= nranks || device < 0 || timeout_ms <= 0 || check_flags(flags))
        return HX_ERR_INVALID;
    const NcclApi* a = nccl();
    if (!a) return HX_ERR_UNSUPPORTED;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device >= ndev) return HX_ERR_INVALID;
    hx_group* g = new hx_group();
    g->nranks = nranks;
    g->flags = flags;
    g->timeout_ms = timeout_ms;
    g->m.resize(1);
    hx_group_member& m = g->m[0];
    m.device = device;
    m.rank = rank;
    int st = setup_member(g, m);
    if (st == HX_OK) {
        DeviceGuard dg(device);
        ncclUniqueId u;
        memcpy(u.internal, id, HX_GROUP_ID_BYTES);
        ncclConfig_t cfg = config_of(flags);
        const ncclResult_t r = a->CommInitRankConfig(&m.comm, nranks, u, rank, &cfg);
        if (r != ncclSuccess && r != ncclInProgress) {
            st = gfail(g, HX_ERR_NCCL, "ncclCommInitRankConfig: %s", nstr(r));
            if (m.comm) a->CommAbort(m.comm);
            m.comm = nullptr;
        } else {
            st = settle(g, m, "communicator initialisation", deadline_of(g));
        }
    }
    *out = g;  // returned even on failure, so hx_group_last_error can explain it
    return st;
}

int hx_group_create(int n, const int* devices, int flags, int timeout_ms, hx_group** out) {
    using namespace hx;
    if (!out) return HX_ERR_INVALID;
    *out = nullptr;
    if (n < 1 || !devices || timeout_ms <= 0 || check_flags(flags)) return HX_ERR_INVALID;
    const NcclApi* a = nccl();
    if (!a) return HX_ERR_UNSUPPORTED;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess) return HX_ERR_CUDA;
    for (int i = 0; i < n; ++i) {
        if (devices[i] < 0 || devices[i] >= ndev) return HX_ERR_INVALID;
        for (int j = 0; j < i; ++j)
            if (devices[j] == devices[i]) return HX_ERR_INVALID;  // one rank per GPU
    }
    hx_group* g = new hx_group();
    g->nranks = n;
    g->flags = flags;
    g->timeout_ms = timeout_ms;
    g->m.resize(n);
    int st = HX_OK;
    for (int i = 0; i < n && st == HX_OK; ++i) {
        g->m[i].device = devices[i];
        g->m[i].rank = i;
        st = setup_member(g, g->m[i]);
    }
    ncclUniqueId u;
    if (st == HX_OK && a->GetUniqueId(&u) != ncclSuccess) st = gfail(g, HX_ERR_NCCL, "ncclGetUniqueId failed");
    if (st == HX_OK) {
        // All ranks of this process join in one NCCL group call.
        a->GroupStart();
        for (int i = 0; i < n && st == HX_OK; ++i) {
            DeviceGuard dg(devices[i]);
            ncclConfig_t cfg = config_of(flags);
            const ncclResult_t r = a->CommInitRankConfig(&g->m[i].comm, n, u, i, &cfg);
            if (r != ncclSuccess && r != ncclInProgress)
                st = gfail(g, HX_ERR_NCCL, "ncclCommInitRankConfig (rank %d): %s", i, nstr(r));
        }
        const ncclResult_t r = a->GroupEnd();
        if (st == HX_OK && r != ncclSuccess && r != ncclInProgress)
            st = gfail(g, HX_ERR_NCCL, "ncclGroupEnd: %s", nstr(r));
        const auto dl = deadline_of(g);
        for (int i = 0; i < n && st == HX_OK; ++i) st = settle(g, g->m[i], "communicator initialisation", dl);
        if (st != HX_OK) abort_all(g);
    }
    *out = g;
    return st;
}

int hx_group_destroy(hx_group* g) {
    using namespace hx;
    if (!g) return HX_OK;
    const NcclApi* a = nccl();
    for (auto& m : g->m) release_member(a, g, m);
    delete g;
    return HX_OK;
}

int hx_group_abort(hx_group* g) {
    if (!g) return HX_ERR_INVALID;
    hx::abort_all(g);
    return HX_OK;
}

int hx_group_set_timeout(hx_group* g, int timeout_ms) {
    if (!g || timeout_ms <= 0) return HX_ERR_INVALID;
    g->timeout_ms = timeout_ms;
    return HX_OK;
}

int hx_group_info(const hx_group* g, int* nranks, int* members, int* nccl_version) {
    if (!g) return HX_ERR_INVALID;
    if (nranks) *nranks = g->nranks;
    if (members) *members = (int)g->m.size();
    if (nccl_version) {
        const hx::NcclApi* a = hx::nccl();
        *nccl_version = a ? a->version : 0;
    }
    return HX_OK;
}

int hx_group_last_error(const hx_group* g, char* buf, uint64_t n) {
    if (!g || !buf || n == 0) return HX_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g->err_mu);
    snprintf(buf, (size_t)n, "%s", g->last_error.c_str());
    return HX_OK;
}

int hx_group_gather_buffer(hx_group* g, int member, uint64_t slot_bytes, void** base) {
    using namespace hx;
    hx_group_member* m = member_of(g, member);
    if (!m || !base || slot_bytes == 0) return HX_ERR_INVALID;
    if (g->aborted) return gfail(g, HX_ERR_NCCL, "the group was aborted");
    if (int st = ensure_buffer(g, *m, slot_bytes)) return st;
    *base = m->buf;
    return HX_OK;
}

int hx_allgather_heads(hx_group* g, int member, hx_ctx* ctx, hx_dtype dtype, const void* shard, void* merged,
                       int B, int Hs, int S, int D, int layout) {
    using namespace hx;
    hx_group_member* mp = member_of(g, member);
    if (!mp || !ctx) return HX_ERR_INVALID;
    hx_group_member& m = *mp;
    if (g->aborted) return gfail(g, HX_ERR_NCCL, "the group was aborted");
    if (ctx->device != m.device)
        return gfail(g, HX_ERR_INVALID, "context device %d is not member %d's device %d", ctx->device, member,
                     m.device);
    if ((dtype != HX_BF16 && dtype != HX_F32) || B < 0 || Hs < 0 || S < 0 || D < 1 || layout < 0 || layout > 2)
        return gfail(g, HX_ERR_INVALID, "hx_allgather_heads: bad dtype, shape or layout");
    const int esize = dtype == HX_BF16 ? 2 : 4;
    const uint64_t count = (uint64_t)B * Hs * S * D;
    if (count == 0) return HX_OK;
    if (!shard) return gfail(g, HX_ERR_INVALID, "hx_allgather_heads: NULL shard");
    if (int st = ensure_buffer(g, m, count * esize)) return st;
    const NcclApi* a = nccl();
    DeviceGuard dg(m.device);
    uint8_t* base = (uint8_t*)m.buf;
    uint8_t* own = base + (uint64_t)m.rank * m.slot_bytes;
    if (cudaEventRecord(m.ready, ctx->stream) != cudaSuccess || cudaStreamWaitEvent(m.stream, m.ready, 0) != cudaSuccess)
        return gfail(g, HX_ERR_CUDA, "hx_allgather_heads: cannot order the exchange after the caller's stream");
    // A shard already in this rank's slot (the forward wrote its output
    // there) is gathered in place.
    const void* send = shard == own ? (const void*)own : shard;
    const ncclResult_t r = a->AllGather(send, base, count, dtype == HX_BF16 ? ncclBfloat16 : ncclFloat32,
                                        m.comm, m.stream);
    if (r != ncclSuccess && r != ncclInProgress) {
        abort_all(g);
        return gfail(g, HX_ERR_NCCL, "ncclAllGather (rank %d): %s; communicator aborted", m.rank, nstr(r));
    }
    if (int st = settle(g, m, "ncclAllGather", deadline_of(g))) return st;
    if (merged && layout == 2) {
        // Shards stored [B, S, H_shard, D]: rank r's slot is B*S rows of
        // H_shard*D elements, which land in columns [r*H_shard*D, ...) of the
        // merged [B*S, H*D] rows. One 2D copy per rank, on the copy engines.
        const size_t w = (size_t)Hs * D * esize;
        for (int r = 0; r < g->nranks; ++r) {
            const cudaError_t e =
                cudaMemcpy2DAsync((uint8_t*)merged + (size_t)r * w, w * (size_t)g->nranks,
                                  base + (uint64_t)r * m.slot_bytes, w, w, (size_t)B * S, cudaMemcpyDeviceToDevice,
                                  m.stream);
            if (e != cudaSuccess) return gfail(g, HX_ERR_CUDA, "head reassembly copy: %s", cudaGetErrorString(e));
        }
    } else if (merged) {
        const uint64_t t0 = launches_of_this_thread();
        const cudaError_t e = reassemble_heads(m.stream, esize, base, merged, g->nranks, B, Hs, S, D, layout,
                                               HX_EXCHANGE_MERGE_SMS ? HX_EXCHANGE_MERGE_SMS : ctx->sm_count);
        ctx->kernel_launches += launches_of_this_thread() - t0;
        if (e != cudaSuccess)
            return gfail(g, HX_ERR_CUDA, "head reassembly: %s", cudaGetErrorString(e));
    }
    if (cudaEventRecord(m.done, m.stream) != cudaSuccess)
        return gfail(g, HX_ERR_CUDA, "hx_allgather_heads: cannot record completion");
    m.pending = true;
    return HX_OK;
}

int hx_group_wait(hx_group* g, int member, hx_ctx* ctx) {
    using namespace hx;
    hx_group_member* m = member_of(g, member);
    if (!m || !ctx || ctx->device != m->device) return HX_ERR_INVALID;
    if (!m->pending) return HX_OK;
    DeviceGuard dg(m->device);
    if (cudaStreamWaitEvent(ctx->stream, m->done, 0) != cudaSuccess)
        return gfail(g, HX_ERR_CUDA, "hx_group_wait: cannot order the caller's stream after the exchange");
    return HX_OK;
}

int hx_group_sync(hx_group* g, int member) {
    using namespace hx;
    hx_group_member* mp = member_of(g, member);
    if (!mp) return HX_ERR_INVALID;
    hx_group_member& m = *mp;
    if (!m.pending) return g->aborted ? gfail(g, HX_ERR_NCCL, "the group was aborted") : HX_OK;
    if (g->aborted) return gfail(g, HX_ERR_NCCL, "the group was aborted");
    const NcclApi* a = nccl();
    DeviceGuard dg(m.device);
    const auto dl = deadline_of(g);
    for (;;) {
        const cudaError_t e = cudaEventQuery(m.done);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return gfail(g, HX_ERR_CUDA, "exchange: %s", cudaGetErrorString(e));
        ncclResult_t st = ncclSuccess;
        if (a->CommGetAsyncError(m.comm, &st) != ncclSuccess || (st != ncclSuccess && st != ncclInProgress)) {
            abort_all(g);
            return gfail(g, HX_ERR_NCCL, "all-gather (rank %d) failed: %s; communicator aborted", m.rank, nstr(st));
        }
        if (Clock::now() > dl) {
            abort_all(g);
            // The aborted communicator's kernels return; drain the side stream.
            drain_member(g, m);
            m.pending = false;
            return gfail(g, HX_ERR_NCCL, "all-gather (rank %d) did not complete within %d ms (a peer has left "
                         "or stalled); communicator aborted", m.rank, g->timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    m.pending = false;
    return HX_OK;
}

}  // extern "C"
