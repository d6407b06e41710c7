// The arena as the device allocator of a whole process's tensors: the two
// functions torch's pluggable-allocator interface calls
// (torch.cuda.memory.CUDAPluggableAllocator), so that every CUDA tensor of a
// training loop — activations, gradients, optimizer state — takes its storage
// from a GpuMemoryArena (src/gpu/arena.rs:13-145: power-of-two bins, slabs
// parked on free and handed out again), as every tensor of the reference does.
//
// One arena per device, on a context of its own whose stream is the arena's
// home stream H: every pool operation (a miss's cudaMallocFromPoolAsync, the
// cudaFreeAsync of a reset) is ordered on H. A slab crossing streams is made
// safe with events: on free, an event recorded on the freeing stream is
// waited on by H and parked with the slab; a later allocation on any stream
// waits for that event before it may touch the slab, and a miss's allocation
// on H is waited on by the allocating stream.
#include <mutex>
#include <unordered_map>
#include <vector>

#include "hx_internal.h"

namespace hx {
namespace {

constexpr int kMaxDevices = 64;

struct TorchArena {
    hx_ctx* ctx = nullptr;
    cudaStream_t home = nullptr;
    std::mutex mu;
    std::unordered_map<void*, cudaEvent_t> freed;  // parked slab -> event of its last use
    std::vector<cudaEvent_t> spare;
};

std::mutex g_mu;
TorchArena* g_arena[kMaxDevices] = {};

TorchArena* arena_for(int device) {
    if (device < 0 || device >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_arena[device] == nullptr) {
        hx_ctx* c = nullptr;
        if (hx_ctx_create(device, &c) != HX_OK) return nullptr;
        TorchArena* a = new TorchArena();  // lives until the process exits (torch frees late)
        a->ctx = c;
        a->home = (cudaStream_t)hx_ctx_stream(c);
        g_arena[device] = a;
    }
    return g_arena[device];
}

cudaEvent_t take_event(TorchArena* a) {
    if (!a->spare.empty()) {
        cudaEvent_t e = a->spare.back();
        a->spare.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    return e;
}

}  // namespace
}  // namespace hx

extern "C" {

void* hx_torch_malloc(size_t size, int device, void* stream_) {
    using namespace hx;
    cudaStream_t stream = (cudaStream_t)stream_;
    TorchArena* a = arena_for(device);
    if (a == nullptr) return nullptr;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    void* p = nullptr;
    {
        std::lock_guard<std::mutex> lk(a->mu);
        const uint64_t misses = a->ctx->arena.misses;
        if (hx_alloc(a->ctx, size ? size : 1, &p) != HX_OK) p = nullptr;
        if (p != nullptr) {
            auto it = a->freed.find(p);
            if (it != a->freed.end()) {  // a parked slab: wait for its last use
                cudaStreamWaitEvent(stream, it->second, 0);
                a->spare.push_back(it->second);
                a->freed.erase(it);
            } else if (a->ctx->arena.misses != misses && stream != a->home) {
                // fresh from the pool on the home stream
                cudaEvent_t e = take_event(a);
                cudaEventRecord(e, a->home);
                cudaStreamWaitEvent(stream, e, 0);
                a->spare.push_back(e);
            }
        }
    }
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    return p;
}

void hx_torch_free(void* ptr, size_t size, int device, void* stream_) {
    using namespace hx;
    cudaStream_t stream = (cudaStream_t)stream_;
    (void)size;
    if (ptr == nullptr) return;
    TorchArena* a = arena_for(device);
    if (a == nullptr) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    {
        std::lock_guard<std::mutex> lk(a->mu);
        cudaEvent_t e = take_event(a);
        cudaEventRecord(e, stream);
        cudaStreamWaitEvent(a->home, e, 0);  // pool operations on the home stream come after this use
        a->freed[ptr] = e;
        hx_free(a->ctx, ptr);
    }
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
}

hx_ctx* hx_torch_arena_context(int device) {
    hx::TorchArena* a = hx::arena_for(device);
    return a ? a->ctx : nullptr;
}

}  // extern "C"
