// Self-test of the device-side failure path that every tcgen05 kernel relies
// on: a bounded mbarrier wait (sm100_ptx.cuh) on a barrier nothing will ever
// complete. After the wait limit the first waiter raises the CTA's abort
// flag and records its site in the context's status word; the other waiter
// sees the flag and leaves too; the kernel ends normally. Nothing faults,
// traps or hangs: the host's next hx_sync reports HX_ERR_TIMEOUT and the
// context stays usable.
#include "sm100_ptx.cuh"

namespace hx {
namespace {

constexpr int kSelftestSite = 99;

__global__ void __launch_bounds__(64, 1) wait_timeout_probe_kernel(DeviceStatus* status) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        ptx::mbar_init(ptx::smem_addr(&bar), 1);  // one arrival completes a phase; none comes
        ptx::fence_mbar_init();
    }
    __syncthreads();
    // One waiter per warp: lane 0 of warp 0 times out and raises the flag,
    // lane 0 of warp 1 leaves on the flag (or on its own limit).
    if (threadIdx.x % 32 == 0)
        (void)ptx::mbar_wait(ptx::smem_addr(&bar), 0, &abort_flag, status, kSelftestSite);
    __syncthreads();
}

}  // namespace

cudaError_t selftest_wait_timeout(cudaStream_t st, DeviceStatus* status) {
    wait_timeout_probe_kernel<<<1, 64, 0, st>>>(status);
    note_launch();
    return cudaGetLastError();
}

}  // namespace hx
