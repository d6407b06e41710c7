// Thin inline-PTX wrappers for the sm_100a features the attention kernels
// use: mbarriers with bounded waits, TMA tensor loads (no multicast), and
// tcgen05 (TMEM allocation, UMMA issue/commit, TMEM loads/stores).
//
// Descriptor formats follow the PTX ISA's tcgen05 "shared memory descriptor"
// and "instruction descriptor" tables (also spelled out in CUTLASS's
// cute/arch/mma_sm100_desc.hpp):
//   smem descriptor: [0,14) start>>4, [16,30) LBO>>4, [32,46) SBO>>4,
//                    [46,48) version=1, [49,52) base offset, [61,64) swizzle
//                    (2 = 128-byte swizzle).
//   instr descriptor (kind::f16): [4,6) D fmt (1=f32), [7,10) A fmt (1=bf16),
//                    [10,13) B fmt, [15] A MN-major, [16] B MN-major,
//                    [17,23) N>>3, [24,29) M>>4.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "hx_internal.h"

namespace hx {
namespace ptx {

// Give up on a device-side wait after this long (the waits here are for
// pipeline stages of a few microseconds; only a broken pipeline reaches it).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier ----------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with `parity` of `bar` to complete. Gives up when the
// CTA's abort flag is raised or after kWaitLimitNs; the first waiter to time
// out raises the flag and records `site` in the device status word, so every
// role of the CTA unwinds and the host reports HX_ERR_TIMEOUT.
__device__ __forceinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                            DeviceStatus* status, int site) {
    const uint64_t t0 = globaltimer();
    for (uint32_t n = 1;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 31u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                *abort_flag = 1;
                if (atomicCAS(&status->code, 0, 1) == 0) {
                    status->where = site;
                    status->block = (int)blockIdx.x;
                }
                return false;
            }
        }
    }
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          DeviceStatus* status, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, abort_flag, status, site);
}

// Waits with a time limit only (ignores the abort flag): used on the way out
// to let this CTA's own asynchronous copies / MMAs finish before its shared
// memory and tensor memory are released.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    for (uint32_t n = 1;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 31u) == 0 && globaltimer() - t0 > kWaitLimitNs) return false;
    }
}

// ---- TMA (tiled tensor loads into this CTA's shared memory, no multicast) ----
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// Plain bulk copy global -> this CTA's smem (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
        : "memory");
}
// Element-wise add of a smem tile into global memory through a tensor map.
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, uint32_t src, int c0,
                                                  int c1, int c2) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(src), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
// Fire-and-forget f32 add in L2 (no return value).
__device__ __forceinline__ void red_add_f32(float* addr, float v) {
    asm volatile("red.global.add.f32 [%0], %1;\n" ::"l"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N of this thread's committed bulk groups still have to
// read their smem sources.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until this thread's committed bulk groups completed.
__device__ __forceinline__ void bulk_wait_group0() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---- tcgen05: TMEM allocation ---------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// ---- tcgen05: MMA ------------------------------------------------------------------
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on `bar` once every tcgen05 operation issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- tcgen05: TMEM <-> registers (32x32b shape: thread t of warp w reaches
// lane 32*(w%4)+t; one 32-bit register per column) ----------------------------------
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

#define HX_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), \
                 "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define HX_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), \
                 "r"(r[i + 4]), "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : HX_R8(0), HX_R8(8), HX_R8(16), HX_R8(24)
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        HX_W8(0), HX_W8(8), HX_W8(16), HX_W8(24)
        : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        HX_W8(0), HX_W8(8)
        : "memory");
}
#undef HX_R8
#undef HX_W8

// Ties registers filled by tcgen05.ld to a point after tcgen05.wait::ld so
// the compiler cannot move their uses above the wait.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t* r) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i])::"memory");
}

// ---- descriptors -----------------------------------------------------------------------
// K-major or MN-major operand tile laid out by TMA with 128-byte swizzle.
// Joins a descriptor's low and high 32-bit words.
__device__ __forceinline__ uint64_t desc_of(uint32_t lo, uint32_t hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
    return d;
}
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) |
           ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major,
                                                      bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
           ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// ---- small numeric helpers ---------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// ---- packed f32x2 arithmetic (sm_100): one instruction for two lanes of
// work, halving the issue slots of elementwise softmax code.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// 2^x for both lanes of an f32x2 pair on the FMA and integer pipes, for
// softmax loops bound by the multi-function unit (one ex2 per 8 cycles per
// warp). x = n + f with n = rint(x) (the 1.5 * 2^23 shifter leaves n in the low
// mantissa bits of t) and f in [-0.5, 0.5]; 2^f is a degree-3 polynomial
// fitted here by iteratively reweighted least squares on 4000 Chebyshev nodes
// for minimax relative error (7.5e-5, a 50th of a bf16 ulp); n is added to the
// result's exponent field. x is clamped below at -125 so the exponent field
// stays normal: results under 2^-125 come out as about 2^-125, which no bf16
// product or f32 row sum of a softmax can tell from 0. Valid for x <= 127.
__device__ __forceinline__ uint64_t ex2_poly_x2(uint64_t x) {
    constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
    float a, b;
    f2_unpack(x, a, b);
    const uint64_t xc = f2_pack(fmaxf(a, -125.f), fmaxf(b, -125.f));
    const uint64_t t = f2_add(xc, f2_pack(kShift, kShift));
    float n0, n1;
    f2_unpack(f2_add(t, f2_pack(-kShift, -kShift)), n0, n1);
    const uint64_t f = f2_add(xc, f2_pack(-n0, -n1));
    uint64_t p = f2_fma(f2_pack(0.05518148094415665f, 0.05518148094415665f), f,
                        f2_pack(0.24261195957660675f, 0.24261195957660675f));
    p = f2_fma(p, f, f2_pack(0.6932591795921326f, 0.6932591795921326f));
    p = f2_fma(p, f, f2_pack(0.9999279975891113f, 0.9999279975891113f));
    float p0, p1, t0, t1;
    f2_unpack(p, p0, p1);
    f2_unpack(t, t0, t1);
    return f2_pack(__int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23)),
                   __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23)));
}
// max of three floats in one instruction (sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// Packs two floats to bf16x2 (round to nearest even): `lo` in bits 0-15.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

}  // namespace ptx
}  // namespace hx
