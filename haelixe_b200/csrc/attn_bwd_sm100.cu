// tcgen05 fused attention backward for sm_100a (bf16 I/O, f32 accumulation,
// head_dim 64 or 128, optional causal mask). Replaces the reference's
// composite backward (src/ops/flash_attention.rs:16-39: recompute P, five
// batched matmuls and a softmax-Jacobian kernel over materialised S x S
// matrices) with three launches that never materialise S x S:
//
//   pre   delta[q] = sum_d dO[q,d] O[q,d]  (the `dot` of the softmax backward,
//         src/kernels/activations.rs:170-176) and zero the f32 dQ accumulator;
//   main  one CTA per (128-key tile, head, batch), K and V resident in smem,
//         looping over query tiles of BQ rows:
//           S^T  = K Q^T      (SS UMMA, M=128 keys, N=BQ)      -> TMEM
//           dP^T = V dO^T     (SS UMMA)                         -> TMEM
//           P^T  = exp2(S^T * scale*log2e - lse*log2e) (mask)   -> TMEM (bf16)
//           dV  += P^T dO     (TS UMMA, A from TMEM, B = dO MN-major)
//           dS^T = P^T (dP^T - delta)                           -> smem (bf16)
//           dK  += dS^T Q     (SS UMMA, dS^T K-major from smem)
//           dQ   = dS K       (SS UMMA from the smem dS tile; for D=128 as
//                              dQ^T = K^T dS^T so M = D = 128)  -> TMEM
//         a drain warpgroup moves each dQ tile TMEM -> registers and adds it
//         into the f32 accumulator in L2 (D=128: red.global.add from the
//         registers; D=64: through an smem staging tile and a bulk tensor
//         reduce-add) while the tensor core moves on;
//   post  dQ = bf16(scale * accumulator), dK already carries the scale.
// The scale on dQ and dK is the factor the reference's backward omits
// (flash_attention.rs:31,34-36).
//
// Warp roles of `main` (512 threads): warp 0 TMA producer (Q, dO tiles and
// the lse/delta rows of each query tile), warp 1 lane 0 the accumulate MMA
// issuer (dV, dK, dQ), warp 3 lane 0 the recompute MMA issuer (S^T, dP^T),
// warp 2 TMEM allocator, warps 4-7 and 8-11 two P/dS warpgroups that split
// each query tile's columns (thread = key row = TMEM lane), warps 12-15 the
// dQ drain warpgroup. All mbarrier waits are bounded (sm100_ptx.cuh).
#include <math.h>
#include <string.h>

#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace hx {
namespace {

using namespace ptx;

constexpr int BK = 128;  // keys per CTA (UMMA M of S^T, dP^T, dV, dK)
constexpr int kThreads = 512;
// Register split (setmaxnreg) per SM sub-partition, one warp of each group:
// control + 2 x P/dS + dQ drain = 512 = 4 x 128 (the launch count, checked on
// the host before every launch); the shares depend on head_dim (BCfg).
constexpr int kRegsLaunch = 128;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct BCfg {
    static constexpr int BQ = D == 128 ? 64 : 128;  // queries per inner tile
    static constexpr bool DQ_T = D == 128;           // dQ computed transposed (M = D)
    // Q/dO/lse/delta ring depth. D=128 uses the 64 KB the register dQ drain
    // freed for a third stage (backward 6.32 -> 6.01 ms on C3).
    static constexpr int QST = D == 128 ? 3 : 2;
    static constexpr int REGS_CTL = D == 128 ? 104 : 64;
    static constexpr int REGS_COMPUTE = D == 128 ? 160 : 168;
    static constexpr int REGS_DRAIN = D == 128 ? 88 : 112;
    static_assert(REGS_CTL + 2 * REGS_COMPUTE + REGS_DRAIN == 4 * kRegsLaunch, "register split");
    static_assert(QST <= 4, "BBars holds 4 ring stages");
    static constexpr int CHUNK_K = BK * 128;         // bytes of a 64-column chunk of a K/V tile
    static constexpr int CHUNK_Q = BQ * 128;         // ... of a Q/dO tile
    static constexpr int CHUNK_DS = BK * 128;        // ... of the dS^T tile (64 queries wide)
    static constexpr int KT = BK * D * 2;
    static constexpr int QT = BQ * D * 2;
    static constexpr int DST = BK * BQ * 2;
    // smem dS^T tiles: two for D=128, so dS(i+1) can be written while dK(i) and
    // dQ(i) still read dS(i); D=64 has room for one.
    static constexpr int NDS = D == 128 ? 2 : 1;
    static constexpr int K_OFF = 0;
    static constexpr int V_OFF = K_OFF + KT;
    static constexpr int Q_OFF = V_OFF + KT;
    static constexpr int DO_OFF = Q_OFF + QST * QT;
    static constexpr int DS_OFF = DO_OFF + QST * QT;
    // dQ drain. D=128: red.global.add straight from the registers loaded from
    // TMEM (each warp instruction adds 32 consecutive floats of a query row);
    // the kernel is bound by shared-memory bandwidth, and this keeps the
    // 2 x 32 KB per query tile of staging writes and bulk-copy reads out of it
    // (backward 4.5 % faster on C3). D=64: an f32 staging tile in smem and a
    // bulk tensor reduce-add (the per-row vector reds measured 20 % slower).
    static constexpr bool DQ_RED = D == 128;
    static constexpr int DQS = BQ * D * 4;           // f32 dQ staging tile for the reduce-add
    // Two staging tiles: the L2 reduce-add of one tile (~0.75 us for 32 KB at
    // the chip's ~5.9 TB/s reduction rate, shared by all SMs) overlaps the
    // drain of the next.
    static constexpr int NDQS = DQ_RED ? 0 : 2;
    static constexpr int DQS_OFF = DS_OFF + NDS * DST;
    static constexpr int LSE_OFF = DQS_OFF + NDQS * DQS;
    static constexpr int DEL_OFF = LSE_OFF + QST * BQ * 4;
    static constexpr int BAR_OFF = DEL_OFF + QST * BQ * 4;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;
    static_assert(SMEM <= 232448, "shared memory per block");
    // TMEM columns. D=128: two S^T buffers (the next tile's K Q^T runs while P of
    // this one is computed) and one dQ^T buffer; D=64: one S^T buffer, two dQ.
    static constexpr int NSB = D == 128 ? 2 : 1;
    // D=128: dS^T is also packed into the S^T buffer's free half, after P^T,
    // and dK reads it from TMEM (TS UMMA) instead of from the smem tile; the
    // buffer is released after dK. D=64 (one S^T buffer) keeps dK on smem.
    static constexpr bool DK_TS = NSB == 2;
    static constexpr int NDQ = D == 128 ? 1 : 2;
    static constexpr int DQ_COLS = DQ_T ? BQ : D;
    static constexpr uint32_t C_S0 = 0, C_DP = NSB * BQ, C_DQ0 = C_DP + BQ,
                              C_DV = C_DQ0 + NDQ * DQ_COLS, C_DK = C_DV + D;
    static_assert(C_DK + D <= 512, "TMEM budget");
};

struct BBars {
    uint64_t kv_full;
    uint64_t q_full[4], q_empty[4];  // indexed by ring stage (QST <= 4)
    uint64_t s_full[2], dp_full;
    // P(i) / dS(i) ready, indexed by i & 1: the P/dS warpgroups can run up to
    // two query tiles ahead of the accumulate issuer (S^T(i+1) does not wait
    // for dV(i)), so one barrier per parity keeps every wait on its own phase.
    uint64_t p_full[2], ds_full[2];
    uint64_t sfree[2];          // S^T buffer b read by dV (accumulate -> recompute issuer)
    uint64_t dpfree;            // dP^T columns loaded by the P/dS warpgroups (-> recompute issuer)
    uint64_t dsfree[2];         // smem dS tile b read by dK and dQ (-> P/dS warpgroups)
    uint64_t dq_full[2], dq_empty[2];
    uint64_t dqs_free, dqs_full;
    uint64_t acc_done, done, done_r;
    uint32_t tmem_base;
    int abort_flag;
};

static_assert(sizeof(BBars) <= 256, "barrier block");

// (batch, head) slices per dispatch group of the backward grid.
#ifndef HX_BWD_HGROUP
#define HX_BWD_HGROUP 2
#endif

struct BwdParams {
    const float* lse2;   // [B*H][S_pad]: lse * log2(e), 0 past S
    const float* delta;  // [B*H][S_pad]: rowsum(dO * O), 0 past S
    int S_pad;
    __nv_bfloat16* dk;
    __nv_bfloat16* dv;
    int64_t sb, sh, ss;  // strides of dk/dv (elements)
    int S, H;
    float scale;
    int causal;
    // (cos, sin) of s * base^(-2i/D) for [S][D/2], or null. When set, dK leaves
    // the kernel rotated back by -theta of its key row: the gradient with
    // respect to K before the rotary embedding (src/kernels/rope.rs:44-82).
    const float2* rope_tab;
    int hgroup;  // (batch, head) slices per dispatch group (see the block mapping)
    float* dq_acc;  // [B*H][S][D] f32 accumulator (D=64: written through tdq by bulk reduce-adds)
    DeviceStatus* status;
};

// Rotation of one (x0, x1) pair by -theta with the reference's unfused
// products and sums (src/kernels/rope.rs:37-38, 67): one rounding per
// operation, no FMA contraction.
__device__ __forceinline__ void rope_rot_back(float x0, float x1, float2 cs, float& y0, float& y1) {
    y0 = __fadd_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    y1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x0, cs.y));
}

__device__ __forceinline__ uint32_t bar_addr(const uint64_t& b) { return smem_addr(&b); }

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t* r) {
#pragma unroll
    for (int c = 0; c < N; c += 32) tmem_ld32(taddr + c, r + c);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                    const __grid_constant__ CUtensorMap tdq, const BwdParams p) {
    using C = BCfg<D>;
    constexpr int BQ = C::BQ;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned base, derived from the shared array itself so that the
    // compiler keeps every access through `sm` in the shared state space.
    uint8_t* sm = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    BBars* bars = (BBars*)(sm + C::BAR_OFF);
    float* s_lse = (float*)(sm + C::LSE_OFF);
    float* s_del = (float*)(sm + C::DEL_OFF);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    // 1D grid in groups of hgroup (batch, head) slices; inside a group the
    // key block varies slowest. Blocks are dispatched in index order, so with
    // causal masking the group's heaviest (first) key blocks go first and the
    // light ones fill the tail (longest first within a group), while the
    // blocks in flight stream only a group's worth of Q, dO and dQ (L2).
    const int nblk = (p.S + BK - 1) / BK;
    const int nbh = (int)(gridDim.x / nblk);
    const int grp = (int)(blockIdx.x / ((unsigned)p.hgroup * nblk));
    const int gs = min(p.hgroup, nbh - grp * p.hgroup);
    const int loc = (int)(blockIdx.x - (unsigned)grp * p.hgroup * nblk);
    const int kb = loc / gs, bhi = grp * p.hgroup + loc % gs;
    const int k0 = kb * BK;
    const int h = bhi % p.H, b = bhi / p.H;
    const int64_t bh = (int64_t)b * p.H + h;
    const int i_start = p.causal ? k0 / BQ : 0;
    const int n_it = (p.S + BQ - 1) / BQ - i_start;
    volatile int* abort_flag = &bars->abort_flag;

    if (threadIdx.x == 0) {
        bars->abort_flag = 0;
        mbar_init(bar_addr(bars->kv_full), 1);
        for (int s = 0; s < C::QST; ++s) {
            mbar_init(bar_addr(bars->q_full[s]), 1);
            mbar_init(bar_addr(bars->q_empty[s]), 1);
        }
        mbar_init(bar_addr(bars->s_full[0]), 1);
        mbar_init(bar_addr(bars->s_full[1]), 1);
        mbar_init(bar_addr(bars->dp_full), 1);
        mbar_init(bar_addr(bars->sfree[0]), 1);
        mbar_init(bar_addr(bars->sfree[1]), 1);
        mbar_init(bar_addr(bars->dpfree), 256);
        mbar_init(bar_addr(bars->dsfree[0]), 1);
        mbar_init(bar_addr(bars->dsfree[1]), 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar_addr(bars->p_full[s]), 256);
            mbar_init(bar_addr(bars->ds_full[s]), 256);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar_addr(bars->dq_full[s]), 1);
            mbar_init(bar_addr(bars->dq_empty[s]), 128);
        }
        mbar_init(bar_addr(bars->dqs_free), 1);
        mbar_init(bar_addr(bars->dqs_full), 128);
        mbar_init(bar_addr(bars->acc_done), 1);
        mbar_init(bar_addr(bars->done), 1);
        mbar_init(bar_addr(bars->done_r), 1);
        fence_mbar_init();
        fence_proxy_async();
    }
    if (warp == 2) {
        tmem_alloc(smem_addr(&bars->tmem_base), 512);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tq);
        prefetch_tmap(&tk);
        prefetch_tmap(&tv);
        prefetch_tmap(&tdo);
        if (!C::DQ_RED) prefetch_tmap(&tdq);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(C::REGS_CTL));
    } else if (warp < 12) {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(C::REGS_COMPUTE));
    } else {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(C::REGS_DRAIN));
    }

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        const uint32_t kvb = bar_addr(bars->kv_full);
        if (lane == 0) {
            mbar_arrive_expect_tx(kvb, 2 * C::KT);
            for (int c = 0; c < D / 64; ++c) {
                tma_load_4d(smem_addr(sm + C::K_OFF + c * C::CHUNK_K), &tk, kvb, c * 64, k0, h, b);
                tma_load_4d(smem_addr(sm + C::V_OFF + c * C::CHUNK_K), &tv, kvb, c * 64, k0, h, b);
            }
        }
        int issued = 0;
        if (lane == 0) {
            for (int it = 0; it < n_it; ++it) {
                const int st = it % C::QST;
                const uint32_t ph = (it / C::QST) & 1;
                const int q0 = (i_start + it) * BQ;
                if (!mbar_wait(bar_addr(bars->q_empty[st]), ph ^ 1, abort_flag, p.status, 40)) break;
                const uint32_t qb = bar_addr(bars->q_full[st]);
                mbar_arrive_expect_tx(qb, 2 * C::QT + 2 * BQ * 4);
                for (int c = 0; c < D / 64; ++c) {
                    tma_load_4d(smem_addr(sm + C::Q_OFF + st * C::QT + c * C::CHUNK_Q), &tq, qb,
                                c * 64, q0, h, b);
                    tma_load_4d(smem_addr(sm + C::DO_OFF + st * C::QT + c * C::CHUNK_Q), &tdo, qb,
                                c * 64, q0, h, b);
                }
                const int64_t row0 = bh * p.S_pad + q0;
                bulk_load(smem_addr(s_lse + st * BQ), p.lse2 + row0, BQ * 4, qb);
                bulk_load(smem_addr(s_del + st * BQ), p.delta + row0, BQ * 4, qb);
                issued = it + 1;
            }
            mbar_wait_drain(kvb, 0);
            for (int it = max(0, issued - C::QST); it < issued; ++it)
                mbar_wait_drain(bar_addr(bars->q_full[it % C::QST]), (it / C::QST) & 1);
        }
        // Teardown stays inside each role branch: no code is shared across the
        // register split.
        __syncwarp();
        tc_fence_before();
        __syncthreads();
    } else if (warp < 4) {
        // ------------------------------------------------------------ MMA issuers
        // Two threads issue MMAs, each waiting only on its own inputs, so one
        // keeps the tensor core fed while the other waits (a single issuing
        // thread leaves the pipe idle during every mbarrier wait):
        //   warp 3 lane 0 (recompute): S^T(i) = K Q^T and dP^T(i) = V dO^T;
        //   warp 1 lane 0 (accumulate): dV += P^T dO, dK += dS^T Q, dQ(i).
        // Buffer hand-offs go through mbarriers: sfree[b] (committed after dV
        // read P^T from S buffer b), dpfree (the P/dS warpgroups have loaded
        // dP^T into registers), dsfree[b] (dK and dQ read smem dS tile b).
        constexpr uint32_t idSP = idesc_bf16_f32(BK, BQ, false, false);
        constexpr uint32_t idAcc = idesc_bf16_f32(BK, D, false, true);
        constexpr uint32_t idDQ =
            C::DQ_T ? idesc_bf16_f32(D, BQ, true, true) : idesc_bf16_f32(BQ, D, true, true);
        constexpr uint64_t kStage = (uint64_t)(C::QT >> 4);  // per-stage descriptor offset
        constexpr int KH = BQ / 32;  // K-steps of dV/dK per warpgroup half (see acc_a)
        constexpr int NS = D / 16;   // K-steps of S^T / dP^T
        constexpr int NA = BQ / 16;  // K-steps of dV / dK
        constexpr int NQ = BK / 16;  // K-steps of dQ
        // K-step offsets (in 16-byte units) of K-major and MN-major operands.
        auto kmaj = [](int kk, int chunk) { return (uint64_t)(((kk / 4) * chunk + (kk % 4) * 32) >> 4); };
        auto mnmaj = [](int kk) { return (uint64_t)((kk * 2048) >> 4); };
        // Descriptor bases, built once: a K-step only adds its byte offset >> 4
        // to the start-address field (every operand lies inside this CTA's smem).
        const uint32_t sK = smem_addr(sm + C::K_OFF), sV = smem_addr(sm + C::V_OFF),
                       sQ = smem_addr(sm + C::Q_OFF), sDO = smem_addr(sm + C::DO_OFF),
                       sDS = smem_addr(sm + C::DS_OFF);
        bool ok = true;
        if (warp == 3 && lane == 0) {
            // -------- recompute issuer
            const uint64_t dKk = sdesc_sw128(sK, 16, 1024);     // K, K-major (A of S^T)
            const uint64_t dVk = sdesc_sw128(sV, 16, 1024);     // V, K-major (A of dP^T)
            const uint64_t dQk0 = sdesc_sw128(sQ, 16, 1024);    // Q stage 0, K-major
            const uint64_t dDOk0 = sdesc_sw128(sDO, 16, 1024);  // dO stage 0, K-major
            ok = mbar_wait(bar_addr(bars->kv_full), 0, abort_flag, p.status, 50);
            for (int it = 0; ok && it < n_it; ++it) {
                const int st = it % C::QST, b = it % C::NSB;
                if (!(ok = mbar_wait(bar_addr(bars->q_full[st]), (it / C::QST) & 1, abort_flag,
                                     p.status, 51)))
                    break;
                // S^T buffer b is free once dV(it - NSB) has read P^T from it.
                if (!(ok = mbar_wait(bar_addr(bars->sfree[b]), ((it / C::NSB) & 1) ^ 1, abort_flag,
                                     p.status, 56)))
                    break;
                tc_fence_after();
                const uint32_t cS = C::C_S0 + (uint32_t)(b * BQ);
                const uint64_t dq = dQk0 + st * kStage, ddo = dDOk0 + st * kStage;
#pragma unroll
                for (int kk = 0; kk < NS; ++kk)
                    umma_ss(tmem + cS, dKk + kmaj(kk, C::CHUNK_K), dq + kmaj(kk, C::CHUNK_Q), idSP, kk > 0);
                umma_commit(bar_addr(bars->s_full[b]));
                // The dP^T columns are free once the P/dS warpgroups loaded dP^T(it - 1).
                if (!(ok = mbar_wait(bar_addr(bars->dpfree), (it & 1) ^ 1, abort_flag, p.status, 57)))
                    break;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < NS; ++kk)
                    umma_ss(tmem + C::C_DP, dVk + kmaj(kk, C::CHUNK_K), ddo + kmaj(kk, C::CHUNK_Q), idSP,
                            kk > 0);
                umma_commit(bar_addr(bars->dp_full));
            }
            umma_commit(bar_addr(bars->done_r));
            mbar_wait_drain(bar_addr(bars->done_r), 0);
        } else if (warp == 1 && lane == 0) {
            // -------- accumulate issuer
            const uint64_t dKm = sdesc_sw128(sK, C::CHUNK_K, 1024);     // K, MN-major (dQ)
            const uint64_t dDSm = sdesc_sw128(sDS, C::CHUNK_DS, 1024);  // dS tile 0, MN-major (dQ)
            const uint64_t dDSk = sdesc_sw128(sDS, 16, 1024);           // dS tile 0, K-major (A of dK)
            constexpr uint64_t kDsTile = (uint64_t)(C::DST >> 4);
            const uint64_t dQm0 = sdesc_sw128(sQ, C::CHUNK_Q, 1024);    // Q stage 0, MN-major
            const uint64_t dDOm0 = sdesc_sw128(sDO, C::CHUNK_Q, 1024);  // dO stage 0, MN-major
            // A column of dV/dK K-step kk: warpgroup g packed its BQ/2 columns at the
            // start of its own f32 columns [g*BQ/2, ...).
            auto acc_a = [](int kk) { return (uint32_t)((kk / KH) * (BQ / 2) + (kk % KH) * 8); };
            for (int it = 0; ok && it < n_it; ++it) {
                const int st = it % C::QST, b = it % C::NSB, db = it % C::NDS;
                const bool first = it == 0;
                const uint32_t cS = C::C_S0 + (uint32_t)(b * BQ);
                const uint64_t dsm = dDSm + db * kDsTile, dsk = dDSk + db * kDsTile;
                const uint64_t dQm = dQm0 + st * kStage, dDOm = dDOm0 + st * kStage;
                if (!(ok = mbar_wait(bar_addr(bars->p_full[it & 1]), (it >> 1) & 1, abort_flag, p.status,
                                     52)))
                    break;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < NA; ++kk)  // dV += P^T dO
                    umma_ts(tmem + C::C_DV, tmem + cS + acc_a(kk), dDOm + mnmaj(kk), idAcc,
                            (first && kk == 0) ? 0u : 1u);
                if (!C::DK_TS) umma_commit(bar_addr(bars->sfree[b]));
                if (!(ok = mbar_wait(bar_addr(bars->ds_full[it & 1]), (it >> 1) & 1, abort_flag, p.status,
                                     54)))
                    break;
                tc_fence_after();
                if constexpr (C::DK_TS) {
#pragma unroll
                    for (int kk = 0; kk < NA; ++kk)  // dK += dS^T Q (dS^T from TMEM, after P^T)
                        umma_ts(tmem + C::C_DK, tmem + cS + acc_a(kk) + BQ / 4, dQm + mnmaj(kk), idAcc,
                                (first && kk == 0) ? 0u : 1u);
                    umma_commit(bar_addr(bars->sfree[b]));
                } else {
#pragma unroll
                    for (int kk = 0; kk < NA; ++kk)  // dK += dS^T Q (dS^T K-major from smem)
                        umma_ss(tmem + C::C_DK, dsk + kmaj(kk, C::CHUNK_DS), dQm + mnmaj(kk), idAcc,
                                (first && kk == 0) ? 0u : 1u);
                }
                // Q(it) and dO(it) are read by nothing after dK(it): S^T(it) and
                // dP^T(it) completed before dS(it) existed.
                umma_commit(bar_addr(bars->q_empty[st]));
                const int dqb = it % C::NDQ;
                if (!(ok = mbar_wait(bar_addr(bars->dq_empty[dqb]), ((it / C::NDQ) & 1) ^ 1,
                                     abort_flag, p.status, 55)))
                    break;
                tc_fence_after();
                const uint32_t cq = C::C_DQ0 + (uint32_t)(dqb * C::DQ_COLS);
#pragma unroll
                for (int kk = 0; kk < NQ; ++kk) {
                    if (C::DQ_T)  // dQ^T = K^T dS^T
                        umma_ss(tmem + cq, dKm + mnmaj(kk), dsm + mnmaj(kk), idDQ, kk > 0);
                    else  // dQ = dS K
                        umma_ss(tmem + cq, dsm + mnmaj(kk), dKm + mnmaj(kk), idDQ, kk > 0);
                }
                umma_commit(bar_addr(bars->dq_full[dqb]));
                umma_commit(bar_addr(bars->dsfree[db]));
            }
            umma_commit(bar_addr(bars->acc_done));
            umma_commit(bar_addr(bars->done));
            mbar_wait_drain(bar_addr(bars->done), 0);
        }
        __syncwarp();
        tc_fence_before();
        __syncthreads();
        if (warp == 2) {  // warp 2 allocated the TMEM; it frees it once every role is done
            tc_fence_after();
            tmem_dealloc(tmem, 512);
        }
    } else if (warp < 12) {
        // ------------------------------------------------------------ P / dS warpgroups
        // Warpgroup g (warps 4-7: g=0, 8-11: g=1) owns columns [g*HC, (g+1)*HC) of
        // every query tile; thread = key row = TMEM lane.
        constexpr int HC = BQ / 2;  // columns per warpgroup
        const int g = (warp - 4) / 4;
        const int wi = warp % 4;
        const int r = wi * 32 + lane;
        const int kr = k0 + r;
        const uint32_t tl = tmem + ((uint32_t)(wi * 32) << 16);
        const float sl2 = p.scale * kLog2e;
        const int c0 = g * HC;  // first column of this warpgroup
        bool ok = true;
        for (int it = 0; it < n_it; ++it) {
            const int st = it % C::QST;
            const uint32_t ph = (it / C::QST) & 1;
            const int q0 = (i_start + it) * BQ;
            const uint32_t cS = C::C_S0 + (uint32_t)((it % C::NSB) * BQ) + c0;
            const uint32_t cD = C::C_DP + c0;
            if (!(ok = mbar_wait(bar_addr(bars->q_full[st]), ph, abort_flag, p.status, 60))) break;
            if (!(ok = mbar_wait(bar_addr(bars->s_full[it % C::NSB]), (it / C::NSB) & 1, abort_flag,
                                 p.status, 61)))
                break;
            tc_fence_after();
            const float* lse2 = s_lse + st * BQ + c0;
            const float* del = s_del + st * BQ + c0;
            // Valid columns [lo, hi) of this row: q < S, key < S, causal q >= key.
            const bool need_mask = (q0 + BQ > p.S) || (k0 + BK > p.S) || (p.causal && k0 + BK - 1 > q0);
            int lo = 0, hi = HC;
            if (need_mask) {
                hi = kr < p.S ? min(HC, p.S - q0 - c0) : 0;
                if (p.causal) lo = max(0, kr - q0 - c0);
            }
            // P^T = exp2(S^T * scale*log2e - lse*log2e) for HC columns, loaded with
            // one wait; the packed result lands on the first HC/2 of these columns.
            uint32_t x[HC];
#pragma unroll
            for (int c = 0; c < HC; c += 32) tmem_ld32(tl + cS + c, x + c);
            tmem_ld_wait();
            reg_fence<HC>(x);
            float pr[HC];
#pragma unroll
            for (int q4 = 0; q4 < HC / 4; ++q4) {
                const float4 l4 = reinterpret_cast<const float4*>(lse2)[q4];
                pr[4 * q4 + 0] = ex2(fmaf(__uint_as_float(x[4 * q4 + 0]), sl2, -l4.x));
                pr[4 * q4 + 1] = ex2(fmaf(__uint_as_float(x[4 * q4 + 1]), sl2, -l4.y));
                pr[4 * q4 + 2] = ex2(fmaf(__uint_as_float(x[4 * q4 + 2]), sl2, -l4.z));
                pr[4 * q4 + 3] = ex2(fmaf(__uint_as_float(x[4 * q4 + 3]), sl2, -l4.w));
            }
            if (need_mask) {
#pragma unroll
                for (int c = 0; c < HC; ++c) pr[c] = (c >= lo && c < hi) ? pr[c] : 0.f;
            }
            uint32_t pk[HC / 2];
#pragma unroll
            for (int i = 0; i < HC / 2; ++i) pk[i] = pack_bf16(pr[2 * i], pr[2 * i + 1]);
#pragma unroll
            for (int c = 0; c < HC / 2; c += 16) tmem_st16(tl + cS + c, pk + c);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(bar_addr(bars->p_full[it & 1]));

            if (!(ok = mbar_wait(bar_addr(bars->dp_full), it & 1, abort_flag, p.status, 62))) break;
            tc_fence_after();
            // dS^T = P^T (dP^T - delta) -> the 128-byte-swizzled smem tile the dK
            // and dQ MMAs read. The dP^T columns are released as soon as they are
            // in registers, so dP^T(it + 1) overlaps the rest of this phase.
#pragma unroll
            for (int c = 0; c < HC; c += 32) tmem_ld32(tl + cD + c, x + c);
            tmem_ld_wait();
            reg_fence<HC>(x);
            tc_fence_before();
            mbar_arrive(bar_addr(bars->dpfree));
#pragma unroll
            for (int q4 = 0; q4 < HC / 4; ++q4) {
                const float4 d4 = reinterpret_cast<const float4*>(del)[q4];
                const float a0 = pr[4 * q4 + 0] * (__uint_as_float(x[4 * q4 + 0]) - d4.x);
                const float a1 = pr[4 * q4 + 1] * (__uint_as_float(x[4 * q4 + 1]) - d4.y);
                const float a2 = pr[4 * q4 + 2] * (__uint_as_float(x[4 * q4 + 2]) - d4.z);
                const float a3 = pr[4 * q4 + 3] * (__uint_as_float(x[4 * q4 + 3]) - d4.w);
                pk[2 * q4] = pack_bf16(a0, a1);
                pk[2 * q4 + 1] = pack_bf16(a2, a3);
            }
            // smem dS tile db is free once dK(it - NDS) and dQ(it - NDS) have read it.
            const int db = it % C::NDS;
            if (!(ok = mbar_wait(bar_addr(bars->dsfree[db]), ((it / C::NDS) & 1) ^ 1, abort_flag,
                                 p.status, 64)))
                break;
            uint8_t* ds_row = sm + C::DS_OFF + db * C::DST + r * 128;
            // smem: 16-byte piece u of the 128-byte row of 64-column chunk k holds
            // columns k*64 + 8u .. +7.
#pragma unroll
            for (int u8 = 0; u8 < HC / 8; ++u8) {
                const int col = c0 + 8 * u8;
                const int chunk = col / 64, u = (col % 64) / 8;
                *reinterpret_cast<uint4*>(ds_row + chunk * C::CHUNK_DS + ((u ^ (r & 7)) * 16)) =
                    make_uint4(pk[4 * u8], pk[4 * u8 + 1], pk[4 * u8 + 2], pk[4 * u8 + 3]);
            }
            if constexpr (C::DK_TS) {  // packed dS^T after this warpgroup's P^T columns
#pragma unroll
                for (int c = 0; c < HC / 2; c += 16) tmem_st16(tl + cS + HC / 2 + c, pk + c);
                tmem_st_wait();
            }
            fence_proxy_async();  // generic-proxy smem writes -> visible to the tensor core
            tc_fence_before();
            mbar_arrive(bar_addr(bars->ds_full[it & 1]));
        }
        // Epilogue: warpgroup 0 stores dV, warpgroup 1 stores dK (times scale).
        if (ok && mbar_wait(bar_addr(bars->acc_done), 0, abort_flag, p.status, 63)) {
            tc_fence_after();
            const bool store = kr < p.S;
            const int64_t off = (int64_t)b * p.sb + (int64_t)h * p.sh + (int64_t)kr * p.ss;
            const uint32_t col = g ? C::C_DK : C::C_DV;
            const float mul = g ? p.scale : 1.f;
            __nv_bfloat16* dst = (g ? p.dk : p.dv) + off;
            const bool rope = g == 1 && p.rope_tab != nullptr;
            const float4* tab4 = reinterpret_cast<const float4*>(p.rope_tab + (int64_t)kr * (D / 2));
#pragma unroll
            for (int c = 0; c < D; c += 32) {
                uint32_t v[32];
                tmem_ld32(tl + col + c, v);
                tmem_ld_wait();
                reg_fence<32>(v);
                if (store && rope) {  // dK: pairs (c+2i, c+2i+1) rotated by -theta(kr)
#pragma unroll
                    for (int i2 = 0; i2 < 8; ++i2) {
                        const float4 t = __ldg(tab4 + c / 4 + i2);  // pairs c/2+2*i2, +1
                        float y0, y1, y2, y3;
                        rope_rot_back(__uint_as_float(v[4 * i2]) * mul, __uint_as_float(v[4 * i2 + 1]) * mul,
                                      make_float2(t.x, t.y), y0, y1);
                        rope_rot_back(__uint_as_float(v[4 * i2 + 2]) * mul, __uint_as_float(v[4 * i2 + 3]) * mul,
                                      make_float2(t.z, t.w), y2, y3);
                        v[4 * i2] = __float_as_uint(y0);
                        v[4 * i2 + 1] = __float_as_uint(y1);
                        v[4 * i2 + 2] = __float_as_uint(y2);
                        v[4 * i2 + 3] = __float_as_uint(y3);
                    }
                    uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint4 o;
                        o.x = pack_bf16(__uint_as_float(v[8 * q4 + 0]), __uint_as_float(v[8 * q4 + 1]));
                        o.y = pack_bf16(__uint_as_float(v[8 * q4 + 2]), __uint_as_float(v[8 * q4 + 3]));
                        o.z = pack_bf16(__uint_as_float(v[8 * q4 + 4]), __uint_as_float(v[8 * q4 + 5]));
                        o.w = pack_bf16(__uint_as_float(v[8 * q4 + 6]), __uint_as_float(v[8 * q4 + 7]));
                        d4[q4] = o;
                    }
                } else if (store) {
                    uint4* d4 = reinterpret_cast<uint4*>(dst + c);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint4 o;
                        o.x = pack_bf16(__uint_as_float(v[8 * q4 + 0]) * mul, __uint_as_float(v[8 * q4 + 1]) * mul);
                        o.y = pack_bf16(__uint_as_float(v[8 * q4 + 2]) * mul, __uint_as_float(v[8 * q4 + 3]) * mul);
                        o.z = pack_bf16(__uint_as_float(v[8 * q4 + 4]) * mul, __uint_as_float(v[8 * q4 + 5]) * mul);
                        o.w = pack_bf16(__uint_as_float(v[8 * q4 + 6]) * mul, __uint_as_float(v[8 * q4 + 7]) * mul);
                        d4[q4] = o;
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();
    } else {
        // ------------------------------------------------------------ dQ drain warpgroup
        // Each dQ tile goes TMEM -> registers, then into the f32 accumulator in L2:
        // D=128 by red.global.add from the registers; D=64 through an f32 staging
        // tile in smem that one thread adds with a bulk tensor reduce-add (the TMA
        // unit does the read-modify-write in L2).
        const int wi = warp % 4;
        const int r = wi * 32 + lane;  // TMEM lane: d (dQ^T) or query row (dQ)
        const uint32_t tl = tmem + ((uint32_t)(wi * 32) << 16);
        const bool elected = (warp == 12 && lane == 0);
        for (int it = 0; it < n_it; ++it) {
            const int buf = it % C::NDQ;
            const int q0 = (i_start + it) * BQ;
            if (!mbar_wait(bar_addr(bars->dq_full[buf]), (it / C::NDQ) & 1, abort_flag, p.status, 70)) break;
            tc_fence_after();
            uint32_t v[C::DQ_COLS];
            tmem_ld_cols<C::DQ_COLS>(tl + C::C_DQ0 + (uint32_t)(buf * C::DQ_COLS), v);
            tmem_ld_wait();
            reg_fence<C::DQ_COLS>(v);
            tc_fence_before();
            mbar_arrive(bar_addr(bars->dq_empty[buf]));
            if constexpr (C::DQ_RED) {
                static_assert(C::DQ_T, "the register drain adds dQ^T rows (lane = d)");
                // a warp adds 32 consecutive floats of one query row per instruction
                float* dst = p.dq_acc + ((int64_t)bh * p.S + q0) * D + r;
                const int nq = min(BQ, p.S - q0);
#pragma unroll
                for (int c = 0; c < BQ; ++c)
                    if (c < nq) red_add_f32(dst + (int64_t)c * D, __uint_as_float(v[c]));
            } else {
                static_assert(!C::DQ_T, "the staging drain writes dQ rows (lane = query row)");
                float* stage = (float*)(sm + C::DQS_OFF + (it % C::NDQS) * C::DQS);
                // The reduce-add that used this staging tile (NDQS tiles ago) must
                // have read it; the NDQS - 1 later ones may still be in flight.
                if (elected) {
                    bulk_wait_group_read<C::NDQS - 1>();
                    mbar_arrive(bar_addr(bars->dqs_free));
                }
                if (!mbar_wait(bar_addr(bars->dqs_free), it & 1, abort_flag, p.status, 71)) break;
                // staging = D/32 128B-swizzled boxes [BQ rows][32 floats]; lane r = query row.
#pragma unroll
                for (int cb = 0; cb < D / 32; ++cb) {
                    uint8_t* row = (uint8_t*)stage + cb * (BQ * 128) + r * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        *reinterpret_cast<uint4*>(row + ((j ^ (r & 7)) * 16)) =
                            make_uint4(v[cb * 32 + 4 * j], v[cb * 32 + 4 * j + 1],
                                       v[cb * 32 + 4 * j + 2], v[cb * 32 + 4 * j + 3]);
                }
                fence_proxy_async();
                mbar_arrive(bar_addr(bars->dqs_full));
                if (elected) {
                    if (!mbar_wait(bar_addr(bars->dqs_full), it & 1, abort_flag, p.status, 72)) break;
#pragma unroll
                    for (int cb = 0; cb < D / 32; ++cb)
                        tma_reduce_add_3d(&tdq, smem_addr((uint8_t*)stage + cb * (BQ * 128)), cb * 32,
                                          q0, (int)bh);
                    bulk_commit_group();
                }
            }
        }
        if (elected) bulk_wait_group0();
        tc_fence_before();
        __syncthreads();
    }
}

// Per row (b, h, s) of the padded [B*H][S_pad] tables: lse2 = lse * log2(e)
// and delta = rowsum(dO * O) in f32 (0 for s >= S), and zero the row of the
// dQ accumulator. D/8 lanes per row, 16-byte loads, 32/(D/8) rows per warp,
// grid-stride over row groups.
template <int D>
__global__ void __launch_bounds__(256) bwd_pre_kernel(const __nv_bfloat16* __restrict__ o,
                                                      const __nv_bfloat16* __restrict__ dout,
                                                      const float* __restrict__ lse,
                                                      float* __restrict__ lse2,
                                                      float* __restrict__ delta,
                                                      float* __restrict__ dq_acc, AttnDims d,
                                                      int S_pad) {
    constexpr int G = D / 8;     // lanes per row
    constexpr int RPW = 32 / G;  // rows per warp
    const int64_t rows = (int64_t)d.B * d.H * S_pad;
    const int lane = threadIdx.x % 32, sub = lane % G;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t r0 = ((int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * RPW; r0 < rows;
         r0 += nwarps * RPW) {
        const int64_t r = r0 + lane / G;
        const bool row_ok = r < rows;
        const int s = row_ok ? (int)(r % S_pad) : 0;
        const int64_t bhi = row_ok ? r / S_pad : 0;
        const bool in_seq = row_ok && s < d.S;
        float acc = 0.f;
        if (in_seq) {
            const int hi = (int)(bhi % d.H), bi = (int)(bhi / d.H);
            const int64_t off = (int64_t)bi * d.sb + (int64_t)hi * d.sh + (int64_t)s * d.ss + sub * 8;
            const uint4 a = *reinterpret_cast<const uint4*>(o + off);
            const uint4 g = *reinterpret_cast<const uint4*>(dout + off);
            const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
            const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 x = __bfloat1622float2(a2[i]), y = __bfloat1622float2(g2[i]);
                acc += x.x * y.x + x.y * y.y;
            }
        }
#pragma unroll
        for (int w = G / 2; w > 0; w >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, w);
        if (row_ok && sub == 0) {
            delta[r] = in_seq ? acc : 0.f;
            lse2[r] = in_seq ? lse[bhi * d.S + s] * kLog2e : 0.f;
        }
        if (in_seq) {
            float4* z = reinterpret_cast<float4*>(dq_acc + (bhi * d.S + s) * D) + sub * 2;
            z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
            z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

// dQ = bf16(scale * accumulator); 8 elements per thread.
template <int D>
__global__ void __launch_bounds__(256) bwd_post_kernel(const float* __restrict__ dq_acc,
                                                       __nv_bfloat16* __restrict__ dq, AttnDims d,
                                                       float scale, const float2* __restrict__ rope_tab) {
    const int64_t n8 = (int64_t)d.B * d.H * d.S * (D / 8);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int c8 = (int)(i % (D / 8));
        const int64_t r = i / (D / 8);
        const int s = (int)(r % d.S);
        const int64_t bhi = r / d.S;
        const int hi = (int)(bhi % d.H), bi = (int)(bhi / d.H);
        const float4* src = reinterpret_cast<const float4*>(dq_acc + r * D + c8 * 8);
        const float4 a = src[0], c = src[1];
        float y[8] = {a.x * scale, a.y * scale, a.z * scale, a.w * scale,
                      c.x * scale, c.y * scale, c.z * scale, c.w * scale};
        if (rope_tab != nullptr) {  // dQ rotated back by -theta(s): pairs 4*c8 .. 4*c8+3
            const float4* t4 = reinterpret_cast<const float4*>(rope_tab + (int64_t)s * (D / 2) + 4 * c8);
            const float4 t01 = t4[0], t23 = t4[1];
            const float2 cs[4] = {make_float2(t01.x, t01.y), make_float2(t01.z, t01.w),
                                  make_float2(t23.x, t23.y), make_float2(t23.z, t23.w)};
#pragma unroll
            for (int k = 0; k < 4; ++k) rope_rot_back(y[2 * k], y[2 * k + 1], cs[k], y[2 * k], y[2 * k + 1]);
        }
        uint4 o;
        o.x = ptx::pack_bf16(y[0], y[1]);
        o.y = ptx::pack_bf16(y[2], y[3]);
        o.z = ptx::pack_bf16(y[4], y[5]);
        o.w = ptx::pack_bf16(y[6], y[7]);
        *reinterpret_cast<uint4*>(dq + (int64_t)bi * d.sb + (int64_t)hi * d.sh + (int64_t)s * d.ss +
                                  c8 * 8) = o;
    }
}

uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

// Workspace: lse2 [B*H][S_pad] | delta [B*H][S_pad] | dQ accumulator [B*H][S][D] (f32).
struct BwdWorkspace {
    float* lse2;
    float* delta;
    float* dq_acc;
    int S_pad;
};

BwdWorkspace carve(void* ws, const AttnDims& d) {
    const int S_pad = (d.S + 127) / 128 * 128;
    const uint64_t tab = align256((uint64_t)d.B * d.H * S_pad * 4);
    BwdWorkspace w;
    w.lse2 = (float*)ws;
    w.delta = (float*)((uint8_t*)ws + tab);
    w.dq_acc = (float*)((uint8_t*)ws + 2 * tab);
    w.S_pad = S_pad;
    return w;
}

template <int D>
cudaError_t launch(cudaStream_t st, int sm_count, DeviceStatus* status, const AttnDims& d,
                   const void* q, const void* k, const void* v, const void* o, const void* dout,
                   const float* lse, void* dq, void* dk, void* dv, void* ws, float scale,
                   int causal, const float2* rope_tab) {
    using C = BCfg<D>;
    const BwdWorkspace w = carve(ws, d);
    const int64_t rows_pad = (int64_t)d.B * d.H * w.S_pad;
    int64_t pre_blocks = (rows_pad / (32 / (D / 8)) + 7) / 8;  // 8 warps per block
    if (pre_blocks > (int64_t)sm_count * 16) pre_blocks = (int64_t)sm_count * 16;
    bwd_pre_kernel<D><<<(unsigned)pre_blocks, 256, 0, st>>>(
        (const __nv_bfloat16*)o, (const __nv_bfloat16*)dout, lse, w.lse2, w.delta, w.dq_acc, d,
        w.S_pad);
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;

    CUtensorMap tq, tk, tv, tdo, tdq;
    if (!make_tmap_bhsd(&tq, q, d.B, d.H, d.S, D, d.sb, d.sh, d.ss, 64, C::BQ) ||
        !make_tmap_bhsd(&tdo, dout, d.B, d.H, d.S, D, d.sb, d.sh, d.ss, 64, C::BQ) ||
        !make_tmap_bhsd(&tk, k, d.B, d.H, d.S, D, d.sb, d.sh, d.ss, 64, BK) ||
        !make_tmap_bhsd(&tv, v, d.B, d.H, d.S, D, d.sb, d.sh, d.ss, 64, BK))
        return cudaErrorInvalidValue;
    // dQ accumulator [B*H][S][D] f32 for the bulk reduce-adds of the D=64 drain:
    // two [BQ][32] boxes with 128-byte swizzle (matches the staging writes).
    // The D=128 drain adds from registers and does not read the map.
    memset(&tdq, 0, sizeof tdq);
    if (!C::DQ_RED && !make_tmap_f32_3d(&tdq, w.dq_acc, D, d.S, (uint64_t)d.B * d.H, 32, C::BQ, true))
        return cudaErrorInvalidValue;
    // setmaxnreg.inc waits until the warp's share fits the block's launch
    // allocation: launch only with exactly the register count the split assumes.
    {
        static int regs = -1;
        if (regs < 0) {
            cudaFuncAttributes fa;
            if (cudaFuncGetAttributes(&fa, attn_bwd_kernel<D>) != cudaSuccess) return cudaErrorInvalidDeviceFunction;
            regs = fa.numRegs;
        }
        if (regs != kRegsLaunch) return cudaErrorInvalidConfiguration;
    }
    e = cudaFuncSetAttribute(attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::SMEM);
    if (e != cudaSuccess) return e;
    BwdParams prm;
    prm.lse2 = w.lse2;
    prm.delta = w.delta;
    prm.S_pad = w.S_pad;
    prm.dk = (__nv_bfloat16*)dk;
    prm.dv = (__nv_bfloat16*)dv;
    prm.sb = d.sb;
    prm.sh = d.sh;
    prm.ss = d.ss;
    prm.S = d.S;
    prm.H = d.H;
    prm.scale = scale;
    prm.causal = causal;
    prm.rope_tab = rope_tab;
    prm.hgroup = HX_BWD_HGROUP;
    prm.dq_acc = w.dq_acc;
    prm.status = status;
    const int64_t main_blocks = (int64_t)((d.S + BK - 1) / BK) * d.H * d.B;
    if (main_blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;  // past the grid's x limit
    dim3 grid((unsigned)main_blocks);
    attn_bwd_kernel<D><<<grid, kThreads, C::SMEM, st>>>(tq, tk, tv, tdo, tdq, prm);
    note_launch();
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;

    const int64_t n8 = (int64_t)d.B * d.H * d.S * (D / 8);
    int64_t blocks = (n8 + 255) / 256;
    if (blocks > (int64_t)sm_count * 32) blocks = (int64_t)sm_count * 32;
    bwd_post_kernel<D><<<(unsigned)blocks, 256, 0, st>>>(w.dq_acc, (__nv_bfloat16*)dq, d, scale, rope_tab);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

bool sm100_bwd_supported(hx_dtype dt, const AttnDims& d) {
    return dt == HX_BF16 && (d.D == 64 || d.D == 128);
}

uint64_t sm100_bwd_workspace_bytes(const AttnDims& d) {
    const uint64_t S_pad = (uint64_t)(d.S + 127) / 128 * 128;
    const uint64_t tab = align256((uint64_t)d.B * d.H * S_pad * 4);
    return 2 * tab + align256((uint64_t)d.B * d.H * d.S * (uint64_t)d.D * 4);
}

cudaError_t sm100_attn_bwd(cudaStream_t st, int sm_count, DeviceStatus* status,
                           const AttnDims& d, const void* q, const void* k, const void* v,
                           const void* o, const void* dout, const float* lse, void* dq, void* dk,
                           void* dv, void* workspace, float scale, int causal,
                           const float2* rope_tab) {
    if (d.D == 64)
        return launch<64>(st, sm_count, status, d, q, k, v, o, dout, lse, dq, dk, dv, workspace,
                          scale, causal, rope_tab);
    if (d.D == 128)
        return launch<128>(st, sm_count, status, d, q, k, v, o, dout, lse, dq, dk, dv, workspace,
                           scale, causal, rope_tab);
    return cudaErrorInvalidValue;
}

}  // namespace hx
