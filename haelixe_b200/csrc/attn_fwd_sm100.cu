// tcgen05 (5th-gen tensor core) fused attention forward for sm_100a,
// bf16 Q/K/V/O with f32 accumulation, head_dim 64 or 128, optional causal
// mask, per-row log-sum-exp out. Replaces the reference's scalar WGSL shader
// (src/gpu/shaders/flash_attention.wgsl:19-123, 16x16 tiles, D fixed at 64)
// behind GpuContext::flash_attention_gpu (src/gpu/mod.rs:1336-1418).
//
// One CTA = 384 threads and two 128-row query tiles of one (batch, head):
//   warp 0      TMA producer: Q tiles once, then a K/V ring of STAGES tiles
//               (128 keys each) with 128-byte swizzle; full/empty mbarriers.
//   warp 1      MMA issuer (one thread): S_w = Q_w K_j^T (SS UMMA, M=N=128)
//               into TMEM, then O_w += P_w V_j (TS UMMA: P read from TMEM,
//               V from smem as an MN-major operand). tcgen05.commit signals
//               the consumers and frees K/V slots.
//               Warp 0 also allocates TMEM (512 columns: S0 | S1 | O0 | O1);
//               warps 2-3 only hold registers for the split below.
//   warps 4-7   softmax warpgroup for query tile 0, warps 8-11 for tile 1:
//               lane l of warp w owns query row 32*(w%4)+l of its tile (the
//               TMEM lane quadrant warp w may access), so row
//               max and row sum need no shuffles. P is written back over S
//               as packed bf16, published in two halves (keys 0-63, then
//               64-127) so the first half of PV runs while the second half is
//               still being exponentiated. O is rescaled in TMEM, before any
//               of P(j) is published, only when the running max grows by more
//               than 2^8 (the stale max is exact after the final division by
//               l, which uses the same max). The two warpgroups take turns on
//               the exponentials (ping-pong mbarriers).
// The MMA order S0(j+1) right after PV0(j) lets softmax of one tile overlap
// the tensor core work of the other.
//
// Every mbarrier wait is bounded (sm100_ptx.cuh): on expiry the CTA raises
// an abort flag, records the site in the context's status word, drains its
// own copies and MMAs, frees its TMEM and exits; hx_sync reports
// HX_ERR_TIMEOUT.
#include <math.h>

#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace hx {
namespace {

using namespace ptx;

constexpr int BM = 128;  // query rows per softmax warpgroup (UMMA M)
constexpr int BN = 128;  // keys per K/V tile
constexpr int NWG = 2;   // query tiles (softmax warpgroups) per CTA
constexpr int kThreads = 384;  // control warpgroup + 2 softmax warpgroups
// Register split (setmaxnreg): the launch gives every thread kRegsLaunch;
// the control warpgroup (TMA, MMA, TMEM allocation) drops to kRegsCtl and
// the softmax warpgroups rise to kRegsSoftmax. Per SM sub-partition (one
// control warp + two softmax warps) that is 56 + 2*224 = 504 <= 3*168.
constexpr int kRegsLaunch = 168;
constexpr int kRegsCtl = 56;
constexpr int kRegsSoftmax = 224;
static_assert(128 * kRegsCtl + 256 * kRegsSoftmax <= kThreads * kRegsLaunch,
              "register split exceeds the launch allocation");
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.0f;  // rescale O only when the max grows by > 2^8

template <int D>
struct Cfg {
    static constexpr int CH = D / 64;              // 64-element (128-byte) swizzle chunks per row
    static constexpr int CHUNK = 128 * 128;        // bytes of one 128-row x 128-byte chunk
    static constexpr int TILE = BM * D * 2;        // one 128-row bf16 tile
    static constexpr int STAGES = D == 128 ? 2 : 4;
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = Q_OFF + NWG * TILE;
    static constexpr int V_OFF = K_OFF + STAGES * TILE;
    static constexpr int BAR_OFF = V_OFF + STAGES * TILE;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;  // + barriers + alignment slack
    static constexpr uint32_t S_COL0 = 0, S_COL1 = 128, O_COL0 = 256, O_COL1 = 256 + D;
};

template <int STAGES>
struct Bars {
    uint64_t q_full;
    uint64_t k_full[STAGES], k_empty[STAGES], v_full[STAGES], v_empty[STAGES];
    uint64_t s_full[NWG], p_full[NWG], o_full[NWG];
    uint64_t p_half[NWG];  // P of the tile's first 64 keys is in TMEM
    uint64_t turn[NWG];  // ping-pong token between the softmax warpgroups
    uint64_t done;
    uint32_t tmem_base;
    int abort_flag;
};

// (batch, head) slices per dispatch group of the forward grid.
#ifndef HX_FWD_HGROUP
#define HX_FWD_HGROUP 8
#endif

struct FwdParams {
    __nv_bfloat16* o;
    float* lse;
    int64_t sb, sh, ss;  // o strides (elements)
    int S, H;
    float sl2;  // scale * log2(e)
    int causal;
    int hgroup;  // (batch, head) slices per dispatch group (see the block mapping)
    DeviceStatus* status;
};

static_assert(sizeof(Bars<4>) <= 256, "barrier block");

__device__ __forceinline__ uint32_t bar_addr(const uint64_t& b) { return smem_addr(&b); }

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const FwdParams p) {
    using C = Cfg<D>;
    using B = Bars<C::STAGES>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned base, derived from the shared array itself so that the
    // compiler keeps every access through `sm` in the shared state space.
    uint8_t* sm = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    B* bars = (B*)(sm + C::BAR_OFF);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    // 1D grid in groups of hgroup (batch, head) slices; inside a group the
    // query block varies slowest. The hardware dispatches blocks in index
    // order, so with causal masking the group's heaviest (last) query blocks
    // of all its slices go first and the light ones fill the tail: longest
    // first within a group (even load at the end of the grid), while the
    // blocks in flight touch only a group's worth of K/V (L2 locality).
    const int nblk = (p.S + NWG * BM - 1) / (NWG * BM);
    const int nbh = (int)(gridDim.x / nblk);
    const int grp = (int)(blockIdx.x / ((unsigned)p.hgroup * nblk));
    const int gs = min(p.hgroup, nbh - grp * p.hgroup);
    const int loc = (int)(blockIdx.x - (unsigned)grp * p.hgroup * nblk);
    const int qi = loc / gs, bhi = grp * p.hgroup + loc % gs;
    const int mblk = p.causal ? nblk - 1 - qi : qi;
    const int m0 = mblk * (NWG * BM);
    const int h = bhi % p.H, b = bhi / p.H;
    const int n_all = (p.S + BN - 1) / BN;
    int n_w[NWG];
#pragma unroll
    for (int w = 0; w < NWG; ++w) {
        const int r0 = m0 + w * BM;
        n_w[w] = r0 >= p.S ? 0 : (p.causal ? min(n_all, (r0 + BM - 1) / BN + 1) : n_all);
    }
    const int n_kv = max(n_w[0], n_w[1]);
    volatile int* abort_flag = &bars->abort_flag;

    if (threadIdx.x == 0) {
        bars->abort_flag = 0;
        mbar_init(bar_addr(bars->q_full), 1);
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(bar_addr(bars->k_full[s]), 1);
            mbar_init(bar_addr(bars->k_empty[s]), 1);
            mbar_init(bar_addr(bars->v_full[s]), 1);
            mbar_init(bar_addr(bars->v_empty[s]), 1);
        }
        for (int w = 0; w < NWG; ++w) {
            mbar_init(bar_addr(bars->s_full[w]), 1);
            mbar_init(bar_addr(bars->p_full[w]), BM);
            mbar_init(bar_addr(bars->p_half[w]), BM);
            mbar_init(bar_addr(bars->o_full[w]), 1);
            mbar_init(bar_addr(bars->turn[w]), BM);
        }
        mbar_init(bar_addr(bars->done), 1);
        fence_mbar_init();
        fence_proxy_async();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(&bars->tmem_base), 512);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tq);
        prefetch_tmap(&tk);
        prefetch_tmap(&tv);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kRegsCtl));
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kRegsSoftmax));
    }

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            const uint32_t qb = bar_addr(bars->q_full);
            mbar_arrive_expect_tx(qb, NWG * C::TILE);
            for (int w = 0; w < NWG; ++w)
                for (int c = 0; c < C::CH; ++c)
                    tma_load_4d(smem_addr(sm + C::Q_OFF + w * C::TILE + c * C::CHUNK), &tq, qb,
                                c * 64, m0 + w * BM, h, b);
            int issued = 0;
            for (int j = 0; j < n_kv; ++j) {
                const int st = j % C::STAGES;
                const uint32_t ph = (j / C::STAGES) & 1;
                if (!mbar_wait(bar_addr(bars->k_empty[st]), ph ^ 1, abort_flag, p.status, 10)) break;
                mbar_arrive_expect_tx(bar_addr(bars->k_full[st]), C::TILE);
                for (int c = 0; c < C::CH; ++c)
                    tma_load_4d(smem_addr(sm + C::K_OFF + st * C::TILE + c * C::CHUNK), &tk,
                                bar_addr(bars->k_full[st]), c * 64, j * BN, h, b);
                if (!mbar_wait(bar_addr(bars->v_empty[st]), ph ^ 1, abort_flag, p.status, 11)) {
                    issued = -(j + 1);  // K of tile j in flight, V not
                    break;
                }
                mbar_arrive_expect_tx(bar_addr(bars->v_full[st]), C::TILE);
                for (int c = 0; c < C::CH; ++c)
                    tma_load_4d(smem_addr(sm + C::V_OFF + st * C::TILE + c * C::CHUNK), &tv,
                                bar_addr(bars->v_full[st]), c * 64, j * BN, h, b);
                issued = j + 1;
            }
            // Drain: the last load of every stage has landed before smem is released.
            mbar_wait_drain(qb, 0);
            const int nk = issued >= 0 ? issued : -issued;
            const int nv = issued >= 0 ? issued : -issued - 1;
            for (int j = max(0, nk - C::STAGES); j < nk; ++j)
                mbar_wait_drain(bar_addr(bars->k_full[j % C::STAGES]), (j / C::STAGES) & 1);
            for (int j = max(0, nv - C::STAGES); j < nv; ++j)
                mbar_wait_drain(bar_addr(bars->v_full[j % C::STAGES]), (j / C::STAGES) & 1);
        }
        __syncwarp();
        // Teardown inside each role branch: no code is shared across the
        // register split. Warp 0 releases TMEM once every role is done.
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    } else if (warp < 4) {
        // ------------------------------------------------------------ MMA issuer (warp 1, lane 0)
        if (warp == 1 && lane == 0) {
            constexpr uint32_t idS = idesc_bf16_f32(BM, BN, false, false);
            constexpr uint32_t idO = idesc_bf16_f32(BM, D, false, true);
            // Descriptors are built once; a K step, a stage or a query tile
            // only moves the start address field (bits 0-13, address >> 4).
            // The high word of every descriptor here is the same (SBO 1024,
            // version, 128-byte swizzle); the low word holds the start address
            // >> 4 (and LBO), so a K step, a stage or a query tile is a 32-bit
            // add to a base built once.
            const uint32_t hi = (uint32_t)(sdesc_sw128(0, 16, 1024) >> 32);
            const uint32_t lQ = (uint32_t)sdesc_sw128(smem_addr(sm + C::Q_OFF), 16, 1024);
            const uint32_t lK = (uint32_t)sdesc_sw128(smem_addr(sm + C::K_OFF), 16, 1024);
            const uint32_t lV = (uint32_t)sdesc_sw128(smem_addr(sm + C::V_OFF), C::CHUNK, 1024);
            constexpr uint32_t kTile = C::TILE >> 4;
            auto kmaj = [](int kk) { return (uint32_t)(((kk / 4) * C::CHUNK + (kk % 4) * 32) >> 4); };
            auto issue_S = [&](int w, int st) {
                const uint32_t dS = tmem + (w ? C::S_COL1 : C::S_COL0);
                const uint32_t dq = lQ + w * kTile, dk = lK + st * kTile;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_ss(dS, desc_of(dq + kmaj(kk), hi), desc_of(dk + kmaj(kk), hi), idS, kk > 0);
                umma_commit(bar_addr(bars->s_full[w]));
            };
            // O_w += P_w V_j over the K steps of keys [half*64, half*64+64).
            auto issue_PV = [&](int w, int st, int j, int half) {
                const uint32_t dO = tmem + (w ? C::O_COL1 : C::O_COL0);
                const uint32_t aP = tmem + (w ? C::S_COL1 : C::S_COL0);
                const uint32_t dv = lV + st * kTile;
#pragma unroll
                for (int kk = half * (BN / 32); kk < (half + 1) * (BN / 32); ++kk)
                    umma_ts(dO, aP + kk * 8, desc_of(dv + kk * (2048 >> 4), hi), idO,
                            (j > 0 || kk > 0) ? 1u : 0u);
                if (half) umma_commit(bar_addr(bars->o_full[w]));
            };
            bool ok = mbar_wait(bar_addr(bars->q_full), 0, abort_flag, p.status, 20);
            if (ok && n_kv > 0) {
                ok = mbar_wait(bar_addr(bars->k_full[0]), 0, abort_flag, p.status, 21);
                if (ok) {
                    tc_fence_after();
                    for (int w = 0; w < NWG; ++w)
                        if (n_w[w] > 0) issue_S(w, 0);
                    umma_commit(bar_addr(bars->k_empty[0]));
                }
            }
            for (int j = 0; ok && j < n_kv; ++j) {
                const int st = j % C::STAGES;
                const uint32_t ph = (j / C::STAGES) & 1;
                const int jn = j + 1, stn = jn % C::STAGES;
                const uint32_t phn = (jn / C::STAGES) & 1;
                if (!(ok = mbar_wait(bar_addr(bars->v_full[st]), ph, abort_flag, p.status, 22))) break;
                tc_fence_after();
                bool k_next = false;
                for (int w = 0; w < NWG && ok; ++w) {
                    if (j < n_w[w]) {
                        // The first half of PV runs while the warpgroup is still
                        // exponentiating the tile's last 64 keys.
                        if (!(ok = mbar_wait(bar_addr(bars->p_half[w]), j & 1, abort_flag, p.status, 25)))
                            break;
                        tc_fence_after();
                        issue_PV(w, st, j, 0);
                        if (!(ok = mbar_wait(bar_addr(bars->p_full[w]), j & 1, abort_flag, p.status, 23)))
                            break;
                        tc_fence_after();
                        issue_PV(w, st, j, 1);
                    }
                    if (jn < n_w[w]) {
                        if (!k_next) {
                            if (!(ok = mbar_wait(bar_addr(bars->k_full[stn]), phn, abort_flag, p.status, 24)))
                                break;
                            tc_fence_after();
                            k_next = true;
                        }
                        issue_S(w, stn);
                    }
                }
                umma_commit(bar_addr(bars->v_empty[st]));
                if (k_next) umma_commit(bar_addr(bars->k_empty[stn]));
            }
            // Drain every MMA this thread issued before TMEM is released.
            umma_commit(bar_addr(bars->done));
            mbar_wait_drain(bar_addr(bars->done), 0);
        }
        __syncwarp();
        tc_fence_before();
        __syncthreads();
    } else {
        // ------------------------------------------------------------ softmax
        const int w = (warp - 4) / 4;
        const int wi = warp % 4;
        const int r = wi * 32 + lane;
        const int row = m0 + w * BM + r;
        const uint32_t tl = tmem + ((uint32_t)(wi * 32) << 16);
        const uint32_t tS = tl + (w ? C::S_COL1 : C::S_COL0);
        const uint32_t tO = tl + (w ? C::O_COL1 : C::O_COL0);
        const int nt = n_w[w];
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            if (!(ok = mbar_wait(bar_addr(bars->s_full[w]), j & 1, abort_flag, p.status, 30))) break;
            tc_fence_after();
            uint32_t s[BN];
            tmem_ld32(tS + 0, s);
            tmem_ld32(tS + 32, s + 32);
            tmem_ld32(tS + 64, s + 64);
            tmem_ld32(tS + 96, s + 96);
            tmem_ld_wait();
            reg_fence<BN>(s);
            const int kbase = j * BN;
            const bool need_mask =
                (kbase + BN > p.S) || (p.causal && kbase + BN - 1 > m0 + w * BM);
            if (need_mask) {
                const int lim = p.causal ? min(p.S - 1, row) : p.S - 1;
#pragma unroll
                for (int c = 0; c < BN; ++c)
                    if (kbase + c > lim) s[c] = __float_as_uint(-INFINITY);
            }
            // Two independent three-input max chains.
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int c = 0; c < BN; c += 4) {
                mx0 = max3(mx0, __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
                mx1 = max3(mx1, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]));
            }
            const float mx = fmaxf(mx0, mx1);
            // Ping-pong: the two warpgroups take turns on the exp2 section (the
            // MUFU is shared), so one runs its exps while the tensor core works
            // on the other's PV and next S. Warpgroup 0 goes first on tile j
            // (after warpgroup 1 finished tile j-1), warpgroup 1 after warpgroup 0
            // finished tile j; a warpgroup with no such partner tile does not wait.
            {
                const int other = n_w[w ^ 1];
                const int jt = w == 0 ? j - 1 : j;  // partner tile that must be done
                if (jt >= 0 && jt < other &&
                    !(ok = mbar_wait(bar_addr(bars->turn[w]), jt & 1, abort_flag, p.status, 33)))
                    break;
            }
            const float m_new = fmaxf(m_run, mx * p.sl2);
            float m_use = m_run, alpha = 1.f;
            bool rescale = false;
            if (j == 0) {
                m_use = m_new;
            } else if (m_new > m_run + kRescaleLog2) {
                m_use = m_new;
                alpha = ex2(m_run - m_new);
                rescale = true;
            }
            l_run *= alpha;
            // O is rescaled before any of P(j) is published (PV(j) accumulates
            // onto it). It already holds all of PV(j-1): the MMA thread issued
            // PV(j-1) before S(j), and S(j) has completed.
            if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
                for (int c = 0; c < D; c += 32) {
                    uint32_t o[32];
                    tmem_ld32(tO + c, o);
                    tmem_ld_wait();
                    reg_fence<32>(o);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(tO + c, o);
                }
            }
            // x = s * scale * log2(e) - m and the row sum run two columns per
            // instruction (f32x2); the exponentials stay on the MUFU.
            const uint64_t sl2x2 = f2_pack(p.sl2, p.sl2);
            const uint64_t negx2 = f2_pack(-m_use, -m_use);
            uint64_t sum_a = f2_pack(0.f, 0.f), sum_b = sum_a;
#pragma unroll
            for (int c = 0; c < BN; c += 32) {
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint64_t x = f2_fma(
                        f2_pack(__uint_as_float(s[c + 2 * i]), __uint_as_float(s[c + 2 * i + 1])),
                        sl2x2, negx2);
                    // D=64 has half the MMA work per tile and is bound by the
                    // multi-function unit: one pair in four goes to the FMA pipe.
                    float p0, p1;
                    if (D == 64 && (i & 3) == 3) {
                        f2_unpack(ex2_poly_x2(x), p0, p1);
                    } else {
                        float x0, x1;
                        f2_unpack(x, x0, x1);
                        p0 = ex2(x0);
                        p1 = ex2(x1);
                    }
                    if (i & 1)
                        sum_b = f2_add(sum_b, f2_pack(p0, p1));
                    else
                        sum_a = f2_add(sum_a, f2_pack(p0, p1));
                    pk[i] = pack_bf16(p0, p1);
                }
                tmem_st16(tS + c / 2, pk);
                if (c == BN / 2 - 32) {  // keys [0, 64) done: publish the first half of P
                    tmem_st_wait();
                    tc_fence_before();
                    mbar_arrive(bar_addr(bars->p_half[w]));
                }
            }
            float s0, s1;
            f2_unpack(f2_add(sum_a, sum_b), s0, s1);
            const float sum = s0 + s1;
            mbar_arrive(bar_addr(bars->turn[w ^ 1]));  // the partner's turn
            l_run += sum;
            m_run = m_use;
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(bar_addr(bars->p_full[w]));
        }
        if (ok && nt > 0 &&
            mbar_wait(bar_addr(bars->o_full[w]), (nt - 1) & 1, abort_flag, p.status, 32)) {
            tc_fence_after();
            const float inv = 1.f / l_run;
            const bool store = row < p.S;
            __nv_bfloat16* orow = p.o + (int64_t)b * p.sb + (int64_t)h * p.sh + (int64_t)row * p.ss;
#pragma unroll
            for (int c = 0; c < D; c += 32) {
                uint32_t o[32];
                tmem_ld32(tO + c, o);
                tmem_ld_wait();
                reg_fence<32>(o);
                if (store) {
                    uint4* dst = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        uint4 v;
                        v.x = pack_bf16(__uint_as_float(o[8 * q4 + 0]) * inv, __uint_as_float(o[8 * q4 + 1]) * inv);
                        v.y = pack_bf16(__uint_as_float(o[8 * q4 + 2]) * inv, __uint_as_float(o[8 * q4 + 3]) * inv);
                        v.z = pack_bf16(__uint_as_float(o[8 * q4 + 4]) * inv, __uint_as_float(o[8 * q4 + 5]) * inv);
                        v.w = pack_bf16(__uint_as_float(o[8 * q4 + 6]) * inv, __uint_as_float(o[8 * q4 + 7]) * inv);
                        dst[q4] = v;
                    }
                }
            }
            if (store)
                p.lse[((int64_t)b * p.H + h) * p.S + row] = (m_run + __log2f(l_run)) * kLn2;
        }
        tc_fence_before();
        __syncthreads();
    }
}

template <int D>
cudaError_t launch(cudaStream_t st, DeviceStatus* status, const AttnDims& d, const void* q,
                   const void* k, const void* v, void* o, float* lse, float scale, int causal) {
    using C = Cfg<D>;
    CUtensorMap tq, tk, tv;
    if (!make_tmap_bhsd(&tq, q, d.B, d.H, d.S, D, d.sb, d.sh, d.ss, 64, BM) ||
        !make_tmap_bhsd(&tk, k, d.B, d.H, d.S, D, d.sb, d.sh, d.ss, 64, BN) ||
        !make_tmap_bhsd(&tv, v, d.B, d.H, d.S, D, d.sb, d.sh, d.ss, 64, BN))
        return cudaErrorInvalidValue;
    // setmaxnreg.inc waits until the warp's share fits the block's launch
    // allocation: launch only with exactly the register count the split assumes.
    {
        static int regs = -1;
        if (regs < 0) {
            cudaFuncAttributes fa;
            if (cudaFuncGetAttributes(&fa, attn_fwd_kernel<D>) != cudaSuccess) return cudaErrorInvalidDeviceFunction;
            regs = fa.numRegs;
        }
        if (regs != kRegsLaunch) return cudaErrorInvalidConfiguration;
    }
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    FwdParams prm;
    prm.o = (__nv_bfloat16*)o;
    prm.lse = lse;
    prm.sb = d.sb;
    prm.sh = d.sh;
    prm.ss = d.ss;
    prm.S = d.S;
    prm.H = d.H;
    prm.sl2 = scale * kLog2e;
    prm.causal = causal;
    prm.hgroup = HX_FWD_HGROUP;
    prm.status = status;
    const int64_t blocks = (int64_t)((d.S + NWG * BM - 1) / (NWG * BM)) * d.H * d.B;
    if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;  // past the grid's x limit
    dim3 grid((unsigned)blocks);
    attn_fwd_kernel<D><<<grid, kThreads, C::SMEM, st>>>(tq, tk, tv, prm);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

bool sm100_supported(hx_dtype dt, const AttnDims& d) {
    return dt == HX_BF16 && (d.D == 64 || d.D == 128);
}

cudaError_t sm100_attn_fwd(cudaStream_t st, int /*sm_count*/, DeviceStatus* status,
                           const AttnDims& d, const void* q, const void* k, const void* v,
                           void* o, float* lse, float scale, int causal) {
    if (d.D == 64) return launch<64>(st, status, d, q, k, v, o, lse, scale, causal);
    if (d.D == 128) return launch<128>(st, status, d, q, k, v, o, lse, scale, causal);
    return cudaErrorInvalidValue;
}

}  // namespace hx
