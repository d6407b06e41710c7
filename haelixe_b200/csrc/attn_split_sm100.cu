// f32 attention on the tcgen05 tensor cores by operand splitting (sm_100a):
// the f32-I/O path of GpuContext::flash_attention_gpu (src/gpu/mod.rs:1336-1418)
// and FlashAttentionOp::backward (src/ops/flash_attention.rs:16-39), whose
// arithmetic the reference does in f32 (src/gpu/shaders/flash_attention.wgsl:
// 19-123, src/tensor.rs:395-397), for head_dim 64 and 128.
//
// Every f32 operand x travels as two fp16 planes of y = x * 2^e, hi = f16(y)
// and lo = f16(y - hi), where the power of two 2^e brings the operand's
// largest magnitude into [2^14, 2^15): |y - hi| <= 2^-11 |y| and lo keeps 11
// more bits, so hi + lo = y (1 + r) with |r| <= 2^-22 (elements below 2^-17
// of the largest keep an absolute error under 2^-39 of it). A product A.B is
// three f16 UMMAs into one f32 TMEM accumulator,
//     A_hi.B_lo + A_lo.B_hi + A_hi.B_hi,
// the dropped A_lo.B_lo being at most 2^-22 |A||B| per term, and the scales
// come off exactly (powers of two) where the accumulators are read. That is
// the precision of a 3xTF32 split at the f16-kind MMA rate (twice kind::tf32)
// and two bytes per plane element, which is what lets Q, K and V of both
// planes stay on chip at head_dim 128. (bf16 planes would carry only 16 bits:
// 2^-16 per operand, too coarse for the 1e-3 bound on weight gradients of
// magnitude ~100 that the f32 layer's tests hold.)
//
// Scales: Q, K, V, dO per tensor from their max-abs (split_stats); P by 2^14
// in the backward (P <= 1) and 2^6 in the forward (P <= 2^8 under lazy
// rescaling); dS by the bound |dS| <= |dP| + |delta| <= 2 D max|dO| max|V|
// (O is a convex combination of V rows). Elements far below a bound keep an
// absolute error under 2^-39 of it, so a loose bound costs no precision that
// matters.
//
//   split_stats max-abs of each f32 operand.
//   split_pre   f32 Q, K, V (and dO) -> contiguous f16 hi/lo planes
//               [B*H][S][D]; in the backward also lse * log2(e),
//               delta = rowsum(dO * O) in f32, and dQ, dK, dV := 0.
//   fwd         two 128-row query tiles per CTA, K/V rings of BN-key tiles:
//               S = Q K^T (SS), P = exp2(S*scale*log2e - m) written back over
//               S as packed hi | lo f16, O += P V (TS, P from TMEM); online
//               softmax with lazy rescaling and ping-pong warpgroups.
//   bwd         one CTA per 128-key tile, K and V resident, looping over query
//               tiles of BQ rows: S^T = K Q^T, dP^T = V dO^T, P^T and
//               dS^T = P^T (dP^T - delta) as hi | lo in TMEM, dV += P^T dO,
//               dK += dS^T Q (TS), dQ from an smem dS tile, added into the f32
//               dQ output by a drain warpgroup (red.global.add). Q and dO
//               have a stage each, released separately (dO after dV, Q after
//               dK), and the MMA order lets the next Q load run behind dK and
//               the next dP^T. dV and dK accumulate in TMEM over segments of
//               2048 queries, each added into the f32 outputs.
//
// Every mbarrier wait is bounded (sm100_ptx.cuh): on expiry the CTA raises an
// abort flag, records the site in the context's status word, drains its own
// copies and MMAs, frees its TMEM and exits; hx_sync reports HX_ERR_TIMEOUT.
#include <math.h>
#include <string.h>

#include <cuda_fp16.h>

#include <algorithm>
#include <initializer_list>

#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace hx {
namespace {

using namespace ptx;

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ uint32_t bar_addr(const uint64_t& b) { return smem_addr(&b); }

// Four consecutive f32 atomic adds in one 16-byte reduction (addr 16-byte aligned).
__device__ __forceinline__ void red_add_v4_f32(float* addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// Packed f16 pair, round to nearest even; the low half holds `lo`.
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ float f16_lo(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xffffu))); }
__device__ __forceinline__ float f16_hi(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

// (a, b) scaled by the power of two s -> packed f16 hi = (f16(a s), f16(b s))
// and lo = (f16(a s - hi_a), f16(b s - hi_b)); the low halves hold a. The
// differences a s - hi_a are exact in f32.
__device__ __forceinline__ void split2(float a, float b, float s, uint32_t& hi, uint32_t& lo) {
    const float ya = a * s, yb = b * s;
    hi = pack_f16(ya, yb);
    lo = pack_f16(ya - f16_lo(hi), yb - f16_hi(hi));
}

// Power of two that brings a non-negative magnitude m (as f32 bits) into
// [2^14, 2^15): 2^(14 - floor(log2 m)); 1 for 0, inf or NaN, and clamped to
// stay a normal f32.
__host__ __device__ __forceinline__ float pow2_scale(uint32_t bits) {
    const int ex = (int)((bits >> 23) & 0xffu);
    if (bits == 0u || ex == 0xff) return 1.f;
    int e = 14 - (ex - 127);
    e = e < -120 ? -120 : (e > 120 ? 120 : e);
    union {
        uint32_t u;
        float f;
    } r;
    r.u = (uint32_t)(e + 127) << 23;
    return r.f;
}
// P planes: the backward's P = exp2(s - lse) is at most 1 and goes in scaled
// by 2^14; the forward's P is relative to a running max that may lag the true
// one by up to 2^kRescaleLog2 = 2^8 (lazy rescaling), so it goes in by 2^6.
constexpr float kPScaleBwd = 16384.f;
constexpr float kPScaleFwd = 64.f;

// Instruction descriptor of a kind::f16 UMMA with f16 A and B (format 0) and
// f32 accumulation: the bf16 descriptor with both operand formats cleared.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn_major, bool b_mn_major) {
    return idesc_bf16_f32(M, N, a_mn_major, b_mn_major) & ~((1u << 7) | (1u << 10));
}

// Operand statistics (device, zeroed before split_stats): f32 bits of the
// max-abs of q, k, v, dout.
struct Stats {
    uint32_t maxabs[4];
};

// Scale of the dS planes from the bound |dS| <= 2 D max|dO| max|V|.
template <int D>
__device__ __forceinline__ float ds_scale(const Stats* st) {
    const float b = 2.f * (float)D * __uint_as_float(st->maxabs[3]) * __uint_as_float(st->maxabs[2]);
    return pow2_scale(__float_as_uint(b));
}

// One f32 operand as its two f16 planes, each contiguous [B*H][S][D].
struct Planes {
    __half* hi;
    __half* lo;
};

struct PreParams {
    const float* src[4];  // q, k, v, dout: strided like AttnDims
    Planes dst[4];
    int n;                // operands to split: 3 (forward) or 4 (backward)
    const float* o;       // backward: O, for delta; null in the forward
    const float* lse;     // backward: [B*H][S]
    float* lse2;          // backward: [B*H][S_pad] lse * log2(e), 0 past S
    float* delta;         // backward: [B*H][S_pad] rowsum(dO * O), 0 past S
    float* dq;            // backward: zeroed, strided like the operands
    float* dk;            // backward: zeroed (the kernel adds dK segments)
    float* dv;            // backward: zeroed (the kernel adds dV segments)
    Stats* stats;         // written by split_stats, read by split_pre
    int S_pad;
};

template <bool VEC>
__device__ __forceinline__ float4 load4(const float* p) {
    if (VEC) return *reinterpret_cast<const float4*>(p);
    return make_float4(p[0], p[1], p[2], p[3]);
}

// Max-abs of each operand: D/4 lanes per row (one float4 each), grid-stride
// over the rows [B*H][S], two rows per lane group per iteration; per-thread
// running maxima (no cross-lane work in the loop), reduced over the block and
// added with one atomicMax per block and operand (non-negative f32 values
// order like their bits). The grid is four blocks per SM: one atomic per warp
// on the same four words had made this pass twice as slow as the split.
template <int D, bool VEC>
__global__ void __launch_bounds__(256) split_stats_kernel(const PreParams p, const AttnDims d) {
    constexpr int G = D / 4;
    constexpr int RPW = 32 / G;
    const int64_t rows = (int64_t)d.B * d.H * d.S;
    const int lane = threadIdx.x % 32, sub = lane % G;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x / 32);
    float mabs[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t r0 = ((int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * RPW; r0 < rows;
         r0 += 2 * nwarps * RPW) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int64_t r = r0 + u * nwarps * RPW + lane / G;
            if (r >= rows) continue;
            // rows < 2^32 (checked on the host): 32-bit divisions
            const uint32_t bhi = (uint32_t)r / (uint32_t)d.S;
            const uint32_t s = (uint32_t)r - bhi * (uint32_t)d.S;
            const uint32_t bb = bhi / (uint32_t)d.H, hh = bhi - bb * (uint32_t)d.H;
            const int64_t off = (int64_t)bb * d.sb + (int64_t)hh * d.sh + (int64_t)s * d.ss + sub * 4;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                if (t < p.n) {
                    const float4 x = load4<VEC>(p.src[t] + off);
                    mabs[t] = fmaxf(mabs[t], fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
                }
            }
        }
    }
    __shared__ float red[8][4];  // [warp][operand]; 256 threads
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        float a = mabs[t];
#pragma unroll
        for (int w = 16; w > 0; w >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, w));
        if (lane == 0) red[threadIdx.x / 32][t] = a;
    }
    __syncthreads();
    if (threadIdx.x < (unsigned)p.n) {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) a = fmaxf(a, red[w][threadIdx.x]);
        atomicMax(&p.stats->maxabs[threadIdx.x], __float_as_uint(a));
    }
}

// D/4 lanes per row (one float4 each), 32/(D/4) rows per warp, grid-stride
// over the padded rows [B*H][S_pad].
template <int D, bool VEC>
__global__ void __launch_bounds__(256) split_pre_kernel(const PreParams p, const AttnDims d) {
    constexpr int G = D / 4;
    constexpr int RPW = 32 / G;
    const int64_t rows = (int64_t)d.B * d.H * p.S_pad;
    const int lane = threadIdx.x % 32, sub = lane % G;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x / 32);
    const bool bwd = p.o != nullptr;
    float sc[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) sc[t] = pow2_scale(p.stats->maxabs[t]);
    for (int64_t r0 = ((int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32) * RPW; r0 < rows;
         r0 += nwarps * RPW) {
        const int64_t r = r0 + lane / G;
        const bool row_ok = r < rows;
        // rows < 2^32 (checked on the host): 32-bit divisions
        const uint32_t bhi = row_ok ? (uint32_t)r / (uint32_t)p.S_pad : 0u;
        const int s = row_ok ? (int)((uint32_t)r - bhi * (uint32_t)p.S_pad) : 0;
        const bool in_seq = row_ok && s < d.S;
        float acc = 0.f;
        if (in_seq) {
            const uint32_t bb = bhi / (uint32_t)d.H, hh = bhi - bb * (uint32_t)d.H;
            const int64_t off = (int64_t)bb * d.sb + (int64_t)hh * d.sh + (int64_t)s * d.ss + sub * 4;
            const int64_t poff = ((int64_t)bhi * d.S + s) * D + sub * 4;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                if (t < p.n) {
                    const float4 x = load4<VEC>(p.src[t] + off);
                    uint2 hi, lo;
                    split2(x.x, x.y, sc[t], hi.x, lo.x);
                    split2(x.z, x.w, sc[t], hi.y, lo.y);
                    *reinterpret_cast<uint2*>(p.dst[t].hi + poff) = hi;
                    *reinterpret_cast<uint2*>(p.dst[t].lo + poff) = lo;
                }
            }
            if (bwd) {
                const float4 a = load4<VEC>(p.o + off), g = load4<VEC>(p.src[3] + off);
                acc = fmaf(a.x, g.x, fmaf(a.y, g.y, fmaf(a.z, g.z, a.w * g.w)));
                float* zs[3] = {p.dq + off, p.dk + off, p.dv + off};
#pragma unroll
                for (int zi = 0; zi < 3; ++zi) {
                    float* z = zs[zi];
                    if (VEC) {
                        *reinterpret_cast<float4*>(z) = make_float4(0.f, 0.f, 0.f, 0.f);
                    } else {
                        z[0] = 0.f;
                        z[1] = 0.f;
                        z[2] = 0.f;
                        z[3] = 0.f;
                    }
                }
            }
        }
        if (bwd) {
#pragma unroll
            for (int w = G / 2; w > 0; w >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, w);
            if (row_ok && sub == 0) {
                p.delta[r] = in_seq ? acc : 0.f;
                p.lse2[r] = in_seq ? p.lse[(int64_t)bhi * d.S + s] * kLog2e : 0.f;
            }
        }
    }
}

// ============================================================================ forward
namespace fwd {

constexpr int BM = 128;         // query rows per softmax warpgroup (UMMA M)
constexpr int NWG = 2;          // query tiles (softmax warpgroups) per CTA
constexpr int kThreads = 384;   // control warpgroup + 2 softmax warpgroups
// setmaxnreg split: the launch gives every thread kRegsLaunch; per SM
// sub-partition (one control warp + two softmax warps) the shares in Cfg add
// up to at most 3 * kRegsLaunch.
constexpr int kRegsLaunch = 168;
constexpr float kRescaleLog2 = 8.0f;  // rescale O only when the max grows by > 2^8

template <int D>
struct Cfg {
    static constexpr int BN = D == 128 ? 64 : 128;  // keys per K/V tile
    static constexpr int KST = 2;                    // K ring stages
    static constexpr int VST = D == 128 ? 1 : 2;     // V ring stages
    static constexpr int CHQ = BM * 128;             // 64-column (128-byte) chunk of a Q plane tile
    static constexpr int CHK = BN * 128;             // ... of a K or V plane tile
    static constexpr int QT = BM * D * 2;            // one plane of a query tile
    static constexpr int KT = BN * D * 2;            // one plane of a key tile
    static constexpr int Q_OFF = 0;                          // [tile][plane]
    static constexpr int K_OFF = Q_OFF + NWG * 2 * QT;       // [stage][plane]
    static constexpr int V_OFF = K_OFF + KST * 2 * KT;       // [stage][plane]
    static constexpr int BAR_OFF = V_OFF + VST * 2 * KT;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;        // + barriers + alignment slack
    static_assert(SMEM <= 232448, "shared memory per block");
    // TMEM: S_w (BN columns; P_w lands on them as hi | lo) and O_w (D columns).
    static constexpr uint32_t S_COL0 = 0, S_COL1 = BN, O_COL0 = 2 * BN, O_COL1 = 2 * BN + D;
    static_assert(O_COL1 + D <= 512, "TMEM budget");
    // Control (the MMA issuer keeps a dozen descriptor bases live) vs softmax
    // (BN scores per thread); the smallest split with no spills.
    static constexpr int REGS_CTL = D == 128 ? 96 : 80;
    static constexpr int REGS_SOFTMAX = D == 128 ? 200 : 208;
    static_assert(128 * REGS_CTL + 256 * REGS_SOFTMAX <= kThreads * kRegsLaunch, "register split");
};

struct Bars {
    uint64_t q_full;
    uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
    uint64_t s_full[NWG], p_full[NWG], o_full[NWG];
    uint64_t turn[NWG];    // ping-pong token between the softmax warpgroups
    uint64_t done;
    uint32_t tmem_base;
    int abort_flag;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

struct Params {
    float* o;
    float* lse;
    int64_t sb, sh, ss;  // o strides (elements)
    int S, H;
    float sl2;  // scale * log2(e)
    int causal;
    int hgroup;  // (batch, head) slices per dispatch group
    int vec;     // o rows 16-byte aligned: float4 stores
    const Stats* stats;  // plane scales of q, k, v
    DeviceStatus* status;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_split_kernel(const __grid_constant__ CUtensorMap tqh, const __grid_constant__ CUtensorMap tql,
                          const __grid_constant__ CUtensorMap tkh, const __grid_constant__ CUtensorMap tkl,
                          const __grid_constant__ CUtensorMap tvh, const __grid_constant__ CUtensorMap tvl,
                          const Params p) {
    using C = Cfg<D>;
    constexpr int BN = C::BN;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    Bars* bars = (Bars*)(sm + C::BAR_OFF);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    // Block mapping: groups of hgroup (batch, head) slices, the query block
    // varying slowest inside a group and, with causal masking, heaviest first.
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
        for (int s = 0; s < 2; ++s) {
            mbar_init(bar_addr(bars->k_full[s]), 1);
            mbar_init(bar_addr(bars->k_empty[s]), 1);
            mbar_init(bar_addr(bars->v_full[s]), 1);
            mbar_init(bar_addr(bars->v_empty[s]), 1);
        }
        for (int w = 0; w < NWG; ++w) {
            mbar_init(bar_addr(bars->s_full[w]), 1);
            mbar_init(bar_addr(bars->p_full[w]), BM);
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
        prefetch_tmap(&tqh);
        prefetch_tmap(&tql);
        prefetch_tmap(&tkh);
        prefetch_tmap(&tkl);
        prefetch_tmap(&tvh);
        prefetch_tmap(&tvl);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(C::REGS_CTL));
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(C::REGS_SOFTMAX));
    }

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            const uint32_t qb = bar_addr(bars->q_full);
            mbar_arrive_expect_tx(qb, NWG * 2 * C::QT);
            for (int w = 0; w < NWG; ++w)
                for (int pl = 0; pl < 2; ++pl)
                    for (int c = 0; c < D / 64; ++c)
                        tma_load_4d(smem_addr(sm + C::Q_OFF + (w * 2 + pl) * C::QT + c * C::CHQ),
                                    pl ? &tql : &tqh, qb, c * 64, m0 + w * BM, h, b);
            int nk = 0, nv = 0;
            for (int j = 0; j < n_kv; ++j) {
                const int sk = j % C::KST, sv = j % C::VST;
                const uint32_t kf = bar_addr(bars->k_full[sk]), vf = bar_addr(bars->v_full[sv]);
                if (!mbar_wait(bar_addr(bars->k_empty[sk]), ((j / C::KST) & 1) ^ 1, abort_flag, p.status, 110))
                    break;
                mbar_arrive_expect_tx(kf, 2 * C::KT);
                for (int pl = 0; pl < 2; ++pl)
                    for (int c = 0; c < D / 64; ++c)
                        tma_load_4d(smem_addr(sm + C::K_OFF + (sk * 2 + pl) * C::KT + c * C::CHK),
                                    pl ? &tkl : &tkh, kf, c * 64, j * BN, h, b);
                nk = j + 1;
                if (!mbar_wait(bar_addr(bars->v_empty[sv]), ((j / C::VST) & 1) ^ 1, abort_flag, p.status, 111))
                    break;
                mbar_arrive_expect_tx(vf, 2 * C::KT);
                for (int pl = 0; pl < 2; ++pl)
                    for (int c = 0; c < D / 64; ++c)
                        tma_load_4d(smem_addr(sm + C::V_OFF + (sv * 2 + pl) * C::KT + c * C::CHK),
                                    pl ? &tvl : &tvh, vf, c * 64, j * BN, h, b);
                nv = j + 1;
            }
            // Drain: the last load into every stage has landed before smem is released.
            mbar_wait_drain(qb, 0);
            for (int j = max(0, nk - C::KST); j < nk; ++j)
                mbar_wait_drain(bar_addr(bars->k_full[j % C::KST]), (j / C::KST) & 1);
            for (int j = max(0, nv - C::VST); j < nv; ++j)
                mbar_wait_drain(bar_addr(bars->v_full[j % C::VST]), (j / C::VST) & 1);
        }
        __syncwarp();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    } else if (warp < 4) {
        // ------------------------------------------------------------ MMA issuer (warp 1, lane 0)
        if (warp == 1 && lane == 0) {
            constexpr uint32_t idS = idesc_f16(BM, BN, false, false);
            constexpr uint32_t idO = idesc_f16(BM, D, false, true);
            // Every descriptor shares the high word (SBO 1024, 128-byte swizzle);
            // a plane, stage, tile or K step only moves the start address in the
            // low word, so each is a 32-bit add to a base built once.
            const uint32_t hi = (uint32_t)(sdesc_sw128(0, 16, 1024) >> 32);
            const uint32_t lQ = (uint32_t)sdesc_sw128(smem_addr(sm + C::Q_OFF), 16, 1024);
            const uint32_t lK = (uint32_t)sdesc_sw128(smem_addr(sm + C::K_OFF), 16, 1024);
            const uint32_t lV = (uint32_t)sdesc_sw128(smem_addr(sm + C::V_OFF), C::CHK, 1024);
            auto kmaj = [](int kk, int chunk) { return (uint32_t)(((kk / 4) * chunk + (kk % 4) * 32) >> 4); };
            // S_w = Q_w K^T as Q_hi K_lo + Q_lo K_hi + Q_hi K_hi.
            auto issue_S = [&](int w, int sk) {
                const uint32_t dS = tmem + (w ? C::S_COL1 : C::S_COL0);
                const uint32_t qh = lQ + (uint32_t)((w * 2 * C::QT) >> 4), ql = qh + (C::QT >> 4);
                const uint32_t kh = lK + (uint32_t)((sk * 2 * C::KT) >> 4), kl = kh + (C::KT >> 4);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_ss(dS, desc_of(qh + kmaj(kk, C::CHQ), hi), desc_of(kl + kmaj(kk, C::CHK), hi), idS,
                            kk > 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_ss(dS, desc_of(ql + kmaj(kk, C::CHQ), hi), desc_of(kh + kmaj(kk, C::CHK), hi), idS, 1u);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    umma_ss(dS, desc_of(qh + kmaj(kk, C::CHQ), hi), desc_of(kh + kmaj(kk, C::CHK), hi), idS, 1u);
                umma_commit(bar_addr(bars->s_full[w]));
            };
            // O_w += P_w V over the K steps of keys [half*BN/2, (half+1)*BN/2):
            // P_hi V_lo + P_lo V_hi + P_hi V_hi, P from TMEM (hi at the S columns'
            // start, lo BN/2 columns on), V as an MN-major operand.
            auto issue_PV = [&](int w, int sv, int j, int half) {
                const uint32_t dO = tmem + (w ? C::O_COL1 : C::O_COL0);
                const uint32_t aP = tmem + (w ? C::S_COL1 : C::S_COL0);
                const uint32_t vh = lV + (uint32_t)((sv * 2 * C::KT) >> 4), vl = vh + (C::KT >> 4);
#pragma unroll
                for (int kk = half * (BN / 32); kk < (half + 1) * (BN / 32); ++kk) {
                    const uint32_t ah = aP + kk * 8, al = ah + BN / 2, off = kk * (2048 >> 4);
                    umma_ts(dO, ah, desc_of(vl + off, hi), idO, (j > 0 || kk > 0) ? 1u : 0u);
                    umma_ts(dO, al, desc_of(vh + off, hi), idO, 1u);
                    umma_ts(dO, ah, desc_of(vh + off, hi), idO, 1u);
                }
                if (half) umma_commit(bar_addr(bars->o_full[w]));
            };
            bool ok = mbar_wait(bar_addr(bars->q_full), 0, abort_flag, p.status, 120);
            if (ok && n_kv > 0) {
                ok = mbar_wait(bar_addr(bars->k_full[0]), 0, abort_flag, p.status, 121);
                if (ok) {
                    tc_fence_after();
                    for (int w = 0; w < NWG; ++w)
                        if (n_w[w] > 0) issue_S(w, 0);
                    umma_commit(bar_addr(bars->k_empty[0]));
                }
            }
            for (int j = 0; ok && j < n_kv; ++j) {
                const int sv = j % C::VST;
                const int jn = j + 1, skn = jn % C::KST;
                if (!(ok = mbar_wait(bar_addr(bars->v_full[sv]), (j / C::VST) & 1, abort_flag, p.status, 122)))
                    break;
                tc_fence_after();
                bool k_next = false;
                for (int w = 0; w < NWG && ok; ++w) {
                    if (j < n_w[w]) {
                        // P is published once per tile: with 64-key tiles two
                        // hand-offs per tile cost more than the early half won
                        // (forward 3.93-3.95 -> 3.76-3.81 ms at D=64, -1.5 % at D=128).
                        if (!(ok = mbar_wait(bar_addr(bars->p_full[w]), j & 1, abort_flag, p.status, 123)))
                            break;
                        tc_fence_after();
                        issue_PV(w, sv, j, 0);
                        issue_PV(w, sv, j, 1);
                    }
                    if (jn < n_w[w]) {
                        if (!k_next) {
                            if (!(ok = mbar_wait(bar_addr(bars->k_full[skn]), (jn / C::KST) & 1, abort_flag,
                                                 p.status, 124)))
                                break;
                            tc_fence_after();
                            k_next = true;
                        }
                        issue_S(w, skn);
                    }
                }
                umma_commit(bar_addr(bars->v_empty[sv]));
                if (k_next) umma_commit(bar_addr(bars->k_empty[skn]));
            }
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
        // S leaves the MMA scaled by sq * sk and O by kPScaleFwd * sv (powers of two).
        const float sq = pow2_scale(p.stats->maxabs[0]), sk = pow2_scale(p.stats->maxabs[1]),
                    sv = pow2_scale(p.stats->maxabs[2]);
        const float sl2 = p.sl2 / (sq * sk);
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; ++j) {
            if (!(ok = mbar_wait(bar_addr(bars->s_full[w]), j & 1, abort_flag, p.status, 130))) break;
            tc_fence_after();
            uint32_t s[BN];
#pragma unroll
            for (int c = 0; c < BN; c += 32) tmem_ld32(tS + c, s + c);
            tmem_ld_wait();
            reg_fence<BN>(s);
            const int kbase = j * BN;
            const bool need_mask = (kbase + BN > p.S) || (p.causal && kbase + BN - 1 > m0 + w * BM);
            if (need_mask) {
                const int lim = p.causal ? min(p.S - 1, row) : p.S - 1;
#pragma unroll
                for (int c = 0; c < BN; ++c)
                    if (kbase + c > lim) s[c] = __float_as_uint(-INFINITY);
            }
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int c = 0; c < BN; c += 4) {
                mx0 = max3(mx0, __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
                mx1 = max3(mx1, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]));
            }
            const float mx = fmaxf(mx0, mx1);
            // Ping-pong on the exponentials: warpgroup 0 takes tile j after
            // warpgroup 1 finished tile j-1, warpgroup 1 after warpgroup 0
            // finished tile j; with no such partner tile there is no wait.
            {
                const int other = n_w[w ^ 1];
                const int jt = w == 0 ? j - 1 : j;
                if (jt >= 0 && jt < other &&
                    !(ok = mbar_wait(bar_addr(bars->turn[w]), jt & 1, abort_flag, p.status, 133)))
                    break;
            }
            const float m_new = fmaxf(m_run, mx * sl2);
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
            // O holds all of PV(j-1) (issued before S(j), which completed) and
            // is rescaled before any of P(j) is published.
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
            const uint64_t sl2x2 = f2_pack(sl2, sl2);
            const uint64_t negx2 = f2_pack(-m_use, -m_use);
            uint64_t sum_a = f2_pack(0.f, 0.f), sum_b = sum_a;
            // P as hi | lo planes over the S columns: hi packed into columns
            // [0, BN/2), lo into [BN/2, BN); all of S is already in registers.
#pragma unroll
            for (int c = 0; c < BN; c += 32) {
                uint32_t ph[16], pl[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint64_t x = f2_fma(
                        f2_pack(__uint_as_float(s[c + 2 * i]), __uint_as_float(s[c + 2 * i + 1])), sl2x2, negx2);
                    float x0, x1;
                    f2_unpack(x, x0, x1);
                    const float p0 = ex2(x0), p1 = ex2(x1);
                    if (i & 1)
                        sum_b = f2_add(sum_b, f2_pack(p0, p1));
                    else
                        sum_a = f2_add(sum_a, f2_pack(p0, p1));
                    split2(p0, p1, kPScaleFwd, ph[i], pl[i]);
                }
                tmem_st16(tS + c / 2, ph);
                tmem_st16(tS + BN / 2 + c / 2, pl);
            }
            float s0, s1;
            f2_unpack(f2_add(sum_a, sum_b), s0, s1);
            mbar_arrive(bar_addr(bars->turn[w ^ 1]));
            l_run += s0 + s1;
            m_run = m_use;
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(bar_addr(bars->p_full[w]));
        }
        if (ok && nt > 0 && mbar_wait(bar_addr(bars->o_full[w]), (nt - 1) & 1, abort_flag, p.status, 132)) {
            tc_fence_after();
            const float inv = 1.f / (l_run * kPScaleFwd * sv);
            const bool store = row < p.S;
            float* orow = p.o + (int64_t)b * p.sb + (int64_t)h * p.sh + (int64_t)row * p.ss;
#pragma unroll
            for (int c = 0; c < D; c += 32) {
                uint32_t o[32];
                tmem_ld32(tO + c, o);
                tmem_ld_wait();
                reg_fence<32>(o);
                if (store) {
                    if (p.vec) {
                        float4* dst = reinterpret_cast<float4*>(orow + c);
#pragma unroll
                        for (int q4 = 0; q4 < 8; ++q4)
                            dst[q4] = make_float4(__uint_as_float(o[4 * q4]) * inv, __uint_as_float(o[4 * q4 + 1]) * inv,
                                                  __uint_as_float(o[4 * q4 + 2]) * inv,
                                                  __uint_as_float(o[4 * q4 + 3]) * inv);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) orow[c + i] = __uint_as_float(o[i]) * inv;
                    }
                }
            }
            if (store) p.lse[((int64_t)b * p.H + h) * p.S + row] = (m_run + __log2f(l_run)) * kLn2;
        }
        tc_fence_before();
        __syncthreads();
    }
}

}  // namespace fwd

// ============================================================================ backward
namespace bwd {

constexpr int BK = 128;  // keys per CTA (UMMA M of S^T, dP^T, dV, dK)
constexpr int kThreads = 512;
// setmaxnreg split per SM sub-partition, one warp of each group: control +
// 2 x P/dS + dQ drain = 4 x the launch's 128.
// The MMA issuer keeps about twenty descriptor bases live: below 128
// registers it spills.
constexpr int kRegsLaunch = 128;
constexpr int kRegsCtl = 128;
constexpr int kRegsCompute = 152;
constexpr int kRegsDrain = 80;
// dV and dK accumulate in TMEM over segments of at most this many queries,
// then the drain warpgroup adds the partial sums into the f32 outputs (zeroed
// by split_pre; RN f32 reductions in L2, fire-and-forget, beside the P/dS work
// of the next tile) and the next segment starts from zero: the error of the
// tensor core's long accumulations (which grew with S: dV 2.4e-4 at S = 16384
// without segments) stays that of a 2048-query sum. Segments of 1024 queries
// cost 5 % of the backward at C3 (two alternations), 2048 about half that.
constexpr int kFlushQueries = 2048;
static_assert(kRegsCtl + 2 * kRegsCompute + kRegsDrain == 4 * kRegsLaunch, "register split");

template <int D>
struct Cfg {
    static constexpr int BQ = D == 128 ? 64 : 128;  // queries per inner tile
    // D=128: dQ^T = K^T dS^T (UMMA M = D); D=64: dQ = dS K (M = BQ). Either
    // way M = 128 and the accumulator has one row per TMEM lane.
    static constexpr bool DQ_T = D == 128;
    static constexpr int HC = BQ / 2;         // query columns per P/dS warpgroup
    static constexpr int FLUSH = kFlushQueries / BQ;  // query tiles per dV/dK segment
    static constexpr int CHK = BK * 128;      // 64-column (128-byte) chunk of a K/V plane tile
    static constexpr int CHQ = BQ * 128;      // ... of a Q/dO plane tile
    static constexpr int CHDS = BK * 128;     // ... of a dS plane tile (64 queries wide)
    static constexpr int KT = BK * D * 2;     // one plane of the K (or V) tile
    static constexpr int QT = BQ * D * 2;     // one plane of a Q (or dO) tile
    static constexpr int DST = BK * BQ * 2;   // one plane of the dS tile
    static constexpr int K_OFF = 0;           // each region: [plane]
    static constexpr int V_OFF = K_OFF + 2 * KT;
    static constexpr int Q_OFF = V_OFF + 2 * KT;
    static constexpr int DO_OFF = Q_OFF + 2 * QT;
    static constexpr int DS_OFF = DO_OFF + 2 * QT;
    static constexpr int LSE_OFF = DS_OFF + 2 * DST;
    static constexpr int DEL_OFF = LSE_OFF + BQ * 4;
    static constexpr int BAR_OFF = DEL_OFF + BQ * 4;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;
    static_assert(SMEM <= 232448, "shared memory per block");
    // TMEM: S^T (BQ columns; P^T lands on them as hi | lo per warpgroup half),
    // dP^T (BQ; then dS^T as hi | lo), the dQ tile, dV and dK.
    static constexpr int DQ_COLS = DQ_T ? BQ : D;
    static constexpr uint32_t C_S = 0, C_DP = BQ, C_DQ = 2 * BQ, C_DV = C_DQ + DQ_COLS, C_DK = C_DV + D;
    static_assert(C_DK + D <= 512, "TMEM budget");
};

struct Bars {
    uint64_t kv_full;
    uint64_t q_full, q_empty;    // Q hi/lo, lse and delta of a query tile
    uint64_t do_full, do_empty;  // dO hi/lo of a query tile (released earlier, after dV)
    uint64_t s_full, dp_full, p_full, ds_full;
    uint64_t dsfree;  // smem dS tile read by dQ (-> P/dS warpgroups)
    uint64_t flush_ready, flush_done;  // dV/dK segment complete (-> drain) / added to the outputs (-> MMA)
    uint64_t dq_full, dq_empty;
    uint64_t acc_done, done;
    uint32_t tmem_base;
    int abort_flag;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

struct Params {
    const float* lse2;   // [B*H][S_pad]: lse * log2(e), 0 past S
    const float* delta;  // [B*H][S_pad]: rowsum(dO * O), 0 past S
    int S_pad;
    float* dq;  // zeroed by split_pre; the drain adds scale * dQ tiles into it
    float* dk;
    float* dv;
    int64_t sb, sh, ss;  // strides of dq/dk/dv (elements)
    int S, H;
    float scale;
    int causal;
    int hgroup;  // (batch, head) slices per dispatch group
    int vec;     // dk/dv rows 16-byte aligned: float4 stores
    const Stats* stats;  // plane scales of q, k, v, dout and the dS bound
    DeviceStatus* status;
};

// dst[0, D) += m * (this lane's D accumulator columns from taddr): TMEM ->
// registers in 32-column pieces, then f32 reductions (16-byte ones when the
// row is aligned) that no later instruction waits for.
template <int D>
__device__ __forceinline__ void add_rows(uint32_t taddr, float m, float* dst, bool valid, bool vec) {
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
        uint32_t v[32];
        tmem_ld32(taddr + c, v);
        tmem_ld_wait();
        reg_fence<32>(v);
        if (!valid) continue;
        if (vec) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
                red_add_v4_f32(dst + c + i, __uint_as_float(v[i]) * m, __uint_as_float(v[i + 1]) * m,
                               __uint_as_float(v[i + 2]) * m, __uint_as_float(v[i + 3]) * m);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) red_add_f32(dst + c + i, __uint_as_float(v[i]) * m);
        }
    }
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_split_kernel(const __grid_constant__ CUtensorMap tkh, const __grid_constant__ CUtensorMap tkl,
                          const __grid_constant__ CUtensorMap tvh, const __grid_constant__ CUtensorMap tvl,
                          const __grid_constant__ CUtensorMap tqh, const __grid_constant__ CUtensorMap tql,
                          const __grid_constant__ CUtensorMap tdoh, const __grid_constant__ CUtensorMap tdol,
                          const Params p) {
    using C = Cfg<D>;
    constexpr int BQ = C::BQ, HC = C::HC;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    Bars* bars = (Bars*)(sm + C::BAR_OFF);
    float* s_lse = (float*)(sm + C::LSE_OFF);
    float* s_del = (float*)(sm + C::DEL_OFF);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    // Groups of hgroup (batch, head) slices, the key block varying slowest
    // inside a group; with causal masking the heaviest (first) key blocks go first.
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
        mbar_init(bar_addr(bars->q_full), 1);
        mbar_init(bar_addr(bars->q_empty), 1);
        mbar_init(bar_addr(bars->do_full), 1);
        mbar_init(bar_addr(bars->do_empty), 1);
        mbar_init(bar_addr(bars->s_full), 1);
        mbar_init(bar_addr(bars->dp_full), 1);
        mbar_init(bar_addr(bars->p_full), 256);
        mbar_init(bar_addr(bars->ds_full), 256);
        mbar_init(bar_addr(bars->dsfree), 1);
        mbar_init(bar_addr(bars->flush_ready), 1);
        mbar_init(bar_addr(bars->flush_done), 128);
        mbar_init(bar_addr(bars->dq_full), 1);
        mbar_init(bar_addr(bars->dq_empty), 128);
        mbar_init(bar_addr(bars->acc_done), 1);
        mbar_init(bar_addr(bars->done), 1);
        fence_mbar_init();
        fence_proxy_async();
    }
    if (warp == 2) {
        tmem_alloc(smem_addr(&bars->tmem_base), 512);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tkh);
        prefetch_tmap(&tkl);
        prefetch_tmap(&tvh);
        prefetch_tmap(&tvl);
        prefetch_tmap(&tqh);
        prefetch_tmap(&tql);
        prefetch_tmap(&tdoh);
        prefetch_tmap(&tdol);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    if (warp < 4) {
        if constexpr (kRegsCtl < kRegsLaunch) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kRegsCtl));
    } else if (warp < 12) {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kRegsCompute));
    } else {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kRegsDrain));
    }

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint32_t kvb = bar_addr(bars->kv_full);
            mbar_arrive_expect_tx(kvb, 4 * C::KT);
            for (int pl = 0; pl < 2; ++pl)
                for (int c = 0; c < D / 64; ++c) {
                    tma_load_4d(smem_addr(sm + C::K_OFF + pl * C::KT + c * C::CHK), pl ? &tkl : &tkh, kvb, c * 64,
                                k0, h, b);
                    tma_load_4d(smem_addr(sm + C::V_OFF + pl * C::KT + c * C::CHK), pl ? &tvl : &tvh, kvb, c * 64,
                                k0, h, b);
                }
            // One stage each: dO(it) once dV(it-1) has read dO(it-1), then Q(it)
            // with its lse and delta rows once dK(it-1) has read Q(it-1).
            int nq = 0, ndo = 0;
            for (int it = 0; it < n_it; ++it) {
                const int q0 = (i_start + it) * BQ;
                if (!mbar_wait(bar_addr(bars->do_empty), (it & 1) ^ 1, abort_flag, p.status, 141)) break;
                const uint32_t db = bar_addr(bars->do_full);
                mbar_arrive_expect_tx(db, 2 * C::QT);
                for (int pl = 0; pl < 2; ++pl)
                    for (int c = 0; c < D / 64; ++c)
                        tma_load_4d(smem_addr(sm + C::DO_OFF + pl * C::QT + c * C::CHQ), pl ? &tdol : &tdoh, db,
                                    c * 64, q0, h, b);
                ndo = it + 1;
                if (!mbar_wait(bar_addr(bars->q_empty), (it & 1) ^ 1, abort_flag, p.status, 140)) break;
                const uint32_t qb = bar_addr(bars->q_full);
                mbar_arrive_expect_tx(qb, 2 * C::QT + 2 * BQ * 4);
                for (int pl = 0; pl < 2; ++pl)
                    for (int c = 0; c < D / 64; ++c)
                        tma_load_4d(smem_addr(sm + C::Q_OFF + pl * C::QT + c * C::CHQ), pl ? &tql : &tqh, qb,
                                    c * 64, q0, h, b);
                const int64_t row0 = bh * p.S_pad + q0;
                bulk_load(smem_addr(s_lse), p.lse2 + row0, BQ * 4, qb);
                bulk_load(smem_addr(s_del), p.delta + row0, BQ * 4, qb);
                nq = it + 1;
            }
            mbar_wait_drain(kvb, 0);
            if (nq > 0) mbar_wait_drain(bar_addr(bars->q_full), (nq - 1) & 1);
            if (ndo > 0) mbar_wait_drain(bar_addr(bars->do_full), (ndo - 1) & 1);
        }
        __syncwarp();
        tc_fence_before();
        __syncthreads();
    } else if (warp < 4) {
        // ------------------------------------------------------------ MMA issuer (warp 1, lane 0)
        // Order: S^T(0), dP^T(0); then per query tile it: dV(it) once P^T is in
        // TMEM (releases dO), dK(it) once dS^T is (releases Q), dP^T(it+1),
        // S^T(it+1), dQ(it). The reload of Q(it+1) runs behind dK(it) and
        // dP^T(it+1), and dQ(it) behind the P phase of tile it+1. Each product
        // is hi.lo + lo.hi + hi.hi over the two planes.
        if (warp == 1 && lane == 0) {
            constexpr uint32_t idSP = idesc_f16(BK, BQ, false, false);
            constexpr uint32_t idAcc = idesc_f16(BK, D, false, true);
            constexpr uint32_t idDQ = C::DQ_T ? idesc_f16(D, BQ, true, true) : idesc_f16(BQ, D, true, true);
            constexpr int NS = D / 16;   // K steps of S^T, dP^T
            constexpr int NA = BQ / 16;  // K steps of dV, dK
            constexpr int NQ = BK / 16;  // K steps of dQ
            constexpr int KH = HC / 16;  // K steps of dV/dK per warpgroup half
            const uint32_t hi = (uint32_t)(sdesc_sw128(0, 16, 1024) >> 32);
            auto lo_of = [](const uint8_t* a, uint32_t lbo) { return (uint32_t)sdesc_sw128(smem_addr(a), lbo, 1024); };
            // K-major bases (A of S^T / dP^T, B of S^T / dP^T) and MN-major bases
            // (B of dV / dK, both operands of dQ); plane 1 is one tile further on.
            const uint32_t kK = lo_of(sm + C::K_OFF, 16), kV = lo_of(sm + C::V_OFF, 16),
                           kQ = lo_of(sm + C::Q_OFF, 16), kDO = lo_of(sm + C::DO_OFF, 16);
            const uint32_t mK = lo_of(sm + C::K_OFF, C::CHK), mQ = lo_of(sm + C::Q_OFF, C::CHQ),
                           mDO = lo_of(sm + C::DO_OFF, C::CHQ), mDS = lo_of(sm + C::DS_OFF, C::CHDS);
            constexpr uint32_t pK = C::KT >> 4, pQ = C::QT >> 4, pDS = C::DST >> 4;
            auto kmaj = [](int kk, int chunk) { return (uint32_t)(((kk / 4) * chunk + (kk % 4) * 32) >> 4); };
            auto mnmaj = [](int kk) { return (uint32_t)((kk * 2048) >> 4); };
            // hi column of K step kk of P^T / dS^T: warpgroup g packed its HC
            // queries as hi into [g*HC, g*HC + HC/2) and lo into the next HC/2.
            auto acc_a = [](int kk) { return (uint32_t)((kk / KH) * HC + (kk % KH) * 8); };
            // A (K-major, chunk ca) x B (K-major, chunk cb) over nk steps, three terms.
            auto kk3 = [&](uint32_t d, uint32_t a, uint32_t a_pl, int ca, uint32_t bb, uint32_t b_pl, int cb, int nk,
                           uint32_t id) {
                for (int kk = 0; kk < nk; ++kk)
                    umma_ss(d, desc_of(a + kmaj(kk, ca), hi), desc_of(bb + b_pl + kmaj(kk, cb), hi), id, kk > 0);
                for (int kk = 0; kk < nk; ++kk)
                    umma_ss(d, desc_of(a + a_pl + kmaj(kk, ca), hi), desc_of(bb + kmaj(kk, cb), hi), id, 1u);
                for (int kk = 0; kk < nk; ++kk)
                    umma_ss(d, desc_of(a + kmaj(kk, ca), hi), desc_of(bb + kmaj(kk, cb), hi), id, 1u);
            };
            // D += A^T(TMEM, hi | lo) x B (MN-major, plane offset b_pl) over NA steps.
            auto ts3 = [&](uint32_t d, uint32_t a_col, uint32_t bb, uint32_t b_pl, bool first) {
                for (int kk = 0; kk < NA; ++kk) {
                    const uint32_t ah = tmem + a_col + acc_a(kk), al = ah + HC / 2;
                    umma_ts(d, ah, desc_of(bb + b_pl + mnmaj(kk), hi), idAcc, (first && kk == 0) ? 0u : 1u);
                    umma_ts(d, al, desc_of(bb + mnmaj(kk), hi), idAcc, 1u);
                    umma_ts(d, ah, desc_of(bb + mnmaj(kk), hi), idAcc, 1u);
                }
            };
            // S^T = K Q^T overwrites P^T(it-1), which dV(it-1), issued earlier by
            // this thread, has read; dP^T = V dO^T likewise after dK(it-1).
            auto issue_S = [&](int it) {
                if (!mbar_wait(bar_addr(bars->q_full), it & 1, abort_flag, p.status, 151)) return false;
                tc_fence_after();
                kk3(tmem + C::C_S, kK, pK, C::CHK, kQ, pQ, C::CHQ, NS, idSP);
                umma_commit(bar_addr(bars->s_full));
                return true;
            };
            auto issue_DP = [&](int it) {
                if (!mbar_wait(bar_addr(bars->do_full), it & 1, abort_flag, p.status, 156)) return false;
                tc_fence_after();
                kk3(tmem + C::C_DP, kV, pK, C::CHK, kDO, pQ, C::CHQ, NS, idSP);
                umma_commit(bar_addr(bars->dp_full));
                return true;
            };
            bool ok = mbar_wait(bar_addr(bars->kv_full), 0, abort_flag, p.status, 150);
            if (ok && n_it > 0) ok = issue_S(0) && issue_DP(0);
            for (int it = 0; ok && it < n_it; ++it) {
                // A new dV/dK segment starts from zero once the last one is in the outputs.
                const bool first = (it % C::FLUSH) == 0;
                if (first && it > 0 &&
                    !(ok = mbar_wait(bar_addr(bars->flush_done), (it / C::FLUSH - 1) & 1, abort_flag, p.status,
                                     157)))
                    break;
                if (!(ok = mbar_wait(bar_addr(bars->p_full), it & 1, abort_flag, p.status, 152))) break;
                tc_fence_after();
                ts3(tmem + C::C_DV, C::C_S, mDO, pQ, first);  // dV += P^T dO
                umma_commit(bar_addr(bars->do_empty));        // dO(it) is read by nothing after dV(it)
                if (!(ok = mbar_wait(bar_addr(bars->ds_full), it & 1, abort_flag, p.status, 154))) break;
                tc_fence_after();
                ts3(tmem + C::C_DK, C::C_DP, mQ, pQ, first);  // dK += dS^T Q
                // Q(it), lse and delta are read by nothing after dK(it).
                umma_commit(bar_addr(bars->q_empty));
                if (it % C::FLUSH == C::FLUSH - 1 && it + 1 < n_it) umma_commit(bar_addr(bars->flush_ready));
                if (it + 1 < n_it && !(ok = issue_DP(it + 1) && issue_S(it + 1))) break;
                if (!(ok = mbar_wait(bar_addr(bars->dq_empty), (it & 1) ^ 1, abort_flag, p.status, 155))) break;
                tc_fence_after();
                const uint32_t dq = tmem + C::C_DQ;
                // D=128: dQ^T = K^T dS^T; D=64: dQ = dS K. Both operands MN-major.
                const uint32_t a0 = C::DQ_T ? mK : mDS, b0 = C::DQ_T ? mDS : mK;
                const uint32_t apl = C::DQ_T ? pK : pDS, bpl = C::DQ_T ? pDS : pK;
                for (int kk = 0; kk < NQ; ++kk)
                    umma_ss(dq, desc_of(a0 + mnmaj(kk), hi), desc_of(b0 + bpl + mnmaj(kk), hi), idDQ, kk > 0);
                for (int kk = 0; kk < NQ; ++kk)
                    umma_ss(dq, desc_of(a0 + apl + mnmaj(kk), hi), desc_of(b0 + mnmaj(kk), hi), idDQ, 1u);
                for (int kk = 0; kk < NQ; ++kk)
                    umma_ss(dq, desc_of(a0 + mnmaj(kk), hi), desc_of(b0 + mnmaj(kk), hi), idDQ, 1u);
                umma_commit(bar_addr(bars->dq_full));
                umma_commit(bar_addr(bars->dsfree));
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
        // Warpgroup g (warps 4-7: g=0, 8-11: g=1) owns query columns
        // [g*HC, (g+1)*HC) of every tile; thread = key row = TMEM lane.
        const int g = (warp - 4) / 4;
        const int wi = warp % 4;
        const int r = wi * 32 + lane;
        const int kr = k0 + r;
        const uint32_t tl = tmem + ((uint32_t)(wi * 32) << 16);
        // S^T leaves the MMA scaled by sk * sq, dP^T by sv * sdo; P^T and dS^T
        // go in scaled by kPScaleBwd and sds (powers of two: exact).
        const float sq = pow2_scale(p.stats->maxabs[0]), sk = pow2_scale(p.stats->maxabs[1]),
                    sv = pow2_scale(p.stats->maxabs[2]), sdo = pow2_scale(p.stats->maxabs[3]);
        const float sds = ds_scale<D>(p.stats);
        const float sl2 = p.scale * kLog2e / (sk * sq);
        const float dpu = 1.f / (sv * sdo);
        const int c0 = g * HC;
        // Warpgroup 0 adds the last segment of dV, warpgroup 1 that of dK
        // (times scale): this thread's key row, into the zeroed outputs.
        const uint32_t acc_col = g ? C::C_DK : C::C_DV;
        const float acc_mul = g ? p.scale / (sds * sq) : 1.f / (kPScaleBwd * sdo);
        float* acc_dst = (g ? p.dk : p.dv) + (int64_t)b * p.sb + (int64_t)h * p.sh + (int64_t)kr * p.ss;
        // The last segment is added like the earlier ones (drain warpgroup).
        auto flush = [&]() { add_rows<D>(tl + acc_col, acc_mul, acc_dst, kr < p.S, p.vec != 0); };
        bool ok = true;
        for (int it = 0; it < n_it; ++it) {
            const int q0 = (i_start + it) * BQ;
            if (!(ok = mbar_wait(bar_addr(bars->q_full), it & 1, abort_flag, p.status, 160))) break;
            if (!(ok = mbar_wait(bar_addr(bars->s_full), it & 1, abort_flag, p.status, 161))) break;
            tc_fence_after();
            const float* lse2 = s_lse + c0;
            const float* del = s_del + c0;
            // Valid columns [lo, hi) of this row: q < S, key < S, causal q >= key.
            const bool need_mask = (q0 + BQ > p.S) || (k0 + BK > p.S) || (p.causal && k0 + BK - 1 > q0);
            int lo = 0, hi = HC;
            if (need_mask) {
                hi = kr < p.S ? min(HC, p.S - q0 - c0) : 0;
                if (p.causal) lo = max(0, kr - q0 - c0);
            }
            uint32_t x[HC];
#pragma unroll
            for (int c = 0; c < HC; c += 32) tmem_ld32(tl + C::C_S + c0 + c, x + c);
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
            // P^T hi | lo over this warpgroup's S^T columns (all loaded above).
#pragma unroll
            for (int c = 0; c < HC; c += 32) {
                uint32_t ph[16], pl[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) split2(pr[c + 2 * i], pr[c + 2 * i + 1], kPScaleBwd, ph[i], pl[i]);
                tmem_st16(tl + C::C_S + c0 + c / 2, ph);
                tmem_st16(tl + C::C_S + c0 + HC / 2 + c / 2, pl);
            }
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(bar_addr(bars->p_full));

            if (!(ok = mbar_wait(bar_addr(bars->dp_full), it & 1, abort_flag, p.status, 162))) break;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < HC; c += 32) tmem_ld32(tl + C::C_DP + c0 + c, x + c);
            tmem_ld_wait();
            reg_fence<HC>(x);
            // dS^T = P^T (dP^T - delta), in place of P^T.
#pragma unroll
            for (int q4 = 0; q4 < HC / 4; ++q4) {
                const float4 d4 = reinterpret_cast<const float4*>(del)[q4];
                pr[4 * q4 + 0] *= fmaf(__uint_as_float(x[4 * q4 + 0]), dpu, -d4.x);
                pr[4 * q4 + 1] *= fmaf(__uint_as_float(x[4 * q4 + 1]), dpu, -d4.y);
                pr[4 * q4 + 2] *= fmaf(__uint_as_float(x[4 * q4 + 2]), dpu, -d4.z);
                pr[4 * q4 + 3] *= fmaf(__uint_as_float(x[4 * q4 + 3]), dpu, -d4.w);
            }
            // The smem dS tile is free once dQ(it - 1) has read it.
            if (!(ok = mbar_wait(bar_addr(bars->dsfree), (it & 1) ^ 1, abort_flag, p.status, 164))) break;
#pragma unroll
            for (int c = 0; c < HC; c += 32) {
                uint32_t dh[16], dl[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) split2(pr[c + 2 * i], pr[c + 2 * i + 1], sds, dh[i], dl[i]);
                // dS^T hi | lo in TMEM over the dP^T columns (A of dK) ...
                tmem_st16(tl + C::C_DP + c0 + c / 2, dh);
                tmem_st16(tl + C::C_DP + c0 + HC / 2 + c / 2, dl);
                // ... and in the 128-byte-swizzled smem tile dQ reads: 16-byte
                // piece u of the row of 64-column chunk k holds columns k*64+8u..+7.
#pragma unroll
                for (int u8 = 0; u8 < 4; ++u8) {
                    const int col = c0 + c + 8 * u8;
                    const int chunk = col / 64, u = (col % 64) / 8;
                    uint8_t* row = sm + C::DS_OFF + chunk * C::CHDS + r * 128 + ((u ^ (r & 7)) * 16);
                    *reinterpret_cast<uint4*>(row) =
                        make_uint4(dh[4 * u8], dh[4 * u8 + 1], dh[4 * u8 + 2], dh[4 * u8 + 3]);
                    *reinterpret_cast<uint4*>(row + C::DST) =
                        make_uint4(dl[4 * u8], dl[4 * u8 + 1], dl[4 * u8 + 2], dl[4 * u8 + 3]);
                }
            }
            tmem_st_wait();
            fence_proxy_async();  // generic-proxy smem writes -> visible to the tensor core
            tc_fence_before();
            mbar_arrive(bar_addr(bars->ds_full));
        }
        // Epilogue: the last segment of dV / dK.
        if (ok && mbar_wait(bar_addr(bars->acc_done), 0, abort_flag, p.status, 163)) {
            tc_fence_after();
            flush();
        }
        tc_fence_before();
        __syncthreads();
    } else {
        // ------------------------------------------------------------ dQ drain warpgroup
        // Each dQ tile goes TMEM -> registers -> red.global.add of scale * dQ
        // into the f32 dQ output (zeroed by split_pre); D=128 lanes are head
        // dims (a warp instruction adds 32 consecutive floats of one query
        // row), D=64 lanes are query rows.
        const int wi = warp % 4;
        const int r = wi * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(wi * 32) << 16);
        float* base = p.dq + (int64_t)b * p.sb + (int64_t)h * p.sh;
        const float mul = p.scale / (ds_scale<D>(p.stats) * pow2_scale(p.stats->maxabs[1]));  // dQ = scale dS K
        // Segment flushes: lane r holds key row k0 + r of the dV and dK accumulators.
        const int kr = k0 + r;
        const float mul_dv = 1.f / (kPScaleBwd * pow2_scale(p.stats->maxabs[3]));
        const float mul_dk = p.scale / (ds_scale<D>(p.stats) * pow2_scale(p.stats->maxabs[0]));
        const int64_t row_off = (int64_t)b * p.sb + (int64_t)h * p.sh + (int64_t)kr * p.ss;

        for (int it = 0; it < n_it; ++it) {
            const int q0 = (i_start + it) * BQ;
            if (it % C::FLUSH == C::FLUSH - 1 && it + 1 < n_it) {  // a dV/dK segment is complete
                if (!mbar_wait(bar_addr(bars->flush_ready), (it / C::FLUSH) & 1, abort_flag, p.status, 165)) break;
                tc_fence_after();
                add_rows<D>(tl + C::C_DV, mul_dv, p.dv + row_off, kr < p.S, p.vec != 0);
                add_rows<D>(tl + C::C_DK, mul_dk, p.dk + row_off, kr < p.S, p.vec != 0);
                tc_fence_before();
                mbar_arrive(bar_addr(bars->flush_done));
            }
            if (!mbar_wait(bar_addr(bars->dq_full), it & 1, abort_flag, p.status, 170)) break;
            tc_fence_after();
            uint32_t v[C::DQ_COLS];
#pragma unroll
            for (int c = 0; c < C::DQ_COLS; c += 32) tmem_ld32(tl + C::C_DQ + c, v + c);
            tmem_ld_wait();
            reg_fence<C::DQ_COLS>(v);
            tc_fence_before();
            mbar_arrive(bar_addr(bars->dq_empty));
            if constexpr (C::DQ_T) {
                const int nq = min(BQ, p.S - q0);
                float* dst = base + (int64_t)q0 * p.ss + r;
#pragma unroll
                for (int c = 0; c < BQ; ++c)
                    if (c < nq) red_add_f32(dst + (int64_t)c * p.ss, __uint_as_float(v[c]) * mul);
            } else {
                if (q0 + r < p.S) {  // one query row per thread: 16-byte vector adds when aligned
                    float* dst = base + (int64_t)(q0 + r) * p.ss;
                    if (p.vec) {
#pragma unroll
                        for (int c = 0; c < D; c += 4)
                            red_add_v4_f32(dst + c, __uint_as_float(v[c]) * mul, __uint_as_float(v[c + 1]) * mul,
                                           __uint_as_float(v[c + 2]) * mul, __uint_as_float(v[c + 3]) * mul);
                    } else {
#pragma unroll
                        for (int c = 0; c < D; ++c) red_add_f32(dst + c, __uint_as_float(v[c]) * mul);
                    }
                }
            }
        }
        tc_fence_before();
        __syncthreads();
    }
}

}  // namespace bwd

// ============================================================================ host side
uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

uint64_t plane_bytes(const AttnDims& d) { return align256((uint64_t)d.B * d.H * d.S * (uint64_t)d.D * 2); }

int s_pad_of(const AttnDims& d) { return (d.S + 127) / 128 * 128; }

uint64_t table_bytes(const AttnDims& d) { return align256((uint64_t)d.B * d.H * s_pad_of(d) * 4); }

// Workspace: the Stats block (256 bytes), then n operands x (hi, lo) planes,
// 256-byte aligned each.
constexpr uint64_t kStatsBytes = 256;
static_assert(sizeof(Stats) <= kStatsBytes, "stats block");

Stats* carve_planes(void* ws, const AttnDims& d, int n, Planes* out) {
    uint8_t* p = (uint8_t*)ws + kStatsBytes;
    const uint64_t pb = plane_bytes(d);
    for (int i = 0; i < n; ++i) {
        out[i].hi = (__half*)p;
        p += pb;
        out[i].lo = (__half*)p;
        p += pb;
    }
    return (Stats*)ws;
}

// float4 access to every operand row: 16-byte aligned bases, strides in
// multiples of 4 elements.
bool vec_ok(const AttnDims& d, std::initializer_list<const void*> ptrs) {
    if (d.ss % 4 || d.sh % 4 || d.sb % 4) return false;
    for (const void* p : ptrs)
        if (((uintptr_t)p & 15u) != 0) return false;
    return true;
}

// A plane [B][H][S][D] (contiguous f16) as a TMA map with box (64, rows).
bool plane_map(CUtensorMap* m, const __half* base, const AttnDims& d, int rows) {
    return make_tmap_bhsd(m, base, d.B, d.H, d.S, d.D, (int64_t)d.H * d.S * d.D, (int64_t)d.S * d.D, d.D, 64,
                          rows, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
}

int64_t pre_blocks(int64_t rows, int D, int sm_count) {
    int64_t blocks = (rows / (32 / (D / 4)) + 7) / 8;  // 8 warps per block
    if (blocks > (int64_t)sm_count * 16) blocks = (int64_t)sm_count * 16;
    return blocks < 1 ? 1 : blocks;
}

// Zeroes the Stats block, gathers the operand statistics, then writes the planes.
template <int D>
cudaError_t launch_pre(cudaStream_t st, int sm_count, const PreParams& pp, const AttnDims& d, bool vec) {
    if ((uint64_t)d.B * d.H * pp.S_pad >= (1ull << 32)) return cudaErrorInvalidConfiguration;  // 32-bit row index
    cudaError_t e = cudaMemsetAsync(pp.stats, 0, sizeof(Stats), st);
    if (e != cudaSuccess) return e;
    const int64_t sb = std::min<int64_t>(pre_blocks((int64_t)d.B * d.H * d.S, D, sm_count), 4 * (int64_t)sm_count);
    if (vec)
        split_stats_kernel<D, true><<<(unsigned)sb, 256, 0, st>>>(pp, d);
    else
        split_stats_kernel<D, false><<<(unsigned)sb, 256, 0, st>>>(pp, d);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int64_t pb = pre_blocks((int64_t)d.B * d.H * pp.S_pad, D, sm_count);
    if (vec)
        split_pre_kernel<D, true><<<(unsigned)pb, 256, 0, st>>>(pp, d);
    else
        split_pre_kernel<D, false><<<(unsigned)pb, 256, 0, st>>>(pp, d);
    note_launch();
    return cudaGetLastError();
}

// setmaxnreg.inc waits until the warp's share fits the block's launch
// allocation: launch only with exactly the register count the split assumes.
template <typename K>
cudaError_t check_regs(K kernel, int want, int* cache) {
    if (*cache < 0) {
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess) return cudaErrorInvalidDeviceFunction;
        *cache = fa.numRegs;
    }
    return *cache == want ? cudaSuccess : cudaErrorInvalidConfiguration;
}

template <int D>
cudaError_t launch_fwd(cudaStream_t st, int sm_count, DeviceStatus* status, const AttnDims& d, const float* q,
                       const float* k, const float* v, float* o, float* lse, float scale, int causal, void* ws) {
    using C = fwd::Cfg<D>;
    Planes pl[3];
    Stats* stats = carve_planes(ws, d, 3, pl);
    PreParams pp;
    memset(&pp, 0, sizeof pp);
    pp.stats = stats;
    pp.src[0] = q;
    pp.src[1] = k;
    pp.src[2] = v;
    for (int i = 0; i < 3; ++i) pp.dst[i] = pl[i];
    pp.n = 3;
    pp.S_pad = d.S;
    const bool vec = vec_ok(d, {q, k, v, o});
    cudaError_t e = launch_pre<D>(st, sm_count, pp, d, vec);
    if (e != cudaSuccess) return e;
    CUtensorMap m[6];
    if (!plane_map(&m[0], pl[0].hi, d, fwd::BM) || !plane_map(&m[1], pl[0].lo, d, fwd::BM) ||
        !plane_map(&m[2], pl[1].hi, d, C::BN) || !plane_map(&m[3], pl[1].lo, d, C::BN) ||
        !plane_map(&m[4], pl[2].hi, d, C::BN) || !plane_map(&m[5], pl[2].lo, d, C::BN))
        return cudaErrorInvalidValue;
    static int regs = -1;
    if ((e = check_regs(fwd::attn_fwd_split_kernel<D>, fwd::kRegsLaunch, &regs)) != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fwd::attn_fwd_split_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    fwd::Params prm;
    prm.o = o;
    prm.lse = lse;
    prm.sb = d.sb;
    prm.sh = d.sh;
    prm.ss = d.ss;
    prm.S = d.S;
    prm.H = d.H;
    prm.sl2 = scale * kLog2e;
    prm.causal = causal;
    prm.hgroup = 8;
    prm.vec = vec ? 1 : 0;
    prm.stats = stats;
    prm.status = status;
    const int64_t blocks = (int64_t)((d.S + fwd::NWG * fwd::BM - 1) / (fwd::NWG * fwd::BM)) * d.H * d.B;
    if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
    fwd::attn_fwd_split_kernel<D><<<(unsigned)blocks, fwd::kThreads, C::SMEM, st>>>(m[0], m[1], m[2], m[3], m[4],
                                                                                    m[5], prm);
    note_launch();
    return cudaGetLastError();
}

template <int D>
cudaError_t launch_bwd(cudaStream_t st, int sm_count, DeviceStatus* status, const AttnDims& d, const float* q,
                       const float* k, const float* v, const float* o, const float* dout, const float* lse,
                       float* dq, float* dk, float* dv, void* ws, float scale, int causal) {
    using C = bwd::Cfg<D>;
    Planes pl[4];
    Stats* stats = carve_planes(ws, d, 4, pl);
    uint8_t* tail = (uint8_t*)ws + kStatsBytes + 8 * plane_bytes(d);
    PreParams pp;
    memset(&pp, 0, sizeof pp);
    pp.stats = stats;
    pp.src[0] = q;
    pp.src[1] = k;
    pp.src[2] = v;
    pp.src[3] = dout;
    for (int i = 0; i < 4; ++i) pp.dst[i] = pl[i];
    pp.n = 4;
    pp.o = o;
    pp.lse = lse;
    pp.lse2 = (float*)tail;
    pp.delta = (float*)(tail + table_bytes(d));
    pp.dq = dq;
    pp.dk = dk;
    pp.dv = dv;
    pp.S_pad = s_pad_of(d);
    const bool vec = vec_ok(d, {q, k, v, o, dout, dq, dk, dv});
    cudaError_t e = launch_pre<D>(st, sm_count, pp, d, vec);
    if (e != cudaSuccess) return e;
    CUtensorMap m[8];
    if (!plane_map(&m[0], pl[1].hi, d, bwd::BK) || !plane_map(&m[1], pl[1].lo, d, bwd::BK) ||
        !plane_map(&m[2], pl[2].hi, d, bwd::BK) || !plane_map(&m[3], pl[2].lo, d, bwd::BK) ||
        !plane_map(&m[4], pl[0].hi, d, C::BQ) || !plane_map(&m[5], pl[0].lo, d, C::BQ) ||
        !plane_map(&m[6], pl[3].hi, d, C::BQ) || !plane_map(&m[7], pl[3].lo, d, C::BQ))
        return cudaErrorInvalidValue;
    static int regs = -1;
    if ((e = check_regs(bwd::attn_bwd_split_kernel<D>, bwd::kRegsLaunch, &regs)) != cudaSuccess) return e;
    e = cudaFuncSetAttribute(bwd::attn_bwd_split_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    bwd::Params prm;
    prm.lse2 = pp.lse2;
    prm.delta = pp.delta;
    prm.S_pad = pp.S_pad;
    prm.dq = dq;
    prm.dk = dk;
    prm.dv = dv;
    prm.sb = d.sb;
    prm.sh = d.sh;
    prm.ss = d.ss;
    prm.S = d.S;
    prm.H = d.H;
    prm.scale = scale;
    prm.causal = causal;
    prm.hgroup = 2;
    prm.vec = vec ? 1 : 0;
    prm.stats = stats;
    prm.status = status;
    const int64_t blocks = (int64_t)((d.S + bwd::BK - 1) / bwd::BK) * d.H * d.B;
    if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
    bwd::attn_bwd_split_kernel<D><<<(unsigned)blocks, bwd::kThreads, C::SMEM, st>>>(m[0], m[1], m[2], m[3], m[4],
                                                                                   m[5], m[6], m[7], prm);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

bool split_supported(hx_dtype dt, const AttnDims& d) { return dt == HX_F32 && (d.D == 64 || d.D == 128); }

uint64_t split_fwd_workspace_bytes(const AttnDims& d) { return kStatsBytes + 6 * plane_bytes(d); }

uint64_t split_bwd_workspace_bytes(const AttnDims& d) {
    return kStatsBytes + 8 * plane_bytes(d) + 2 * table_bytes(d);
}

cudaError_t split_attn_fwd(cudaStream_t st, int sm_count, DeviceStatus* status, const AttnDims& d, const void* q,
                           const void* k, const void* v, void* o, float* lse, float scale, int causal, void* ws) {
    const float *fq = (const float*)q, *fk = (const float*)k, *fv = (const float*)v;
    if (d.D == 64) return launch_fwd<64>(st, sm_count, status, d, fq, fk, fv, (float*)o, lse, scale, causal, ws);
    if (d.D == 128) return launch_fwd<128>(st, sm_count, status, d, fq, fk, fv, (float*)o, lse, scale, causal, ws);
    return cudaErrorInvalidValue;
}

cudaError_t split_attn_bwd(cudaStream_t st, int sm_count, DeviceStatus* status, const AttnDims& d, const void* q,
                           const void* k, const void* v, const void* o, const void* dout, const float* lse,
                           void* dq, void* dk, void* dv, void* ws, float scale, int causal) {
    const float *fq = (const float*)q, *fk = (const float*)k, *fv = (const float*)v, *fo = (const float*)o,
                *fdo = (const float*)dout;
    if (d.D == 64)
        return launch_bwd<64>(st, sm_count, status, d, fq, fk, fv, fo, fdo, lse, (float*)dq, (float*)dk, (float*)dv,
                              ws, scale, causal);
    if (d.D == 128)
        return launch_bwd<128>(st, sm_count, status, d, fq, fk, fv, fo, fdo, lse, (float*)dq, (float*)dk, (float*)dv,
                               ws, scale, causal);
    return cudaErrorInvalidValue;
}

}  // namespace hx
