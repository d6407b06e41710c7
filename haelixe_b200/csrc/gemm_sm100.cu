// tcgen05 GEMM for the Linear layers around the attention (bf16 operands,
// f32 accumulation, bf16 out), replacing the reference's CPU matmul behind
// Linear::forward (src/nn/linear.rs:54-56: y = x W + b with W stored
// [in, out]; src/kernels/matmul.rs:31-126) for the device-resident layer.
//
// Row-major C[M, N] = A'[M, K] B'[K, N] (+ bias[N]) (+ R[M, N]) where
//   A' = A (K-major: A[m * lda + k])   or A^T (MN-major: A[k * lda + m]),
//   B' = B (MN-major: B[k * ldb + n])  or B^T (K-major: B[n * ldb + k]).
// The three Linear products are (K-major, MN-major) for y = x W,
// (K-major, K-major) for dx = dy W^T and (MN-major, MN-major) for
// dW = x^T dy; UMMA reads both majors straight from the TMA tiles, so no
// operand is transposed in memory.
//
// Persistent kernel, one CTA per SM, tiles of BM x BN (BM = 128 or 256):
//   warp 0     TMA producer: per 64-wide K block, the A tile (BM x 64) and
//              the B tile (BN x 64), 128-byte swizzle, into a STAGES ring;
//   warp 1     MMA issuer (one thread): per K block and 128-row half of A,
//              4 UMMAs (M=128, N=BN, K=16); the B tile in smem serves both
//              halves, so a 256 x 256 tile reads a third less operand data
//              from L2 per FLOP than a 128 x 256 one (the kernel is bound by
//              L2 -> SM bandwidth when K is small). With BM = 128 the two
//              TMEM accumulators (2 x BN columns) alternate between tiles so
//              the epilogue of tile t overlaps the main loop of tile t + 1;
//              with BM = 256 the two halves fill TMEM and the epilogue is
//              exposed once per tile;
//   warp 2     TMEM allocation;
//   warps 4-7 (and 8-11 for BM = 256)  epilogue: thread = output row (TMEM
//              lane), 32 columns per tcgen05.ld, + bias + residual in f32,
//              one bf16 rounding, 16-byte stores.
// Tiles are visited in groups of 8 M-tiles (consecutive CTAs share B tiles
// in L2). All mbarrier waits are bounded (sm100_ptx.cuh).
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace hx {
namespace {

using namespace ptx;

constexpr int GBK = 64;   // K per stage (one 128-byte swizzle atom of bf16)
constexpr int kGroupM = 8;

template <int BM, int BN>
struct GCfg {
    static constexpr int HALVES = BM / 128;            // UMMA M = 128 per half
    static constexpr int NBUF = HALVES == 1 ? 2 : 1;   // accumulator sets (alternating tiles)
    static constexpr int TMEM_COLS = NBUF * HALVES * BN;
    static constexpr int THREADS = 128 + HALVES * 128;
    static constexpr int A_HALF = 128 * GBK * 2;
    static constexpr int A_BYTES = HALVES * A_HALF;
    static constexpr int B_BYTES = BN * GBK * 2;
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int STAGES = 196608 / STAGE < 8 ? 196608 / STAGE : 8;
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;
    static_assert(TMEM_COLS <= 512, "tensor memory");
    static_assert(SMEM <= 232448, "shared memory per block");
    static_assert(STAGE % 1024 == 0, "stage buffers on 1024-byte boundaries");
};

struct GBars {
    uint64_t full[8], empty[8];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t done;
    uint32_t tmem_base;
    int abort_flag;
};
static_assert(sizeof(GBars) <= 256, "barrier block");

struct GemmParams {
    __nv_bfloat16* c;
    const __nv_bfloat16* r;     // residual [M, N] (may alias c) or null
    const __nv_bfloat16* bias;  // [N] or null
    int64_t ldc, ldr;
    int M, N, K;
    int tiles_m, tiles_n;
    DeviceStatus* status;
};

__device__ __forceinline__ uint32_t gbar(const uint64_t& b) { return smem_addr(&b); }

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mt, int& nt) {
    const int per_group = kGroupM * tiles_n;
    const int g = t / per_group;
    const int first = g * kGroupM;
    const int gm = min(kGroupM, tiles_m - first);
    const int in = t - g * per_group;
    mt = first + in % gm;
    nt = in / gm;
}

template <int BM, int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(GCfg<BM, BN>::THREADS, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                     const GemmParams p) {
    using C = GCfg<BM, BN>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    GBars* bars = (GBars*)(sm + C::BAR_OFF);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int ntiles = p.tiles_m * p.tiles_n;
    const int nk = (p.K + GBK - 1) / GBK;
    volatile int* abort_flag = &bars->abort_flag;

    if (threadIdx.x == 0) {
        bars->abort_flag = 0;
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(gbar(bars->full[s]), 1);
            mbar_init(gbar(bars->empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(gbar(bars->acc_full[b]), 1);
            mbar_init(gbar(bars->acc_empty[b]), C::HALVES * 128);
        }
        mbar_init(gbar(bars->done), 1);
        fence_mbar_init();
        fence_proxy_async();
    }
    if (warp == 2) {
        tmem_alloc(smem_addr(&bars->tmem_base), C::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&ta);
        prefetch_tmap(&tb);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x) {
                int mt, nt;
                tile_coords(t, p.tiles_m, p.tiles_n, mt, nt);
                const int m0 = mt * BM, n0 = nt * BN;
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    if (!(ok = mbar_wait(gbar(bars->empty[s]), ((it / C::STAGES) & 1) ^ 1, abort_flag,
                                         p.status, 80)))
                        break;
                    const uint32_t fb = gbar(bars->full[s]);
                    mbar_arrive_expect_tx(fb, C::STAGE);
                    const uint32_t sa = smem_addr(sm + s * C::STAGE), sb = sa + C::A_BYTES;
                    const int k0 = kb * GBK;
                    if (A_MN) {  // BM/64 boxes of 64 M x 64 K (a half = two boxes)
#pragma unroll
                        for (int c = 0; c < BM / 64; ++c) tma_load_2d(sa + c * 8192, &ta, fb, m0 + c * 64, k0);
                    } else {     // one box of 64 K x 128 M per half
#pragma unroll
                        for (int h = 0; h < C::HALVES; ++h) tma_load_2d(sa + h * C::A_HALF, &ta, fb, k0, m0 + h * 128);
                    }
                    if (B_MN) {  // BN/64 boxes of 64 N x 64 K
#pragma unroll
                        for (int c = 0; c < BN / 64; ++c) tma_load_2d(sb + c * 8192, &tb, fb, n0 + c * 64, k0);
                    } else {     // one box of 64 K x BN N
                        tma_load_2d(sb, &tb, fb, k0, n0);
                    }
                }
            }
            // Let the last copies land before the CTA's smem goes away.
            for (int j = max(0, it - C::STAGES); j < it; ++j)
                mbar_wait_drain(gbar(bars->full[j % C::STAGES]), (j / C::STAGES) & 1);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(128, BN, A_MN, B_MN);
            const uint32_t s0 = smem_addr(sm);
            // A: K-major 128 rows x 128 B (SBO 1024, K step 32 B) or MN-major
            // two 64-element chunks 8 KB apart (LBO 8192, SBO 1024, K step 2 KB).
            const uint64_t da0 = A_MN ? sdesc_sw128(s0, 8192, 1024) : sdesc_sw128(s0, 16, 1024);
            const uint64_t db0 = B_MN ? sdesc_sw128(s0 + C::A_BYTES, 8192, 1024)
                                      : sdesc_sw128(s0 + C::A_BYTES, 16, 1024);
            constexpr uint64_t kStep = (A_MN ? 2048 : 32) >> 4, kStepB = (B_MN ? 2048 : 32) >> 4;
            constexpr uint64_t kStage = (uint64_t)C::STAGE >> 4;
            int it = 0, lt = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++lt) {
                const int b = lt % C::NBUF;
                if (!(ok = mbar_wait(gbar(bars->acc_empty[b]), ((lt / C::NBUF) & 1) ^ 1, abort_flag, p.status,
                                     81)))
                    break;
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(b * C::HALVES * BN);
                for (int kb = 0; kb < nk; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    if (!(ok = mbar_wait(gbar(bars->full[s]), (it / C::STAGES) & 1, abort_flag, p.status, 82)))
                        break;
                    tc_fence_after();
                    const uint64_t da = da0 + s * kStage, db = db0 + s * kStage;
#pragma unroll
                    for (int kk = 0; kk < GBK / 16; ++kk)
#pragma unroll
                        for (int h = 0; h < C::HALVES; ++h)
                            umma_ss(acc + (uint32_t)(h * BN), da + h * (C::A_HALF >> 4) + kk * kStep,
                                    db + kk * kStepB, idesc, (kb | kk) ? 1u : 0u);
                    umma_commit(gbar(bars->empty[s]));
                }
                if (ok) umma_commit(gbar(bars->acc_full[b]));
            }
            umma_commit(gbar(bars->done));
            mbar_wait_drain(gbar(bars->done), 0);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ------------------------------------------------------------ epilogue
        const int half = (warp - 4) / 4;  // which 128-row half of the tile
        const int wi = warp % 4;          // TMEM lane quadrant of this warp
        const int row = half * 128 + wi * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(wi * 32) << 16) + (uint32_t)(half * BN);
        const bool vec_ok = (p.ldc % 8 == 0) && (p.r == nullptr || p.ldr % 8 == 0);
        int lt = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++lt) {
            const int b = lt % C::NBUF;
            if (!mbar_wait(gbar(bars->acc_full[b]), (lt / C::NBUF) & 1, abort_flag, p.status, 83)) break;
            tc_fence_after();
            int mt, nt;
            tile_coords(t, p.tiles_m, p.tiles_n, mt, nt);
            const int m = mt * BM + row;
            const bool row_ok = m < p.M;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                uint32_t v[32];
                __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the guarded stores
                tmem_ld32(tl + (uint32_t)(b * C::HALVES * BN + c), v);
                tmem_ld_wait();
                reg_fence<32>(v);
                const int n0 = nt * BN + c;
                if (!row_ok || n0 >= p.N) continue;
                float y[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) y[j] = __uint_as_float(v[j]);
                const bool full = vec_ok && n0 + 32 <= p.N;
                if (p.bias) {
                    if (full) {
                        const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + n0);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint4 u = __ldg(b4 + q);
                            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 f = __bfloat1622float2(h2[e]);
                                y[8 * q + 2 * e] += f.x;
                                y[8 * q + 2 * e + 1] += f.y;
                            }
                        }
                    } else {
                        for (int j = 0; j < 32 && n0 + j < p.N; ++j) y[j] += __bfloat162float(p.bias[n0 + j]);
                    }
                }
                const int64_t ro = (int64_t)m * p.ldr + n0;
                if (p.r) {
                    if (full) {
                        const uint4* r4 = reinterpret_cast<const uint4*>(p.r + ro);
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const uint4 u = r4[q];
                            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float2 f = __bfloat1622float2(h2[e]);
                                y[8 * q + 2 * e] += f.x;
                                y[8 * q + 2 * e + 1] += f.y;
                            }
                        }
                    } else {
                        for (int j = 0; j < 32 && n0 + j < p.N; ++j) y[j] += __bfloat162float(p.r[ro + j]);
                    }
                }
                __nv_bfloat16* dst = p.c + (int64_t)m * p.ldc + n0;
                if (full) {
                    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        d4[q] = make_uint4(pack_bf16(y[8 * q], y[8 * q + 1]), pack_bf16(y[8 * q + 2], y[8 * q + 3]),
                                           pack_bf16(y[8 * q + 4], y[8 * q + 5]),
                                           pack_bf16(y[8 * q + 6], y[8 * q + 7]));
                } else {
                    for (int j = 0; j < 32 && n0 + j < p.N; ++j) dst[j] = __float2bfloat16_rn(y[j]);
                }
            }
            tc_fence_before();
            mbar_arrive(gbar(bars->acc_empty[b]));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int BM, int BN, bool A_MN, bool B_MN>
cudaError_t launch_gemm(cudaStream_t st, int sm_count, const CUtensorMap& ta, const CUtensorMap& tb,
                        const GemmParams& p) {
    using C = GCfg<BM, BN>;
    auto kern = gemm_bf16_kernel<BM, BN, A_MN, B_MN>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    const int tiles = p.tiles_m * p.tiles_n;
    const int grid = tiles < sm_count ? tiles : sm_count;
    kern<<<grid, C::THREADS, C::SMEM, st>>>(ta, tb, p);
    note_launch();
    return cudaGetLastError();
}

// Fraction of the last wave's SMs that have work (1 = no tail).
double wave_fill(int tiles, int sm_count) {
    const int waves = (tiles + sm_count - 1) / sm_count;
    return (double)tiles / ((double)waves * sm_count);
}

}  // namespace

bool gemm_bf16_supported(bool a_mn, bool b_mn, int M, int N, int K, const void* A, int64_t lda, const void* B,
                         int64_t ldb, const void* C, int64_t ldc, const void* R, int64_t ldr, const void* bias) {
    auto al16 = [](const void* q) { return ((uintptr_t)q & 15u) == 0; };
    if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !C) return false;
    if (!al16(A) || !al16(B) || !al16(C) || (R && !al16(R)) || (bias && !al16(bias))) return false;
    if (lda % 8 || ldb % 8 || ldc % 8 || (R && ldr % 8)) return false;  // TMA strides: multiples of 16 bytes
    if (lda < (a_mn ? M : K) || ldb < (b_mn ? N : K) || ldc < N || (R && ldr < N)) return false;
    if (b_mn && N % 8) return false;
    return true;
}

cudaError_t gemm_bf16(cudaStream_t st, int sm_count, DeviceStatus* status, bool a_mn, bool b_mn, int M, int N,
                      int K, const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                      const void* R, int64_t ldr, const void* bias, int tile) {
    if (!gemm_bf16_supported(a_mn, b_mn, M, N, K, A, lda, B, ldb, C, ldc, R, ldr, bias))
        return cudaErrorNotSupported;
    // Tile shape: 256 x 256 reads the least operand data per FLOP but exposes
    // its epilogue once per tile and fills waves coarsely, so it pays only
    // when the main loop is long (K >= 4096) and there are enough tiles;
    // measured on the block stack's shapes, 128 x 256 (epilogue overlapped)
    // won every K = 2048 product. 128 x 128 serves narrow outputs. `tile`
    // (1, 2, 3) forces one of them.
    auto tiles_of = [&](int bm, int bn) { return ((M + bm - 1) / bm) * ((N + bn - 1) / bn); };
    int BM = 128, BN = N > 128 ? 256 : 128;
    if (tile == 0 && N > 128 && M > 128 && K >= 4096 && tiles_of(256, 256) * 10 >= 17 * sm_count &&
        wave_fill(tiles_of(256, 256), sm_count) >= 0.85)
        BM = 256;
    if (tile == 1) BM = 128, BN = 128;
    if (tile == 2) BM = 128, BN = 256;
    if (tile == 3) BM = 256, BN = 256;
    CUtensorMap ta, tb;
    const bool ok_a = a_mn ? make_tmap_2d_ld(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, 64, 64)
                           : make_tmap_2d_ld(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, 128);
    const bool ok_b = b_mn ? make_tmap_2d_ld(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, 64, 64)
                           : make_tmap_2d_ld(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, BN);
    if (!ok_a) return cudaErrorInvalidValue;       // the A operand's tensor map was refused
    if (!ok_b) return cudaErrorInvalidPitchValue;  // the B operand's tensor map was refused
    GemmParams p;
    p.c = (__nv_bfloat16*)C;
    p.r = (const __nv_bfloat16*)R;
    p.bias = (const __nv_bfloat16*)bias;
    p.ldc = ldc;
    p.ldr = ldr;
    p.M = M;
    p.N = N;
    p.K = K;
    p.tiles_m = (M + BM - 1) / BM;
    p.tiles_n = (N + BN - 1) / BN;
    p.status = status;
#define HX_GEMM_CASE(bm, bn, amn, bmn)                     \
    if (BM == bm && BN == bn && a_mn == amn && b_mn == bmn) \
        return launch_gemm<bm, bn, amn, bmn>(st, sm_count, ta, tb, p);
#define HX_GEMM_SHAPES(amn, bmn) \
    HX_GEMM_CASE(256, 256, amn, bmn) HX_GEMM_CASE(128, 256, amn, bmn) HX_GEMM_CASE(128, 128, amn, bmn)
    HX_GEMM_SHAPES(false, true)
    HX_GEMM_SHAPES(false, false)
    HX_GEMM_SHAPES(true, true)
#undef HX_GEMM_SHAPES
#undef HX_GEMM_CASE
    return cudaErrorNotSupported;  // (A MN-major, B K-major) is not a Linear product
}

}  // namespace hx
