// SIMT (CUDA-core FFMA) fused attention: the f32-I/O path and the path for
// head dims the tcgen05 kernels do not cover (any D <= 256, f32 or bf16).
//
// Forward: one block per (16 query rows, head, batch); 16 threads per row
// keep the online-softmax state (row max m, row sum l, O accumulators) of
// one row, as the reference shader's per-row state (flash_attention.wgsl:
// 30-38, 86-109) but with the row reductions done once per row by warp
// shuffles instead of by every thread, keys beyond S masked to -inf (the
// shader pads them with score 0, flash_attention.wgsl:63-69), an optional
// causal mask, and the per-row log-sum-exp stored for the backward.
//
// Backward: delta = rowsum(dO * O) (the `dot` of the reference's softmax
// backward, src/kernels/activations.rs:170-176, which equals rowsum(dP * P)),
// then a key-stationary kernel for dK, dV and a query-stationary kernel for
// dQ, each recomputing P = exp(scale * q.k - lse) - the decomposition of
// src/ops/flash_attention.rs:16-39 without materialising the S x S matrices.
// No atomics: results are deterministic.
#include <math.h>

#include "hx_internal.h"

namespace hx {
namespace {

constexpr int kRows = 16;  // rows (queries or keys) per block
constexpr int kTpr = 16;   // threads per row
constexpr int kTile = 32;  // keys (or queries) per inner tile
constexpr int kMaxD = 256;
constexpr int kCols = kMaxD / kTpr;  // output columns per thread, max
constexpr int kThreads = kRows * kTpr;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename T>
__device__ __forceinline__ float ldf(const T* p);
template <>
__device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) {
    return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ void stf(T* p, float v);
template <>
__device__ __forceinline__ void stf<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void stf<__nv_bfloat16>(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float half_warp_max(float x) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o, 16));
    return x;
}
__device__ __forceinline__ float half_warp_sum(float x) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o, 16);
    return x;
}

// Loads `rows` rows of a [.., S, D] operand starting at sequence index r0
// into smem (row pitch D+1 floats), zero-filling rows at or beyond S.
template <typename T>
__device__ __forceinline__ void load_rows(float* dst, const T* src, int64_t base, int64_t ss,
                                          int r0, int rows, int S, int D) {
    const int DP = D + 1;
    for (int idx = threadIdx.x; idx < rows * D; idx += blockDim.x) {
        const int r = idx / D, c = idx - r * D;
        const int s = r0 + r;
        dst[r * DP + c] = (s < S) ? ldf(src + base + (int64_t)s * ss + c) : 0.f;
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) simt_fwd_kernel(const T* __restrict__ q,
                                                            const T* __restrict__ k,
                                                            const T* __restrict__ v,
                                                            T* __restrict__ o,
                                                            float* __restrict__ lse, AttnDims d,
                                                            float scale_log2, int causal) {
    extern __shared__ float smem[];
    const int D = d.D, DP = D + 1, S = d.S;
    float* sq = smem;               // kRows x DP
    float* sk = sq + kRows * DP;    // kTile x DP
    float* sv = sk + kTile * DP;    // kTile x DP
    float* sp = sv + kTile * DP;    // kRows x (kTile+1)
    const int bi = blockIdx.z, hi = blockIdx.y;
    const int64_t base = (int64_t)bi * d.sb + (int64_t)hi * d.sh;
    const int row = threadIdx.x / kTpr, t = threadIdx.x % kTpr;
    const int q0 = blockIdx.x * kRows;
    const int qi = q0 + row;

    load_rows(sq, q, base, d.ss, q0, kRows, S, D);
    float m = -INFINITY, l = 0.f;
    float acc[kCols];
#pragma unroll
    for (int c = 0; c < kCols; ++c) acc[c] = 0.f;

    const int kend = causal ? min(S, q0 + kRows) : S;
    for (int k0 = 0; k0 < kend; k0 += kTile) {
        __syncthreads();
        load_rows(sk, k, base, d.ss, k0, kTile, S, D);
        load_rows(sv, v, base, d.ss, k0, kTile, S, D);
        __syncthreads();
        float s[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = t + kTpr * u, kj = k0 + j;
            float dot = 0.f;
            for (int c = 0; c < D; ++c) dot += sq[row * DP + c] * sk[j * DP + c];
            const bool valid = kj < S && (!causal || kj <= qi);
            s[u] = valid ? dot * scale_log2 : -INFINITY;
        }
        const float mx = half_warp_max(fmaxf(s[0], s[1]));
        const float m_new = fmaxf(m, mx);
        // m_new is finite from the first tile on (key 0 is never masked).
        const float alpha = exp2f(m - m_new);
        const float p0 = exp2f(s[0] - m_new), p1 = exp2f(s[1] - m_new);
        l = l * alpha + half_warp_sum(p0 + p1);
        m = m_new;
        sp[row * (kTile + 1) + t] = p0;
        sp[row * (kTile + 1) + t + kTpr] = p1;
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const int col = t + kTpr * c;
            if (col < D) {
                float a = acc[c] * alpha;
                for (int j = 0; j < kTile; ++j) a += sp[row * (kTile + 1) + j] * sv[j * DP + col];
                acc[c] = a;
            }
        }
        __syncwarp();
    }
    if (qi < S) {
        const float inv_l = 1.f / l;
        T* orow = o + base + (int64_t)qi * d.ss;
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const int col = t + kTpr * c;
            if (col < D) stf(orow + col, acc[c] * inv_l);
        }
        if (t == 0 && lse != nullptr)
            lse[((int64_t)bi * d.H + hi) * S + qi] = (m + log2f(l)) * kLn2;
    }
}

// delta[b,h,s] = sum_d dO[b,h,s,d] * O[b,h,s,d]; one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) delta_kernel(const T* __restrict__ o,
                                                    const T* __restrict__ dout,
                                                    float* __restrict__ delta, AttnDims d) {
    const int64_t rows = (int64_t)d.B * d.H * d.S;
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32;
    const int lane = threadIdx.x % 32;
    if (r >= rows) return;
    const int s = (int)(r % d.S);
    const int64_t bh = r / d.S;
    const int hi = (int)(bh % d.H), bi = (int)(bh / d.H);
    const int64_t off = (int64_t)bi * d.sb + (int64_t)hi * d.sh + (int64_t)s * d.ss;
    float acc = 0.f;
    for (int c = lane; c < d.D; c += 32) acc += ldf(o + off + c) * ldf(dout + off + c);
#pragma unroll
    for (int w = 16; w > 0; w >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, w);
    if (lane == 0) delta[r] = acc;
}

// dK, dV for 16 keys per block; loops over query tiles.
template <typename T>
__global__ void __launch_bounds__(kThreads) simt_dkdv_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const T* __restrict__ dout, const float* __restrict__ lse, const float* __restrict__ delta,
    T* __restrict__ dk, T* __restrict__ dv, AttnDims d, float scale, int causal) {
    extern __shared__ float smem[];
    const int D = d.D, DP = D + 1, S = d.S;
    float* skr = smem;               // kRows x DP   (this block's keys)
    float* svr = skr + kRows * DP;   // kRows x DP
    float* sq = svr + kRows * DP;    // kTile x DP
    float* sdo = sq + kTile * DP;    // kTile x DP
    float* sp = sdo + kTile * DP;    // kRows x (kTile+1)
    float* sds = sp + kRows * (kTile + 1);
    float* slse = sds + kRows * (kTile + 1);  // kTile
    float* sdel = slse + kTile;               // kTile
    const int bi = blockIdx.z, hi = blockIdx.y;
    const int64_t base = (int64_t)bi * d.sb + (int64_t)hi * d.sh;
    const int64_t rbase = ((int64_t)bi * d.H + hi) * S;
    const int row = threadIdx.x / kTpr, t = threadIdx.x % kTpr;
    const int k0 = blockIdx.x * kRows;
    const int kj = k0 + row;
    const float scale_log2 = scale * kLog2e;

    load_rows(skr, k, base, d.ss, k0, kRows, S, D);
    load_rows(svr, v, base, d.ss, k0, kRows, S, D);
    float adk[kCols], adv[kCols];
#pragma unroll
    for (int c = 0; c < kCols; ++c) adk[c] = adv[c] = 0.f;

    const int qstart = causal ? (k0 / kTile) * kTile : 0;
    for (int q0 = qstart; q0 < S; q0 += kTile) {
        __syncthreads();
        load_rows(sq, q, base, d.ss, q0, kTile, S, D);
        load_rows(sdo, dout, base, d.ss, q0, kTile, S, D);
        for (int i = threadIdx.x; i < kTile; i += blockDim.x) {
            const int qi = q0 + i;
            slse[i] = qi < S ? lse[rbase + qi] * kLog2e : 0.f;
            sdel[i] = qi < S ? delta[rbase + qi] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int i = t + kTpr * u, qi = q0 + i;
            float s = 0.f, dp = 0.f;
            for (int c = 0; c < D; ++c) {
                s += skr[row * DP + c] * sq[i * DP + c];
                dp += svr[row * DP + c] * sdo[i * DP + c];
            }
            const bool valid = qi < S && kj < S && (!causal || kj <= qi);
            const float p = valid ? exp2f(s * scale_log2 - slse[i]) : 0.f;
            sp[row * (kTile + 1) + i] = p;
            sds[row * (kTile + 1) + i] = p * (dp - sdel[i]);
        }
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const int col = t + kTpr * c;
            if (col < D) {
                float a = adv[c], b = adk[c];
                for (int i = 0; i < kTile; ++i) {
                    a += sp[row * (kTile + 1) + i] * sdo[i * DP + col];
                    b += sds[row * (kTile + 1) + i] * sq[i * DP + col];
                }
                adv[c] = a;
                adk[c] = b;
            }
        }
        __syncwarp();
    }
    if (kj < S) {
        T* dkrow = dk + base + (int64_t)kj * d.ss;
        T* dvrow = dv + base + (int64_t)kj * d.ss;
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const int col = t + kTpr * c;
            if (col < D) {
                stf(dkrow + col, adk[c] * scale);
                stf(dvrow + col, adv[c]);
            }
        }
    }
}

// dQ for 16 queries per block; loops over key tiles.
template <typename T>
__global__ void __launch_bounds__(kThreads) simt_dq_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
    const T* __restrict__ dout, const float* __restrict__ lse, const float* __restrict__ delta,
    T* __restrict__ dq, AttnDims d, float scale, int causal) {
    extern __shared__ float smem[];
    const int D = d.D, DP = D + 1, S = d.S;
    float* sq = smem;               // kRows x DP
    float* sdo = sq + kRows * DP;   // kRows x DP
    float* sk = sdo + kRows * DP;   // kTile x DP
    float* sv = sk + kTile * DP;    // kTile x DP
    float* sds = sv + kTile * DP;   // kRows x (kTile+1)
    const int bi = blockIdx.z, hi = blockIdx.y;
    const int64_t base = (int64_t)bi * d.sb + (int64_t)hi * d.sh;
    const int64_t rbase = ((int64_t)bi * d.H + hi) * S;
    const int row = threadIdx.x / kTpr, t = threadIdx.x % kTpr;
    const int q0 = blockIdx.x * kRows;
    const int qi = q0 + row;
    const float scale_log2 = scale * kLog2e;

    load_rows(sq, q, base, d.ss, q0, kRows, S, D);
    load_rows(sdo, dout, base, d.ss, q0, kRows, S, D);
    const float lse2 = qi < S ? lse[rbase + qi] * kLog2e : 0.f;
    const float del = qi < S ? delta[rbase + qi] : 0.f;
    float acc[kCols];
#pragma unroll
    for (int c = 0; c < kCols; ++c) acc[c] = 0.f;

    const int kend = causal ? min(S, q0 + kRows) : S;
    for (int k0 = 0; k0 < kend; k0 += kTile) {
        __syncthreads();
        load_rows(sk, k, base, d.ss, k0, kTile, S, D);
        load_rows(sv, v, base, d.ss, k0, kTile, S, D);
        __syncthreads();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = t + kTpr * u, kj = k0 + j;
            float s = 0.f, dp = 0.f;
            for (int c = 0; c < D; ++c) {
                s += sq[row * DP + c] * sk[j * DP + c];
                dp += sdo[row * DP + c] * sv[j * DP + c];
            }
            const bool valid = qi < S && kj < S && (!causal || kj <= qi);
            const float p = valid ? exp2f(s * scale_log2 - lse2) : 0.f;
            sds[row * (kTile + 1) + j] = p * (dp - del);
        }
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const int col = t + kTpr * c;
            if (col < D) {
                float a = acc[c];
                for (int j = 0; j < kTile; ++j) a += sds[row * (kTile + 1) + j] * sk[j * DP + col];
                acc[c] = a;
            }
        }
        __syncwarp();
    }
    if (qi < S) {
        T* row_out = dq + base + (int64_t)qi * d.ss;
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const int col = t + kTpr * c;
            if (col < D) stf(row_out + col, acc[c] * scale);
        }
    }
}

template <typename T>
cudaError_t launch_fwd(cudaStream_t st, const AttnDims& d, const void* q, const void* k,
                       const void* v, void* o, float* lse, float scale, int causal) {
    const int DP = d.D + 1;
    const size_t smem = sizeof(float) * (size_t)(kRows * DP + 2 * kTile * DP + kRows * (kTile + 1));
    cudaError_t e = cudaFuncSetAttribute(simt_fwd_kernel<T>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((d.S + kRows - 1) / kRows, d.H, d.B);
    simt_fwd_kernel<T><<<grid, kThreads, smem, st>>>((const T*)q, (const T*)k, (const T*)v,
                                                     (T*)o, lse, d, scale * kLog2e, causal);
    note_launch();
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_bwd(cudaStream_t st, const AttnDims& d, const void* q, const void* k,
                       const void* v, const void* o, const void* dout, const float* lse,
                       void* dq, void* dk, void* dv, float* delta, float scale, int causal) {
    const int64_t rows = (int64_t)d.B * d.H * d.S;
    delta_kernel<T><<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>((const T*)o,
                                                                       (const T*)dout, delta, d);
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int DP = d.D + 1;
    dim3 grid((d.S + kRows - 1) / kRows, d.H, d.B);
    const size_t smem_kv =
        sizeof(float) * (size_t)(2 * kRows * DP + 2 * kTile * DP + 2 * kRows * (kTile + 1) + 2 * kTile);
    e = cudaFuncSetAttribute(simt_dkdv_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_kv);
    if (e != cudaSuccess) return e;
    simt_dkdv_kernel<T><<<grid, kThreads, smem_kv, st>>>(
        (const T*)q, (const T*)k, (const T*)v, (const T*)dout, lse, delta, (T*)dk, (T*)dv, d,
        scale, causal);
    note_launch();
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem_q = sizeof(float) * (size_t)(2 * kRows * DP + 2 * kTile * DP + kRows * (kTile + 1));
    e = cudaFuncSetAttribute(simt_dq_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_q);
    if (e != cudaSuccess) return e;
    simt_dq_kernel<T><<<grid, kThreads, smem_q, st>>>((const T*)q, (const T*)k, (const T*)v,
                                                      (const T*)dout, lse, delta, (T*)dq, d,
                                                      scale, causal);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t simt_attn_fwd(cudaStream_t st, hx_dtype dt, const AttnDims& d, const void* q,
                          const void* k, const void* v, void* o, float* lse, float scale,
                          int causal) {
    if (dt == HX_F32) return launch_fwd<float>(st, d, q, k, v, o, lse, scale, causal);
    return launch_fwd<__nv_bfloat16>(st, d, q, k, v, o, lse, scale, causal);
}

cudaError_t simt_attn_bwd(cudaStream_t st, hx_dtype dt, const AttnDims& d, const void* q,
                          const void* k, const void* v, const void* o, const void* dout,
                          const float* lse, void* dq, void* dk, void* dv, float* delta,
                          float scale, int causal) {
    if (dt == HX_F32)
        return launch_bwd<float>(st, d, q, k, v, o, dout, lse, dq, dk, dv, delta, scale, causal);
    return launch_bwd<__nv_bfloat16>(st, d, q, k, v, o, dout, lse, dq, dk, dv, delta, scale,
                                     causal);
}

}  // namespace hx
