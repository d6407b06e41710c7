// Device kernels of the training step around the attention stack: the
// cross-entropy loss (Tensor::cross_entropy, src/tensor.rs:754-801, with
// src/kernels/loss.rs:46-117), the AdamW update (src/optim.rs:128-199) and a
// token embedding (the reference has none; it gathers rows of a
// [vocab, hidden] table).
//
// All of them are HBM-bound integer/element work: coalesced 4- and 16-byte
// accesses, grids sized to the SM count, no tensor cores.
#include "hx_internal.h"

namespace hx {
namespace {

template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i) {
    if constexpr (sizeof(T) == 2)
        return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    else
        return reinterpret_cast<const float*>(p)[i];
}
template <typename T>
__device__ __forceinline__ void stf(T* p, int64_t i, float v) {
    if constexpr (sizeof(T) == 2)
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float*>(p)[i] = v;
}

// ---- cross-entropy ---------------------------------------------------------------
// One CTA per row of logits. Pass 1 keeps a per-thread running (max, sum of
// exp(x - max)) and merges them across the CTA: the log-sum-exp of
// loss.rs:69-72 without a separate max pass. Pass 2 re-reads the row (an L2
// hit: one row is at most a few hundred KB) and writes the gradient
// (softmax - onehot) / rows of loss.rs:86-117 directly, so the probabilities
// the reference keeps for its backward are never stored. The row loss
// lse - x[target] goes to row_loss[r]; a second, single-CTA kernel sums the
// rows in a fixed order and divides by the row count (loss.rs:80-81).
// A target outside [0, classes) makes that row's loss NaN (the reference
// panics on the out-of-range index), so the mean loss is NaN.
constexpr int CE_THREADS = 512;

__device__ __forceinline__ void ms_merge(float& m, float& s, float m2, float s2) {
    if (m2 > m) {
        s = s * expf(m - m2) + s2;  // m == -inf with s == 0 gives 0 * 0
        m = m2;
    } else if (m2 != -INFINITY) {
        s = s + s2 * expf(m2 - m);
    }
}

// 16-byte loads of 8 bf16 / 4 f32 logits as f32.
template <typename T>
__device__ __forceinline__ void vld16(const T* p, float (&f)[16 / sizeof(T)]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    if constexpr (sizeof(T) == 4) {
        f[0] = __uint_as_float(u.x), f[1] = __uint_as_float(u.y);
        f[2] = __uint_as_float(u.z), f[3] = __uint_as_float(u.w);
    } else {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
            f[2 * i] = t.x, f[2 * i + 1] = t.y;
        }
    }
}
template <typename T>
__device__ __forceinline__ void vst16(T* p, const float (&f)[16 / sizeof(T)]) {
    uint4 u;
    if constexpr (sizeof(T) == 4) {
        u.x = __float_as_uint(f[0]), u.y = __float_as_uint(f[1]);
        u.z = __float_as_uint(f[2]), u.w = __float_as_uint(f[3]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        u.x = w[0], u.y = w[1], u.z = w[2], u.w = w[3];
    }
    *reinterpret_cast<uint4*>(p) = u;
}

// exp of arguments <= 0 (logit - running max) with the hardware exp2
// (__expf): a few 1e-7 relative, far inside the loss's tolerance.
__device__ __forceinline__ void ms_add(float& m, float& s, float v) {
    if (v > m) {
        s = s * __expf(m - v) + 1.f;
        m = v;
    } else if (m != -INFINITY) {  // -inf logits add exp(-inf) = 0
        s += __expf(v - m);
    }
}

// VEC: 16-byte accesses (classes a multiple of 16 / sizeof(T), rows 16-byte aligned).
template <typename T, bool VEC>
__global__ void __launch_bounds__(CE_THREADS) cross_entropy_kernel(const T* __restrict__ logits,
                                                                   const uint32_t* __restrict__ targets,
                                                                   float* __restrict__ row_loss,
                                                                   T* __restrict__ dlogits, int rows, int classes) {
    constexpr int N = VEC ? 16 / sizeof(T) : 1;
    __shared__ float sm[CE_THREADS / 32], ss[CE_THREADS / 32];
    const int r = blockIdx.x;
    const T* x = logits + (int64_t)r * classes;
    const int nv = classes / N;
    float m = -INFINITY, s = 0.f;
    for (int j = threadIdx.x; j < nv; j += CE_THREADS) {
        if constexpr (VEC) {
            float v[N];
            vld16(x + (int64_t)j * N, v);
#pragma unroll
            for (int k = 0; k < N; ++k) ms_add(m, s, v[k]);
        } else {
            ms_add(m, s, ldf(x, j));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        ms_merge(m, s, m2, s2);
    }
    const int wid = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) {
        sm[wid] = m;
        ss[wid] = s;
    }
    __syncthreads();
    m = -INFINITY;
    s = 0.f;
    for (int w = 0; w < CE_THREADS / 32; ++w) ms_merge(m, s, sm[w], ss[w]);  // same order in every thread
    const uint32_t t = targets[r];
    const bool valid = t < (uint32_t)classes;
    if (threadIdx.x == 0) row_loss[r] = valid ? (logf(s) + m) - ldf(x, (int64_t)t) : __int_as_float(0x7fc00000);
    if (dlogits == nullptr) return;
    T* dx = dlogits + (int64_t)r * classes;
    const float inv_s = 1.f / s, inv_rows = 1.f / (float)rows;
    for (int j = threadIdx.x; j < nv; j += CE_THREADS) {
        if constexpr (VEC) {
            float v[N];
            vld16(x + (int64_t)j * N, v);
#pragma unroll
            for (int k = 0; k < N; ++k) {
                float p = __expf(v[k] - m) * inv_s;
                if ((uint32_t)(j * N + k) == t) p -= 1.f;
                v[k] = p * inv_rows;
            }
            vst16(dx + (int64_t)j * N, v);
        } else {
            float p = __expf(ldf(x, j) - m) * inv_s;
            if ((uint32_t)j == t) p -= 1.f;
            stf(dx, j, p * inv_rows);
        }
    }
}

// loss = (sum over rows of row_loss) / rows, one CTA, fixed summation order.
__global__ void __launch_bounds__(1024) mean_kernel(const float* __restrict__ v, float* __restrict__ out, int n) {
    __shared__ float part[32];
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x % 32 == 0) part[threadIdx.x / 32] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < (int)blockDim.x / 32; ++w) t += part[w];
        out[0] = t / (float)n;
    }
}

// ---- AdamW -----------------------------------------------------------------------
// One launch updates up to ADAM_MAX_TENSORS tensors (a multi-tensor apply):
// the tensor table travels by value in the kernel parameters; the blocks walk
// a flattened list of ADAM_CHUNK-element chunks. Per element, in the
// reference's order and rounding (optim.rs:177-191; every product and sum
// rounded once, no contraction):
//   p -= (lr wd) p
//   m  = b1 m + (1 - b1) g
//   v  = b2 v + ((1 - b2) g) g
//   p -= (lr (m / bc1)) / (sqrt(v / bc2) + eps)
// and, when the tensor has a low-precision copy, that copy = bf16(p).
constexpr int ADAM_MAX_TENSORS = 48;
constexpr int ADAM_CHUNK = 16384;

struct AdamTable {
    hx_adamw_tensor t[ADAM_MAX_TENSORS];
    int64_t chunk_start[ADAM_MAX_TENSORS + 1];  // prefix sums of the tensors' chunk counts
    int count;
};
static_assert(sizeof(AdamTable) + 64 < 4000, "AdamW table must fit the 4 KB kernel-parameter space");

struct AdamHyper {
    float lr_wd, b1, one_m_b1, b2, one_m_b2, bc1, bc2, lr, eps;
};

__device__ __forceinline__ void adam_elem(float& p, float g, float& m, float& v, const AdamHyper& h) {
    p = __fsub_rn(p, __fmul_rn(h.lr_wd, p));
    m = __fadd_rn(__fmul_rn(h.b1, m), __fmul_rn(h.one_m_b1, g));
    v = __fadd_rn(__fmul_rn(h.b2, v), __fmul_rn(__fmul_rn(h.one_m_b2, g), g));
    const float m_hat = __fdiv_rn(m, h.bc1);
    const float v_hat = __fdiv_rn(v, h.bc2);
    p = __fsub_rn(p, __fdiv_rn(__fmul_rn(h.lr, m_hat), __fadd_rn(__fsqrt_rn(v_hat), h.eps)));
}

__global__ void __launch_bounds__(256) adamw_kernel(const __grid_constant__ AdamTable tab, const AdamHyper h) {
    const int64_t total = tab.chunk_start[tab.count];
    int ti = 0;
    for (int64_t c = blockIdx.x; c < total; c += gridDim.x) {
        while (c >= tab.chunk_start[ti + 1]) ++ti;  // chunks are visited in increasing order
        const hx_adamw_tensor& t = tab.t[ti];
        const int64_t base = (c - tab.chunk_start[ti]) * ADAM_CHUNK;
        const int64_t end = min((int64_t)t.n, base + ADAM_CHUNK);
        const bool vec = ((reinterpret_cast<uintptr_t>(t.param) | reinterpret_cast<uintptr_t>(t.m) |
                           reinterpret_cast<uintptr_t>(t.v)) & 15) == 0 &&
                         (t.grad_dtype == HX_F32 ? (reinterpret_cast<uintptr_t>(t.grad) & 15) == 0
                                                 : (reinterpret_cast<uintptr_t>(t.grad) & 7) == 0) &&
                         (reinterpret_cast<uintptr_t>(t.param_lowp) & 7) == 0;
        if (vec) {
            const int64_t nvec = (end - base) / 4;
            for (int64_t k = threadIdx.x; k < nvec; k += blockDim.x) {
                const int64_t i = base + 4 * k;
                float4 p = *reinterpret_cast<const float4*>(t.param + i);
                float4 m = *reinterpret_cast<const float4*>(t.m + i);
                float4 v = *reinterpret_cast<const float4*>(t.v + i);
                float g[4];
                if (t.grad_dtype == HX_F32) {
                    const float4 gg = *reinterpret_cast<const float4*>(static_cast<const float*>(t.grad) + i);
                    g[0] = gg.x, g[1] = gg.y, g[2] = gg.z, g[3] = gg.w;
                } else {
                    const uint2 gg = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(t.grad) + i);
                    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&gg.x);
                    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&gg.y);
                    g[0] = __low2float(a), g[1] = __high2float(a), g[2] = __low2float(b), g[3] = __high2float(b);
                }
                adam_elem(p.x, g[0], m.x, v.x, h);
                adam_elem(p.y, g[1], m.y, v.y, h);
                adam_elem(p.z, g[2], m.z, v.z, h);
                adam_elem(p.w, g[3], m.w, v.w, h);
                *reinterpret_cast<float4*>(t.param + i) = p;
                *reinterpret_cast<float4*>(t.m + i) = m;
                *reinterpret_cast<float4*>(t.v + i) = v;
                if (t.param_lowp) {
                    __nv_bfloat162 a = __floats2bfloat162_rn(p.x, p.y), b = __floats2bfloat162_rn(p.z, p.w);
                    uint2 o;
                    o.x = *reinterpret_cast<uint32_t*>(&a);
                    o.y = *reinterpret_cast<uint32_t*>(&b);
                    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(t.param_lowp) + i) = o;
                }
            }
        }
        for (int64_t i = (vec ? base + (end - base) / 4 * 4 : base) + threadIdx.x; i < end; i += blockDim.x) {
            float p = t.param[i], m = t.m[i], v = t.v[i];
            const float g = t.grad_dtype == HX_F32 ? static_cast<const float*>(t.grad)[i]
                                                   : __bfloat162float(static_cast<const __nv_bfloat16*>(t.grad)[i]);
            adam_elem(p, g, m, v, h);
            t.param[i] = p;
            t.m[i] = m;
            t.v[i] = v;
            if (t.param_lowp) static_cast<__nv_bfloat16*>(t.param_lowp)[i] = __float2bfloat16_rn(p);
        }
    }
}

// ---- embedding -------------------------------------------------------------------
// out[t, :] = table[ids[t], :], one warp per token, 16-byte accesses when the
// row width allows. An id outside the table writes a NaN row.
template <typename T>
__global__ void __launch_bounds__(256) embedding_fwd_kernel(const T* __restrict__ table,
                                                            const uint32_t* __restrict__ ids, T* __restrict__ out,
                                                            int64_t tokens, int vocab, int dim) {
    const int lane = threadIdx.x % 32;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    const int per16 = 16 / sizeof(T);
    for (int64_t tk = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; tk < tokens; tk += nw) {
        const uint32_t id = ids[tk];
        T* o = out + tk * dim;
        if (id >= (uint32_t)vocab) {
            for (int j = lane; j < dim; j += 32) stf(o, j, __int_as_float(0x7fc00000));
            continue;
        }
        const T* src = table + (int64_t)id * dim;
        if (dim % per16 == 0 && ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
            for (int j = lane; j < dim / per16; j += 32)
                reinterpret_cast<uint4*>(o)[j] = reinterpret_cast<const uint4*>(src)[j];
        } else {
            for (int j = lane; j < dim; j += 32) o[j] = src[j];
        }
    }
}

// dtable[ids[t], :] += dout[t, :] in f32 (red.global.add); ids outside the
// table are skipped.
template <typename T>
__global__ void __launch_bounds__(256) embedding_bwd_kernel(const T* __restrict__ dout,
                                                            const uint32_t* __restrict__ ids,
                                                            float* __restrict__ dtable, int64_t tokens, int vocab,
                                                            int dim) {
    const int lane = threadIdx.x % 32;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t tk = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; tk < tokens; tk += nw) {
        const uint32_t id = ids[tk];
        if (id >= (uint32_t)vocab) continue;
        float* d = dtable + (int64_t)id * dim;
        const T* g = dout + tk * dim;
        for (int j = lane; j < dim; j += 32) atomicAdd(d + j, ldf(g, j));
    }
}

int grid_cap(int64_t work, int per_block, int cap) {
    int64_t b = (work + per_block - 1) / per_block;
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t cross_entropy(cudaStream_t st, hx_dtype dt, const void* logits, const uint32_t* targets,
                          float* row_loss, float* loss, void* dlogits, int rows, int classes) {
    const int n16 = dt == HX_BF16 ? 8 : 4;
    const bool vec = classes % n16 == 0 && ((reinterpret_cast<uintptr_t>(logits) |
                                              reinterpret_cast<uintptr_t>(dlogits)) & 15) == 0;
    if (dt == HX_BF16) {
        auto* lg = (const __nv_bfloat16*)logits;
        auto* dl = (__nv_bfloat16*)dlogits;
        if (vec)
            cross_entropy_kernel<__nv_bfloat16, true><<<rows, CE_THREADS, 0, st>>>(lg, targets, row_loss, dl, rows,
                                                                                  classes);
        else
            cross_entropy_kernel<__nv_bfloat16, false><<<rows, CE_THREADS, 0, st>>>(lg, targets, row_loss, dl, rows,
                                                                                   classes);
    } else {
        if (vec)
            cross_entropy_kernel<float, true><<<rows, CE_THREADS, 0, st>>>((const float*)logits, targets, row_loss,
                                                                          (float*)dlogits, rows, classes);
        else
            cross_entropy_kernel<float, false><<<rows, CE_THREADS, 0, st>>>((const float*)logits, targets, row_loss,
                                                                           (float*)dlogits, rows, classes);
    }
    note_launch();
    mean_kernel<<<1, 1024, 0, st>>>(row_loss, loss, rows);
    note_launch();
    return cudaGetLastError();
}

cudaError_t adamw_step(cudaStream_t st, int sm_count, const hx_adamw_tensor* tensors, int count, float lr,
                       float beta1, float beta2, float eps, float weight_decay, float bc1, float bc2) {
    AdamHyper h;
    h.lr_wd = lr * weight_decay;  // optim.rs:180 evaluates self.lr * self.weight_decay first
    h.b1 = beta1;
    h.one_m_b1 = 1.0f - beta1;
    h.b2 = beta2;
    h.one_m_b2 = 1.0f - beta2;
    h.bc1 = bc1;
    h.bc2 = bc2;
    h.lr = lr;
    h.eps = eps;
    for (int first = 0; first < count; first += ADAM_MAX_TENSORS) {
        AdamTable tab;
        tab.count = count - first < ADAM_MAX_TENSORS ? count - first : ADAM_MAX_TENSORS;
        tab.chunk_start[0] = 0;
        for (int i = 0; i < tab.count; ++i) {
            tab.t[i] = tensors[first + i];
            tab.chunk_start[i + 1] = tab.chunk_start[i] + (int64_t)((tab.t[i].n + ADAM_CHUNK - 1) / ADAM_CHUNK);
        }
        for (int i = tab.count; i < ADAM_MAX_TENSORS; ++i) tab.chunk_start[i + 1] = tab.chunk_start[tab.count];
        const int64_t chunks = tab.chunk_start[tab.count];
        if (chunks == 0) continue;
        const int grid = grid_cap(chunks, 1, sm_count * 8);
        adamw_kernel<<<grid, 256, 0, st>>>(tab, h);
        note_launch();
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t embedding_fwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* table, const uint32_t* ids,
                          void* out, int64_t tokens, int vocab, int dim) {
    const int grid = grid_cap(tokens, 8, sm_count * 8);
    if (dt == HX_BF16)
        embedding_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)table, ids,
                                                                 (__nv_bfloat16*)out, tokens, vocab, dim);
    else
        embedding_fwd_kernel<float><<<grid, 256, 0, st>>>((const float*)table, ids, (float*)out, tokens, vocab,
                                                         dim);
    note_launch();
    return cudaGetLastError();
}

cudaError_t embedding_bwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* dout, const uint32_t* ids,
                          float* dtable, int64_t tokens, int vocab, int dim) {
    const int grid = grid_cap(tokens, 8, sm_count * 8);
    if (dt == HX_BF16)
        embedding_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)dout, ids, dtable, tokens,
                                                                 vocab, dim);
    else
        embedding_bwd_kernel<float><<<grid, 256, 0, st>>>((const float*)dout, ids, dtable, tokens, vocab, dim);
    note_launch();
    return cudaGetLastError();
}

}  // namespace hx
