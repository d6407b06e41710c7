// Device kernels of the layers around the fused attention
// (MultiHeadAttention::forward, src/nn/attention.rs:46-98, and the
// TransformerBlock's FeedForward, src/nn/mlp.rs): RMSNorm forward and
// backward (src/kernels/rms_norm.rs:20-132), GELU forward and backward
// (src/kernels/activations.rs:192-237), the bias / residual rows of Linear
// (src/nn/linear.rs:54-56, src/nn/transformer.rs:32-37) and the bias
// gradient's column sums. The Linear GEMMs themselves are plain cuBLAS calls
// (hx_api.cu).
//
// All of them are HBM-bound element or row work. Each kernel has a vector
// form (16-byte accesses: 8 bf16 or 4 f32 per thread, chosen when the row
// width and the pointers allow it) and a scalar form for the rest.
//
// RMSNorm: f32 statistics in the reference's expression order:
// inv_rms = 1 / sqrt(sum_sq / hidden + eps), y = (x * inv_rms) * w. The
// backward recomputes inv_rms, then per row dot = sum_j g_j w_j x_j,
//   dx_j = g_j w_j inv_rms - x_j (inv_rms^3 dot / hidden),
//   dw_j += g_j x_j inv_rms  (summed over the rows, by the column reduction).
#include "hx_internal.h"

namespace hx {
namespace {

template <typename T>
struct Vec {
    static constexpr int N = 16 / sizeof(T);  // elements per 16-byte access
};

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i) {
    if constexpr (sizeof(T) == 2)
        return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    else
        return reinterpret_cast<const float*>(p)[i];
}
template <typename T>
__device__ __forceinline__ void st(T* p, int64_t i, float v) {
    if constexpr (sizeof(T) == 2)
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float*>(p)[i] = v;
}

// 16-byte load / store of Vec<T>::N elements at p (16-byte aligned), as f32.
template <typename T>
__device__ __forceinline__ void vld(const T* p, float (&f)[Vec<T>::N]) {
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
__device__ __forceinline__ void vst(T* p, const float (&f)[Vec<T>::N]) {
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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float inv_rms_of(float sum_sq, int hidden, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum_sq, (float)hidden), eps)));
}

// ---- RMSNorm forward: one warp per row -----------------------------------------
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                          T* __restrict__ y, int rows, int hidden, float eps) {
    constexpr int N = VEC ? Vec<T>::N : 1;
    const int lane = threadIdx.x % 32;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    const int nv = hidden / N;
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += nw) {
        const T* xr = x + r * hidden;
        T* yr = y + r * hidden;
        float ss = 0.f;
        for (int j = lane; j < nv; j += 32) {
            if constexpr (VEC) {
                float v[N];
                vld(xr + j * N, v);
#pragma unroll
                for (int k = 0; k < N; ++k) ss = __fadd_rn(ss, __fmul_rn(v[k], v[k]));
            } else {
                const float v = ld(xr, j);
                ss = __fadd_rn(ss, __fmul_rn(v, v));
            }
        }
        const float inv = inv_rms_of(warp_sum(ss), hidden, eps);
        for (int j = lane; j < nv; j += 32) {
            if constexpr (VEC) {
                float v[N], wv[N];
                vld(xr + j * N, v);
                vld(w + j * N, wv);
#pragma unroll
                for (int k = 0; k < N; ++k) v[k] = __fmul_rn(__fmul_rn(v[k], inv), wv[k]);
                vst(yr + j * N, v);
            } else {
                st(yr, j, __fmul_rn(__fmul_rn(ld(xr, j), inv), ld(w, j)));
            }
        }
    }
}

// ---- RMSNorm backward ------------------------------------------------------------
// dx: one warp per row (statistics, then dx from a second, cached read of
// the row); inv_rms of each row is kept for dw. dw is a column reduction of
// (g * x) * inv_rms over the rows (col_partial_kernel / col_final_kernel).
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) rmsnorm_bwd_dx_kernel(const T* __restrict__ g, const T* __restrict__ x,
                                                             const T* __restrict__ w, T* __restrict__ dx,
                                                             float* __restrict__ row_inv, int rows, int hidden,
                                                             float eps) {
    constexpr int N = VEC ? Vec<T>::N : 1;
    const int lane = threadIdx.x % 32;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    const float inv_h = 1.0f / (float)hidden;
    const int nv = hidden / N;
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += nw) {
        const T* xr = x + r * hidden;
        const T* gr = g + r * hidden;
        T* dxr = dx + r * hidden;
        float ss = 0.f, dot = 0.f;
        for (int j = lane; j < nv; j += 32) {
            if constexpr (VEC) {
                float xv[N], gv[N], wv[N];
                vld(xr + j * N, xv);
                vld(gr + j * N, gv);
                vld(w + j * N, wv);
#pragma unroll
                for (int k = 0; k < N; ++k) {
                    ss = __fadd_rn(ss, __fmul_rn(xv[k], xv[k]));
                    dot = __fadd_rn(dot, __fmul_rn(__fmul_rn(gv[k], wv[k]), xv[k]));
                }
            } else {
                const float xv = ld(xr, j), gv = ld(gr, j), wv = ld(w, j);
                ss = __fadd_rn(ss, __fmul_rn(xv, xv));
                dot = __fadd_rn(dot, __fmul_rn(__fmul_rn(gv, wv), xv));
            }
        }
        const float inv = inv_rms_of(warp_sum(ss), hidden, eps);
        dot = warp_sum(dot);
        const float c = __fmul_rn(__fmul_rn(__fmul_rn(__fmul_rn(inv, inv), inv), dot), inv_h);
        if (lane == 0) row_inv[r] = inv;
        for (int j = lane; j < nv; j += 32) {
            if constexpr (VEC) {
                float xv[N], gv[N], wv[N];
                vld(xr + j * N, xv);
                vld(gr + j * N, gv);
                vld(w + j * N, wv);
#pragma unroll
                for (int k = 0; k < N; ++k)
                    gv[k] = __fsub_rn(__fmul_rn(__fmul_rn(gv[k], wv[k]), inv), __fmul_rn(xv[k], c));
                vst(dxr + j * N, gv);
            } else {
                const float xv = ld(xr, j), gv = ld(gr, j), wv = ld(w, j);
                st(dxr, j, __fsub_rn(__fmul_rn(__fmul_rn(gv, wv), inv), __fmul_rn(xv, c)));
            }
        }
    }
}

// ---- rows of Linear's C operand ----------------------------------------------------
// y[r, c] = res[r, c] + b[c] (either may be NULL): the rows a GEMM with
// beta = 1 then adds x w onto, which folds Linear's bias add and the
// block's residual add into the GEMM's epilogue. Thread = N columns (its
// bias held in registers), grid.y strides the rows.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) rows_init_kernel(T* y, const T* res,  // res may alias y
                                                        const T* __restrict__ b, int64_t rows, int cols) {
    constexpr int N = VEC ? Vec<T>::N : 1;
    const int cv = blockIdx.x * blockDim.x + threadIdx.x;
    if (cv >= cols / N) return;
    float bv[N];
#pragma unroll
    for (int k = 0; k < N; ++k) bv[k] = 0.f;
    if (b) {
        if constexpr (VEC) {
            vld(b + cv * N, bv);
        } else {
            bv[0] = ld(b, cv);
        }
    }
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const int64_t o = r * cols + (int64_t)cv * N;
        float v[N];
        if (res) {
            if constexpr (VEC) {
                vld(res + o, v);
            } else {
                v[0] = ld(res, o);
            }
#pragma unroll
            for (int k = 0; k < N; ++k) v[k] += bv[k];
        } else {
#pragma unroll
            for (int k = 0; k < N; ++k) v[k] = bv[k];
        }
        if constexpr (VEC) {
            vst(y + o, v);
        } else {
            st(y, o, v[0]);
        }
    }
}

// ---- column reductions (bias gradient, RMSNorm weight gradient) --------------------
// Stage 1: thread = N adjacent columns of one stripe of rows; it sums
// a[r, c] (times b[r, c] and row_scale[r] when given, as (a * b) * scale)
// over its stripe and stores the sums to partial[stripe, c]. Stage 2: one
// thread per column adds the stripes in order. No atomics: the result does
// not depend on scheduling.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) col_partial_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                          const float* __restrict__ row_scale,
                                                          float* __restrict__ partial, int64_t rows, int cols,
                                                          int64_t rows_per_stripe) {
    constexpr int N = VEC ? Vec<T>::N : 1;
    const int cv = blockIdx.x * blockDim.x + threadIdx.x;
    if (cv >= cols / N) return;
    const int64_t r0 = (int64_t)blockIdx.y * rows_per_stripe;
    const int64_t r1 = min(rows, r0 + rows_per_stripe);
    float s[N];
#pragma unroll
    for (int k = 0; k < N; ++k) s[k] = 0.f;
#pragma unroll 4
    for (int64_t r = r0; r < r1; ++r) {
        const int64_t o = r * cols + (int64_t)cv * N;
        float v[N], u[N];
        if constexpr (VEC) {
            vld(a + o, v);
            if (b) vld(b + o, u);
        } else {
            v[0] = ld(a, o);
            if (b) u[0] = ld(b, o);
        }
        const float sc = row_scale ? row_scale[r] : 1.f;
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const float t = b ? __fmul_rn(__fmul_rn(v[k], u[k]), sc) : v[k];
            s[k] = __fadd_rn(s[k], t);
        }
    }
    float* out = partial + (int64_t)blockIdx.y * cols + (int64_t)cv * N;
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = s[k];
}

// Stage 2, a block of 32 columns x 8 stripe groups: group q adds stripes
// q, q + 8, ... of its column; the 8 group sums are then added in order.
template <typename T>
__global__ void __launch_bounds__(256) col_final_kernel(const float* __restrict__ partial, int stripes, int cols,
                                                        T* __restrict__ out) {
    __shared__ float part[8][33];
    const int cx = threadIdx.x % 32, q = threadIdx.x / 32;
    const int c = blockIdx.x * 32 + cx;
    float s = 0.f;
    if (c < cols) {
#pragma unroll 4
        for (int i = q; i < stripes; i += 8) s = __fadd_rn(s, partial[(int64_t)i * cols + c]);
    }
    part[q][cx] = s;
    __syncthreads();
    if (q == 0 && c < cols) {
        float t = part[0][cx];
#pragma unroll
        for (int k = 1; k < 8; ++k) t = __fadd_rn(t, part[k][cx]);
        st(out, c, t);
    }
}

// ---- GELU, tanh form (activations.rs:192-237) ---------------------------------------
// u = c (x + 0.044715 x^3), c = sqrt(2/pi). The reference's
// 0.5 x (1 + tanh(u)) is evaluated as x s with s = 0.5 (1 + tanh(u)) =
// 1 / (1 + exp(-2u)) (the same function, one exp and one division), and its
// derivative 0.5 (1 + tanh u) + 0.5 x (1 - tanh^2 u) u' as s + 2 x s (1 - s) u',
// with u' = c (1 + 3 * 0.044715 x^2).
// FAST (bf16 outputs, whose rounding is 2^-9): the hardware exp2 and
// reciprocal (__expf, __fdividef), a few 1e-7 relative; f32 outputs use the
// correctly rounded expf and division.
template <bool FAST>
__device__ __forceinline__ float gelu_s(float x) {
    const float c = 0.7978845608028654f;
    const float u = c * (x + 0.044715f * (x * x * x));
    if constexpr (FAST)
        return __fdividef(1.0f, 1.0f + __expf(-2.0f * u));
    else
        return 1.0f / (1.0f + expf(-2.0f * u));
}
template <bool FAST>
__device__ __forceinline__ float gelu_f(float x) { return x * gelu_s<FAST>(x); }
template <bool FAST>
__device__ __forceinline__ float gelu_d(float g, float x) {
    const float c = 0.7978845608028654f;
    const float s = gelu_s<FAST>(x);
    const float du = c * (1.0f + 3.0f * 0.044715f * (x * x));
    return g * (s + 2.0f * x * s * (1.0f - s) * du);
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) gelu_fwd_kernel(const T* x, T* y, int64_t n) {  // x, y may alias
    constexpr int N = VEC ? Vec<T>::N : 1;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nv = n / N;
    for (int64_t i = t0; i < nv; i += stride) {
        if constexpr (VEC) {
            float v[N];
            vld(x + i * N, v);
#pragma unroll
            for (int k = 0; k < N; ++k) v[k] = gelu_f<(sizeof(T) == 2)>(v[k]);
            vst(y + i * N, v);
        } else {
            st(y, i, gelu_f<(sizeof(T) == 2)>(ld(x, i)));
        }
    }
    for (int64_t i = nv * N + t0; i < n; i += stride) st(y, i, gelu_f<(sizeof(T) == 2)>(ld(x, i)));  // ragged tail
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) gelu_bwd_kernel(const T* __restrict__ g, const T* __restrict__ x,
                                                       T* __restrict__ dx, int64_t n) {
    constexpr int N = VEC ? Vec<T>::N : 1;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nv = n / N;
    for (int64_t i = t0; i < nv; i += stride) {
        if constexpr (VEC) {
            float gv[N], xv[N];
            vld(g + i * N, gv);
            vld(x + i * N, xv);
#pragma unroll
            for (int k = 0; k < N; ++k) gv[k] = gelu_d<(sizeof(T) == 2)>(gv[k], xv[k]);
            vst(dx + i * N, gv);
        } else {
            st(dx, i, gelu_d<(sizeof(T) == 2)>(ld(g, i), ld(x, i)));
        }
    }
    for (int64_t i = nv * N + t0; i < n; i += stride) st(dx, i, gelu_d<(sizeof(T) == 2)>(ld(g, i), ld(x, i)));
}

// out = a + b element-wise (kernels/binary.rs:40-60 for equal shapes: the
// gradient accumulation of the autograd walk, tensor.rs:211-214); out may
// alias a or b.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) add_kernel(const T* a, const T* b, T* out, int64_t n) {
    constexpr int N = VEC ? Vec<T>::N : 1;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nv = n / N;
    for (int64_t i = t0; i < nv; i += stride) {
        if constexpr (VEC) {
            float x[N], y[N];
            vld(a + i * N, x);
            vld(b + i * N, y);
#pragma unroll
            for (int k = 0; k < N; ++k) x[k] += y[k];
            vst(out + i * N, x);
        } else {
            st(out, i, ld(a, i) + ld(b, i));
        }
    }
    for (int64_t i = nv * N + t0; i < n; i += stride) st(out, i, ld(a, i) + ld(b, i));
}

int grid_for(int64_t work, int per_block, int cap) {
    int64_t b = (work + per_block - 1) / per_block;
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Grid for a (column vectors) x (row stripes) kernel: enough blocks to fill
// the GPU, at least min_rows rows per stripe.
dim3 col_grid(int ncv, int64_t rows, int sm_count, int min_rows) {
    const int gx = (ncv + 255) / 256;
    int64_t gy = (rows + min_rows - 1) / min_rows;
    const int64_t cap = (int64_t)sm_count * 8 / gx;
    if (gy > cap) gy = cap;
    if (gy > 65535) gy = 65535;
    return dim3(gx, (unsigned)(gy < 1 ? 1 : gy));
}

template <typename T>
cudaError_t rmsnorm_fwd_t(cudaStream_t st, int sm_count, const T* x, const T* w, T* y, int rows, int hidden,
                          float eps) {
    const int grid = grid_for(rows, 8, sm_count * 8);
    if (hidden % Vec<T>::N == 0 && aligned16(x) && aligned16(w) && aligned16(y))
        rmsnorm_fwd_kernel<T, true><<<grid, 256, 0, st>>>(x, w, y, rows, hidden, eps);
    else
        rmsnorm_fwd_kernel<T, false><<<grid, 256, 0, st>>>(x, w, y, rows, hidden, eps);
    note_launch();
    return cudaGetLastError();
}

// Stripes for a column reduction: enough threads (about 96 K column-vector
// threads in all) to keep HBM busy, at least 4 rows per stripe.
int64_t col_stripes(int ncv, int64_t rows) {
    int64_t gy = (98304 + ncv - 1) / ncv;
    if (gy > (rows + 3) / 4) gy = (rows + 3) / 4;
    if (gy > 65535) gy = 65535;
    return gy < 1 ? 1 : gy;
}

// sum over rows of a (* b * row_scale) into out[cols] (TO = T or float).
// `scratch` holds col_scratch_floats(rows, cols) floats.
template <typename T, typename TO>
cudaError_t col_reduce(cudaStream_t st, const T* a, const T* b, const float* row_scale, TO* out,
                       float* scratch, int64_t rows, int cols) {
    const bool vec = cols % Vec<T>::N == 0 && aligned16(a) && aligned16(b);
    const int ncv = vec ? cols / Vec<T>::N : cols;
    const int64_t gy = col_stripes(ncv, rows);
    const int64_t per = (rows + gy - 1) / gy;
    const dim3 grid((ncv + 255) / 256, (unsigned)gy);
    if (vec)
        col_partial_kernel<T, true><<<grid, 256, 0, st>>>(a, b, row_scale, scratch, rows, cols, per);
    else
        col_partial_kernel<T, false><<<grid, 256, 0, st>>>(a, b, row_scale, scratch, rows, cols, per);
    note_launch();
    col_final_kernel<TO><<<(cols + 31) / 32, 256, 0, st>>>(scratch, (int)gy, cols, out);
    note_launch();
    return cudaGetLastError();
}

template <typename T>
cudaError_t rmsnorm_bwd_t(cudaStream_t st, int sm_count, const T* g, const T* x, const T* w, T* dx, float* dw,
                          float* scratch, int rows, int hidden, float eps) {
    const int grid = grid_for(rows, 8, sm_count * 8);
    float* row_inv = scratch;
    if (hidden % Vec<T>::N == 0 && aligned16(g) && aligned16(x) && aligned16(w) && aligned16(dx))
        rmsnorm_bwd_dx_kernel<T, true><<<grid, 256, 0, st>>>(g, x, w, dx, row_inv, rows, hidden, eps);
    else
        rmsnorm_bwd_dx_kernel<T, false><<<grid, 256, 0, st>>>(g, x, w, dx, row_inv, rows, hidden, eps);
    note_launch();
    // dw_j = sum over rows of (g_j x_j) inv_rms
    return col_reduce<T, float>(st, g, x, row_inv, dw, scratch + rows, rows, hidden);
}

template <typename T>
cudaError_t gelu_fwd_t(cudaStream_t st, int sm_count, const T* x, T* y, int64_t n) {
    const bool vec = aligned16(x) && aligned16(y);
    const int grid = grid_for(vec ? n / Vec<T>::N + 1 : n, 256, sm_count * 8);
    if (vec)
        gelu_fwd_kernel<T, true><<<grid, 256, 0, st>>>(x, y, n);
    else
        gelu_fwd_kernel<T, false><<<grid, 256, 0, st>>>(x, y, n);
    note_launch();
    return cudaGetLastError();
}

template <typename T>
cudaError_t gelu_bwd_t(cudaStream_t st, int sm_count, const T* g, const T* x, T* dx, int64_t n) {
    const bool vec = aligned16(g) && aligned16(x) && aligned16(dx);
    const int grid = grid_for(vec ? n / Vec<T>::N + 1 : n, 256, sm_count * 8);
    if (vec)
        gelu_bwd_kernel<T, true><<<grid, 256, 0, st>>>(g, x, dx, n);
    else
        gelu_bwd_kernel<T, false><<<grid, 256, 0, st>>>(g, x, dx, n);
    note_launch();
    return cudaGetLastError();
}

template <typename T>
cudaError_t add_t(cudaStream_t st, int sm_count, const T* a, const T* b, T* out, int64_t n) {
    const bool vec = aligned16(a) && aligned16(b) && aligned16(out);
    const int grid = grid_for(vec ? n / Vec<T>::N + 1 : n, 256, sm_count * 8);
    if (vec)
        add_kernel<T, true><<<grid, 256, 0, st>>>(a, b, out, n);
    else
        add_kernel<T, false><<<grid, 256, 0, st>>>(a, b, out, n);
    note_launch();
    return cudaGetLastError();
}

template <typename T>
cudaError_t rows_init_t(cudaStream_t st, int sm_count, T* y, const T* res, const T* b, int64_t rows, int cols) {
    const bool vec = cols % Vec<T>::N == 0 && aligned16(y) && aligned16(res) && aligned16(b);
    const int ncv = vec ? cols / Vec<T>::N : cols;
    const dim3 grid = col_grid(ncv, rows, sm_count, 4);
    if (vec)
        rows_init_kernel<T, true><<<grid, 256, 0, st>>>(y, res, b, rows, cols);
    else
        rows_init_kernel<T, false><<<grid, 256, 0, st>>>(y, res, b, rows, cols);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t rmsnorm_fwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* x, const void* w, void* y,
                        int rows, int hidden, float eps) {
    if (dt == HX_BF16)
        return rmsnorm_fwd_t(st, sm_count, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, (__nv_bfloat16*)y,
                             rows, hidden, eps);
    return rmsnorm_fwd_t(st, sm_count, (const float*)x, (const float*)w, (float*)y, rows, hidden, eps);
}

int64_t col_scratch_floats(int64_t rows, int cols) {
    // stripes are fewest for the widest thread count; cols / 8 column vectors bounds every form from above
    return col_stripes(cols / 8 > 0 ? cols / 8 : 1, rows) * (int64_t)cols;
}

int64_t rmsnorm_bwd_scratch_floats(int64_t rows, int hidden) { return rows + col_scratch_floats(rows, hidden); }

cudaError_t rmsnorm_bwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* g, const void* x, const void* w,
                        void* dx, float* dw, float* scratch, int rows, int hidden, float eps) {
    if (dt == HX_BF16)
        return rmsnorm_bwd_t(st, sm_count, (const __nv_bfloat16*)g, (const __nv_bfloat16*)x,
                             (const __nv_bfloat16*)w, (__nv_bfloat16*)dx, dw, scratch, rows, hidden, eps);
    return rmsnorm_bwd_t(st, sm_count, (const float*)g, (const float*)x, (const float*)w, (float*)dx, dw, scratch,
                         rows, hidden, eps);
}

cudaError_t gelu_fwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* x, void* y, int64_t n) {
    if (dt == HX_BF16) return gelu_fwd_t(st, sm_count, (const __nv_bfloat16*)x, (__nv_bfloat16*)y, n);
    return gelu_fwd_t(st, sm_count, (const float*)x, (float*)y, n);
}

cudaError_t gelu_bwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* g, const void* x, void* dx, int64_t n) {
    if (dt == HX_BF16)
        return gelu_bwd_t(st, sm_count, (const __nv_bfloat16*)g, (const __nv_bfloat16*)x, (__nv_bfloat16*)dx, n);
    return gelu_bwd_t(st, sm_count, (const float*)g, (const float*)x, (float*)dx, n);
}

cudaError_t add(cudaStream_t st, int sm_count, hx_dtype dt, const void* a, const void* b, void* out, int64_t n) {
    if (dt == HX_BF16)
        return add_t(st, sm_count, (const __nv_bfloat16*)a, (const __nv_bfloat16*)b, (__nv_bfloat16*)out, n);
    return add_t(st, sm_count, (const float*)a, (const float*)b, (float*)out, n);
}

cudaError_t rows_init(cudaStream_t st, int sm_count, hx_dtype dt, void* y, const void* res, const void* b,
                      int64_t rows, int cols) {
    if (dt == HX_BF16)
        return rows_init_t(st, sm_count, (__nv_bfloat16*)y, (const __nv_bfloat16*)res, (const __nv_bfloat16*)b,
                           rows, cols);
    return rows_init_t(st, sm_count, (float*)y, (const float*)res, (const float*)b, rows, cols);
}

cudaError_t col_sum(cudaStream_t st, hx_dtype dt, const void* dy, void* db, float* scratch, int64_t rows,
                    int cols) {
    if (dt == HX_BF16)
        return col_reduce<__nv_bfloat16, __nv_bfloat16>(st, (const __nv_bfloat16*)dy, nullptr, nullptr,
                                                        (__nv_bfloat16*)db, scratch, rows, cols);
    return col_reduce<float, float>(st, (const float*)dy, nullptr, nullptr, (float*)db, scratch, rows, cols);
}

}  // namespace hx
