// Device kernels of the layers around the fused attention
// (MultiHeadAttention::forward, src/nn/attention.rs:46-98, and the
// TransformerBlock's FeedForward, src/nn/mlp.rs): RMSNorm forward and
// backward (src/kernels/rms_norm.rs:20-132), GELU forward and backward
// (src/kernels/activations.rs:192-237) and the bias broadcast / column-sum
// kernels of Linear (src/nn/linear.rs:54-56). The Linear GEMMs themselves are
// plain cuBLAS calls (hx_api.cu).
//
// RMSNorm: one warp per row, f32 statistics. The forward keeps the
// reference's expression order: inv_rms = 1 / sqrt(sum_sq / hidden + eps),
// y = (x * inv_rms) * w. The backward recomputes inv_rms, then
//   dot = sum_j g_j w_j x_j,
//   dx_j = g_j w_j inv_rms - x_j inv_rms^3 dot / hidden,
//   dw_j += g_j x_j inv_rms  (summed over rows: per-block shared-memory
//                             partial sums, then one atomic add per column).
#include "hx_internal.h"

namespace hx {
namespace {

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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float inv_rms_of(float sum_sq, int hidden, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum_sq, (float)hidden), eps)));
}

template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                          T* __restrict__ y, int rows, int hidden, float eps) {
    const int lane = threadIdx.x % 32;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += nw) {
        const T* xr = x + r * hidden;
        float ss = 0.f;
        for (int j = lane; j < hidden; j += 32) {
            const float v = ld(xr, j);
            ss = __fadd_rn(ss, __fmul_rn(v, v));
        }
        const float inv = inv_rms_of(warp_sum(ss), hidden, eps);
        T* yr = y + r * hidden;
        for (int j = lane; j < hidden; j += 32) st(yr, j, __fmul_rn(__fmul_rn(ld(xr, j), inv), ld(w, j)));
    }
}

// dw must be zeroed before the launch; dynamic smem = hidden floats.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const T* __restrict__ g, const T* __restrict__ x,
                                                          const T* __restrict__ w, T* __restrict__ dx,
                                                          float* __restrict__ dw, int rows, int hidden,
                                                          float eps) {
    extern __shared__ float sdw[];
    for (int j = threadIdx.x; j < hidden; j += blockDim.x) sdw[j] = 0.f;
    __syncthreads();
    const int lane = threadIdx.x % 32;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    const float inv_h = 1.0f / (float)hidden;
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += nw) {
        const T* xr = x + r * hidden;
        const T* gr = g + r * hidden;
        float ss = 0.f, dot = 0.f;
        for (int j = lane; j < hidden; j += 32) {
            const float xv = ld(xr, j), gv = ld(gr, j), wv = ld(w, j);
            ss = __fadd_rn(ss, __fmul_rn(xv, xv));
            dot = __fadd_rn(dot, __fmul_rn(__fmul_rn(gv, wv), xv));
        }
        const float inv = inv_rms_of(warp_sum(ss), hidden, eps);
        dot = warp_sum(dot);
        const float inv3 = __fmul_rn(__fmul_rn(inv, inv), inv);
        const float c = __fmul_rn(__fmul_rn(inv3, dot), inv_h);
        T* dxr = dx + r * hidden;
        for (int j = lane; j < hidden; j += 32) {
            const float xv = ld(xr, j), gv = ld(gr, j), wv = ld(w, j);
            st(dxr, j, __fsub_rn(__fmul_rn(__fmul_rn(gv, wv), inv), __fmul_rn(xv, c)));
            atomicAdd(&sdw[j], __fmul_rn(__fmul_rn(gv, xv), inv));
        }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < hidden; j += blockDim.x) atomicAdd(&dw[j], sdw[j]);
}

// y[r, c] = b[c]: the bias rows a GEMM with beta = 1 then adds x w onto.
template <typename T>
__global__ void __launch_bounds__(256) bias_rows_kernel(T* __restrict__ y, const T* __restrict__ b,
                                                        int64_t rows, int cols) {
    const int64_t n = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = b[i % cols];
}

// db[c] = sum_r dy[r, c] in f32; one thread per column, rows strided over the grid's y.
template <typename T>
__global__ void __launch_bounds__(256) col_sum_kernel(const T* __restrict__ dy, float* __restrict__ acc,
                                                      int64_t rows, int cols) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    float s = 0.f;
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) s += ld(dy, r * cols + c);
    atomicAdd(&acc[c], s);
}

template <typename T>
__global__ void __launch_bounds__(256) store_f32_kernel(const float* __restrict__ a, T* __restrict__ out, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) st(out, i, a[i]);
}

// GELU, tanh form (activations.rs:200-206): c = sqrt(2/pi),
// y = 0.5 x (1 + tanh(c (x + 0.044715 x^3))).
template <typename T>
__global__ void __launch_bounds__(256) gelu_fwd_kernel(const T* x, T* y, int64_t n) {  // x, y may alias
    const float c = 0.7978845608028654f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = ld(x, i);
        const float t = tanhf(c * (v + 0.044715f * (v * v * v)));
        st(y, i, 0.5f * v * (1.0f + t));
    }
}

// Its exact derivative (activations.rs:222-234):
// dx = g (0.5 (1 + t) + 0.5 x (1 - t^2) c (1 + 3 * 0.044715 x^2)).
template <typename T>
__global__ void __launch_bounds__(256) gelu_bwd_kernel(const T* __restrict__ g, const T* __restrict__ x,
                                                       T* __restrict__ dx, int64_t n) {
    const float c = 0.7978845608028654f;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = ld(x, i);
        const float t = tanhf(c * (v + 0.044715f * (v * v * v)));
        const float sech2 = 1.0f - t * t;
        const float d_inner = c * (1.0f + 3.0f * 0.044715f * (v * v));
        st(dx, i, ld(g, i) * (0.5f * (1.0f + t) + 0.5f * v * sech2 * d_inner));
    }
}

int grid_for(int64_t work, int per_block, int sm_count) {
    int64_t b = (work + per_block - 1) / per_block;
    const int64_t cap = (int64_t)sm_count * 8;
    if (b > cap) b = cap;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t rmsnorm_fwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* x, const void* w, void* y,
                        int rows, int hidden, float eps) {
    const int grid = grid_for(rows, 8, sm_count);
    if (dt == HX_BF16)
        rmsnorm_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)w,
                                                               (__nv_bfloat16*)y, rows, hidden, eps);
    else
        rmsnorm_fwd_kernel<float><<<grid, 256, 0, st>>>((const float*)x, (const float*)w, (float*)y, rows, hidden, eps);
    note_launch();
    return cudaGetLastError();
}

cudaError_t rmsnorm_bwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* g, const void* x, const void* w,
                        void* dx, float* dw, int rows, int hidden, float eps) {
    cudaError_t e = cudaMemsetAsync(dw, 0, sizeof(float) * (size_t)hidden, st);
    if (e != cudaSuccess) return e;
    const int grid = grid_for(rows, 8, sm_count);
    const size_t smem = sizeof(float) * (size_t)hidden;
    if (dt == HX_BF16) {
        e = cudaFuncSetAttribute(rmsnorm_bwd_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return e;
        rmsnorm_bwd_kernel<__nv_bfloat16><<<grid, 256, smem, st>>>(
            (const __nv_bfloat16*)g, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, (__nv_bfloat16*)dx, dw, rows,
            hidden, eps);
    } else {
        e = cudaFuncSetAttribute(rmsnorm_bwd_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        rmsnorm_bwd_kernel<float><<<grid, 256, smem, st>>>((const float*)g, (const float*)x, (const float*)w,
                                                           (float*)dx, dw, rows, hidden, eps);
    }
    note_launch();
    return cudaGetLastError();
}

cudaError_t gelu_fwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* x, void* y, int64_t n) {
    const int grid = grid_for(n, 256, sm_count * 4);
    if (dt == HX_BF16)
        gelu_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y, n);
    else
        gelu_fwd_kernel<float><<<grid, 256, 0, st>>>((const float*)x, (float*)y, n);
    note_launch();
    return cudaGetLastError();
}

cudaError_t gelu_bwd(cudaStream_t st, int sm_count, hx_dtype dt, const void* g, const void* x, void* dx, int64_t n) {
    const int grid = grid_for(n, 256, sm_count * 4);
    if (dt == HX_BF16)
        gelu_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)g, (const __nv_bfloat16*)x,
                                                            (__nv_bfloat16*)dx, n);
    else
        gelu_bwd_kernel<float><<<grid, 256, 0, st>>>((const float*)g, (const float*)x, (float*)dx, n);
    note_launch();
    return cudaGetLastError();
}

cudaError_t bias_rows(cudaStream_t st, int sm_count, hx_dtype dt, void* y, const void* b, int64_t rows, int cols) {
    const int grid = grid_for(rows * cols, 256, sm_count * 4);
    if (dt == HX_BF16)
        bias_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((__nv_bfloat16*)y, (const __nv_bfloat16*)b, rows, cols);
    else
        bias_rows_kernel<float><<<grid, 256, 0, st>>>((float*)y, (const float*)b, rows, cols);
    note_launch();
    return cudaGetLastError();
}

cudaError_t col_sum(cudaStream_t st, hx_dtype dt, const void* dy, void* db, float* scratch, int64_t rows, int cols) {
    cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(float) * (size_t)cols, st);
    if (e != cudaSuccess) return e;
    dim3 grid((cols + 255) / 256, (unsigned)(rows < 256 ? rows : 256));
    if (dt == HX_BF16) {
        col_sum_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)dy, scratch, rows, cols);
        note_launch();
        store_f32_kernel<__nv_bfloat16><<<(cols + 255) / 256, 256, 0, st>>>(scratch, (__nv_bfloat16*)db, cols);
    } else {
        col_sum_kernel<float><<<grid, 256, 0, st>>>((const float*)dy, scratch, rows, cols);
        note_launch();
        store_f32_kernel<float><<<(cols + 255) / 256, 256, 0, st>>>(scratch, (float*)db, cols);
    }
    note_launch();
    return cudaGetLastError();
}

}  // namespace hx
