// Rotary position embedding on [B, H, S, D] views (src/kernels/rope.rs:5-82).
//
// One thread per rotated pair (2i, 2i+1). The per-pair frequency
// base^(-(2i)/D) is computed once on the host with the same f32 powf the
// reference uses (rope.rs:28) and passed in, so theta = s * freq is the
// reference's f32 product bit for bit; each output is one rounded multiply
// per term and one rounded add/sub (rope.rs:37-38), without FMA contraction.
#include "hx_internal.h"

namespace hx {
namespace {

struct FreqTable {
    float f[128];  // D <= 256
};

template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
    if constexpr (sizeof(T) == 4) {
        return *reinterpret_cast<const float*>(p);
    } else {
        return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
    }
}
template <typename T>
__device__ __forceinline__ void stf(T* p, float v) {
    if constexpr (sizeof(T) == 4) {
        *reinterpret_cast<float*>(p) = v;
    } else {
        *reinterpret_cast<__nv_bfloat16*>(p) = __float2bfloat16_rn(v);
    }
}

template <typename T>
__global__ void __launch_bounds__(256) rope_kernel(const T* x, T* out,
                                                   AttnDims d, FreqTable tab, float sign) {
    const int half = d.D / 2;
    const int64_t pairs = (int64_t)d.B * d.H * d.S * half;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < pairs;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(idx % half);
        int64_t r = idx / half;
        const int s = (int)(r % d.S);
        r /= d.S;
        const int h = (int)(r % d.H);
        const int b = (int)(r / d.H);
        const int64_t off = (int64_t)b * d.sb + (int64_t)h * d.sh + (int64_t)s * d.ss + 2 * i;
        float theta = __fmul_rn((float)s, tab.f[i]);
        if (sign < 0.f) theta = -theta;
        float sn, cs;
        sincosf(theta, &sn, &cs);
        const float x0 = ldf(x + off), x1 = ldf(x + off + 1);
        const float y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        stf(out + off, y0);
        stf(out + off + 1, y1);
    }
}

}  // namespace

cudaError_t rope_apply(cudaStream_t st, hx_dtype dt, const AttnDims& d, const void* x, void* out,
                       const float* inv_freq_host, float sign) {
    FreqTable tab{};
    for (int i = 0; i < d.D / 2; ++i) tab.f[i] = inv_freq_host[i];
    const int64_t pairs = (int64_t)d.B * d.H * d.S * (d.D / 2);
    const int blocks = (int)((pairs + 255) / 256 < 148 * 32 ? (pairs + 255) / 256 : 148 * 32);
    if (dt == HX_F32) {
        rope_kernel<float><<<blocks, 256, 0, st>>>((const float*)x, (float*)out, d, tab, sign);
        note_launch();
    } else {
        rope_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
            (const __nv_bfloat16*)x, (__nv_bfloat16*)out, d, tab, sign);
        note_launch();
    }
    return cudaGetLastError();
}

}  // namespace hx
