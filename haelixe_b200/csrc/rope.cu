// Rotary position embedding on [B, H, S, D] views (src/kernels/rope.rs:5-82).
//
// The per-pair frequency base^(-(2i)/D) is computed once on the host with
// the same f32 powf expression the reference uses (rope.rs:27-28). A table
// of (cos, sin) of theta = s * freq for every (s, i) is built once per
// (S, D, base) on the device and cached in the context, so the per-call
// kernel is a pure stream over x (HBM-bound) instead of one sincos per
// element per head. Each output is one rounded multiply per term and one
// rounded add/sub (rope.rs:37-38), without FMA contraction; the backward
// rotates by -theta (rope.rs:67): cos(-t) = cos(t), sin(-t) = -sin(t).
#include "hx_internal.h"

namespace hx {
namespace {

struct FreqTable {
    float f[128];  // D <= 256
};

// tab[s * half + i] = (cos(s * freq_i), sin(s * freq_i))
__global__ void __launch_bounds__(256) rope_table_kernel(float2* __restrict__ tab, int S, int half,
                                                         FreqTable ft) {
    const int64_t n = (int64_t)S * half;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int i = (int)(idx % half);
        const int s = (int)(idx / half);
        const float theta = __fmul_rn((float)s, ft.f[i]);
        float sn, cs;
        sincosf(theta, &sn, &cs);
        tab[idx] = make_float2(cs, sn);
    }
}

__device__ __forceinline__ void rot(float x0, float x1, float2 cs, float sign, float& y0,
                                    float& y1) {
    const float sn = cs.y * sign;
    y0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, sn));
    y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs.x));
}

// x / 2^k and x % 2^k when k >= 0 (a power-of-two divisor), else plain
// division: the row index splits into (b, h, s, group) without integer
// divides for the usual power-of-two S, H and D.
template <typename I>
__device__ __forceinline__ I div_by(I x, I v, int k) { return k >= 0 ? (x >> k) : x / v; }
template <typename I>
__device__ __forceinline__ I mod_by(I x, I v, int k) { return k >= 0 ? (x & (v - 1)) : x % v; }

// One thread per 4 pairs (8 elements) of a row; rows are [.., S, D] with
// element strides; D % 8 == 0 on this path. I is the index type: 32-bit
// when the host has checked that the index space and one grid stride fit,
// else 64-bit. gk, sk, hk: log2 of D/8, S, H, or -1 when not a power of two.
// x2/out2 (optional): a second tensor of the same shape and strides, rotated
// in the same launch (Q and K before attention): its index space follows the
// first one's.
template <typename T, typename I>
__global__ void __launch_bounds__(256) rope_kernel8(const T* x, T* out, const T* x2, T* out2,
                                                    const float2* __restrict__ tab, AttnDims d, float sign,
                                                    int gk, int sk, int hk) {
    const int half = d.D / 2;
    const I groups = (I)(d.D / 8), S = (I)d.S, H = (I)d.H;
    const I total1 = (I)d.B * H * S * groups;
    const I total = x2 ? 2 * total1 : total1;
    const I stride = (I)gridDim.x * (I)blockDim.x;
    for (I idx0 = (I)blockIdx.x * (I)blockDim.x + (I)threadIdx.x; idx0 < total; idx0 += stride) {
        const bool second = idx0 >= total1;
        const I idx = second ? idx0 - total1 : idx0;
        const T* src = second ? x2 : x;
        T* dst = second ? out2 : out;
        const int g = (int)mod_by(idx, groups, gk);
        I r = div_by(idx, groups, gk);
        const int s = (int)mod_by(r, S, sk);
        r = div_by(r, S, sk);
        const int h = (int)mod_by(r, H, hk);
        const int b = (int)div_by(r, H, hk);
        const int64_t off = (int64_t)b * d.sb + (int64_t)h * d.sh + (int64_t)s * d.ss + 8 * g;
        const float4* t4 = reinterpret_cast<const float4*>(tab + (int64_t)s * half + 4 * g);
        const float4 c01 = t4[0], c23 = t4[1];
        const float2 cs[4] = {make_float2(c01.x, c01.y), make_float2(c01.z, c01.w),
                              make_float2(c23.x, c23.y), make_float2(c23.z, c23.w)};
        float v[8], y[8];
        if constexpr (sizeof(T) == 2) {
            const uint4 raw = *reinterpret_cast<const uint4*>(src + off);
            const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __bfloat1622float2(p2[k]);
                v[2 * k] = f.x;
                v[2 * k + 1] = f.y;
            }
        } else {
            const float4 a = *reinterpret_cast<const float4*>(src + off);
            const float4 c = *reinterpret_cast<const float4*>(src + off + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) rot(v[2 * k], v[2 * k + 1], cs[k], sign, y[2 * k], y[2 * k + 1]);
        if constexpr (sizeof(T) == 2) {
            uint4 o;
            __nv_bfloat162* q2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int k = 0; k < 4; ++k) q2[k] = __floats2bfloat162_rn(y[2 * k], y[2 * k + 1]);
            *reinterpret_cast<uint4*>(dst + off) = o;
        } else {
            *reinterpret_cast<float4*>(dst + off) = make_float4(y[0], y[1], y[2], y[3]);
            *reinterpret_cast<float4*>(dst + off + 4) = make_float4(y[4], y[5], y[6], y[7]);
        }
    }
}

// General layout: one thread per pair.
template <typename T>
__global__ void __launch_bounds__(256) rope_kernel1(const T* x, T* out, const float2* __restrict__ tab,
                                                    AttnDims d, float sign) {
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
        float x0, x1, y0, y1;
        if constexpr (sizeof(T) == 2) {
            x0 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[off]);
            x1 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[off + 1]);
        } else {
            x0 = reinterpret_cast<const float*>(x)[off];
            x1 = reinterpret_cast<const float*>(x)[off + 1];
        }
        rot(x0, x1, tab[(int64_t)s * half + i], sign, y0, y1);
        if constexpr (sizeof(T) == 2) {
            reinterpret_cast<__nv_bfloat16*>(out)[off] = __float2bfloat16_rn(y0);
            reinterpret_cast<__nv_bfloat16*>(out)[off + 1] = __float2bfloat16_rn(y1);
        } else {
            reinterpret_cast<float*>(out)[off] = y0;
            reinterpret_cast<float*>(out)[off + 1] = y1;
        }
    }
}

template <typename T>
cudaError_t launch_rope(cudaStream_t st, int sm_count, const AttnDims& d, const void* x, void* out,
                        const float2* tab, float sign, const void* x2 = nullptr, void* out2 = nullptr) {
    const int eb = (int)sizeof(T);
    const bool vec = d.D % 8 == 0 && ((uintptr_t)x % 16 == 0) && ((uintptr_t)out % 16 == 0) &&
                     (d.ss * eb) % 16 == 0 && (d.sh * eb) % 16 == 0 && (d.sb * eb) % 16 == 0;
    if (x2 != nullptr) {  // one launch for both tensors: the vector kernel only
        if (!vec || (uintptr_t)x2 % 16 || (uintptr_t)out2 % 16) {
            cudaError_t e = launch_rope<T>(st, sm_count, d, x, out, tab, sign);
            return e != cudaSuccess ? e : launch_rope<T>(st, sm_count, d, x2, out2, tab, sign);
        }
    }
    const int64_t work = (int64_t)d.B * d.H * d.S * (vec ? d.D / 8 : d.D / 2) * (x2 ? 2 : 1);
    int64_t blocks = (work + 255) / 256;
    const int64_t cap = (int64_t)sm_count * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    auto log2_of = [](int64_t v) { return (v > 0 && (v & (v - 1)) == 0) ? __builtin_ctzll((uint64_t)v) : -1; };
    const int gk = log2_of(d.D / 8), sk = log2_of(d.S), hk = log2_of(d.H);
    if (vec && work + blocks * 256 < (int64_t(1) << 32))
        rope_kernel8<T, uint32_t><<<(unsigned)blocks, 256, 0, st>>>((const T*)x, (T*)out, (const T*)x2, (T*)out2,
                                                                  tab, d, sign, gk, sk, hk);
    else if (vec)
        rope_kernel8<T, int64_t><<<(unsigned)blocks, 256, 0, st>>>((const T*)x, (T*)out, (const T*)x2, (T*)out2,
                                                                 tab, d, sign, gk, sk, hk);
    else
        rope_kernel1<T><<<(unsigned)blocks, 256, 0, st>>>((const T*)x, (T*)out, tab, d, sign);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t rope_table(cudaStream_t st, int S, int D, const float* inv_freq_host, float2* tab) {
    FreqTable ft{};
    for (int i = 0; i < D / 2; ++i) ft.f[i] = inv_freq_host[i];
    const int64_t n = (int64_t)S * (D / 2);
    int64_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    rope_table_kernel<<<(unsigned)blocks, 256, 0, st>>>(tab, S, D / 2, ft);
    note_launch();
    return cudaGetLastError();
}

cudaError_t rope_apply(cudaStream_t st, int sm_count, hx_dtype dt, const AttnDims& d,
                       const void* x, void* out, const float2* tab, float sign, const void* x2, void* out2) {
    if (dt == HX_F32) return launch_rope<float>(st, sm_count, d, x, out, tab, sign, x2, out2);
    return launch_rope<__nv_bfloat16>(st, sm_count, d, x, out, tab, sign, x2, out2);
}

}  // namespace hx
