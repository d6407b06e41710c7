// The attention layer's modules (src/nn) in the C++ host layer: Linear,
// RMSNorm and MultiHeadAttention, each op recorded on the autograd graph like
// the reference's Op nodes, every byte of compute in the CUDA library.
#include <cmath>
#include <random>

#include "haelixe.hpp"

namespace haelixe {
namespace {

void check(hx_ctx* c, int status) {
    if (status == HX_OK) return;
    char buf[512] = {0};
    hx_last_error(c, buf, sizeof(buf));
    throw Error("haelixe_cuda error " + std::to_string(status) + ": " + (buf[0] ? buf : hx_status_string(status)));
}

hx_ctx* ctx_of(const Tensor& t, const char* who) {
    if (!t.device.is_cuda()) throw Error(std::string(who) + ": the nn layers run on CUDA tensors");
    if (t.dtype != DType::F32) throw Error(std::string(who) + ": the nn layers are f32, the reference's GPU dtype");
    return t.device.context()->raw();
}

bool contiguous(const Tensor& t) { return t.strides == t.shape.contiguous_strides() && t.byte_offset == 0; }

size_t last_dim(const Tensor& t) { return t.shape.dims().empty() ? 1 : t.shape.dims().back(); }

// A buffer with `strides` over shape (a permutation of a contiguous block).
Tensor empty_strided(const Shape& shape, const std::vector<int64_t>& strides, const Device& dev) {
    return Tensor::empty(DType::F32, shape, dev).view(shape, strides);
}

// nn/linear.rs:54-56 and the matmul + add backward it records.
class LinearOp : public Op {
  public:
    Tensor x, w, b;
    LinearOp(Tensor x_, Tensor w_, Tensor b_) : x(std::move(x_)), w(std::move(w_)), b(std::move(b_)) {}
    const char* name() const override { return "Linear"; }
    std::vector<std::optional<Tensor>> backward(const Tensor& dy) const override {
        hx_ctx* c = ctx_of(dy, "Linear backward");
        if (!contiguous(dy)) throw Error("Linear backward: gradient must be contiguous");
        const int in = (int)w.shape.dims()[0], out = (int)w.shape.dims()[1];
        const int rows = (int)(x.shape.num_elements() / in);
        Tensor dx = Tensor::empty(DType::F32, x.shape, x.device);
        Tensor dw = Tensor::empty(DType::F32, w.shape, w.device);
        Tensor db = Tensor::empty(DType::F32, b.shape, b.device);
        check(c, hx_linear_bwd(c, HX_F32, x.data_ptr(), w.data_ptr(), dy.data_ptr(), dx.data_ptr_mut(),
                               dw.data_ptr_mut(), db.data_ptr_mut(), rows, in, out));
        return {dx, dw, db};
    }
};

// kernels/rms_norm.rs:57-132.
class RMSNormOp : public Op {
  public:
    Tensor x, w;
    float eps;
    RMSNormOp(Tensor x_, Tensor w_, float e) : x(std::move(x_)), w(std::move(w_)), eps(e) {}
    const char* name() const override { return "RMSNorm"; }
    std::vector<std::optional<Tensor>> backward(const Tensor& dy) const override {
        hx_ctx* c = ctx_of(dy, "RMSNorm backward");
        if (!contiguous(dy)) throw Error("RMSNorm backward: gradient must be contiguous");
        const int hidden = (int)last_dim(x);
        const int rows = (int)(x.shape.num_elements() / hidden);
        Tensor dx = Tensor::empty(DType::F32, x.shape, x.device);
        Tensor dw = Tensor::empty(DType::F32, w.shape, w.device);
        check(c, hx_rmsnorm_bwd(c, HX_F32, dy.data_ptr(), x.data_ptr(), w.data_ptr(), dx.data_ptr_mut(),
                                static_cast<float*>(dw.data_ptr_mut()), rows, hidden, eps));
        return {dx, dw};
    }
};

// The fused attention on strided [B, H, S, D] views, with RoPE applied to q
// and k first (nn/attention.rs:76-78); the backward returns the gradients of
// q and k before the rotation (rope_backward fused into the kernels).
class AttentionRopeOp : public Op {
  public:
    Tensor qr, kr, v, o, lse;
    hx_attn_shape shape;
    float scale, rope_base;
    bool causal;
    AttentionRopeOp(Tensor qr_, Tensor kr_, Tensor v_, Tensor o_, Tensor lse_, hx_attn_shape s, float sc, bool ca,
                    float rb)
        : qr(std::move(qr_)), kr(std::move(kr_)), v(std::move(v_)), o(std::move(o_)), lse(std::move(lse_)),
          shape(s), scale(sc), rope_base(rb), causal(ca) {}
    const char* name() const override { return "FlashAttention"; }
    std::vector<std::optional<Tensor>> backward(const Tensor& dout) const override {
        hx_ctx* c = ctx_of(dout, "FlashAttention backward");
        if (dout.strides != o.strides) throw Error("FlashAttention backward: gradient not in O's layout");
        Tensor dq = empty_strided(o.shape, o.strides, o.device);
        Tensor dk = empty_strided(o.shape, o.strides, o.device);
        Tensor dv = empty_strided(o.shape, o.strides, o.device);
        check(c, hx_attn_bwd_rope_strided(c, HX_F32, &shape, qr.data_ptr(), kr.data_ptr(), v.data_ptr(), o.data_ptr(),
                                          dout.data_ptr(), static_cast<const float*>(lse.data_ptr()),
                                          dq.data_ptr_mut(), dk.data_ptr_mut(), dv.data_ptr_mut(), nullptr, 0,
                                          scale, causal ? 1 : 0, rope_base));
        return {dq, dk, dv};
    }
};

// A view on the graph: `t` seen with another shape / strides.
Tensor graph_view(const Tensor& t, Shape shape, std::vector<int64_t> strides) {
    Tensor v = t.view(shape, strides);
    if (!t.requires_grad) return v;
    return v.with_node(std::make_shared<ViewOp>(t.shape, t.strides, strides), {t});
}

}  // namespace

Linear::Linear(size_t in_features, size_t out_features, const Device& device, uint64_t seed) {
    // nn/linear.rs: weight uniform in +-sqrt(6 / in), bias zeros.
    std::mt19937_64 g(seed);
    const float bound = std::sqrt(6.0f / (float)in_features);
    std::uniform_real_distribution<float> u(-bound, bound);
    std::vector<float> w(in_features * out_features);
    for (auto& x : w) x = u(g);
    weight = Tensor::from_slice(DType::F32, Shape{in_features, out_features}, w).to(device).requires_grad_(true);
    bias = Tensor::from_slice(DType::F32, Shape{out_features}, std::vector<float>(out_features, 0.f))
               .to(device)
               .requires_grad_(true);
}

Tensor Linear::forward(const Tensor& x) const {
    hx_ctx* c = ctx_of(x, "Linear");
    if (!contiguous(x)) throw Error("Linear: input must be contiguous");
    const size_t in = weight.shape.dims()[0], out = weight.shape.dims()[1];
    if (last_dim(x) != in) throw Error("Linear: input width does not match in_features");
    std::vector<size_t> yd = x.shape.dims();
    yd.back() = out;
    Tensor y = Tensor::empty(DType::F32, Shape(yd), x.device);
    check(c, hx_linear_fwd(c, HX_F32, x.data_ptr(), weight.data_ptr(), bias.data_ptr(), y.data_ptr_mut(),
                           (int)(x.shape.num_elements() / in), (int)in, (int)out));
    if (x.requires_grad || weight.requires_grad || bias.requires_grad)
        return y.with_node(std::make_shared<LinearOp>(x, weight, bias), {x, weight, bias});
    return y;
}

RMSNorm::RMSNorm(size_t hidden, const Device& device) {
    weight = Tensor::from_slice(DType::F32, Shape{hidden}, std::vector<float>(hidden, 1.f)).to(device).requires_grad_(true);
}

Tensor RMSNorm::forward(const Tensor& x) const {
    hx_ctx* c = ctx_of(x, "RMSNorm");
    if (!contiguous(x)) throw Error("RMSNorm: input must be contiguous");
    const int hidden = (int)last_dim(x);
    Tensor y = Tensor::empty(DType::F32, x.shape, x.device);
    check(c, hx_rmsnorm_fwd(c, HX_F32, x.data_ptr(), weight.data_ptr(), y.data_ptr_mut(),
                            (int)(x.shape.num_elements() / hidden), hidden, eps));
    if (x.requires_grad || weight.requires_grad)
        return y.with_node(std::make_shared<RMSNormOp>(x, weight, eps), {x, weight});
    return y;
}

MultiHeadAttention::MultiHeadAttention(size_t hidden, size_t heads, const Device& device, bool causal_,
                                       uint64_t seed)
    : norm(hidden, device),
      q_proj(hidden, hidden, device, seed * 4 + 1),
      k_proj(hidden, hidden, device, seed * 4 + 2),
      v_proj(hidden, hidden, device, seed * 4 + 3),
      out_proj(hidden, hidden, device, seed * 4 + 4),
      num_heads(heads),
      head_dim(heads ? hidden / heads : 0),
      causal(causal_) {
    if (heads == 0 || hidden % heads) throw Error("hidden_dim must be divisible by num_heads");  // attention.rs:24-28
}

Tensor MultiHeadAttention::forward(const Tensor& x) const {
    hx_ctx* c = ctx_of(x, "MultiHeadAttention");
    const auto& d = x.shape.dims();
    if (d.size() != 3) throw Error("MultiHeadAttention: input is [B, S, hidden]");
    const size_t B = d[0], S = d[1], Hd = d[2], H = num_heads, D = head_dim;
    const float scale = 1.0f / std::sqrt((float)D);

    const Tensor n = norm.forward(x);                                    // 1. pre-norm
    const Tensor q = q_proj.forward(n), k = k_proj.forward(n), v = v_proj.forward(n);  // 2. projections
    // 3. heads: [B, S, H*D] seen as [B, H, S, D] (attention.rs:62-73 without the copies)
    const Shape hs{B, H, S, D};
    const std::vector<int64_t> hst{(int64_t)(S * Hd), (int64_t)D, (int64_t)Hd, 1};
    const Tensor qh = graph_view(q, hs, hst), kh = graph_view(k, hs, hst), vh = graph_view(v, hs, hst);
    // 4-5. RoPE on q and k, then the fused attention
    hx_attn_shape shp{(int32_t)B, (int32_t)H, (int32_t)S, (int32_t)D, hst[0], hst[1], hst[2]};
    Tensor qr = empty_strided(hs, hst, x.device), kr = empty_strided(hs, hst, x.device);
    check(c, hx_rope_fwd(c, HX_F32, &shp, qh.data_ptr(), qr.data_ptr_mut(), rope_base));
    check(c, hx_rope_fwd(c, HX_F32, &shp, kh.data_ptr(), kr.data_ptr_mut(), rope_base));
    Tensor o = empty_strided(hs, hst, x.device);
    Tensor lse = Tensor::empty(DType::F32, Shape{B * H * S}, x.device);
    check(c, hx_attn_fwd_strided(c, HX_F32, &shp, qr.data_ptr(), kr.data_ptr(), vh.data_ptr(), o.data_ptr_mut(),
                                 static_cast<float*>(lse.data_ptr_mut()), scale, causal ? 1 : 0));
    const Tensor att = o.with_node(std::make_shared<AttentionRopeOp>(qr, kr, vh, o, lse, shp, scale, causal, rope_base),
                                   {qh, kh, vh});
    // 6. merge: O's memory is already [B, S, H, D] (attention.rs:91-94 without the copies)
    const Shape ms{B, S, Hd};
    const Tensor merged = graph_view(att, ms, ms.contiguous_strides());
    return out_proj.forward(merged);  // 7. output projection
}

std::vector<Tensor*> MultiHeadAttention::parameters() {
    return {&norm.weight,  &q_proj.weight, &q_proj.bias,   &k_proj.weight, &k_proj.bias,
            &v_proj.weight, &v_proj.bias,  &out_proj.weight, &out_proj.bias};
}

}  // namespace haelixe
