// Parity tests of the C++ host side (haelixe_b200/host) against the CPU
// oracle, written like the reference's own tests (tests/tensor_tests.rs:
// tensors built with from_slice, compared with assert_tensor_eq at a
// tolerance, gradients taken through the autograd graph).
//
// TEST INFRASTRUCTURE: this program links the oracle (oracle/liboracle.so)
// as the checker; the host library under test does not.
//
//   test_haelixe_host             all tests (needs a CUDA GPU)
//   test_haelixe_host --cpu-only  the tests that need no GPU
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

#include "haelixe.hpp"

extern "C" {
int ora_attn_fwd(const float* q, const float* k, const float* v, float* o, float* lse, int BH, int S, int D,
                 float scale, int causal);
int ora_attn_bwd(const float* q, const float* k, const float* v, const float* dout, float* dq, float* dk,
                 float* dv, int BH, int S, int D, float scale, int causal, int ref_compat);
void ora_round_bf16(const float* x, float* y, long n);
void ora_matmul(const float* a, const float* b, float* out, long m, long k, long n);
void ora_rms_norm_fwd(const float* x, const float* w, float* out, long rows, int hidden, float eps);
void ora_rms_norm_bwd(const float* g, const float* x, const float* w, float* dx, float* dw, long rows, int hidden,
                      float eps);
void ora_rope_fwd(const float* x, float* out, long tokens, int S, int D, float base);
void ora_rope_bwd(const float* g, float* out, long tokens, int S, int D, float base);
}

using haelixe::Device;
using haelixe::DType;
using haelixe::Shape;
using haelixe::Tensor;

namespace {

struct Failure {
    std::string what;
};

void require(bool ok, const std::string& what) {
    if (!ok) throw Failure{what};
}

// tests/tensor_tests.rs assert_tensor_eq: max |a - b| <= tol.
void assert_tensor_eq(const std::vector<float>& got, const std::vector<float>& want, float tol,
                      const std::string& name) {
    require(got.size() == want.size(), name + ": length mismatch");
    float worst = 0.f;
    for (size_t i = 0; i < got.size(); ++i) {
        const float e = std::fabs(got[i] - want[i]);
        if (!(e <= worst)) worst = e;  // NaN-propagating max
    }
    char buf[160];
    std::snprintf(buf, sizeof(buf), "%s: max |err| %.3g > %.3g", name.c_str(), worst, tol);
    require(worst <= tol, buf);
}

std::vector<float> randn(size_t n, unsigned seed, bool bf16) {
    std::mt19937 g(seed);
    std::normal_distribution<float> nd(0.f, 1.f);
    std::vector<float> v(n);
    for (auto& x : v) x = nd(g);
    if (bf16) ora_round_bf16(v.data(), v.data(), (long)n);
    return v;
}

// ---- tests that need no GPU --------------------------------------------------------

void test_contiguous_strides() {
    const Shape s{2, 3, 4};
    require(s.contiguous_strides() == std::vector<int64_t>({12, 4, 1}), "strides");
    require(s.num_elements() == 24, "num_elements");
}

void test_bf16_roundtrip() {  // tests/tensor_tests.rs:93-102
    const Tensor t = Tensor::from_slice(DType::BF16, Shape{3}, {1.0f, -2.5f, 3.14f});
    const auto back = t.to_vec_f32();
    require(back[0] == 1.0f && back[1] == -2.5f, "exact values survive");
    require(std::fabs(back[2] - 3.14f) < 0.01f, "3.14 rounds to the nearest bf16");
    require(back[2] == 3.140625f, "round to nearest even");
}

void test_flash_attention_requires_gpu() {  // tensor.rs:652
    const Tensor q = Tensor::from_slice(DType::F32, Shape{1, 2, 4}, std::vector<float>(8, 0.5f));
    try {
        (void)q.flash_attention(q, q, 0.5f);
    } catch (const haelixe::Error& e) {
        require(std::string(e.what()).find("FlashAttention currently requires GPU") != std::string::npos,
                std::string("message: ") + e.what());
        return;
    }
    throw Failure{"a CPU tensor must not run the attention"};
}

struct Scale2 : haelixe::Op {
    const char* name() const override { return "Scale2"; }
    std::vector<std::optional<Tensor>> backward(const Tensor& g) const override {
        auto v = g.to_vec_f32();
        for (auto& x : v) x *= 2.f;
        return {Tensor::from_slice(DType::F32, g.shape, v)};
    }
};

void test_topo_sort_and_seeded_backward() {  // autograd.rs:82-110, tensor.rs:240-266
    const Tensor leaf = Tensor::from_slice(DType::F32, Shape{2}, {1.f, 2.f}).requires_grad_(true);
    const Tensor mid = Tensor::from_slice(DType::F32, Shape{2}, {2.f, 4.f}).with_node(std::make_shared<Scale2>(), {leaf});
    const Tensor out = Tensor::from_slice(DType::F32, Shape{2}, {4.f, 8.f}).with_node(std::make_shared<Scale2>(), {mid});
    const auto order = out.topo_sort();
    require(order.size() == 3 && order[0].id == out.id && order[2].id == leaf.id, "loss -> leaves order");
    const auto grads = out.backward_with_seed(Tensor::from_slice(DType::F32, Shape{2}, {1.f, 1.f}));
    assert_tensor_eq(grads.at(leaf.id.value).to_vec_f32(), {4.f, 4.f}, 0.f, "d out / d leaf");
}

// ---- GPU tests -------------------------------------------------------------------

void attention_case(DType dt, int BH, int S, int D, bool causal, float tol) {
    const bool bf = dt == DType::BF16;
    const size_t n = (size_t)BH * S * D;
    const auto q = randn(n, 11, bf), k = randn(n, 12, bf), v = randn(n, 13, bf), dout = randn(n, 14, bf);
    const float scale = 1.0f / std::sqrt((float)D);
    const Device cuda = Device::cuda();
    const Shape sh{(size_t)BH, (size_t)S, (size_t)D};
    const Tensor qt = Tensor::from_slice(dt, sh, q).to(cuda).requires_grad_(true);
    const Tensor kt = Tensor::from_slice(dt, sh, k).to(cuda).requires_grad_(true);
    const Tensor vt = Tensor::from_slice(dt, sh, v).to(cuda).requires_grad_(true);
    const Tensor o = causal ? qt.flash_attention_causal(kt, vt, scale) : qt.flash_attention(kt, vt, scale);
    require(o.node && std::string(o.node->op->name()) == "FlashAttention", "the output carries the op");
    const auto grads = o.backward_with_seed(Tensor::from_slice(dt, sh, dout).to(cuda));

    std::vector<float> ro(n), rdq(n), rdk(n), rdv(n);
    require(ora_attn_fwd(q.data(), k.data(), v.data(), ro.data(), nullptr, BH, S, D, scale, causal) == 0, "oracle");
    require(ora_attn_bwd(q.data(), k.data(), v.data(), dout.data(), rdq.data(), rdk.data(), rdv.data(), BH, S, D,
                         scale, causal, 0) == 0,
            "oracle");
    assert_tensor_eq(o.to_vec_f32(), ro, tol, "O");
    assert_tensor_eq(grads.at(qt.id.value).to_vec_f32(), rdq, tol, "dQ");
    assert_tensor_eq(grads.at(kt.id.value).to_vec_f32(), rdk, tol, "dK");
    assert_tensor_eq(grads.at(vt.id.value).to_vec_f32(), rdv, tol, "dV");
}

// The path's parity tolerances: max-abs 1e-3 for f32 I/O, 2e-2 for bf16 I/O.
void test_flash_attention_f32_matches_oracle() { attention_case(DType::F32, 2, 80, 64, false, 1e-3f); }
void test_flash_attention_f32_causal_matches_oracle() { attention_case(DType::F32, 3, 77, 32, true, 1e-3f); }
void test_flash_attention_bf16_causal_matches_oracle() { attention_case(DType::BF16, 2, 320, 128, true, 2e-2f); }
void test_flash_attention_bf16_d64_matches_oracle() { attention_case(DType::BF16, 2, 200, 64, false, 2e-2f); }

void test_to_roundtrip_is_exact() {
    for (DType dt : {DType::F32, DType::BF16}) {
        const auto v = randn(1000, 5, dt == DType::BF16);
        const Tensor t = Tensor::from_slice(dt, Shape{10, 100}, v);
        const Tensor back = t.to(Device::cuda()).to(Device::cpu());
        require(back.device.is_cpu() && back.to_vec_f32() == t.to_vec_f32(), "host -> device -> host");
    }
}

void test_arena_slab_returns_on_last_drop() {  // arena.rs:113-131
    const auto ctx = haelixe::CudaContext::get(0);
    const Shape sh{3, 1000};
    { const Tensor a = Tensor::empty(DType::F32, sh, Device::cuda()); }
    const auto before = ctx->arena_stats();
    {
        const Tensor b = Tensor::empty(DType::F32, sh, Device::cuda());
        const Tensor alias = b;  // shares the storage: the slab stays out while either lives
        (void)alias;
    }
    const auto after = ctx->arena_stats();
    require(after.hits == before.hits + 1, "the dropped slab is reused from its bin");
}

void test_gradient_through_to() {  // tests/tensor_tests.rs:105-115
    const int BH = 1, S = 64, D = 64;
    const size_t n = (size_t)BH * S * D;
    const Shape sh{1, 64, 64};
    const Tensor q = Tensor::from_slice(DType::F32, sh, randn(n, 21, false)).requires_grad_(true);
    const Tensor k = Tensor::from_slice(DType::F32, sh, randn(n, 22, false)).requires_grad_(true);
    const Tensor v = Tensor::from_slice(DType::F32, sh, randn(n, 23, false)).requires_grad_(true);
    const Device cuda = Device::cuda();
    const Tensor o = q.to(cuda).flash_attention(k.to(cuda), v.to(cuda), 0.125f);
    const auto grads = o.backward_with_seed(Tensor::from_slice(DType::F32, sh, randn(n, 24, false)).to(cuda));
    for (const Tensor* leaf : {&q, &k, &v}) {
        auto it = grads.find(leaf->id.value);
        require(it != grads.end(), "every CPU leaf receives a gradient");
        require(it->second.device.is_cpu(), "the gradient comes back to the leaf's device");
        require(it->second.shape == sh, "gradient shape");
    }
}

// ---- the attention layer (nn/attention.rs:46-98) -----------------------------------

using Vec = std::vector<float>;

Vec transpose(const Vec& a, size_t rows, size_t cols) {
    Vec t(a.size());
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) t[c * rows + r] = a[r * cols + c];
    return t;
}

Vec matmul(const Vec& a, const Vec& b, size_t m, size_t k, size_t n) {
    Vec out(m * n);
    ora_matmul(a.data(), b.data(), out.data(), (long)m, (long)k, (long)n);
    return out;
}

Vec col_sum(const Vec& a, size_t rows, size_t cols) {
    Vec s(cols, 0.f);
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) s[c] += a[r * cols + c];
    return s;
}

struct MhaParams {
    Vec norm_w, w[4], b[4];  // q, k, v, o; weights [in, out]
};

struct MhaGrads {
    Vec y, dx, norm_w, w[4], b[4];
};

// MultiHeadAttention::forward and its backward composed from the oracle's
// kernels, in the reference's op order (the C restatement of oracle.py's
// mha_forward / mha_backward).
MhaGrads mha_oracle(const Vec& x, const MhaParams& p, const Vec& dy, size_t B, size_t S, size_t H, size_t D,
                    bool causal) {
    const size_t Hd = H * D, rows = B * S;
    const float scale = 1.0f / std::sqrt((float)D), eps = 1e-5f, base = 10000.0f;
    auto split = [&](const Vec& t) {  // [B, S, H*D] -> [B*H, S, D]
        Vec o(t.size());
        for (size_t b = 0; b < B; ++b)
            for (size_t s = 0; s < S; ++s)
                for (size_t h = 0; h < H; ++h)
                    for (size_t d = 0; d < D; ++d) o[((b * H + h) * S + s) * D + d] = t[(b * S + s) * Hd + h * D + d];
        return o;
    };
    auto merge = [&](const Vec& t) {  // the inverse
        Vec o(t.size());
        for (size_t b = 0; b < B; ++b)
            for (size_t s = 0; s < S; ++s)
                for (size_t h = 0; h < H; ++h)
                    for (size_t d = 0; d < D; ++d) o[(b * S + s) * Hd + h * D + d] = t[((b * H + h) * S + s) * D + d];
        return o;
    };
    auto rope = [&](const Vec& t, bool fwd) {
        Vec o(t.size());
        (fwd ? ora_rope_fwd : ora_rope_bwd)(t.data(), o.data(), (long)(B * H * S), (int)S, (int)D, base);
        return o;
    };
    MhaGrads g;
    Vec n(rows * Hd);
    ora_rms_norm_fwd(x.data(), p.norm_w.data(), n.data(), (long)rows, (int)Hd, eps);
    Vec proj[3];
    for (int c = 0; c < 3; ++c) {
        proj[c] = matmul(n, p.w[c], rows, Hd, Hd);
        for (size_t r = 0; r < rows; ++r)
            for (size_t j = 0; j < Hd; ++j) proj[c][r * Hd + j] += p.b[c][j];
    }
    const Vec qr = rope(split(proj[0]), true), kr = rope(split(proj[1]), true), vs = split(proj[2]);
    Vec o(qr.size());
    ora_attn_fwd(qr.data(), kr.data(), vs.data(), o.data(), nullptr, (int)(B * H), (int)S, (int)D, scale, causal);
    const Vec om = merge(o);
    g.y = matmul(om, p.w[3], rows, Hd, Hd);
    for (size_t r = 0; r < rows; ++r)
        for (size_t j = 0; j < Hd; ++j) g.y[r * Hd + j] += p.b[3][j];
    g.w[3] = matmul(transpose(om, rows, Hd), dy, Hd, rows, Hd);
    g.b[3] = col_sum(dy, rows, Hd);
    const Vec dout = split(matmul(dy, transpose(p.w[3], Hd, Hd), rows, Hd, Hd));
    Vec dq(qr.size()), dk(qr.size()), dv(qr.size());
    ora_attn_bwd(qr.data(), kr.data(), vs.data(), dout.data(), dq.data(), dk.data(), dv.data(), (int)(B * H), (int)S,
                 (int)D, scale, causal, 0);
    const Vec dproj[3] = {merge(rope(dq, false)), merge(rope(dk, false)), merge(dv)};
    Vec dn(rows * Hd, 0.f);
    for (int c = 0; c < 3; ++c) {
        g.w[c] = matmul(transpose(n, rows, Hd), dproj[c], Hd, rows, Hd);
        g.b[c] = col_sum(dproj[c], rows, Hd);
        const Vec t = matmul(dproj[c], transpose(p.w[c], Hd, Hd), rows, Hd, Hd);
        for (size_t i = 0; i < dn.size(); ++i) dn[i] += t[i];
    }
    g.dx.resize(rows * Hd);
    g.norm_w.resize(Hd);
    ora_rms_norm_bwd(dn.data(), x.data(), p.norm_w.data(), g.dx.data(), g.norm_w.data(), (long)rows, (int)Hd, eps);
    return g;
}

void mha_case(bool causal) {
    const size_t B = 2, S = 128, H = 4, D = 64, Hd = H * D;  // the reference's CPU-runnable layer shape
    std::mt19937 gen(99);
    std::uniform_real_distribution<float> uw(-std::sqrt(6.0f / Hd), std::sqrt(6.0f / Hd)), ub(-0.1f, 0.1f),
        un(0.5f, 1.5f);
    MhaParams p;
    p.norm_w.resize(Hd);
    for (auto& v : p.norm_w) v = un(gen);
    for (int c = 0; c < 4; ++c) {
        p.w[c].resize(Hd * Hd);
        p.b[c].resize(Hd);
        for (auto& v : p.w[c]) v = uw(gen);
        for (auto& v : p.b[c]) v = ub(gen);
    }
    const Vec x = randn(B * S * Hd, 31, false), dy = randn(B * S * Hd, 32, false);
    const Device cuda = Device::cuda();
    haelixe::MultiHeadAttention mha(Hd, H, cuda, causal);
    auto param = [&](const Vec& v, Shape s) { return Tensor::from_slice(DType::F32, s, v).to(cuda).requires_grad_(true); };
    mha.norm.weight = param(p.norm_w, Shape{Hd});
    haelixe::Linear* lin[4] = {&mha.q_proj, &mha.k_proj, &mha.v_proj, &mha.out_proj};
    for (int c = 0; c < 4; ++c) {
        lin[c]->weight = param(p.w[c], Shape{Hd, Hd});
        lin[c]->bias = param(p.b[c], Shape{Hd});
    }
    const Tensor xt = param(x, Shape{B, S, Hd});
    const Tensor y = mha.forward(xt);
    const auto grads = y.backward_with_seed(Tensor::from_slice(DType::F32, Shape{B, S, Hd}, dy).to(cuda));
    const MhaGrads r = mha_oracle(x, p, dy, B, S, H, D, causal);
    const float tol = 1e-3f;  // f32 I/O
    assert_tensor_eq(y.to_vec_f32(), r.y, tol, "y");
    assert_tensor_eq(grads.at(xt.id.value).to_vec_f32(), r.dx, tol, "dx");
    assert_tensor_eq(grads.at(mha.norm.weight.id.value).to_vec_f32(), r.norm_w, tol, "d norm_w");
    const char* names[4] = {"q", "k", "v", "o"};
    for (int c = 0; c < 4; ++c) {
        assert_tensor_eq(grads.at(lin[c]->weight.id.value).to_vec_f32(), r.w[c], tol, std::string("d w") + names[c]);
        assert_tensor_eq(grads.at(lin[c]->bias.id.value).to_vec_f32(), r.b[c], tol, std::string("d b") + names[c]);
    }
}

void test_multi_head_attention_matches_oracle() { mha_case(false); }
void test_multi_head_attention_causal_matches_oracle() { mha_case(true); }

void test_multi_head_attention_rejects_bad_heads() {  // attention.rs:24-28
    try {
        haelixe::MultiHeadAttention bad(10, 3, Device::cpu());
    } catch (const haelixe::Error& e) {
        require(std::string(e.what()).find("divisible") != std::string::npos, e.what());
        return;
    }
    throw Failure{"hidden_dim % num_heads != 0 must be refused"};
}

}  // namespace

int main(int argc, char** argv) {
    const bool cpu_only = argc > 1 && std::strcmp(argv[1], "--cpu-only") == 0;
    struct Case {
        const char* name;
        std::function<void()> fn;
        bool gpu;
    };
    const std::vector<Case> cases = {
        {"contiguous_strides", test_contiguous_strides, false},
        {"bf16_roundtrip", test_bf16_roundtrip, false},
        {"flash_attention_requires_gpu", test_flash_attention_requires_gpu, false},
        {"topo_sort_and_seeded_backward", test_topo_sort_and_seeded_backward, false},
        {"flash_attention_f32_matches_oracle", test_flash_attention_f32_matches_oracle, true},
        {"flash_attention_f32_causal_matches_oracle", test_flash_attention_f32_causal_matches_oracle, true},
        {"flash_attention_bf16_causal_matches_oracle", test_flash_attention_bf16_causal_matches_oracle, true},
        {"flash_attention_bf16_d64_matches_oracle", test_flash_attention_bf16_d64_matches_oracle, true},
        {"to_roundtrip_is_exact", test_to_roundtrip_is_exact, true},
        {"arena_slab_returns_on_last_drop", test_arena_slab_returns_on_last_drop, true},
        {"gradient_through_to", test_gradient_through_to, true},
        {"multi_head_attention_matches_oracle", test_multi_head_attention_matches_oracle, true},
        {"multi_head_attention_causal_matches_oracle", test_multi_head_attention_causal_matches_oracle, true},
        {"multi_head_attention_rejects_bad_heads", test_multi_head_attention_rejects_bad_heads, false},
    };
    int failed = 0, ran = 0;
    for (const auto& c : cases) {
        if (cpu_only && c.gpu) continue;
        ++ran;
        try {
            c.fn();
            std::printf("ok %s\n", c.name);
        } catch (const Failure& f) {
            ++failed;
            std::printf("FAILED %s: %s\n", c.name, f.what.c_str());
        } catch (const std::exception& e) {
            ++failed;
            std::printf("FAILED %s: exception: %s\n", c.name, e.what());
        }
    }
    std::printf("%d of %d passed\n", ran - failed, ran);
    return failed == 0 ? 0 : 1;
}
