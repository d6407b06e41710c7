// Implementation of the C++ host side (haelixe.hpp) over the C ABI.
#include "haelixe.hpp"

#include <atomic>
#include <cstring>
#include <mutex>
#include <unordered_set>

namespace haelixe {
namespace {

std::string last_error(hx_ctx* c, int status) {
    char buf[512] = {0};
    if (c) hx_last_error(c, buf, sizeof(buf));
    std::string msg = buf[0] ? buf : hx_status_string(status);
    return "haelixe_cuda error " + std::to_string(status) + ": " + msg;
}

void check(hx_ctx* c, int status) {
    if (status != HX_OK) throw Error(last_error(c, status));
}

hx_dtype code_of(DType dt) { return dt == DType::BF16 ? HX_BF16 : HX_F32; }

// f32 -> bf16 bits, round to nearest, ties to even; NaN stays a quiet NaN.
uint16_t bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float bf16_value(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// The contiguous [BH, S, D] view the attention entry points take.
void dims3(const Tensor& t, int* bh, int* s, int* d) {
    const auto& dm = t.shape.dims();
    if (dm.size() != 3) throw Error("flash_attention expects [BH, S, D] tensors");
    if (t.strides != t.shape.contiguous_strides() || t.byte_offset != 0)
        throw Error("flash_attention expects contiguous tensors");
    *bh = (int)dm[0];
    *s = (int)dm[1];
    *d = (int)dm[2];
}

}  // namespace

size_t size_in_bytes(DType dt) { return dt == DType::BF16 ? 2 : 4; }

size_t Shape::num_elements() const {
    size_t n = 1;
    for (size_t d : dims_) n *= d;
    return n;
}

std::vector<int64_t> Shape::contiguous_strides() const {
    std::vector<int64_t> s(dims_.size());
    int64_t acc = 1;
    for (size_t i = dims_.size(); i-- > 0;) {
        s[i] = acc;
        acc *= (int64_t)dims_[i];
    }
    return s;
}

// ---- contexts and the arena ------------------------------------------------------

CudaContext::CudaContext(int device) : device_(device) { check(nullptr, hx_ctx_create(device, &raw_)); }

CudaContext::~CudaContext() {
    if (raw_) hx_ctx_destroy(raw_);
}

void CudaContext::sync() const { check(raw_, hx_sync(raw_)); }

hx_arena_stats CudaContext::arena_stats() const {
    hx_arena_stats s{};
    check(raw_, hx_arena_stats_get(raw_, &s));
    return s;
}

std::shared_ptr<CudaContext> CudaContext::get(int device) {
    // Process-lifetime contexts, deliberately never destroyed: a static map's
    // destructor would run at exit after the CUDA runtime's own teardown.
    static std::mutex mu;
    static auto* contexts = new std::unordered_map<int, std::shared_ptr<CudaContext>>();
    std::lock_guard<std::mutex> lk(mu);
    auto it = contexts->find(device);
    if (it != contexts->end()) return it->second;
    auto c = std::make_shared<CudaContext>(device);
    (*contexts)[device] = c;
    return c;
}

CudaAllocation::CudaAllocation(std::shared_ptr<CudaContext> ctx, uint64_t bytes) : ctx_(std::move(ctx)) {
    check(ctx_->raw(), hx_alloc(ctx_->raw(), bytes, &ptr_));
    size_ = hx_bin_size(bytes);
}

CudaAllocation::~CudaAllocation() {
    if (ptr_) hx_free(ctx_->raw(), ptr_);
}

TensorId TensorId::next() {
    static std::atomic<uint64_t> counter{1};
    return TensorId{counter.fetch_add(1)};
}

// ---- tensors ---------------------------------------------------------------------

Tensor Tensor::empty(DType dtype, Shape shape, const Device& device) {
    Tensor t;
    t.id = TensorId::next();
    t.dtype = dtype;
    t.strides = shape.contiguous_strides();
    t.shape = std::move(shape);
    t.storage = std::make_shared<Storage>();
    t.device = device;
    const uint64_t bytes = (uint64_t)t.shape.num_elements() * size_in_bytes(dtype);
    if (device.is_cuda())
        t.storage->cuda = std::make_shared<CudaAllocation>(device.context(), bytes);
    else
        t.storage->host.resize(bytes);
    return t;
}

Tensor Tensor::from_slice(DType dtype, Shape shape, const std::vector<float>& data) {
    if (data.size() != shape.num_elements()) throw Error("from_slice: data length does not match the shape");
    Tensor t = empty(dtype, std::move(shape));
    if (dtype == DType::F32) {
        std::memcpy(t.storage->host.data(), data.data(), data.size() * 4);
    } else {
        auto* out = reinterpret_cast<uint16_t*>(t.storage->host.data());
        for (size_t i = 0; i < data.size(); ++i) out[i] = bf16_bits(data[i]);
    }
    return t;
}

Tensor Tensor::requires_grad_(bool rg) const {
    Tensor t = *this;
    t.requires_grad = rg;
    return t;
}

const void* Tensor::data_ptr() const {
    const uint8_t* base = device.is_cuda() ? static_cast<const uint8_t*>(storage->cuda->ptr()) : storage->host.data();
    return base + byte_offset;
}

void* Tensor::data_ptr_mut() { return const_cast<void*>(data_ptr()); }

Tensor Tensor::to(const Device& dst) const {
    if (device == dst) return *this;
    if (strides != shape.contiguous_strides())
        throw Error("to: only contiguous tensors move between devices on this path");
    const uint64_t bytes = (uint64_t)shape.num_elements() * size_in_bytes(dtype);
    Tensor out = empty(dtype, shape, dst);
    if (device.is_cpu() && dst.is_cuda()) {
        hx_ctx* c = dst.context()->raw();
        check(c, hx_copy_h2d(c, out.data_ptr_mut(), data_ptr(), bytes));
    } else if (device.is_cuda() && dst.is_cpu()) {
        hx_ctx* c = device.context()->raw();
        check(c, hx_copy_d2h(c, out.data_ptr_mut(), data_ptr(), bytes));
    } else {  // CUDA -> another CUDA context: through the host
        Tensor host = to(Device::cpu());
        Tensor moved = host.to(dst);
        out.storage = moved.storage;
    }
    out.requires_grad = requires_grad;
    if (requires_grad) return out.with_node(std::make_shared<ToDeviceOp>(device), {*this});
    return out;
}

std::vector<float> Tensor::to_vec_f32() const {
    const Tensor h = device.is_cuda() ? to(Device::cpu()) : *this;
    if (h.strides != h.shape.contiguous_strides()) throw Error("to_vec_f32: tensor is not contiguous");
    const size_t n = h.shape.num_elements();
    std::vector<float> out(n);
    if (dtype == DType::F32) {
        std::memcpy(out.data(), h.data_ptr(), n * 4);
    } else {
        const auto* b = static_cast<const uint16_t*>(h.data_ptr());
        for (size_t i = 0; i < n; ++i) out[i] = bf16_value(b[i]);
    }
    return out;
}

Tensor Tensor::flash_attention(const Tensor& k, const Tensor& v, float scale) const {
    return flash_attention_ex(k, v, scale, false);
}

Tensor Tensor::flash_attention_causal(const Tensor& k, const Tensor& v, float scale) const {
    return flash_attention_ex(k, v, scale, true);
}

Tensor Tensor::flash_attention_ex(const Tensor& k, const Tensor& v, float scale, bool causal) const {
    if (!device.is_cuda()) throw Error("FlashAttention currently requires GPU");  // tensor.rs:652
    if (k.device != device || v.device != device || k.dtype != dtype || v.dtype != dtype ||
        !(k.shape == shape) || !(v.shape == shape))
        throw Error("flash_attention: q, k, v must share device, dtype and shape");
    int bh, s, d;
    dims3(*this, &bh, &s, &d);
    dims3(k, &bh, &s, &d);
    dims3(v, &bh, &s, &d);
    Tensor out = empty(dtype, shape, device);
    Tensor lse = empty(DType::F32, Shape{(size_t)bh, (size_t)s}, device);
    hx_ctx* c = device.context()->raw();
    check(c, hx_flash_attention_fwd(c, code_of(dtype), data_ptr(), k.data_ptr(), v.data_ptr(),
                                    out.data_ptr_mut(), static_cast<float*>(lse.data_ptr_mut()), bh, s, d,
                                    scale, causal ? 1 : 0));
    if (requires_grad || k.requires_grad || v.requires_grad) {
        auto op = std::make_shared<FlashAttentionOp>(*this, k, v, scale, out, lse, causal);
        return out.with_node(op, {*this, k, v});
    }
    return out;
}

std::vector<std::optional<Tensor>> FlashAttentionOp::backward(const Tensor& grad_out) const {
    int bh, s, d;
    dims3(q, &bh, &s, &d);
    Tensor g = grad_out.device == q.device ? grad_out : grad_out.to(q.device);
    if (g.dtype != q.dtype || !(g.shape == q.shape)) throw Error("FlashAttention backward: bad grad_out");
    dims3(g, &bh, &s, &d);
    Tensor dq = Tensor::empty(q.dtype, q.shape, q.device);
    Tensor dk = Tensor::empty(q.dtype, q.shape, q.device);
    Tensor dv = Tensor::empty(q.dtype, q.shape, q.device);
    hx_ctx* c = q.device.context()->raw();
    check(c, hx_flash_attention_bwd(c, code_of(q.dtype), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                    g.data_ptr(), static_cast<const float*>(lse.data_ptr()), dq.data_ptr_mut(),
                                    dk.data_ptr_mut(), dv.data_ptr_mut(), nullptr, 0, bh, s, d, scale,
                                    causal ? 1 : 0));
    return {dq, dk, dv};  // parent order [q, k, v], flash_attention.rs:38
}

std::vector<std::optional<Tensor>> ToDeviceOp::backward(const Tensor& grad_out) const {
    return {grad_out.to(source)};
}

Tensor Tensor::view(Shape new_shape, std::vector<int64_t> new_strides) const {
    if (new_strides.size() != new_shape.dims().size()) throw Error("view: one stride per dimension");
    Tensor t = *this;
    t.id = TensorId::next();
    t.shape = std::move(new_shape);
    t.strides = std::move(new_strides);
    t.requires_grad = false;
    t.node = nullptr;
    return t;
}

Tensor add(const Tensor& a, const Tensor& b) {
    if (a.device != b.device || a.dtype != b.dtype || !(a.shape == b.shape) || a.strides != b.strides)
        throw Error("add: operands must share device, dtype, shape and strides");
    const size_t n = a.shape.num_elements();
    // Dense layouts only (contiguous, or a permutation of a contiguous block):
    // the element order then is the same in a, b and the result.
    Tensor out = Tensor::empty(a.dtype, a.shape, a.device).view(a.shape, a.strides);
    if (a.device.is_cuda()) {
        hx_ctx* c = a.device.context()->raw();
        check(c, hx_add(c, code_of(a.dtype), a.data_ptr(), b.data_ptr(), out.data_ptr_mut(), n));
    } else {
        if (a.dtype != DType::F32) throw Error("add: CPU tensors are f32 on this path");
        const float* x = static_cast<const float*>(a.data_ptr());
        const float* y = static_cast<const float*>(b.data_ptr());
        float* z = static_cast<float*>(out.data_ptr_mut());
        for (size_t i = 0; i < n; ++i) z[i] = x[i] + y[i];
    }
    return out;
}

std::vector<std::optional<Tensor>> ViewOp::backward(const Tensor& grad_out) const {
    if (grad_out.strides != view_strides)
        throw Error("View backward: the gradient is not in the view's memory layout");
    return {grad_out.view(src_shape, src_strides)};
}

// ---- autograd ----------------------------------------------------------------------

Tensor Tensor::with_node(std::shared_ptr<Op> op, std::vector<Tensor> parents) const {
    Tensor t = *this;
    t.node = std::make_shared<Node>(Node{std::move(op), std::move(parents)});
    t.requires_grad = true;
    return t;
}

std::vector<Tensor> Tensor::topo_sort() const {
    std::unordered_set<uint64_t> visited;
    std::vector<Tensor> sorted;
    // Iterative post-order DFS: parents before children.
    struct Frame {
        Tensor t;
        size_t next;
    };
    std::vector<Frame> stack;
    stack.push_back({*this, 0});
    visited.insert(id.value);
    while (!stack.empty()) {
        Frame& f = stack.back();
        const size_t np = f.t.node ? f.t.node->parents.size() : 0;
        if (f.next < np) {
            const Tensor& p = f.t.node->parents[f.next++];
            if (visited.insert(p.id.value).second) stack.push_back({p, 0});
        } else {
            sorted.push_back(f.t);
            stack.pop_back();
        }
    }
    return std::vector<Tensor>(sorted.rbegin(), sorted.rend());  // loss -> leaves
}

std::unordered_map<uint64_t, Tensor> Tensor::backward_with_seed(const Tensor& seed) const {
    std::unordered_map<uint64_t, Tensor> grads;
    grads.emplace(id.value, seed);
    for (const Tensor& t : topo_sort()) {
        auto it = grads.find(t.id.value);
        if (it == grads.end() || !t.node) continue;
        const Tensor grad_out = it->second;
        std::vector<std::optional<Tensor>> pg = t.node->op->backward(grad_out);
        for (size_t i = 0; i < t.node->parents.size() && i < pg.size(); ++i) {
            if (!pg[i]) continue;
            const uint64_t pid = t.node->parents[i].id.value;
            auto have = grads.find(pid);
            if (have == grads.end())
                grads.emplace(pid, *pg[i]);
            else  // a tensor used more than once: gradients sum (tensor.rs:211-214)
                have->second = add(have->second, *pg[i]);
        }
    }
    return grads;
}

}  // namespace haelixe
