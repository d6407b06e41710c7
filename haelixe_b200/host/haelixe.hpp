// C++ host side of haelixe's attention path, above the C ABI
// (include/haelixe_cuda.h). It mirrors the crate's own types for this path,
// with the same names, argument meaning and error behaviour:
//
//   Device           <- src/device.rs:5-33 (Cpu, plus the Cuda variant the path adds)
//   CudaAllocation   <- the arena slab of src/gpu/arena.rs, returned to its bin
//                       when the last reference drops (the Arc rule, arena.rs:113-131)
//   Tensor           <- src/tensor.rs:25-39 (id, dtype, shape, strides, shared
//                       storage, byte offset, device, requires_grad, node)
//   Tensor::to       <- src/tensor.rs:299-356 (upload / download)
//   Tensor::flash_attention <- src/tensor.rs:644-666
//   FlashAttentionOp <- src/ops/flash_attention.rs (backward -> [dq, dk, dv])
//   Op, Node, with_node, topo_sort, backward_with_seed
//                    <- src/autograd.rs:55-118, src/tensor.rs:240-266 (gradients
//                       that meet are summed with add, kernels/binary.rs:40)
//   Linear, RMSNorm, MultiHeadAttention
//                    <- src/nn/linear.rs, src/nn/rms_norm.rs, src/nn/attention.rs:46-98
//                       (f32, the reference's GPU dtype; heads split and merged
//                       as strided views of the projections, not copies)
//
// The reference panics on misuse (tensor.rs:652 "FlashAttention currently
// requires GPU"); this layer throws haelixe::Error with the same text, and
// with the library's message when a C ABI call fails. No CPU fallback exists
// for the attention: a CPU tensor is an error, as in the reference.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "haelixe_cuda.h"

namespace haelixe {

class Error : public std::runtime_error {
  public:
    explicit Error(const std::string& what) : std::runtime_error(what) {}
};

// src/dtype.rs: the two dtypes of this path (f32 storage, bf16 storage).
enum class DType { F32, BF16 };
size_t size_in_bytes(DType dt);

// src/layout.rs Shape: row-major dims with contiguous strides.
class Shape {
  public:
    Shape() = default;
    Shape(std::initializer_list<size_t> dims) : dims_(dims) {}
    explicit Shape(std::vector<size_t> dims) : dims_(std::move(dims)) {}
    const std::vector<size_t>& dims() const { return dims_; }
    size_t num_elements() const;
    std::vector<int64_t> contiguous_strides() const;
    bool operator==(const Shape& o) const { return dims_ == o.dims_; }

  private:
    std::vector<size_t> dims_;
};

// One library context per GPU (hx_ctx): stream, arena, device status word.
class CudaContext {
  public:
    explicit CudaContext(int device);
    ~CudaContext();
    CudaContext(const CudaContext&) = delete;
    CudaContext& operator=(const CudaContext&) = delete;
    hx_ctx* raw() const { return raw_; }
    int device() const { return device_; }
    void sync() const;  // waits for the stream; reports a device-side timeout
    hx_arena_stats arena_stats() const;
    // The shared context of `device` (Device::cuda() hands out the same one).
    static std::shared_ptr<CudaContext> get(int device);

  private:
    hx_ctx* raw_ = nullptr;
    int device_ = 0;
};

// src/device.rs: where a tensor's data lives.
class Device {
  public:
    enum class Kind { Cpu, Cuda };
    static Device cpu() { return Device(Kind::Cpu, nullptr); }
    static Device cuda(int ordinal = 0) { return Device(Kind::Cuda, CudaContext::get(ordinal)); }
    bool is_cpu() const { return kind_ == Kind::Cpu; }
    bool is_cuda() const { return kind_ == Kind::Cuda; }
    const std::shared_ptr<CudaContext>& context() const { return ctx_; }
    // Same device: both CPU, or the same CUDA context.
    bool operator==(const Device& o) const { return kind_ == o.kind_ && ctx_ == o.ctx_; }
    bool operator!=(const Device& o) const { return !(*this == o); }

  private:
    Device(Kind k, std::shared_ptr<CudaContext> c) : kind_(k), ctx_(std::move(c)) {}
    Kind kind_;
    std::shared_ptr<CudaContext> ctx_;
};

// An arena slab (hx_alloc); the destructor returns it to its bin (hx_free).
class CudaAllocation {
  public:
    CudaAllocation(std::shared_ptr<CudaContext> ctx, uint64_t bytes);
    ~CudaAllocation();
    CudaAllocation(const CudaAllocation&) = delete;
    CudaAllocation& operator=(const CudaAllocation&) = delete;
    void* ptr() const { return ptr_; }
    uint64_t size() const { return size_; }  // hx_bin_size(bytes)

  private:
    std::shared_ptr<CudaContext> ctx_;
    void* ptr_ = nullptr;
    uint64_t size_ = 0;
};

// src/storage.rs CpuStorage with the Cuda backing the path adds.
struct Storage {
    std::vector<uint8_t> host;
    std::shared_ptr<CudaAllocation> cuda;
};

struct TensorId {
    uint64_t value = 0;
    static TensorId next();
    bool operator==(const TensorId& o) const { return value == o.value; }
};

class Tensor;

// src/autograd.rs:55-65
class Op {
  public:
    virtual ~Op() = default;
    virtual const char* name() const = 0;
    // Given the gradient of the output, the gradients of the inputs (parent order).
    virtual std::vector<std::optional<Tensor>> backward(const Tensor& grad_output) const = 0;
};

struct Node;

class Tensor {
  public:
    TensorId id;
    DType dtype = DType::F32;
    Shape shape;
    std::vector<int64_t> strides;
    std::shared_ptr<Storage> storage;
    size_t byte_offset = 0;
    Device device = Device::cpu();
    bool requires_grad = false;
    std::shared_ptr<Node> node;

    // Uninitialised storage of `shape` on `device` (tensor.rs:61-76 for the CPU).
    static Tensor empty(DType dtype, Shape shape, const Device& device = Device::cpu());
    // A CPU tensor from f32 values; BF16 rounds each to the nearest bf16, ties
    // to even (half::bf16::from_f32, as tensor.rs:706 converts).
    static Tensor from_slice(DType dtype, Shape shape, const std::vector<float>& data);
    Tensor requires_grad_(bool requires_grad) const;  // tensor.rs:112-115

    Tensor to(const Device& device) const;  // tensor.rs:299-356
    std::vector<float> to_vec_f32() const;  // contiguous values as f32 (downloads a CUDA tensor)

    // softmax(scale q k^T) v over [BH, S, D] (tensor.rs:644-666). The causal
    // form is the mask this path adds. Panics (throws) for a CPU tensor.
    Tensor flash_attention(const Tensor& k, const Tensor& v, float scale) const;
    Tensor flash_attention_causal(const Tensor& k, const Tensor& v, float scale) const;

    // A tensor sharing this one's storage with another shape / strides (no copy;
    // no autograd node: see ViewOp).
    Tensor view(Shape shape, std::vector<int64_t> strides) const;

    Tensor with_node(std::shared_ptr<Op> op, std::vector<Tensor> parents) const;  // autograd.rs:68-78
    std::vector<Tensor> topo_sort() const;                                         // autograd.rs:82-110
    // Reverse-mode AD from a seed gradient (tensor.rs:240-266): every tensor of
    // the graph, keyed by id value, to its gradient.
    std::unordered_map<uint64_t, Tensor> backward_with_seed(const Tensor& seed) const;

    const void* data_ptr() const;  // device or host address of element 0
    void* data_ptr_mut();

  private:
    Tensor flash_attention_ex(const Tensor& k, const Tensor& v, float scale, bool causal) const;
};

struct Node {
    std::shared_ptr<Op> op;
    std::vector<Tensor> parents;
};

// src/ops/flash_attention.rs, keeping the forward's O and log-sum-exp: the
// backward recomputes the softmax from them inside the fused kernels.
class FlashAttentionOp : public Op {
  public:
    Tensor q, k, v;
    float scale;
    Tensor o, lse;
    bool causal;
    FlashAttentionOp(Tensor q_, Tensor k_, Tensor v_, float scale_, Tensor o_, Tensor lse_, bool causal_)
        : q(std::move(q_)), k(std::move(k_)), v(std::move(v_)), scale(scale_), o(std::move(o_)),
          lse(std::move(lse_)), causal(causal_) {}
    const char* name() const override { return "FlashAttention"; }
    std::vector<std::optional<Tensor>> backward(const Tensor& grad_out) const override;
};

// Element-wise a + b of same-shape, same-layout tensors on one device
// (kernels/binary.rs:40-60 without broadcasting).
Tensor add(const Tensor& a, const Tensor& b);

// A reinterpretation of the parent's storage (shape / strides change, no
// data moves): the backward hands the gradient back with the parent's shape
// and strides, which needs the gradient in the view's memory layout.
class ViewOp : public Op {
  public:
    Shape src_shape;
    std::vector<int64_t> src_strides, view_strides;
    ViewOp(Shape s, std::vector<int64_t> ss, std::vector<int64_t> vs)
        : src_shape(std::move(s)), src_strides(std::move(ss)), view_strides(std::move(vs)) {}
    const char* name() const override { return "View"; }
    std::vector<std::optional<Tensor>> backward(const Tensor& grad_out) const override;
};

// ---- nn (src/nn) ---------------------------------------------------------------

// src/nn/linear.rs:54-56: y = x w + b with w stored [in, out].
class Linear {
  public:
    Tensor weight, bias;
    Linear(size_t in_features, size_t out_features, const Device& device, uint64_t seed);
    Tensor forward(const Tensor& x) const;
};

// src/nn/rms_norm.rs: weight initialised to ones, eps 1e-5.
class RMSNorm {
  public:
    Tensor weight;
    float eps = 1e-5f;
    RMSNorm(size_t hidden, const Device& device);
    Tensor forward(const Tensor& x) const;
};

// src/nn/attention.rs:5-98: pre-RMSNorm, Q/K/V projections, heads as strided
// views, RoPE (base 10000, attention.rs:76) on Q and K, the fused attention
// with scale 1/sqrt(head_dim), heads merged by a view, output projection.
// `causal` adds the mask the reference's layer lacks (false reproduces it).
class MultiHeadAttention {
  public:
    RMSNorm norm;
    Linear q_proj, k_proj, v_proj, out_proj;
    size_t num_heads, head_dim;
    bool causal;
    float rope_base = 10000.0f;
    MultiHeadAttention(size_t hidden, size_t num_heads, const Device& device, bool causal = false,
                       uint64_t seed = 0);
    Tensor forward(const Tensor& x) const;  // x: [B, S, hidden]
    std::vector<Tensor*> parameters();
};

// Moves a tensor across devices in the graph (the ContiguousOp node that
// tensor.rs:347-353 attaches): the gradient goes back to the source device.
class ToDeviceOp : public Op {
  public:
    Device source;
    explicit ToDeviceOp(Device src) : source(std::move(src)) {}
    const char* name() const override { return "ToDevice"; }
    std::vector<std::optional<Tensor>> backward(const Tensor& grad_out) const override;
};

}  // namespace haelixe
