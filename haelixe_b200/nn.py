"""Device-resident layers around the fused kernel.

Mirrors haelixe's `nn` modules: `RMSNorm` (src/nn/rms_norm.rs,
kernels/rms_norm.rs), `Linear` (src/nn/linear.rs), `MultiHeadAttention`
(src/nn/attention.rs:46-98), `FeedForward` (src/nn/mlp.rs) and
`TransformerBlock` (src/nn/transformer.rs), plus the pieces a language-model
training step over a block stack needs: a token `Embedding` (the reference
has none), `cross_entropy` (src/tensor.rs:754-801) and `BlockStack`. Every op
runs on the GPU through the library's C ABI: RMSNorm and GELU kernels, Linear
as cuBLAS GEMMs (weights stored [in, out] as in linear.rs:41) with the bias
and the block's residual add folded into the GEMM's C operand, and the fused
attention with RoPE. The reference's head split/merge copies
(`view -> transpose -> view`, attention.rs:62-73, 91-94) become strided
[B, H, S, D] views of the projection outputs: no data moves. Gradients flow
through torch.autograd, one Function per op, like the reference's `Op` nodes.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _native as N
from .attention import _DTYPES, context, flash_attention


def _p(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _ctx(t: torch.Tensor):
    if not t.is_cuda:
        raise RuntimeError("the attention block runs on CUDA tensors")
    if t.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {t.dtype}; f32 and bf16 are supported")
    c = context(t.device.index)
    c.use_stream()
    return c


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, x, w, eps):
        c = _ctx(x)
        x = x.contiguous()
        hidden = x.shape[-1]
        y = torch.empty_like(x)
        N.check(N.lib().hx_rmsnorm_fwd(c.handle, _DTYPES[x.dtype], _p(x), _p(w.contiguous()), _p(y),
                                       x.numel() // hidden, hidden, float(eps)), c.handle)
        fctx.save_for_backward(x, w)
        fctx.eps = eps
        return y

    @staticmethod
    def backward(fctx, dy):
        x, w = fctx.saved_tensors
        c = _ctx(x)
        dy = dy.contiguous()
        hidden = x.shape[-1]
        dx = torch.empty_like(x)
        dw = torch.empty(hidden, dtype=torch.float32, device=x.device)
        N.check(N.lib().hx_rmsnorm_bwd(c.handle, _DTYPES[x.dtype], _p(dy), _p(x), _p(w.contiguous()), _p(dx),
                                       _p(dw), x.numel() // hidden, hidden, float(fctx.eps)), c.handle)
        return dx, dw.to(w.dtype), None


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, x, w, b, r=None):
        c = _ctx(x)
        in_f, out_f = w.shape
        x2 = x.reshape(-1, in_f).contiguous()
        y = torch.empty(x2.shape[0], out_f, dtype=x.dtype, device=x.device)
        bp = _p(None if b is None else b.contiguous())
        if r is None:
            N.check(N.lib().hx_linear_fwd(c.handle, _DTYPES[x.dtype], _p(x2), _p(w.contiguous()), bp, _p(y),
                                          x2.shape[0], in_f, out_f), c.handle)
        else:
            r2 = r.reshape(x2.shape[0], out_f).contiguous()
            N.check(N.lib().hx_linear_residual_fwd(c.handle, _DTYPES[x.dtype], _p(x2), _p(w.contiguous()), bp,
                                                   _p(r2), _p(y), x2.shape[0], in_f, out_f), c.handle)
        fctx.save_for_backward(x2, w)
        fctx.in_shape, fctx.has_bias, fctx.has_res = x.shape, b is not None, r is not None
        return y.view(*x.shape[:-1], out_f)

    @staticmethod
    def backward(fctx, dy):
        x2, w = fctx.saved_tensors
        c = _ctx(x2)
        in_f, out_f = w.shape
        dy2 = dy.reshape(-1, out_f).contiguous()
        need_x, need_w, need_b = fctx.needs_input_grad[:3]
        dx = torch.empty_like(x2) if need_x else None
        dw = torch.empty_like(w) if need_w else None
        db = torch.empty(out_f, dtype=w.dtype, device=w.device) if (need_b and fctx.has_bias) else None
        N.check(N.lib().hx_linear_bwd(c.handle, _DTYPES[x2.dtype], _p(x2), _p(w.contiguous()), _p(dy2), _p(dx),
                                      _p(dw), _p(db), x2.shape[0], in_f, out_f), c.handle)
        dr = dy if fctx.has_res else None  # y = r + ...: the residual's gradient is dy itself
        return (None if dx is None else dx.view(fctx.in_shape)), dw, db, dr


class _GeluFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, x):
        c = _ctx(x)
        x = x.contiguous()
        y = torch.empty_like(x)
        N.check(N.lib().hx_gelu_fwd(c.handle, _DTYPES[x.dtype], _p(x), _p(y), x.numel()), c.handle)
        fctx.save_for_backward(x)
        return y

    @staticmethod
    def backward(fctx, dy):
        (x,) = fctx.saved_tensors
        c = _ctx(x)
        dy = dy.contiguous()
        dx = torch.empty_like(x)
        N.check(N.lib().hx_gelu_bwd(c.handle, _DTYPES[x.dtype], _p(dy), _p(x), _p(dx), x.numel()), c.handle)
        return dx


def _ids(ids: torch.Tensor) -> torch.Tensor:
    if ids.dtype not in (torch.int32, torch.int64, torch.uint32):
        raise TypeError("token ids / targets must be an integer tensor")
    return ids.reshape(-1).to(torch.int32).contiguous()  # read as uint32 by the kernels


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, ids, table):
        c = _ctx(table)
        vocab, dim = table.shape
        flat = _ids(ids)
        out = torch.empty(flat.numel(), dim, dtype=table.dtype, device=table.device)
        N.check(N.lib().hx_embedding_fwd(c.handle, _DTYPES[table.dtype], _p(table.contiguous()), _p(flat), _p(out),
                                         flat.numel(), vocab, dim), c.handle)
        fctx.save_for_backward(flat)
        fctx.vocab, fctx.table_dtype = vocab, table.dtype
        return out.view(*ids.shape, dim)

    @staticmethod
    def backward(fctx, dout):
        (flat,) = fctx.saved_tensors
        c = _ctx(dout)
        dim = dout.shape[-1]
        dout = dout.contiguous()
        dtable = torch.zeros(fctx.vocab, dim, dtype=torch.float32, device=dout.device)
        N.check(N.lib().hx_embedding_bwd(c.handle, _DTYPES[dout.dtype], _p(dout), _p(flat), _p(dtable),
                                         flat.numel(), fctx.vocab, dim), c.handle)
        return None, dtable.to(fctx.table_dtype)


class _CrossEntropyFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, logits, targets):
        c = _ctx(logits)
        rows, classes = logits.shape
        logits = logits.contiguous()
        flat = _ids(targets)
        if flat.numel() != rows:
            raise ValueError("targets length must match the number of logit rows")
        loss = torch.empty((), dtype=torch.float32, device=logits.device)
        dlogits = torch.empty_like(logits) if fctx.needs_input_grad[0] else None
        N.check(N.lib().hx_cross_entropy(c.handle, _DTYPES[logits.dtype], _p(logits), _p(flat), _p(loss),
                                         _p(dlogits), rows, classes), c.handle)
        fctx.dlogits = dlogits
        return loss

    @staticmethod
    def backward(fctx, _dloss):
        # Like ops/cross_entropy.rs:18-50 the loss is the graph's root: the
        # stored (softmax - onehot) / rows is the gradient, the upstream one is 1.
        d, fctx.dlogits = fctx.dlogits, None
        return d, None


def gelu(x: torch.Tensor) -> torch.Tensor:
    """Tensor::gelu (kernels/activations.rs:192-237, tanh form) with its backward."""
    return _GeluFn.apply(x)


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """table[ids]: [..., dim] rows of a [vocab, dim] table; its gradient is a scatter-add."""
    return _EmbeddingFn.apply(ids, table)


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Tensor::cross_entropy (src/tensor.rs:754-801): mean over rows of
    logsumexp(row) - row[target], a device scalar; logits [rows, classes]."""
    return _CrossEntropyFn.apply(logits, targets)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """kernels/rms_norm.rs:20-55 over the last dimension, with its backward."""
    return _RMSNormFn.apply(x, weight, float(eps))


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x @ weight + bias with weight stored [in, out] (nn/linear.rs:54-56);
    `residual` (same shape as the output) is added in the same GEMM, the
    residual add of nn/transformer.rs:32, 37."""
    return _LinearFn.apply(x, weight, bias, residual)


class RMSNorm:
    """src/nn/rms_norm.rs: weight initialised to ones, eps 1e-5."""

    def __init__(self, hidden_dim: int, device=None, dtype=torch.float32):
        self.weight = torch.ones(hidden_dim, device=device, dtype=dtype, requires_grad=True)
        self.eps = 1e-5

    def forward(self, x):
        return rms_norm(x, self.weight, self.eps)

    __call__ = forward

    def parameters(self):
        return [self.weight]


class Linear:
    """src/nn/linear.rs: weight [in, out] uniform in +-sqrt(6 / in), bias zeros."""

    def __init__(self, in_features: int, out_features: int, device=None, dtype=torch.float32,
                 generator: Optional[torch.Generator] = None):
        bound = math.sqrt(6.0 / in_features)
        w = torch.rand(in_features, out_features, generator=generator, dtype=torch.float32) * 2 * bound - bound
        self.weight = w.to(device=device, dtype=dtype).requires_grad_()
        self.bias = torch.zeros(out_features, device=device, dtype=dtype, requires_grad=True)

    def forward(self, x, residual=None):
        return linear(x, self.weight, self.bias, residual)

    __call__ = forward

    def parameters(self):
        return [self.weight, self.bias]


class MultiHeadAttention:
    """src/nn/attention.rs:5-98: pre-RMSNorm, Q/K/V projections, heads as strided
    views, RoPE (base 10000, attention.rs:76) on Q and K, the fused attention
    with scale 1/sqrt(head_dim), heads merged by a view, output projection.
    `causal` adds the mask the reference's layer lacks (False reproduces it)."""

    def __init__(self, hidden_dim: int, num_heads: int, device=None, dtype=torch.float32,
                 rope_base: float = 10000.0, causal: bool = False, seed: Optional[int] = None):
        if hidden_dim % num_heads:
            raise ValueError("hidden_dim must be divisible by num_heads")
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        self.num_heads, self.head_dim = num_heads, hidden_dim // num_heads
        self.rope_base, self.causal = float(rope_base), bool(causal)
        self.norm = RMSNorm(hidden_dim, device, dtype)
        self.q_proj, self.k_proj, self.v_proj, self.out_proj = (
            Linear(hidden_dim, hidden_dim, device, dtype, g) for _ in range(4))

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S, Hd = x.shape
        H, D = self.num_heads, self.head_dim
        n = self.norm(x)

        def heads(t):  # [B, S, H*D] -> [B, H, S, D] view (attention.rs:62-73 without the copies)
            return t.view(B, S, H, D).transpose(1, 2)

        q, k, v = heads(self.q_proj(n)), heads(self.k_proj(n)), heads(self.v_proj(n))
        o = flash_attention(q, k, v, 1.0 / math.sqrt(D), self.causal, rope_base=self.rope_base)
        # [B, H, S, D] with [B, S, H, D] memory: the head merge is a view (attention.rs:91-94)
        return self.out_proj(o.transpose(1, 2).reshape(B, S, Hd), residual)

    __call__ = forward

    def parameters(self):
        return (self.norm.parameters() + self.q_proj.parameters() + self.k_proj.parameters()
                + self.v_proj.parameters() + self.out_proj.parameters())


class FeedForward:
    """src/nn/mlp.rs: linear1 (hidden -> 4 hidden), GELU, linear2 (4 hidden -> hidden)."""

    def __init__(self, hidden_dim: int, device=None, dtype=torch.float32, seed: Optional[int] = None):
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        self.linear1 = Linear(hidden_dim, 4 * hidden_dim, device, dtype, g)
        self.linear2 = Linear(4 * hidden_dim, hidden_dim, device, dtype, g)

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.linear2(gelu(self.linear1(x)), residual)

    __call__ = forward

    def parameters(self):
        return self.linear1.parameters() + self.linear2.parameters()


class TransformerBlock:
    """src/nn/transformer.rs:17-40, pre-norm with residuals:
    x = x + mha(norm1(x)); x = x + mlp(norm2(x)). The MultiHeadAttention
    keeps its own pre-RMSNorm (nn/attention.rs:53), so the attention input is
    normalised twice, as in the reference. Each residual add is folded into
    the GEMM of the branch's last projection."""

    def __init__(self, hidden_dim: int, num_heads: int, device=None, dtype=torch.float32,
                 rope_base: float = 10000.0, causal: bool = False, seed: Optional[int] = None):
        self.norm1 = RMSNorm(hidden_dim, device, dtype)
        self.mha = MultiHeadAttention(hidden_dim, num_heads, device, dtype, rope_base, causal, seed)
        self.norm2 = RMSNorm(hidden_dim, device, dtype)
        self.mlp = FeedForward(hidden_dim, device, dtype, None if seed is None else seed + 1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.mha(self.norm1(x), residual=x)
        return self.mlp(self.norm2(x), residual=x)

    __call__ = forward

    def parameters(self):
        return (self.norm1.parameters() + self.mha.parameters() + self.norm2.parameters()
                + self.mlp.parameters())


class Embedding:
    """A [vocab, dim] token table (the reference has no embedding layer)."""

    def __init__(self, vocab: int, dim: int, device=None, dtype=torch.float32,
                 generator: Optional[torch.Generator] = None):
        w = torch.randn(vocab, dim, generator=generator, dtype=torch.float32) * 0.02
        self.weight = w.to(device=device, dtype=dtype).requires_grad_()

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        return embedding(ids, self.weight)

    __call__ = forward

    def parameters(self):
        return [self.weight]


class BlockStack:
    """A language model over TransformerBlocks: token embedding, `layers`
    blocks, a final RMSNorm and an output Linear to `vocab` logits.
    forward(ids [B, S]) -> logits [B*S, vocab]; loss(ids, targets) adds the
    cross-entropy. `init_std` (e.g. 0.02) re-draws every Linear weight from
    N(0, init_std^2) instead of linear.rs's uniform init."""

    def __init__(self, vocab: int, hidden_dim: int, num_heads: int, layers: int, device=None,
                 dtype=torch.float32, rope_base: float = 10000.0, causal: bool = True,
                 init_std: Optional[float] = None, seed: int = 0):
        g = torch.Generator().manual_seed(seed)
        self.embed = Embedding(vocab, hidden_dim, device, dtype, g)
        self.blocks = [TransformerBlock(hidden_dim, num_heads, device, dtype, rope_base, causal, seed + 2 * i + 1)
                       for i in range(layers)]
        self.norm = RMSNorm(hidden_dim, device, dtype)
        self.head = Linear(hidden_dim, vocab, device, dtype, g)
        if init_std is not None:
            with torch.no_grad():
                for p in self.parameters():
                    if p.dim() == 2 and p is not self.embed.weight:
                        w = torch.randn(p.shape, generator=g, dtype=torch.float32) * init_std
                        p.copy_(w.to(p.device, p.dtype))

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        x = self.embed(ids)
        for blk in self.blocks:
            x = blk(x)
        return self.head(self.norm(x)).reshape(-1, self.head.weight.shape[1])

    __call__ = forward

    def loss(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        return cross_entropy(self(ids), targets)

    def parameters(self):
        ps = self.embed.parameters()
        for blk in self.blocks:
            ps += blk.parameters()
        return ps + self.norm.parameters() + self.head.parameters()
