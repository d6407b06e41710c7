"""Device-resident attention block around the fused kernel.

Mirrors haelixe's `nn` modules for the attention layer: `RMSNorm`
(src/nn/rms_norm.rs, kernels/rms_norm.rs), `Linear` (src/nn/linear.rs) and
`MultiHeadAttention` (src/nn/attention.rs:46-98), with every op on the GPU
through the library's C ABI: RMSNorm kernels, Linear as cuBLAS GEMMs (weights
stored [in, out] as in linear.rs:41) plus bias kernels, and the fused
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
    def forward(fctx, x, w, b):
        c = _ctx(x)
        in_f, out_f = w.shape
        x2 = x.reshape(-1, in_f).contiguous()
        y = torch.empty(x2.shape[0], out_f, dtype=x.dtype, device=x.device)
        N.check(N.lib().hx_linear_fwd(c.handle, _DTYPES[x.dtype], _p(x2), _p(w.contiguous()),
                                      _p(None if b is None else b.contiguous()), _p(y), x2.shape[0], in_f,
                                      out_f), c.handle)
        fctx.save_for_backward(x2, w)
        fctx.in_shape, fctx.has_bias = x.shape, b is not None
        return y.view(*x.shape[:-1], out_f)

    @staticmethod
    def backward(fctx, dy):
        x2, w = fctx.saved_tensors
        c = _ctx(x2)
        in_f, out_f = w.shape
        dy2 = dy.reshape(-1, out_f).contiguous()
        need_x, need_w, need_b = fctx.needs_input_grad
        dx = torch.empty_like(x2) if need_x else None
        dw = torch.empty_like(w) if need_w else None
        db = torch.empty(out_f, dtype=w.dtype, device=w.device) if (need_b and fctx.has_bias) else None
        N.check(N.lib().hx_linear_bwd(c.handle, _DTYPES[x2.dtype], _p(x2), _p(w.contiguous()), _p(dy2), _p(dx),
                                      _p(dw), _p(db), x2.shape[0], in_f, out_f), c.handle)
        return (None if dx is None else dx.view(fctx.in_shape)), dw, db


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """kernels/rms_norm.rs:20-55 over the last dimension, with its backward."""
    return _RMSNormFn.apply(x, weight, float(eps))


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x @ weight + bias with weight stored [in, out] (nn/linear.rs:54-56)."""
    return _LinearFn.apply(x, weight, bias)


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

    def forward(self, x):
        return linear(x, self.weight, self.bias)

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

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, S, Hd = x.shape
        H, D = self.num_heads, self.head_dim
        n = self.norm(x)

        def heads(t):  # [B, S, H*D] -> [B, H, S, D] view (attention.rs:62-73 without the copies)
            return t.view(B, S, H, D).transpose(1, 2)

        q, k, v = heads(self.q_proj(n)), heads(self.k_proj(n)), heads(self.v_proj(n))
        o = flash_attention(q, k, v, 1.0 / math.sqrt(D), self.causal, rope_base=self.rope_base)
        # [B, H, S, D] with [B, S, H, D] memory: the head merge is a view (attention.rs:91-94)
        return self.out_proj(o.transpose(1, 2).reshape(B, S, Hd))

    __call__ = forward

    def parameters(self):
        return (self.norm.parameters() + self.q_proj.parameters() + self.k_proj.parameters()
                + self.v_proj.parameters() + self.out_proj.parameters())
