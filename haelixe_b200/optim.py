"""AdamW on the GPU (src/optim.rs:87-199), for bf16 storage with f32 master weights.

`AdamW(lr)` keeps the reference's defaults (beta1 0.9, beta2 0.999, eps 1e-8,
weight decay 0.01, optim.rs:106-115), `set_lr`, `step(params_and_grads)` and
`zero_grad`. The moments are f32 zeros allocated at a parameter's first step
(optim.rs:147-153). A bf16 parameter also gets an f32 master copy: the update
runs on the master and writes the rounded bf16 weights back into the
parameter in the same kernel. All tensors of one step go through one
hx_adamw_step call (a multi-tensor kernel: one launch per 48 tensors).
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N
from .attention import _DTYPES, context


class AdamW:
    def __init__(self, lr: float, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
                 weight_decay: float = 0.01):
        self.lr, self.beta1, self.beta2, self.eps, self.weight_decay = lr, beta1, beta2, eps, weight_decay
        self.step_count = 0
        self.state: dict[int, tuple] = {}

    def set_lr(self, new_lr: float) -> None:
        self.lr = new_lr

    def _state_for(self, p: torch.Tensor):
        st = self.state.get(id(p))
        if st is None:
            master = p.detach().float().contiguous() if p.dtype != torch.float32 else None
            m = torch.zeros(p.numel(), dtype=torch.float32, device=p.device)
            v = torch.zeros_like(m)
            st = (p, master, m, v)  # p keeps the id alive
            self.state[id(p)] = st
        return st

    def step(self, params_and_grads) -> None:
        self.step_count += 1  # optim.rs:130
        table, keep, dev = [], [], None
        for p, g in params_and_grads:
            if g is None:
                continue
            if not (p.is_cuda and p.is_contiguous()):
                raise ValueError("AdamW parameters must be contiguous CUDA tensors")
            if p.dtype not in _DTYPES or g.dtype not in _DTYPES:
                raise TypeError("AdamW supports f32 and bf16 parameters and gradients")
            dev = p.device.index if dev is None else dev
            _, master, m, v = self._state_for(p)
            g = g.contiguous()
            keep.append(g)
            t = N.AdamWTensor()
            t.param = (master if master is not None else p).data_ptr()
            t.grad = g.data_ptr()
            t.m, t.v = m.data_ptr(), v.data_ptr()
            t.param_lowp = p.data_ptr() if master is not None else None
            t.n = p.numel()
            t.grad_dtype = _DTYPES[g.dtype]
            table.append(t)
        if not table:
            return
        c = context(dev)
        c.use_stream()
        arr = (N.AdamWTensor * len(table))(*table)
        N.check(N.lib().hx_adamw_step(c.handle, ctypes.cast(arr, ctypes.c_void_p), len(table), self.lr,
                                      self.beta1, self.beta2, self.eps, self.weight_decay, self.step_count),
                c.handle)

    def zero_grad(self) -> None:
        """The reference keeps no gradient buffers (optim.rs:193-199); neither does this."""
