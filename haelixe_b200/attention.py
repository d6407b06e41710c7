"""Host-side mirror of haelixe's attention interface over the C ABI.

Reference interface mirrored (paths inside sethigris/haelixe):
  * `Tensor::flash_attention(&self, k, v, scale) -> Tensor` (src/tensor.rs:644-666)
    -> `flash_attention(q, k, v, scale, causal=False)`; like the reference it
    attaches a `FlashAttentionOp` autograd node when q requires grad.
  * `FlashAttentionOp { q, k, v, scale }` with `name() == "FlashAttention"` and
    `backward(grad_out) -> [dQ, dK, dV]` (src/ops/flash_attention.rs:3-40); the
    CUDA variant also keeps `o` and `lse`, so the backward recomputes P from
    the saved statistics instead of re-running softmax.
  * `Device::Cuda` / `GpuContext` (src/device.rs:5-26, src/gpu/mod.rs:38) ->
    `CudaContext`; `GpuMemoryArena` / `GpuAllocation` (src/gpu/arena.rs) ->
    `CudaContext.allocate()` / `CudaAllocation` (slab returns to its bin when
    the last Python reference drops, the Arc rule of arena.rs:113-131).
  * `rope_forward` / `rope_backward` (src/kernels/rope.rs:5-82).

Device memory is held in torch CUDA tensors (plumbing only); every byte of
compute runs in libhaelixe_cuda.so. Errors raise `HxError` (the reference
panics).
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional

import torch

from . import _native as N

_DTYPES = {torch.float32: N.HX_F32, torch.bfloat16: N.HX_BF16}


class CudaAllocation:
    """A binned slab from the context's arena; returned to its bin on drop."""

    def __init__(self, ctx: "CudaContext", nbytes: int):
        self._ctx = ctx
        p = ctypes.c_void_p()
        N.check(N.lib().hx_alloc(ctx.handle, nbytes, ctypes.byref(p)), ctx.handle)
        self.ptr = p.value
        self.size = int(N.lib().hx_bin_size(nbytes))

    def __del__(self):
        ctx = getattr(self, "_ctx", None)
        if ctx is not None and ctx.handle and self.ptr:
            N.lib().hx_free(ctx.handle, self.ptr)
            self.ptr = None


class CudaContext:
    """One per device: stream, binning arena, device status word."""

    def __init__(self, device: int = 0):
        self.device = int(device)
        h = ctypes.c_void_p()
        st = N.lib().hx_ctx_create(self.device, ctypes.byref(h))
        N.check(st)
        self.handle = h.value
        self._stream = None  # raw stream last handed to hx_ctx_set_stream

    def close(self) -> None:
        if self.handle:
            N.lib().hx_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def use_stream(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Enqueue the context's work on `stream` (default: torch's current
        stream on this device). The library call is made only when the stream
        changes."""
        raw = stream.cuda_stream if stream is not None else torch._C._cuda_getCurrentRawStream(self.device)
        if raw != self._stream:
            N.check(N.lib().hx_ctx_set_stream(self.handle, ctypes.c_void_p(raw)), self.handle)
            self._stream = raw

    def sync(self) -> None:
        N.check(N.lib().hx_sync(self.handle), self.handle)

    def allocate(self, nbytes: int) -> CudaAllocation:
        return CudaAllocation(self, nbytes)

    def arena_stats(self) -> dict:
        s = N.ArenaStats()
        N.check(N.lib().hx_arena_stats_get(self.handle, ctypes.byref(s)), self.handle)
        return {f: int(getattr(s, f)) for f, _ in N.ArenaStats._fields_}

    def set_arena_limit(self, nbytes: int) -> None:
        """Caps the arena's held bytes (0 removes the cap): past it allocations fail with OOM."""
        N.check(N.lib().hx_arena_set_limit(self.handle, int(nbytes)), self.handle)

    def arena_reset(self) -> None:
        N.check(N.lib().hx_arena_reset(self.handle), self.handle)

    @property
    def last_path(self) -> str:
        return {0: "none", 1: "simt", 2: "tcgen05"}[N.lib().hx_last_path(self.handle)]

    def force_simt(self, on: bool) -> None:
        N.check(N.lib().hx_set_force_simt(self.handle, int(bool(on))), self.handle)


_ctx_lock = threading.Lock()
_contexts: dict[int, CudaContext] = {}


def context(device: Optional[int] = None) -> CudaContext:
    """The cached context of `device` (default: torch's current device)."""
    dev = torch.cuda.current_device() if device is None else int(device)
    with _ctx_lock:
        c = _contexts.get(dev)
        if c is None:
            c = CudaContext(dev)
            _contexts[dev] = c
    return c


def bin_size(nbytes: int) -> int:
    return int(N.lib().hx_bin_size(nbytes))


def _shape_of(t: torch.Tensor) -> N.AttnShape:
    """[BH,S,D] or [B,H,S,D] (last dim contiguous) -> hx_attn_shape."""
    if t.dim() == 3:
        BH, S, D = t.shape
        sb, ss = t.stride(0), t.stride(1)
        return N.AttnShape(BH, 1, S, D, sb, sb, ss)
    if t.dim() == 4:
        B, H, S, D = t.shape
        return N.AttnShape(B, H, S, D, t.stride(0), t.stride(1), t.stride(2))
    raise ValueError(f"attention operands are [BH,S,D] or [B,H,S,D], got {tuple(t.shape)}")


def _same_strides(a: torch.Tensor, b: torch.Tensor) -> bool:
    # The stride of a dimension of size 1 never moves an address, so it may differ.
    return all(n == 1 or x == y for n, x, y in zip(a.shape, a.stride(), b.stride()))


def _check_operands(*ts: torch.Tensor) -> None:
    t0 = ts[0]
    for t in ts:
        if not t.is_cuda:
            # The reference panics here too: "FlashAttention currently requires GPU" (tensor.rs:652).
            raise RuntimeError("FlashAttention requires CUDA tensors")
        if t.dtype not in _DTYPES:
            raise TypeError(f"unsupported dtype {t.dtype}; f32 and bf16 are supported")
        if t.dtype != t0.dtype or t.shape != t0.shape or t.device != t0.device:
            raise ValueError("q, k, v (and gradients) must share dtype, shape and device")
        if t.stride(-1) != 1:
            raise ValueError("the head dimension must be contiguous")
        if t.dim() == 4 and not _same_strides(t, t0):
            raise ValueError("strided operands must share strides")


def _like(t: torch.Tensor) -> torch.Tensor:
    """An uninitialised tensor with exactly t's strides: every operand of one
    call is addressed through the same [B, H, S, D] strides."""
    return torch.empty_strided(t.shape, t.stride(), dtype=t.dtype, device=t.device)


def _check_outputs(ref: torch.Tensor, *outs: Optional[torch.Tensor]) -> None:
    for t in outs:
        if t is not None and (t.shape != ref.shape or not _same_strides(t, ref) or t.dtype != ref.dtype
                              or t.device != ref.device):
            raise ValueError("output tensors must have the inputs' shape, strides, dtype and device")


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def attn_forward(q, k, v, scale: float, causal: bool = False, out=None, lse=None):
    """Runs the fused forward. Returns (o, lse[B*H*S] f32)."""
    _check_operands(q, k, v)
    ctx = context(q.device.index)
    ctx.use_stream()
    shp = _shape_of(q)
    _check_outputs(q, out)
    if out is None:
        out = _like(q)
    if lse is None:
        lse = torch.empty(shp.B * shp.H * shp.S, device=q.device, dtype=torch.float32)
    N.check(N.lib().hx_attn_fwd_strided(ctx.handle, _DTYPES[q.dtype], ctypes.byref(shp),
                                        _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(lse),
                                        float(scale), int(bool(causal))), ctx.handle)
    return out, lse


def attn_backward(q, k, v, o, lse, dout, scale: float, causal: bool = False,
                  dq=None, dk=None, dv=None, rope_base: Optional[float] = None):
    """Runs the fused backward. Returns (dq, dk, dv).

    With rope_base, q and k are the rotary-embedded tensors the forward used and
    dq, dk are returned with respect to the tensors before the rotation
    (rope_backward fused into the backward's last writes of dq and dk).
    """
    if not _same_strides(dout, q):  # e.g. a contiguous upstream gradient of a strided view
        dout = _like(q).copy_(dout)
    _check_operands(q, k, v, o, dout)
    ctx = context(q.device.index)
    ctx.use_stream()
    shp = _shape_of(q)
    _check_outputs(q, dq, dk, dv)
    dq = _like(q) if dq is None else dq
    dk = _like(q) if dk is None else dk
    dv = _like(q) if dv is None else dv
    if rope_base is None:
        N.check(N.lib().hx_attn_bwd_strided(ctx.handle, _DTYPES[q.dtype], ctypes.byref(shp),
                                            _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dout),
                                            _ptr(lse), _ptr(dq), _ptr(dk), _ptr(dv), None, 0,
                                            float(scale), int(bool(causal))), ctx.handle)
    else:
        N.check(N.lib().hx_attn_bwd_rope_strided(ctx.handle, _DTYPES[q.dtype], ctypes.byref(shp),
                                                 _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dout),
                                                 _ptr(lse), _ptr(dq), _ptr(dk), _ptr(dv), None, 0,
                                                 float(scale), int(bool(causal)),
                                                 float(rope_base)), ctx.handle)
    return dq, dk, dv


class FlashAttentionOp:
    """Autograd node of the fused attention (src/ops/flash_attention.rs:3-40).

    With rope_base set, q and k held here are the rotated tensors and the
    gradients returned are those of the tensors before the rotation.
    """

    def __init__(self, q, k, v, scale: float, o, lse, causal: bool = False,
                 rope_base: Optional[float] = None):
        self.q, self.k, self.v, self.scale = q, k, v, float(scale)
        self.o, self.lse, self.causal = o, lse, bool(causal)
        self.rope_base = rope_base

    def name(self) -> str:
        return "FlashAttention"

    def backward(self, grad_out: torch.Tensor) -> list:
        """Gradients for the parents in the order [q, k, v] (ops/flash_attention.rs:38)."""
        dq, dk, dv = attn_backward(self.q, self.k, self.v, self.o, self.lse, grad_out,
                                   self.scale, self.causal, rope_base=self.rope_base)
        return [dq, dk, dv]


class _FlashAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, q, k, v, scale, causal, rope_base):
        q, k = q.detach(), k.detach()
        if rope_base is not None:
            q, k = rope_forward(q, rope_base), rope_forward(k, rope_base)
        v = v.detach()
        o, lse = attn_forward(q, k, v, scale, causal)
        # Saved through save_for_backward, not as attributes: o is this node's
        # own output, and holding it on the context would make a reference
        # cycle (node -> o -> o.grad_fn = node) that only the cyclic garbage
        # collector frees, keeping every step's q, k, v, o and lse alive.
        fctx.save_for_backward(q, k, v, o, lse)
        fctx.scale, fctx.causal, fctx.rope_base = scale, causal, rope_base
        return o

    @staticmethod
    def backward(fctx, grad_out):
        q, k, v, o, lse = fctx.saved_tensors
        op = FlashAttentionOp(q, k, v, fctx.scale, o, lse, fctx.causal, fctx.rope_base)
        dq, dk, dv = op.backward(grad_out)
        return dq, dk, dv, None, None, None


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                    causal: bool = False, rope_base: Optional[float] = None) -> torch.Tensor:
    """softmax(scale * q k^T [causal]) v on CUDA (Tensor::flash_attention, tensor.rs:644).

    q, k, v: [B*H, S, D] (the reference's layout) or [B, H, S, D] views with a
    contiguous head dim; f32 or bf16. When any input requires grad, the result
    carries a FlashAttentionOp node, as `with_node` does in the reference
    (tensor.rs:655-663). With rope_base, q and k are rotated first (the order of
    MultiHeadAttention::forward, nn/attention.rs:76-78) and the backward returns
    their gradients before the rotation.
    """
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return _FlashAttentionFn.apply(q, k, v, float(scale), bool(causal),
                                       None if rope_base is None else float(rope_base))
    if rope_base is not None:
        q, k = rope_forward(q, rope_base), rope_forward(k, rope_base)
    o, _ = attn_forward(q, k, v, scale, causal)
    return o


def use_arena_allocator() -> None:
    """Routes every CUDA tensor this process allocates from now on through the
    library's arena (one per device: power-of-two bins, slabs parked on free
    and reused), as every tensor of the reference lives in its GpuMemoryArena
    (src/gpu/arena.rs:13-145). Call it before the first CUDA allocation."""
    alloc = torch.cuda.memory.CUDAPluggableAllocator(N.LIB_PATH, "hx_torch_malloc", "hx_torch_free")
    torch.cuda.memory.change_current_allocator(alloc)


def torch_arena_stats(device: int = 0) -> dict:
    """Statistics of the arena behind use_arena_allocator() on `device`."""
    c = N.lib().hx_torch_arena_context(device)
    if not c:
        raise RuntimeError("no arena for this device")
    st = N.ArenaStats()
    N.check(N.lib().hx_arena_stats_get(c, ctypes.byref(st)))
    return {f: getattr(st, f) for f, _ in N.ArenaStats._fields_}


def rope_forward(x: torch.Tensor, base: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Interleaved-pair RoPE on [BH,S,D] / [B,H,S,D] (kernels/rope.rs:5-44)."""
    _check_operands(x)
    ctx = context(x.device.index)
    ctx.use_stream()
    _check_outputs(x, out)
    out = _like(x) if out is None else out
    shp = _shape_of(x)
    N.check(N.lib().hx_rope_fwd(ctx.handle, _DTYPES[x.dtype], ctypes.byref(shp), _ptr(x),
                                _ptr(out), float(base)), ctx.handle)
    return out


def rope_forward_qk(q: torch.Tensor, k: torch.Tensor, base: float, out_q: Optional[torch.Tensor] = None,
                    out_k: Optional[torch.Tensor] = None):
    """rope_forward of q and k (same shape and strides) in one launch."""
    _check_operands(q, k)
    if q.shape != k.shape or not _same_strides(q, k):
        raise ValueError("q and k must have the same shape and strides")
    ctx = context(q.device.index)
    ctx.use_stream()
    _check_outputs(q, out_q)
    _check_outputs(k, out_k)
    out_q = _like(q) if out_q is None else out_q
    out_k = _like(k) if out_k is None else out_k
    if not (_same_strides(out_q, q) and _same_strides(out_k, k)):
        raise ValueError("outputs must have the strides of the inputs")
    shp = _shape_of(q)
    N.check(N.lib().hx_rope_fwd_qk(ctx.handle, _DTYPES[q.dtype], ctypes.byref(shp), _ptr(q), _ptr(k),
                                   _ptr(out_q), _ptr(out_k), float(base)), ctx.handle)
    return out_q, out_k


def rope_backward(g: torch.Tensor, base: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Inverse rotation (kernels/rope.rs:46-82)."""
    _check_operands(g)
    ctx = context(g.device.index)
    ctx.use_stream()
    _check_outputs(g, out)
    out = _like(g) if out is None else out
    shp = _shape_of(g)
    N.check(N.lib().hx_rope_bwd(ctx.handle, _DTYPES[g.dtype], ctypes.byref(shp), _ptr(g),
                                _ptr(out), float(base)), ctx.handle)
    return out
