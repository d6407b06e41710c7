"""ctypes front end of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by the smoke check in
__graft_entry__.py and by the CPU-baseline leg of bench.py. The product
library never imports it. See attn_oracle.c for what each function restates
in the reference (src/ops/flash_attention.rs, src/kernels/*.rs).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_F = ctypes.POINTER(ctypes.c_float)


def build(force: bool = False) -> str:
    """Compile liboracle.so with the Makefile beside this file."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        i, f, l = ctypes.c_int, ctypes.c_float, ctypes.c_long
        L.ora_attn_fwd.argtypes = [_F, _F, _F, _F, _F, i, i, i, f, i]
        L.ora_attn_fwd_f64.argtypes = L.ora_attn_fwd.argtypes
        L.ora_attn_bwd.argtypes = [_F, _F, _F, _F, _F, _F, _F, i, i, i, f, i, i]
        L.ora_attn_bwd_f64.argtypes = L.ora_attn_bwd.argtypes
        L.ora_attn_fwd.restype = L.ora_attn_fwd_f64.restype = i
        L.ora_attn_bwd.restype = L.ora_attn_bwd_f64.restype = i
        L.ora_softmax.argtypes = [_F, _F, l, l]
        L.ora_softmax_backward.argtypes = [_F, _F, _F, l, l]
        L.ora_rope_fwd.argtypes = [_F, _F, l, i, i, f]
        L.ora_rope_bwd.argtypes = [_F, _F, l, i, i, f]
        L.ora_round_bf16.argtypes = [_F, _F, l]
        L.ora_matmul.argtypes = [_F, _F, _F, l, l, l]
        L.ora_rms_norm_fwd.argtypes = [_F, _F, _F, l, i, f]
        L.ora_rms_norm_bwd.argtypes = [_F, _F, _F, _F, _F, l, i, f]
        L.ora_set_threads.argtypes = [i]
        L.ora_num_threads.restype = i
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a: np.ndarray):
    return a.ctypes.data_as(_F)


def set_threads(n: int) -> None:
    lib().ora_set_threads(int(n))


def num_threads() -> int:
    return int(lib().ora_num_threads())


def softmax(x) -> np.ndarray:
    x = _f32(x)
    n = x.shape[-1]
    y = np.empty_like(x)
    lib().ora_softmax(_p(x), _p(y), x.size // n, n)
    return y


def softmax_backward(dy, y) -> np.ndarray:
    dy, y = _f32(dy), _f32(y)
    n = y.shape[-1]
    dx = np.empty_like(y)
    lib().ora_softmax_backward(_p(dy), _p(y), _p(dx), y.size // n, n)
    return dx


def attn_fwd(q, k, v, scale: float, causal: bool, f64: bool = False):
    """O[BH,S,D] and LSE[BH,S] of softmax(scale Q K^T [causal]) V."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    BH, S, D = q.shape
    o = np.empty_like(q)
    lse = np.empty((BH, S), np.float32)
    fn = lib().ora_attn_fwd_f64 if f64 else lib().ora_attn_fwd
    rc = fn(_p(q), _p(k), _p(v), _p(o), _p(lse), BH, S, D, float(scale), int(bool(causal)))
    if rc != 0:
        raise MemoryError("oracle forward could not allocate its S x S buffers")
    return o, lse


def attn_bwd(q, k, v, do, scale: float, causal: bool, f64: bool = False, ref_compat: bool = False):
    """(dQ, dK, dV) of the attention forward above for upstream gradient dO."""
    q, k, v, do = _f32(q), _f32(k), _f32(v), _f32(do)
    BH, S, D = q.shape
    dq, dk, dv = np.empty_like(q), np.empty_like(q), np.empty_like(q)
    fn = lib().ora_attn_bwd_f64 if f64 else lib().ora_attn_bwd
    rc = fn(_p(q), _p(k), _p(v), _p(do), _p(dq), _p(dk), _p(dv), BH, S, D, float(scale),
            int(bool(causal)), int(bool(ref_compat)))
    if rc != 0:
        raise MemoryError("oracle backward could not allocate its S x S buffers")
    return dq, dk, dv


def rope_fwd(x, base: float) -> np.ndarray:
    """x: [..., S, D]; rotation by position s = token % S (kernels/rope.rs:24)."""
    x = _f32(x)
    S, D = x.shape[-2], x.shape[-1]
    out = np.empty_like(x)
    lib().ora_rope_fwd(_p(x), _p(out), x.size // D, S, D, float(base))
    return out


def rope_bwd(g, base: float) -> np.ndarray:
    g = _f32(g)
    S, D = g.shape[-2], g.shape[-1]
    out = np.empty_like(g)
    lib().ora_rope_bwd(_p(g), _p(out), g.size // D, S, D, float(base))
    return out


def round_bf16(x) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    lib().ora_round_bf16(_p(x), _p(y), x.size)
    return y


def matmul(a, b) -> np.ndarray:
    """Row-major a[m, k] @ b[k, n] with the reference's blocked loop (kernels/matmul.rs)."""
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    out = np.empty((m, n), np.float32)
    lib().ora_matmul(_p(a), _p(b), _p(out), m, k, n)
    return out


def rms_norm_fwd(x, w, eps: float = 1e-5) -> np.ndarray:
    """kernels/rms_norm.rs:20-55 over the last dimension."""
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    lib().ora_rms_norm_fwd(_p(x), _p(w), _p(out), x.size // x.shape[-1], x.shape[-1], float(eps))
    return out


def rms_norm_bwd(g, x, w, eps: float = 1e-5):
    """kernels/rms_norm.rs:57-132: (dx, dw)."""
    g, x, w = _f32(g), _f32(x), _f32(w)
    dx = np.empty_like(x)
    dw = np.empty(x.shape[-1], np.float32)
    lib().ora_rms_norm_bwd(_p(g), _p(x), _p(w), _p(dx), _p(dw), x.size // x.shape[-1], x.shape[-1],
                           float(eps))
    return dx, dw


def mha_forward_backward(x, p: dict, dy, heads: int, rope_base: float = 10000.0, eps: float = 1e-5,
                         causal: bool = False):
    """MultiHeadAttention::forward (src/nn/attention.rs:46-98) on the CPU with
    its backward through every op it records. x, dy: [B, S, hidden]; p holds
    norm_w [hidden], wq/wk/wv/wo [hidden, hidden] (stored [in, out],
    nn/linear.rs:41) and bq/bk/bv/bo [hidden]. Returns (y, grads) with grads
    keyed dx, norm_w, wq, bq, ... as in p."""
    x, dy = _f32(x), _f32(dy)
    B, S, Hd = x.shape
    H, D = heads, Hd // heads
    scale = 1.0 / float(np.sqrt(np.float32(D)))
    rows = B * S
    x2 = x.reshape(rows, Hd)
    n = rms_norm_fwd(x2, p["norm_w"], eps)                        # 1. pre-norm
    proj = {c: matmul(n, p["w" + c]) + p["b" + c] for c in "qkv"}  # 2. Linear = matmul + add

    def split(t):  # 3. [B, S, Hd] -> [B*H, S, D] (view, transpose(1, 2), view)
        return np.ascontiguousarray(t.reshape(B, S, H, D).transpose(0, 2, 1, 3)).reshape(B * H, S, D)

    def merge(t):  # 6. [B*H, S, D] -> [B, S, Hd]
        return np.ascontiguousarray(t.reshape(B, H, S, D).transpose(0, 2, 1, 3)).reshape(rows, Hd)

    q, k, v = (split(proj[c]) for c in "qkv")
    qr, kr = rope_fwd(q, rope_base), rope_fwd(k, rope_base)        # 4. RoPE on Q and K
    o, _ = attn_fwd(qr, kr, v, scale, causal)                      # 5. attention
    om = merge(o)
    y = matmul(om, p["wo"]) + p["bo"]                              # 7. out_proj
    # backward, in reverse
    g = {}
    dy2 = dy.reshape(rows, Hd)
    g["wo"] = matmul(np.ascontiguousarray(om.T), dy2)
    g["bo"] = dy2.sum(axis=0, dtype=np.float32)
    dom = matmul(dy2, np.ascontiguousarray(p["wo"].T))
    do = split(dom.reshape(B, S, Hd))
    dq, dk, dv = attn_bwd(qr, kr, v, do, scale, causal)
    dq, dk = rope_bwd(dq, rope_base), rope_bwd(dk, rope_base)
    dn = np.zeros((rows, Hd), np.float32)
    for c, dt in zip("qkv", (dq, dk, dv)):
        dproj = merge(dt)
        g["w" + c] = matmul(np.ascontiguousarray(n.T), dproj)
        g["b" + c] = dproj.sum(axis=0, dtype=np.float32)
        dn += matmul(dproj, np.ascontiguousarray(p["w" + c].T))
    g["dx"], g["norm_w"] = rms_norm_bwd(dn, x2, p["norm_w"], eps)
    g["dx"] = g["dx"].reshape(B, S, Hd)
    return y.reshape(B, S, Hd), g
