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
        L.ora_attn_rows.argtypes = [_F, _F, _F, _F, _F, _F, _F, _F, _F, i, i, i, f, i, i]
        L.ora_attn_rows_f64.argtypes = L.ora_attn_rows.argtypes
        L.ora_attn_rows.restype = L.ora_attn_rows_f64.restype = i
        L.ora_attn_bwd.restype = L.ora_attn_bwd_f64.restype = i
        L.ora_softmax.argtypes = [_F, _F, l, l]
        L.ora_softmax_backward.argtypes = [_F, _F, _F, l, l]
        L.ora_rope_fwd.argtypes = [_F, _F, l, i, i, f]
        L.ora_rope_bwd.argtypes = [_F, _F, l, i, i, f]
        L.ora_round_bf16.argtypes = [_F, _F, l]
        L.ora_matmul.argtypes = [_F, _F, _F, l, l, l]
        L.ora_rms_norm_fwd.argtypes = [_F, _F, _F, l, i, f]
        L.ora_rms_norm_bwd.argtypes = [_F, _F, _F, _F, _F, l, i, f]
        u32p = ctypes.POINTER(ctypes.c_uint32)
        L.ora_gelu_fwd.argtypes = [_F, _F, l]
        L.ora_gelu_bwd.argtypes = [_F, _F, _F, l]
        L.ora_cross_entropy_fwd.argtypes = [_F, u32p, _F, l, l]
        L.ora_cross_entropy_fwd.restype = f
        L.ora_cross_entropy_bwd.argtypes = [_F, u32p, _F, l, l]
        L.ora_adamw_step.argtypes = [_F, _F, _F, _F, l, f, f, f, f, f, i]
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


def attn_rows(q, k, v, do, scale: float, causal: bool, rows: int = 2048, f64: bool = False):
    """(O, LSE, dQ, dK, dV) by blocks of `rows` query rows: the results of
    attn_fwd and attn_bwd bit for bit, without S x S buffers, so that a whole
    S = 32768 slice fits in host memory (3 x rows x S floats of scratch)."""
    q, k, v, do = _f32(q), _f32(k), _f32(v), _f32(do)
    BH, S, D = q.shape
    o, dq, dk, dv = (np.empty_like(q) for _ in range(4))
    lse = np.empty((BH, S), np.float32)
    fn = lib().ora_attn_rows_f64 if f64 else lib().ora_attn_rows
    rc = fn(_p(q), _p(k), _p(v), _p(do), _p(o), _p(lse), _p(dq), _p(dk), _p(dv), BH, S, D,
            float(scale), int(bool(causal)), int(rows))
    if rc != 0:
        raise MemoryError("oracle could not allocate its row-block buffers")
    return o, lse, dq, dk, dv


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


def mha_forward(x, p: dict, heads: int, rope_base: float = 10000.0, eps: float = 1e-5, causal: bool = False):
    """MultiHeadAttention::forward (src/nn/attention.rs:46-98) on the CPU.
    x: [B, S, hidden]; p holds norm_w [hidden], wq/wk/wv/wo [hidden, hidden]
    (stored [in, out], nn/linear.rs:41) and bq/bk/bv/bo [hidden]. Returns
    (y, cache) with cache the inputs mha_backward needs."""
    x = _f32(x)
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
    cache = dict(x2=x2, n=n, qr=qr, kr=kr, v=v, om=om, p=p, shape=(B, S, H, D), scale=scale,
                 rope_base=rope_base, eps=eps, causal=causal, split=split, merge=merge)
    return y.reshape(B, S, Hd), cache


def mha_backward(dy, cache):
    """The backward of mha_forward through every op it records; grads keyed
    dx, norm_w, wq, bq, ... as in p."""
    B, S, H, D = cache["shape"]
    Hd, rows = H * D, B * S
    p, split, merge = cache["p"], cache["split"], cache["merge"]
    g = {}
    dy2 = _f32(dy).reshape(rows, Hd)
    g["wo"] = matmul(np.ascontiguousarray(cache["om"].T), dy2)
    g["bo"] = dy2.sum(axis=0, dtype=np.float32)
    dom = matmul(dy2, np.ascontiguousarray(p["wo"].T))
    do = split(dom.reshape(B, S, Hd))
    dq, dk, dv = attn_bwd(cache["qr"], cache["kr"], cache["v"], do, cache["scale"], cache["causal"])
    dq, dk = rope_bwd(dq, cache["rope_base"]), rope_bwd(dk, cache["rope_base"])
    dn = np.zeros((rows, Hd), np.float32)
    for c, dt in zip("qkv", (dq, dk, dv)):
        dproj = merge(dt)
        g["w" + c] = matmul(np.ascontiguousarray(cache["n"].T), dproj)
        g["b" + c] = dproj.sum(axis=0, dtype=np.float32)
        dn += matmul(dproj, np.ascontiguousarray(p["w" + c].T))
    g["dx"], g["norm_w"] = rms_norm_bwd(dn, cache["x2"], p["norm_w"], cache["eps"])
    g["dx"] = g["dx"].reshape(B, S, Hd)
    return g


def mha_forward_backward(x, p: dict, dy, heads: int, rope_base: float = 10000.0, eps: float = 1e-5,
                         causal: bool = False):
    """mha_forward then mha_backward: (y, grads)."""
    y, cache = mha_forward(x, p, heads, rope_base, eps, causal)
    return y, mha_backward(dy, cache)


def block_forward(x, p: dict, heads: int, rope_base: float = 10000.0, eps: float = 1e-5, causal: bool = False):
    """TransformerBlock::forward (src/nn/transformer.rs:26-40) with
    FeedForward (src/nn/mlp.rs): x1 = x + mha(norm1(x)),
    y = x1 + linear2(gelu(linear1(norm2(x1)))). p holds norm1_w, norm2_w,
    mha (a dict for mha_forward), w1 [hidden, 4 hidden], b1, w2, b2."""
    x = _f32(x)
    B, S, Hd = x.shape
    rows = B * S
    x2 = x.reshape(rows, Hd)
    n1 = rms_norm_fwd(x2, p["norm1_w"], eps)
    a, mcache = mha_forward(n1.reshape(B, S, Hd), p["mha"], heads, rope_base, eps, causal)
    x1 = x2 + a.reshape(rows, Hd)
    n2 = rms_norm_fwd(x1, p["norm2_w"], eps)
    h = matmul(n2, p["w1"]) + p["b1"]
    gg = gelu_fwd(h)
    y = x1 + (matmul(gg, p["w2"]) + p["b2"])
    cache = dict(x2=x2, n1=n1, mcache=mcache, x1=x1, n2=n2, h=h, gg=gg, p=p, eps=eps, shape=(B, S, Hd))
    return y.reshape(B, S, Hd), cache


def block_backward(dy, cache):
    """The backward of block_forward: grads keyed dx, norm1_w, norm2_w, w1,
    b1, w2, b2 and mha (the dict of mha_backward without its dx)."""
    B, S, Hd = cache["shape"]
    rows, p, eps = B * S, cache["p"], cache["eps"]
    dy2 = _f32(dy).reshape(rows, Hd)
    g = {}
    g["w2"] = matmul(np.ascontiguousarray(cache["gg"].T), dy2)
    g["b2"] = dy2.sum(axis=0, dtype=np.float32)
    dh = gelu_bwd(matmul(dy2, np.ascontiguousarray(p["w2"].T)), cache["h"])
    g["w1"] = matmul(np.ascontiguousarray(cache["n2"].T), dh)
    g["b1"] = dh.sum(axis=0, dtype=np.float32)
    dn2 = matmul(dh, np.ascontiguousarray(p["w1"].T))
    dx1_n, g["norm2_w"] = rms_norm_bwd(dn2, cache["x1"], p["norm2_w"], eps)
    dx1 = dy2 + dx1_n
    mg = mha_backward(dx1.reshape(B, S, Hd), cache["mcache"])
    dn1 = mg.pop("dx").reshape(rows, Hd)
    g["mha"] = mg
    dx_n, g["norm1_w"] = rms_norm_bwd(dn1, cache["x2"], p["norm1_w"], eps)
    g["dx"] = (dx1 + dx_n).reshape(B, S, Hd)
    return g


def stack_forward_backward(ids, targets, p: dict, heads: int, rope_base: float = 10000.0, eps: float = 1e-5,
                           causal: bool = True):
    """A language model over TransformerBlocks: embedding rows, the blocks
    of p["blocks"], a final RMSNorm (norm_w), an output Linear (head_w
    [hidden, vocab], head_b) and the mean cross-entropy against targets.
    Returns (loss, grads) with grads keyed embed, blocks (a list of
    block_backward dicts), norm_w, head_w, head_b."""
    ids = np.asarray(ids)
    B, S = ids.shape
    vocab, Hd = p["embed"].shape
    x = embedding_fwd(p["embed"], ids.reshape(-1)).reshape(B, S, Hd)
    caches = []
    for bp in p["blocks"]:
        x, c = block_forward(x, bp, heads, rope_base, eps, causal)
        caches.append(c)
    x2 = x.reshape(B * S, Hd)
    n = rms_norm_fwd(x2, p["norm_w"], eps)
    logits = matmul(n, p["head_w"]) + p["head_b"]
    loss, dlogits = cross_entropy(logits, np.asarray(targets).reshape(-1))
    g = {"head_w": matmul(np.ascontiguousarray(n.T), dlogits), "head_b": dlogits.sum(axis=0, dtype=np.float32)}
    dn = matmul(dlogits, np.ascontiguousarray(p["head_w"].T))
    dx, g["norm_w"] = rms_norm_bwd(dn, x2, p["norm_w"], eps)
    dx = dx.reshape(B, S, Hd)
    g["blocks"] = [None] * len(caches)
    for i in range(len(caches) - 1, -1, -1):
        bg = block_backward(dx, caches[i])
        dx = bg.pop("dx")
        g["blocks"][i] = bg
    g["embed"] = embedding_bwd(dx.reshape(B * S, Hd), ids.reshape(-1), vocab)
    return loss, g


def gelu_fwd(x) -> np.ndarray:
    """kernels/activations.rs:192-209 (tanh form)."""
    x = _f32(x)
    y = np.empty_like(x)
    lib().ora_gelu_fwd(_p(x), _p(y), x.size)
    return y


def gelu_bwd(g, x) -> np.ndarray:
    """kernels/activations.rs:211-237."""
    g, x = _f32(g), _f32(x)
    dx = np.empty_like(x)
    lib().ora_gelu_bwd(_p(g), _p(x), _p(dx), x.size)
    return dx


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)


def cross_entropy(logits, targets):
    """kernels/loss.rs:46-117: (mean loss, dlogits) for logits [rows, classes]."""
    logits, targets = _f32(logits), _u32(targets)
    rows, classes = logits.shape
    probs = np.empty_like(logits)
    u32p = ctypes.POINTER(ctypes.c_uint32)
    loss = lib().ora_cross_entropy_fwd(_p(logits), targets.ctypes.data_as(u32p), _p(probs), rows, classes)
    grads = np.empty_like(logits)
    lib().ora_cross_entropy_bwd(_p(probs), targets.ctypes.data_as(u32p), _p(grads), rows, classes)
    return float(loss), grads


def adamw_step(p, g, m, v, lr: float, step: int, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
               weight_decay: float = 0.01):
    """optim.rs:128-191 on copies: returns (p, m, v) after one step."""
    p, m, v = (np.array(_f32(a), copy=True) for a in (p, m, v))
    g = _f32(g)
    lib().ora_adamw_step(_p(p), _p(g), _p(m), _p(v), p.size, lr, beta1, beta2, eps, weight_decay, int(step))
    return p, m, v


def embedding_fwd(table, ids) -> np.ndarray:
    """Row gather table[ids] (no reference counterpart: the crate has no embedding)."""
    return _f32(table)[_u32(ids)]


def embedding_bwd(dout, ids, vocab: int) -> np.ndarray:
    """Scatter-add of the rows of dout into a [vocab, dim] f32 table."""
    dout = _f32(dout)
    d = np.zeros((vocab, dout.shape[-1]), np.float32)
    np.add.at(d, _u32(ids), dout.reshape(-1, dout.shape[-1]))
    return d
