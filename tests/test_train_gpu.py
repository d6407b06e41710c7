"""GPU parity of the training step around the block stack, through the C ABI,
against the CPU oracle: GELU (kernels/activations.rs:192-237), cross-entropy
(kernels/loss.rs:46-117), AdamW (optim.rs:128-199, bit-exact for f32), the
embedding, Linear with the residual folded in, TransformerBlock
(nn/transformer.rs + nn/mlp.rs) and a two-block BlockStack training step.

Tolerances: max-abs 1e-3 (f32) for element kernels and f32 blocks; bf16
blocks round every intermediate to bf16, so they are checked by relative L2
error (2 %) against the oracle on the same bf16-rounded inputs.
"""
import ctypes

import numpy as np
import pytest
import torch

import haelixe_b200 as hx
from haelixe_b200 import _native as N
from oracle import oracle as ora

pytestmark = pytest.mark.gpu

F32, BF16 = torch.float32, torch.bfloat16
DT = [pytest.param(F32, id="f32"), pytest.param(BF16, id="bf16")]


def _dev(a, dtype, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dtype).cuda()
    return t.requires_grad_() if grad else t


def _rnd(a, dtype):
    return ora.round_bf16(a) if dtype == BF16 else np.asarray(a, np.float32)


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("n", [1, 1000, 1 << 20])
def test_gelu_matches_oracle(dtype, n):
    rng = np.random.default_rng(n)
    x = _rnd(rng.standard_normal(n).astype(np.float32) * 3, dtype)
    g = _rnd(rng.standard_normal(n).astype(np.float32), dtype)
    xt = _dev(x, dtype, grad=True)
    y = hx.nn.gelu(xt)
    y.backward(_dev(g, dtype))
    tol = 1e-5 if dtype == F32 else 8e-3  # relative to max(1, |ref|); bf16 rounds the output (2^-9)
    for got, ref in ((y, ora.gelu_fwd(x)), (xt.grad, ora.gelu_bwd(g, x))):
        assert (np.abs(_np(got) - ref) / np.maximum(1.0, np.abs(ref))).max() < tol


def test_gelu_in_place():
    x = np.linspace(-5, 5, 4097, dtype=np.float32)
    t = _dev(x, F32)
    c = hx.context()
    c.use_stream()
    N.check(N.lib().hx_gelu_fwd(c.handle, 0, ctypes.c_void_p(t.data_ptr()), ctypes.c_void_p(t.data_ptr()),
                                t.numel()), c.handle)
    c.sync()
    assert np.abs(_np(t) - ora.gelu_fwd(x)).max() < 1e-5


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("rows,classes", [(1, 3), (37, 101), (64, 32000), (5, 70001)])
def test_cross_entropy_matches_oracle(dtype, rows, classes):
    rng = np.random.default_rng(rows * classes)
    logits = _rnd(rng.standard_normal((rows, classes)).astype(np.float32) * 4, dtype)
    t = rng.integers(0, classes, rows).astype(np.int32)
    lt = _dev(logits, dtype, grad=True)
    loss = hx.nn.cross_entropy(lt, torch.from_numpy(t).cuda())
    loss.backward()
    rl, rg = ora.cross_entropy(logits, t.astype(np.uint32))
    assert abs(loss.item() - rl) < 1e-4 * max(1.0, abs(rl))
    # f32: the oracle (like loss.rs:70) sums exp() over a row left to right,
    # the kernel in a tree; over 70001 classes the left-to-right sum drifts by
    # ~1e-4 relative, so the kernel is also held to a float64 evaluation.
    tol = 1e-4 if dtype == F32 else 1e-2 / rows
    assert np.abs(_np(lt.grad) - rg).max() < tol
    if dtype == F32:
        l64 = logits.astype(np.float64)
        p64 = np.exp(l64 - l64.max(1, keepdims=True))
        p64 /= p64.sum(1, keepdims=True)
        p64[np.arange(rows), t] -= 1.0
        assert np.abs(_np(lt.grad) - p64 / rows).max() < 1e-6


def test_cross_entropy_reference_vector_and_edges():
    """tests/tensor_tests.rs:79-90 ([3, 4, 5], target 1); -inf logits; a target
    out of range gives a NaN loss instead of the reference's panic."""
    lt = _dev(np.array([[3.0, 4.0, 5.0], [0.0, -np.inf, 1.0]], np.float32), F32, grad=True)
    loss = hx.nn.cross_entropy(lt, torch.tensor([1, 2], dtype=torch.int32).cuda())
    loss.backward()
    e = np.exp([-2.0, -1.0, 0.0])
    l0 = np.log(e.sum()) + 1.0
    l1 = np.log(1.0 + np.exp(-1.0)) + 1.0 - 1.0
    assert abs(loss.item() - (l0 + l1) / 2) < 1e-5
    g = _np(lt.grad)
    assert g[1, 1] == 0.0 and np.isfinite(g).all()
    bad = hx.nn.cross_entropy(_dev(np.zeros((2, 4), np.float32), F32), torch.tensor([0, 4]).cuda())
    assert np.isnan(bad.item())


def _adam_table(items):
    arr = (N.AdamWTensor * len(items))()
    for i, (p, g, m, v, low) in enumerate(items):
        arr[i].param, arr[i].grad, arr[i].m, arr[i].v = p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr()
        arr[i].param_lowp = low.data_ptr() if low is not None else None
        arr[i].n = p.numel()
        arr[i].grad_dtype = 1 if g.dtype == BF16 else 0
    return arr


@pytest.mark.parametrize("gdtype", DT)
def test_adamw_multi_tensor_matches_oracle(gdtype):
    """61 tensors (two launches of the 48-tensor table), odd sizes and
    unaligned views (the scalar tail path), 4 steps. f32 gradients: bit-exact."""
    rng = np.random.default_rng(11)
    sizes = [int(s) for s in rng.integers(1, 40000, 60)] + [70001]
    c = hx.context()
    c.use_stream()  # the step's kernels run in order with torch's copies and frees
    host, dev = [], []
    for i, n in enumerate(sizes):
        off = i % 3  # element offset into a larger buffer: breaks 16-byte alignment for some
        p = rng.standard_normal(n).astype(np.float32)
        pbuf = torch.zeros(n + off, dtype=F32, device="cuda")
        pbuf[off:] = torch.from_numpy(p).cuda()
        mv = torch.zeros(2, n + off, dtype=F32, device="cuda")
        low = torch.zeros(n, dtype=BF16, device="cuda") if i % 2 else None
        host.append([p, np.zeros(n, np.float32), np.zeros(n, np.float32)])
        dev.append((pbuf[off:], mv[0, off:], mv[1, off:], low))
    for step in range(1, 5):
        grads = [_rnd(rng.standard_normal(n).astype(np.float32), gdtype) for n in sizes]
        gd = [_dev(g, gdtype) for g in grads]
        arr = _adam_table([(p, g, m, v, low) for (p, m, v, low), g in zip(dev, gd)])
        N.check(N.lib().hx_adamw_step(c.handle, ctypes.cast(arr, ctypes.c_void_p), len(sizes), 1e-3, 0.9, 0.999,
                                      1e-8, 0.01, step), c.handle)
        for h, g in zip(host, grads):
            h[0], h[1], h[2] = ora.adamw_step(h[0], g, h[1], h[2], 1e-3, step)
    c.sync()
    for (p, m, v, low), (rp, rm, rv) in zip(dev, host):
        assert np.array_equal(_np(p), rp) and np.array_equal(_np(m), rm) and np.array_equal(_np(v), rv)
        if low is not None:
            assert np.array_equal(_np(low), ora.round_bf16(rp))


def test_adamw_rejects_bad_arguments():
    c = hx.context()
    c.use_stream()
    with pytest.raises(hx.HxError):
        N.check(N.lib().hx_adamw_step(c.handle, None, 1, 1e-3, 0.9, 0.999, 1e-8, 0.01, 1), c.handle)
    p = torch.zeros(4, device="cuda")
    arr = _adam_table([(p, p, p, p, None)])
    with pytest.raises(hx.HxError):
        N.check(N.lib().hx_adamw_step(c.handle, ctypes.cast(arr, ctypes.c_void_p), 1, 1e-3, 0.9, 0.999, 1e-8,
                                      0.01, 0), c.handle)


@pytest.mark.parametrize("dtype", DT)
def test_embedding_matches_oracle(dtype):
    rng = np.random.default_rng(12)
    V, Dm, T = 97, 200, 333
    table = _rnd(rng.standard_normal((V, Dm)).astype(np.float32), dtype)
    ids = rng.integers(0, V, (3, T // 3)).astype(np.int32)
    g = _rnd(rng.standard_normal((3, T // 3, Dm)).astype(np.float32), dtype)
    tt = _dev(table, dtype, grad=True)
    out = hx.nn.embedding(torch.from_numpy(ids).cuda(), tt)
    out.backward(_dev(g, dtype))
    assert np.array_equal(_np(out), ora.embedding_fwd(table, ids.reshape(-1)).reshape(3, T // 3, Dm))
    ref = ora.embedding_bwd(g.reshape(-1, Dm), ids.reshape(-1), V)
    tol = 1e-5 if dtype == F32 else 2e-2 * max(1.0, np.abs(ref).max())
    assert np.abs(_np(tt.grad) - ref).max() < tol


@pytest.mark.parametrize("dtype", DT)
def test_linear_residual_matches_oracle(dtype):
    rng = np.random.default_rng(13)
    rows, fin, fout = 75, 128, 96
    x, w, b, r, g = (_rnd(a, dtype) for a in (rng.standard_normal((rows, fin)).astype(np.float32),
                                               rng.standard_normal((fin, fout)).astype(np.float32) * 0.1,
                                               rng.standard_normal(fout).astype(np.float32),
                                               rng.standard_normal((rows, fout)).astype(np.float32),
                                               rng.standard_normal((rows, fout)).astype(np.float32)))
    xt, wt, bt, rt = (_dev(a, dtype, grad=True) for a in (x, w, b, r))
    y = hx.nn.linear(xt, wt, bt, residual=rt)
    y.backward(_dev(g, dtype))
    ry = r + (ora.matmul(x, w) + b)
    tol = 1e-3 if dtype == F32 else 3e-2
    for name, got, ref in (("y", y, ry), ("dr", rt.grad, g), ("db", bt.grad, g.sum(0)),
                           ("dx", xt.grad, ora.matmul(g, np.ascontiguousarray(w.T)))):
        err = np.abs(_np(got) - ref).max() / max(1.0, np.abs(ref).max())
        assert err < tol, (name, err)


def _block_params(rng, Hd, dtype):
    p = {"norm1_w": rng.uniform(0.5, 1.5, Hd), "norm2_w": rng.uniform(0.5, 1.5, Hd),
         "w1": rng.standard_normal((Hd, 4 * Hd)) * (1 / np.sqrt(Hd)), "b1": rng.uniform(-0.1, 0.1, 4 * Hd),
         "w2": rng.standard_normal((4 * Hd, Hd)) * (0.5 / np.sqrt(4 * Hd)), "b2": rng.uniform(-0.1, 0.1, Hd),
         "mha": {"norm_w": rng.uniform(0.5, 1.5, Hd)}}
    for c in "qkvo":
        p["mha"]["w" + c] = rng.standard_normal((Hd, Hd)) * (1 / np.sqrt(Hd))
        p["mha"]["b" + c] = rng.uniform(-0.1, 0.1, Hd)
    cast = lambda d: {k: cast(v) if isinstance(v, dict) else _rnd(v.astype(np.float32), dtype) for k, v in d.items()}
    return cast(p)


def _block_tensors(blk):
    m = blk.mha
    t = {"norm1_w": blk.norm1.weight, "norm2_w": blk.norm2.weight, "w1": blk.mlp.linear1.weight,
         "b1": blk.mlp.linear1.bias, "w2": blk.mlp.linear2.weight, "b2": blk.mlp.linear2.bias,
         "mha": {"norm_w": m.norm.weight}}
    for c, lin in zip("qkvo", (m.q_proj, m.k_proj, m.v_proj, m.out_proj)):
        t["mha"]["w" + c], t["mha"]["b" + c] = lin.weight, lin.bias
    return t


def _load(tensors, p):
    with torch.no_grad():
        for k, v in p.items():
            if isinstance(v, dict):
                _load(tensors[k], v)
            else:
                tensors[k].copy_(torch.from_numpy(v))


def _check(tensors, ref, dtype, path=""):
    for k, r in ref.items():
        if isinstance(r, dict):
            _check(tensors[k], r, dtype, path + k + ".")
            continue
        got = _np(tensors[k].grad)
        if dtype == F32:
            err = np.abs(got - r).max() / max(1.0, np.abs(r).max())
            assert err < 1e-3, (path + k, err)
        else:
            rel = np.linalg.norm(got - r) / max(np.linalg.norm(r), 1e-6)
            assert rel < 2e-2, (path + k, rel)


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_transformer_block_matches_oracle(dtype, causal):
    B, S, H, D = 2, 128, 2, 64
    Hd = H * D
    rng = np.random.default_rng(14)
    p = _block_params(rng, Hd, dtype)
    x = _rnd(rng.standard_normal((B, S, Hd)).astype(np.float32), dtype)
    dy = _rnd(rng.standard_normal((B, S, Hd)).astype(np.float32), dtype)
    blk = hx.nn.TransformerBlock(Hd, H, device="cuda", dtype=dtype, causal=causal)
    tens = _block_tensors(blk)
    _load(tens, p)
    xt = _dev(x, dtype, grad=True)
    y = blk(xt)
    y.backward(_dev(dy, dtype))
    ry, cache = ora.block_forward(x, p, H, causal=causal)
    rg = ora.block_backward(dy, cache)
    for name, got, ref in (("y", y, ry), ("dx", xt.grad, rg.pop("dx"))):
        got = _np(got)
        if dtype == F32:
            assert np.abs(got - ref).max() < 1e-3, name
        else:
            assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-2, name
    _check(tens, rg, dtype)


@pytest.mark.parametrize("dtype", DT)
def test_block_stack_step_matches_oracle(dtype):
    """A two-block stack (vocab 300, hidden 128, 2 heads x 64, causal): loss,
    every gradient, then one AdamW step on every parameter."""
    B, S, H, D, V, L = 2, 64, 2, 64, 300, 2
    Hd = H * D
    rng = np.random.default_rng(15)
    model = hx.nn.BlockStack(V, Hd, H, L, device="cuda", dtype=dtype, causal=True)
    p = {"embed": _rnd(rng.standard_normal((V, Hd)).astype(np.float32) * 0.5, dtype),
         "blocks": [_block_params(rng, Hd, dtype) for _ in range(L)],
         "norm_w": _rnd(rng.uniform(0.5, 1.5, Hd).astype(np.float32), dtype),
         "head_w": _rnd(rng.standard_normal((Hd, V)).astype(np.float32) * (1 / np.sqrt(Hd)), dtype),
         "head_b": _rnd(rng.uniform(-0.1, 0.1, V).astype(np.float32), dtype)}
    tens = {"embed": model.embed.weight, "blocks": [_block_tensors(b) for b in model.blocks],
            "norm_w": model.norm.weight, "head_w": model.head.weight, "head_b": model.head.bias}
    for bt, bp in zip(tens["blocks"], p["blocks"]):
        _load(bt, bp)
    _load({k: tens[k] for k in ("embed", "norm_w", "head_w", "head_b")},
          {k: p[k] for k in ("embed", "norm_w", "head_w", "head_b")})
    ids = rng.integers(0, V, (B, S))
    targets = rng.integers(0, V, B * S)
    loss = model.loss(torch.from_numpy(ids).cuda(), torch.from_numpy(targets).cuda())
    loss.backward()
    rl, rg = ora.stack_forward_backward(ids, targets, p, H, causal=True)
    assert abs(loss.item() - rl) < (1e-4 if dtype == F32 else 2e-2) * max(1.0, abs(rl))
    for k in ("embed", "norm_w", "head_w", "head_b"):
        _check({k: tens[k]}, {k: rg[k]}, dtype)
    for bt, bg in zip(tens["blocks"], rg["blocks"]):
        _check(bt, bg, dtype)
    # one optimizer step: every parameter against the oracle's AdamW on the GPU's own gradients
    params = model.parameters()
    before = [_np(q) for q in params]
    grads = [_np(q.grad) for q in params]
    opt = hx.optim.AdamW(1e-3)
    opt.step([(q, q.grad) for q in params])
    for q, b0, g in zip(params, before, grads):
        rp, _, _ = ora.adamw_step(b0, g, np.zeros_like(b0), np.zeros_like(b0), 1e-3, 1)
        if dtype == F32:
            assert np.array_equal(_np(q), rp)
        else:
            assert np.array_equal(_np(q), ora.round_bf16(rp))


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("rows,fin,fout", [(70, 100, 75), (33, 64, 8), (1, 9, 3)])
def test_row_kernels_vector_and_scalar_forms(dtype, rows, fin, fout):
    """RMSNorm, Linear (+ residual, bias gradient) and GELU on widths that are
    and are not multiples of the 16-byte vector, with tiles of rows that do
    not fill a block, against the oracle."""
    rng = np.random.default_rng(rows * 1000 + fin)
    x = _rnd(rng.standard_normal((rows, fin)).astype(np.float32), dtype)
    nw = _rnd(rng.uniform(0.5, 1.5, fin).astype(np.float32), dtype)
    gn = _rnd(rng.standard_normal((rows, fin)).astype(np.float32), dtype)
    w = _rnd(rng.standard_normal((fin, fout)).astype(np.float32) * 0.1, dtype)
    b = _rnd(rng.standard_normal(fout).astype(np.float32), dtype)
    r = _rnd(rng.standard_normal((rows, fout)).astype(np.float32), dtype)
    g = _rnd(rng.standard_normal((rows, fout)).astype(np.float32), dtype)
    tol = 1e-3 if dtype == F32 else 3e-2

    def close(name, got, ref):
        err = np.abs(_np(got) - ref).max() / max(1.0, np.abs(ref).max())
        assert err < tol, (name, err)

    xt, nwt = _dev(x, dtype, grad=True), _dev(nw, dtype, grad=True)
    n = hx.nn.rms_norm(xt, nwt)
    n.backward(_dev(gn, dtype))
    rdx, rdw = ora.rms_norm_bwd(gn, x, nw)
    close("norm", n, ora.rms_norm_fwd(x, nw))
    close("norm dx", xt.grad, rdx)
    close("norm dw", nwt.grad, rdw)

    xt2, wt, bt, rt = (_dev(a, dtype, grad=True) for a in (x, w, b, r))
    y = hx.nn.linear(xt2, wt, bt, residual=rt)
    y.backward(_dev(g, dtype))
    close("y", y, r + (ora.matmul(x, w) + b))
    close("db", bt.grad, g.sum(0))
    close("dw", wt.grad, ora.matmul(np.ascontiguousarray(x.T), g))

    # GELU on an unaligned view (one element in): the scalar form
    buf = _dev(np.concatenate([[0.0], x.reshape(-1)]).astype(np.float32), dtype)
    xv = buf[1:].detach().requires_grad_()
    gy = hx.nn.gelu(xv)
    gy.backward(_dev(gn.reshape(-1)[: x.size] if gn.size >= x.size else np.ones(x.size, np.float32), dtype))
    close("gelu", gy, ora.gelu_fwd(x.reshape(-1)))
