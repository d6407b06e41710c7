"""CPU tests of the oracle's training-step restatements: GELU
(kernels/activations.rs:192-237), cross-entropy (kernels/loss.rs:46-117),
AdamW (optim.rs:128-199) and the TransformerBlock / block-stack compositions
(nn/transformer.rs, nn/mlp.rs), each pinned to the reference's own test
vectors where it has some and to float64 autograd models otherwise."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as ora


def _torch_rope(x, base):
    D = x.shape[-1]
    S = x.shape[-2]
    i = torch.arange(D // 2, dtype=torch.float64)
    theta = base ** (-2.0 * i / D)
    ang = torch.arange(S, dtype=torch.float64)[:, None] * theta[None, :]
    c, s = torch.cos(ang), torch.sin(ang)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def _rms(x, w, eps=1e-5):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w


def _gelu64(x):
    c = math.sqrt(2.0 / math.pi)
    return 0.5 * x * (1.0 + torch.tanh(c * (x + 0.044715 * x ** 3)))


def _torch_mha(x, pt, H, causal, base=10000.0):
    B, S, Hd = x.shape
    D = Hd // H
    n = _rms(x, pt["norm_w"])

    def split(t):
        return t.reshape(B, S, H, D).transpose(1, 2)

    q, k, v = (split(n @ pt["w" + c] + pt["b" + c]) for c in "qkv")
    q, k = _torch_rope(q, base), _torch_rope(k, base)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(D)
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
    o = torch.softmax(s, -1) @ v
    return o.transpose(1, 2).reshape(B, S, Hd) @ pt["wo"] + pt["bo"]


def _torch_block(x, pt, H, causal):
    x1 = x + _torch_mha(_rms(x, pt["norm1_w"]), pt["mha"], H, causal)
    h = _rms(x1, pt["norm2_w"]) @ pt["w1"] + pt["b1"]
    return x1 + _gelu64(h) @ pt["w2"] + pt["b2"]


def _block_params(rng, Hd):
    p = {"norm1_w": rng.uniform(0.5, 1.5, Hd).astype(np.float32),
         "norm2_w": rng.uniform(0.5, 1.5, Hd).astype(np.float32),
         "w1": (rng.standard_normal((Hd, 4 * Hd)) * 0.2).astype(np.float32),
         "b1": rng.uniform(-0.1, 0.1, 4 * Hd).astype(np.float32),
         "w2": (rng.standard_normal((4 * Hd, Hd)) * 0.1).astype(np.float32),
         "b2": rng.uniform(-0.1, 0.1, Hd).astype(np.float32),
         "mha": {"norm_w": rng.uniform(0.5, 1.5, Hd).astype(np.float32)}}
    for c in "qkvo":
        p["mha"]["w" + c] = (rng.standard_normal((Hd, Hd)) * 0.2).astype(np.float32)
        p["mha"]["b" + c] = rng.uniform(-0.1, 0.1, Hd).astype(np.float32)
    return p


def _to_torch(p):
    if isinstance(p, dict):
        return {k: _to_torch(v) for k, v in p.items()}
    if isinstance(p, list):
        return [_to_torch(v) for v in p]
    return torch.tensor(p, dtype=torch.float64, requires_grad=True)


def _compare_grads(g, pt, tol):
    if isinstance(pt, dict):
        for k in pt:
            _compare_grads(g[k], pt[k], tol)
    elif isinstance(pt, list):
        for a, b in zip(g, pt):
            _compare_grads(a, b, tol)
    else:
        ref = pt.grad.numpy()
        err = np.abs(np.asarray(g) - ref).max() / max(1.0, np.abs(ref).max())
        assert err < tol, err


def test_gelu_matches_tanh_form_and_its_autograd():
    x = np.linspace(-8, 8, 4001, dtype=np.float32)
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    yt = _gelu64(xt)
    g = np.random.default_rng(0).standard_normal(x.size).astype(np.float32)
    yt.backward(torch.tensor(g, dtype=torch.float64))
    assert np.abs(ora.gelu_fwd(x) - yt.detach().numpy()).max() < 2e-6
    assert np.abs(ora.gelu_bwd(g, x) - xt.grad.numpy()).max() < 1e-5


def test_gelu_finite_difference_reference_points():
    """tests/tensor_tests.rs:172-179 checks the GELU gradient at these points."""
    x = np.array([-2.0, -0.5, 0.0, 0.5, 2.0], np.float32)
    h = 1e-3
    num = (ora.gelu_fwd(x + h).astype(np.float64) - ora.gelu_fwd(x - h)) / (2 * h)
    assert np.abs(ora.gelu_bwd(np.ones_like(x), x) - num).max() < 1e-2


def test_cross_entropy_reference_vector():
    """tests/tensor_tests.rs:79-90: row [3, 4, 5] with target 1."""
    loss, grad = ora.cross_entropy(np.array([[3.0, 4.0, 5.0]], np.float32), [1])
    e = np.exp(np.array([-2.0, -1.0, 0.0]))
    assert abs(loss - (math.log(e.sum()) + 5.0 - 4.0)) < 1e-5
    assert np.abs(grad - (e / e.sum() - np.array([0, 1, 0]))).max() < 1e-6


def test_cross_entropy_matches_torch():
    rng = np.random.default_rng(1)
    logits = (rng.standard_normal((37, 101)) * 3).astype(np.float32)
    t = rng.integers(0, 101, 37).astype(np.uint32)
    loss, grad = ora.cross_entropy(logits, t)
    lt = torch.tensor(logits, dtype=torch.float64, requires_grad=True)
    ref = torch.nn.functional.cross_entropy(lt, torch.tensor(t.astype(np.int64)))
    ref.backward()
    assert abs(loss - ref.item()) < 1e-5
    assert np.abs(grad - lt.grad.numpy()).max() < 1e-6


def _adamw_scalar(p, g, m, v, lr, step, b1=0.9, b2=0.999, eps=1e-8, wd=0.01):
    """optim.rs:177-191 element by element with numpy float32 scalars."""
    f = np.float32
    r1 = r2 = f(1)
    a1, a2, n = f(b1), f(b2), step
    while True:  # square-and-multiply, one f32 rounding per product
        if n & 1:
            r1 = f(r1 * a1)
            r2 = f(r2 * a2)
        n //= 2
        if n == 0:
            break
        a1, a2 = f(a1 * a1), f(a2 * a2)
    bc1, bc2 = f(1) - r1, f(1) - r2
    p, m, v = p.copy(), m.copy(), v.copy()
    for i in range(p.size):
        gi = f(g[i])
        p[i] = f(p[i] - f(f(f(lr) * f(wd)) * p[i]))
        m[i] = f(f(f(b1) * m[i]) + f(f(f(1) - f(b1)) * gi))
        v[i] = f(f(f(b2) * v[i]) + f(f(f(f(1) - f(b2)) * gi) * gi))
        mh, vh = f(m[i] / bc1), f(v[i] / bc2)
        p[i] = f(p[i] - f(f(f(lr) * mh) / f(np.sqrt(vh) + f(eps))))
    return p, m, v


def test_adamw_port_is_bit_exact_to_scalar_restatement():
    rng = np.random.default_rng(2)
    n = 257
    p = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    p2, m2, v2 = p.copy(), m.copy(), v.copy()
    for step in range(1, 6):
        g = rng.standard_normal(n).astype(np.float32)
        p, m, v = ora.adamw_step(p, g, m, v, 1e-3, step)
        p2, m2, v2 = _adamw_scalar(p2, g, m2, v2, 1e-3, step)
        assert np.array_equal(p, p2) and np.array_equal(m, m2) and np.array_equal(v, v2), step


def test_adamw_port_tracks_torch_adamw():
    """torch.optim.AdamW computes the same update with a different grouping of
    the bias corrections; the two agree to rounding."""
    rng = np.random.default_rng(3)
    n = 1000
    p0 = rng.standard_normal(n).astype(np.float32)
    pt = torch.tensor(p0.astype(np.float64), requires_grad=True)
    opt = torch.optim.AdamW([pt], lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    p, m, v = p0.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    for step in range(1, 11):
        g = rng.standard_normal(n).astype(np.float32)
        p, m, v = ora.adamw_step(p, g, m, v, 1e-2, step)
        pt.grad = torch.tensor(g.astype(np.float64))
        opt.step()
    assert np.abs(p - pt.detach().numpy()).max() < 1e-5


@pytest.mark.parametrize("causal", [False, True])
def test_block_composition_matches_autograd(causal):
    B, S, H, D = 2, 10, 2, 8
    Hd = H * D
    rng = np.random.default_rng(4)
    x = rng.standard_normal((B, S, Hd), dtype=np.float32)
    dy = rng.standard_normal((B, S, Hd), dtype=np.float32)
    p = _block_params(rng, Hd)
    y, cache = ora.block_forward(x, p, H, causal=causal)
    g = ora.block_backward(dy, cache)
    pt = _to_torch(p)
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    yt = _torch_block(xt, pt, H, causal)
    yt.backward(torch.tensor(dy, dtype=torch.float64))
    assert np.abs(y - yt.detach().numpy()).max() < 2e-4
    assert np.abs(g["dx"] - xt.grad.numpy()).max() < 2e-4
    g.pop("dx")
    _compare_grads(g, pt, 5e-4)


def test_stack_composition_matches_autograd():
    B, S, H, D, V, L = 2, 8, 2, 8, 23, 2
    Hd = H * D
    rng = np.random.default_rng(5)
    ids = rng.integers(0, V, (B, S))
    targets = rng.integers(0, V, B * S)
    p = {"embed": (rng.standard_normal((V, Hd)) * 0.5).astype(np.float32),
         "blocks": [_block_params(rng, Hd) for _ in range(L)],
         "norm_w": rng.uniform(0.5, 1.5, Hd).astype(np.float32),
         "head_w": (rng.standard_normal((Hd, V)) * 0.2).astype(np.float32),
         "head_b": rng.uniform(-0.1, 0.1, V).astype(np.float32)}
    loss, g = ora.stack_forward_backward(ids, targets, p, H, causal=True)
    pt = _to_torch(p)
    x = pt["embed"][torch.tensor(ids)]
    for bp in pt["blocks"]:
        x = _torch_block(x, bp, H, True)
    logits = _rms(x.reshape(B * S, Hd), pt["norm_w"]) @ pt["head_w"] + pt["head_b"]
    lt = torch.nn.functional.cross_entropy(logits, torch.tensor(targets))
    lt.backward()
    assert abs(loss - lt.item()) < 1e-4
    _compare_grads(g, pt, 5e-4)
