"""Pins the CPU oracle before it is trusted as the parity checker.

1. The reference's own softmax known-answer vectors and finite-difference
   tolerances (tests/golden/softmax_golden.json, extracted by make_golden.py
   from haelixe-lab/src/main.rs and tests/tensor_tests.rs).
2. The f32 restatement against an f64 evaluation of the same formulas.
3. Attention gradients against finite differences (EPS/TOL of the reference).
4. An independent implementation (torch CPU, f64 autograd) of the same math.
5. The documented departures from the reference (scale on dQ/dK, causal mask).
6. The row-block restatement (used for slices too long for S x S buffers)
   against the plain oracle, bit for bit.
"""
import json
import math
import os

import numpy as np
import pytest
import torch

from oracle import oracle as ora

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "softmax_golden.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


def test_softmax_golden_vectors(golden):
    for case in golden["softmax_cases"]:
        x = np.array(case["input"], np.float32).reshape(case["shape"])
        y = ora.softmax(x)
        kind = case["kind"]
        if kind == "softmax_forward":
            assert np.all(np.abs(y.ravel() - np.array(case["expected"])) < case["abs_tol"]), case["name"]
        elif kind == "softmax_finite":
            assert np.all(np.isfinite(y)), case["name"]
        elif kind == "softmax_simplex":
            assert np.all(np.abs(y.sum(-1) - 1.0) < case["abs_tol"]), case["name"]
            assert np.all((y >= 0) & (y <= 1)), case["name"]
        elif kind == "softmax_backward":
            dy = np.array(case["seed"], np.float32).reshape(case["shape"])
            dx = ora.softmax_backward(dy, y)
            assert np.all(np.abs(dx.ravel() - np.array(case["expected"])) < case["abs_tol"]), case["name"]
        elif kind == "softmax_sum_grad":
            dx = ora.softmax_backward(np.ones_like(y), y)
            assert np.all(np.abs(dx) < case["abs_tol"]), case["name"]
        else:
            raise AssertionError(f"unknown golden kind {kind}")


def test_softmax_finite_difference(golden):
    fd = golden["finite_difference"]
    eps, tol = fd["eps"], fd["tol"]
    x = np.array(fd["softmax_input"], np.float32)[None, :]
    w = np.array([0.3, -1.2, 0.7], np.float32)[None, :]  # loss = sum(w * softmax(x))
    y = ora.softmax(x)
    analytic = ora.softmax_backward(w, y)
    num = np.zeros_like(x)
    for i in range(x.shape[1]):
        xp, xm = x.copy(), x.copy()
        xp[0, i] += eps
        xm[0, i] -= eps
        num[0, i] = ((ora.softmax(xp) * w).sum() - (ora.softmax(xm) * w).sum()) / (2 * eps)
    assert np.max(np.abs(analytic - num)) < tol


def _inputs(BH, S, D, seed=0, bf16=False):
    rng = np.random.default_rng(seed)
    t = [rng.standard_normal((BH, S, D), dtype=np.float32) for _ in range(4)]
    if bf16:
        t = [ora.round_bf16(a) for a in t]
    return t


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S,D", [(1, 8), (17, 16), (64, 64), (130, 32)])
def test_f32_port_matches_f64(S, D, causal):
    q, k, v, do = _inputs(2, S, D, seed=S + D)
    scale = 1.0 / math.sqrt(D)
    o32, l32 = ora.attn_fwd(q, k, v, scale, causal)
    o64, l64 = ora.attn_fwd(q, k, v, scale, causal, f64=True)
    assert np.max(np.abs(o32 - o64)) < 2e-5
    assert np.max(np.abs(l32 - l64)) < 2e-5
    g32 = ora.attn_bwd(q, k, v, do, scale, causal)
    g64 = ora.attn_bwd(q, k, v, do, scale, causal, f64=True)
    for a, b in zip(g32, g64):
        assert np.max(np.abs(a - b)) < 5e-5


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("BH,S,D,rows", [(2, 1, 64, 64), (2, 300, 64, 128), (1, 1000, 128, 256),
                                         (1, 1000, 128, 192), (2, 513, 64, 64), (1, 4096, 128, 1024),
                                         (1, 129, 32, 4096)])
def test_row_block_oracle_is_the_plain_oracle_bit_for_bit(BH, S, D, rows, causal):
    q, k, v, do = _inputs(BH, S, D, seed=3 * S + D)
    scale = 1.0 / math.sqrt(D)
    o, lse = ora.attn_fwd(q, k, v, scale, causal)
    g = ora.attn_bwd(q, k, v, do, scale, causal)
    got = ora.attn_rows(q, k, v, do, scale, causal, rows)
    for name, a, b in zip(("O", "LSE", "dQ", "dK", "dV"), (o, lse) + g, got):
        assert np.array_equal(a, b), (name, float(np.abs(a - b).max()))


@pytest.mark.parametrize("causal", [False, True])
def test_attention_finite_difference(golden, causal):
    """d/dx of sum(O * G) by central differences at the reference's EPS/TOL."""
    eps, tol = golden["finite_difference"]["eps"], golden["finite_difference"]["tol"]
    BH, S, D = 1, 6, 4
    q, k, v, g = _inputs(BH, S, D, seed=11)
    scale = 0.5
    dq, dk, dv = ora.attn_bwd(q, k, v, g, scale, causal, f64=True)
    rng = np.random.default_rng(3)

    def loss(qq, kk, vv):
        o, _ = ora.attn_fwd(qq, kk, vv, scale, causal, f64=True)
        return float((o.astype(np.float64) * g).sum())

    for which, grad in ((0, dq), (1, dk), (2, dv)):
        for _ in range(6):
            idx = (0, int(rng.integers(S)), int(rng.integers(D)))
            args = [q.copy(), k.copy(), v.copy()]
            args[which][idx] += eps
            lp = loss(*args)
            args[which][idx] -= 2 * eps
            lm = loss(*args)
            num = (lp - lm) / (2 * eps)
            assert abs(num - grad[idx]) < tol, (which, idx, num, grad[idx])


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_matches_independent_torch_f64(causal):
    BH, S, D = 3, 33, 16
    q, k, v, do = _inputs(BH, S, D, seed=5)
    scale = 1.0 / math.sqrt(D)
    o, lse = ora.attn_fwd(q, k, v, scale, causal)
    dq, dk, dv = ora.attn_bwd(q, k, v, do, scale, causal)
    tq, tk, tv = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (q, k, v))
    s = (tq @ tk.transpose(1, 2)) * scale
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
    to = torch.softmax(s, -1) @ tv
    to.backward(torch.tensor(do, dtype=torch.float64))
    assert np.max(np.abs(o - to.detach().numpy())) < 1e-5
    assert np.max(np.abs(lse - torch.logsumexp(s, -1).detach().numpy())) < 1e-5
    for mine, ref in ((dq, tq.grad), (dk, tk.grad), (dv, tv.grad)):
        assert np.max(np.abs(mine - ref.numpy())) < 2e-5


def test_ref_compat_omits_scale_on_dq_dk():
    """The reference's backward (ops/flash_attention.rs:31,34-36) lacks `* scale`."""
    q, k, v, do = _inputs(2, 20, 8, seed=9)
    scale = 0.25
    dq, dk, dv = ora.attn_bwd(q, k, v, do, scale, True)
    rq, rk, rv = ora.attn_bwd(q, k, v, do, scale, True, ref_compat=True)
    np.testing.assert_allclose(rq * scale, dq, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(rk * scale, dk, rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(rv, dv)


def test_causal_first_row_is_first_value():
    q, k, v, _ = _inputs(2, 9, 8, seed=1)
    o, lse = ora.attn_fwd(q, k, v, 0.3, True)
    np.testing.assert_allclose(o[:, 0], v[:, 0], rtol=0, atol=1e-6)
    s00 = (q[:, 0] * k[:, 0]).sum(-1) * 0.3
    np.testing.assert_allclose(lse[:, 0], s00, rtol=0, atol=1e-5)


def test_gradient_identities():
    """sum_j dK_j = 0 and sum_j dV_j = sum_i dO_i (softmax rows sum to 1)."""
    q, k, v, do = _inputs(2, 40, 16, seed=21)
    for causal in (False, True):
        dq, dk, dv = ora.attn_bwd(q, k, v, do, 0.25, causal, f64=True)
        assert np.max(np.abs(dk.sum(1))) < 1e-4
        np.testing.assert_allclose(dv.sum(1), do.sum(1), atol=1e-4)


def test_rope_matches_f64_rotation_and_inverts():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((3, 50, 64), dtype=np.float32)
    base = 10000.0
    y = ora.rope_fwd(x, base)
    S, D = 50, 64
    i = np.arange(D // 2)
    theta = np.arange(S)[:, None] * np.power(base, -(2.0 * i) / D)[None, :]
    c, s = np.cos(theta), np.sin(theta)
    x0, x1 = x[..., 0::2].astype(np.float64), x[..., 1::2].astype(np.float64)
    ref = np.empty_like(x, dtype=np.float64)
    ref[..., 0::2] = x0 * c - x1 * s
    ref[..., 1::2] = x0 * s + x1 * c
    assert np.max(np.abs(y - ref)) < 1e-4
    np.testing.assert_array_equal(y[:, 0], x[:, 0])  # position 0 is the identity
    z = ora.rope_bwd(y, base)
    assert np.max(np.abs(z - x)) < 1e-4


def test_bf16_rounding_is_round_to_nearest_even():
    rng = np.random.default_rng(4)
    x = np.concatenate([rng.standard_normal(10000, dtype=np.float32) * 10,
                        np.array([1.0 + 2**-8, 1.0 + 3 * 2**-8, -0.0, 65504.0, 1e-40], np.float32)])
    mine = ora.round_bf16(x)
    ref = torch.tensor(x).to(torch.bfloat16).to(torch.float32).numpy()
    np.testing.assert_array_equal(mine, ref)


# ---- the attention block around the kernel (nn/attention.rs, kernels/rms_norm.rs) ----

def _torch_rope(x, base):
    """Interleaved-pair rotation by s * base^(-2i/D), in float64 (kernels/rope.rs:23-40)."""
    S, D = x.shape[-2], x.shape[-1]
    i = torch.arange(D // 2, dtype=torch.float64)
    freq = base ** (-(2 * i) / D)
    th = torch.arange(S, dtype=torch.float64)[:, None] * freq[None, :]
    c, s = torch.cos(th), torch.sin(th)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    return torch.stack((x0 * c - x1 * s, x0 * s + x1 * c), dim=-1).reshape(x.shape)


def test_rms_norm_matches_autograd():
    rng = np.random.default_rng(11)
    x = rng.standard_normal((7, 48), dtype=np.float32)
    w = rng.standard_normal(48, dtype=np.float32)
    g = rng.standard_normal((7, 48), dtype=np.float32)
    xt, wt = (torch.tensor(a, dtype=torch.float64, requires_grad=True) for a in (x, w))
    yt = xt / torch.sqrt((xt * xt).mean(-1, keepdim=True) + 1e-5) * wt
    yt.backward(torch.tensor(g, dtype=torch.float64))
    y = ora.rms_norm_fwd(x, w)
    dx, dw = ora.rms_norm_bwd(g, x, w)
    assert np.abs(y - yt.detach().numpy()).max() < 1e-5
    assert np.abs(dx - xt.grad.numpy()).max() < 1e-4
    assert np.abs(dw - wt.grad.numpy()).max() < 1e-4


@pytest.mark.parametrize("causal", [False, True])
def test_mha_composition_matches_autograd(causal):
    """oracle.mha_forward_backward against a float64 autograd model of
    MultiHeadAttention::forward (nn/attention.rs:46-98)."""
    B, S, H, D = 2, 12, 2, 8
    Hd = H * D
    rng = np.random.default_rng(5)
    x = rng.standard_normal((B, S, Hd), dtype=np.float32)
    dy = rng.standard_normal((B, S, Hd), dtype=np.float32)
    p = {"norm_w": rng.uniform(0.5, 1.5, Hd).astype(np.float32)}
    for c in "qkvo":
        p["w" + c] = (rng.uniform(-1, 1, (Hd, Hd)) * np.sqrt(6 / Hd)).astype(np.float32)
        p["b" + c] = rng.uniform(-0.1, 0.1, Hd).astype(np.float32)
    y, g = ora.mha_forward_backward(x, p, dy, H, rope_base=10000.0, causal=causal)
    pt = {k: torch.tensor(v, dtype=torch.float64, requires_grad=True) for k, v in p.items()}
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    n = xt / torch.sqrt((xt * xt).mean(-1, keepdim=True) + 1e-5) * pt["norm_w"]

    def split(t):
        return t.reshape(B, S, H, D).transpose(1, 2)

    q, k, v = (split(n @ pt["w" + c] + pt["b" + c]) for c in "qkv")
    q, k = _torch_rope(q, 10000.0), _torch_rope(k, 10000.0)
    s = (q @ k.transpose(-1, -2)) / np.sqrt(D)
    if causal:
        s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
    o = torch.softmax(s, -1) @ v
    yt = o.transpose(1, 2).reshape(B, S, Hd) @ pt["wo"] + pt["bo"]
    yt.backward(torch.tensor(dy, dtype=torch.float64))
    assert np.abs(y - yt.detach().numpy()).max() < 1e-4
    assert np.abs(g["dx"] - xt.grad.numpy()).max() < 1e-4
    for key in p:
        assert np.abs(g[key] - pt[key].grad.numpy()).max() < 2e-4, key
