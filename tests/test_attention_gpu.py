"""GPU parity of the fused attention (through the C ABI) against the CPU oracle.

Tolerances (max-abs, for O and every gradient): 1e-3 for f32 I/O and 2e-2
for bf16 I/O with f32 accumulation, with the oracle run in f32 on the same
bf16-rounded inputs. bf16 outputs are rounded to bf16, whose spacing exceeds
2e-2 above magnitude 4; for such elements the bound is widened to one bf16
spacing of the oracle value (`_bf16_tol`).
"""
import ctypes
import math

import numpy as np
import pytest
import torch

import haelixe_b200 as hx
from haelixe_b200 import _native as N
from oracle import oracle as ora

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-3, torch.bfloat16: 2e-2}


def _host(shape, seed, dtype):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal(shape, dtype=np.float32)
    return ora.round_bf16(a) if dtype == torch.bfloat16 else a


def _dev(a, dtype):
    return torch.from_numpy(a).to(dtype).cuda()


def _bf16_tol(ref, tol):
    # one bf16 spacing (2^(e-7)) where it exceeds the absolute tolerance
    mag = np.abs(ref)
    spacing = np.exp2(np.floor(np.log2(np.maximum(mag, 1e-30))) - 7)
    return np.maximum(tol, spacing)


def _check(name, got, ref, dtype):
    got = got.float().cpu().numpy().reshape(ref.shape)
    tol = TOL[dtype]
    err = np.abs(got - ref)
    bound = _bf16_tol(ref, tol) if dtype == torch.bfloat16 else tol
    bad = err > bound
    assert not bad.any(), (f"{name}: max_abs_err={err.max():.3g} at {np.unravel_index(err.argmax(), err.shape)}"
                           f" ({bad.sum()} elements over the bound)")
    return float(err.max())


CASES = [
    # (BH, S, D)
    (2, 1, 64), (2, 17, 64), (3, 128, 64), (2, 129, 64), (2, 255, 128), (2, 256, 128),
    (1, 384, 128), (2, 300, 64), (1, 97, 32), (2, 65, 80), (1, 70, 256), (1, 130, 16),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("BH,S,D", CASES)
def test_fwd_bwd_matches_oracle(BH, S, D, causal, dtype):
    seed = BH * 1000 + S * 7 + D
    q, k, v, do = (_host((BH, S, D), seed + i, dtype) for i in range(4))
    scale = 1.0 / math.sqrt(D)
    qd, kd, vd, dod = (_dev(a, dtype) for a in (q, k, v, do))
    ctx = hx.context()
    expect = "tcgen05" if D in (64, 128) else "simt"  # f32 there: bf16 hi/lo operand planes
    o, lse = hx.attn_forward(qd, kd, vd, scale, causal)
    assert ctx.last_path == expect
    dq, dk, dv = hx.attn_backward(qd, kd, vd, o, lse, dod, scale, causal)
    assert ctx.last_path == expect
    torch.cuda.synchronize()
    ro, rlse = ora.attn_fwd(q, k, v, scale, causal)
    rdq, rdk, rdv = ora.attn_bwd(q, k, v, do, scale, causal)
    _check("O", o, ro, dtype)
    assert np.max(np.abs(lse.cpu().numpy().reshape(rlse.shape) - rlse)) < 1e-3
    _check("dQ", dq, rdq, dtype)
    _check("dK", dk, rdk, dtype)
    _check("dV", dv, rdv, dtype)


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_bf16_paths_agree_with_simt(causal):
    """The tcgen05 path (when selected) and the SIMT path give the same answer."""
    BH, S, D = 4, 512, 128
    q, k, v, do = (_dev(_host((BH, S, D), 50 + i, torch.bfloat16), torch.bfloat16) for i in range(4))
    ctx = hx.context()
    outs = []
    for force in (False, True):
        ctx.force_simt(force)
        o, lse = hx.attn_forward(q, k, v, 0.088, causal)
        g = hx.attn_backward(q, k, v, o, lse, do, 0.088, causal)
        outs.append([o.float(), lse] + [t.float() for t in g])
    ctx.force_simt(False)
    for a, b in zip(*outs):
        a, b = a.cpu().numpy(), b.cpu().numpy()
        # both sides are bf16-rounded: allow 2e-2 or two bf16 spacings
        assert (np.abs(a - b) <= 2 * _bf16_tol(b, 1e-2)).all(), np.abs(a - b).max()


def test_strided_bshd_layout_matches_contiguous():
    """[B,S,H,D] storage (the projection layout of nn/attention.rs:57-73) viewed
    as [B,H,S,D] without copies gives the same result as the contiguous call."""
    B, S, H, D = 2, 200, 3, 64
    base = [torch.from_numpy(_host((B, S, H, D), 70 + i, torch.bfloat16)).to(torch.bfloat16).cuda()
            for i in range(4)]
    views = [t.permute(0, 2, 1, 3) for t in base]  # [B,H,S,D], stride_s = H*D
    o, lse = hx.attn_forward(*views[:3], 0.125, True)
    g = hx.attn_backward(*views[:3], o, lse, views[3], 0.125, True)
    cont = [t.contiguous() for t in views]
    o2, lse2 = hx.attn_forward(*cont[:3], 0.125, True)
    g2 = hx.attn_backward(*cont[:3], o2, lse2, cont[3], 0.125, True)
    assert (o.float() - o2.float()).abs().max().item() < 2e-2
    for a, b in zip(g, g2):
        assert (a.float() - b.float()).abs().max().item() < 2e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_autograd_node(dtype):
    BH, S, D = 2, 96, 64
    q, k, v, g = (_dev(_host((BH, S, D), 90 + i, dtype), dtype) for i in range(4))
    for t in (q, k, v):
        t.requires_grad_(True)
    o = hx.flash_attention(q, k, v, 0.125, causal=True)
    o.backward(g)
    o2, lse2 = hx.attn_forward(q.detach(), k.detach(), v.detach(), 0.125, True)
    op = hx.FlashAttentionOp(q.detach(), k.detach(), v.detach(), 0.125, o2, lse2, True)
    assert op.name() == "FlashAttention"
    grads = op.backward(g)
    for t, ref in zip((q, k, v), grads):
        assert torch.equal(t.grad, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("base", [10000.0, 500000.0])
def test_rope_matches_oracle(dtype, base):
    BH, S, D = 3, 257, 128
    x = _host((BH, S, D), 5, dtype)
    xd = _dev(x, dtype)
    y = hx.rope_forward(xd, base)
    z = hx.rope_backward(y, base)
    ref = ora.rope_fwd(x, base)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert np.max(np.abs(y.float().cpu().numpy() - ref)) < tol
    refz = ora.rope_bwd(y.float().cpu().numpy(), base)
    assert np.max(np.abs(z.float().cpu().numpy() - refz)) < tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("shape", [(2, 3, 257, 128), (1, 4, 1024, 64), (2, 2, 33, 40)])
def test_rope_qk_one_launch_equals_two(shape, dtype):
    """hx_rope_fwd_qk rotates Q and K exactly as two hx_rope_fwd calls do
    (one launch; layouts the vector kernel cannot take run as two)."""
    q = torch.from_numpy(_host(shape, 31, dtype)).to(dtype).cuda()
    k = torch.from_numpy(_host(shape, 32, dtype)).to(dtype).cuda()
    ctx = hx.context()
    ref_q, ref_k = hx.rope_forward(q, 500000.0), hx.rope_forward(k, 500000.0)  # also builds the table
    n0 = N.lib().hx_kernel_launches(ctx.handle)
    qr, kr = hx.rope_forward_qk(q, k, 500000.0)
    n1 = N.lib().hx_kernel_launches(ctx.handle)
    assert torch.equal(qr, ref_q) and torch.equal(kr, ref_k)
    if shape[-1] % 8 == 0:
        assert n1 - n0 == 1


def test_arena_bins_and_reuse():
    ctx = hx.CudaContext(0)
    try:
        a = ctx.allocate(4000)
        assert a.size == 4096
        p = a.ptr
        del a  # last reference: slab goes back to the 4096 bin
        s = ctx.arena_stats()
        assert s["cached_slabs"] == 1 and s["cached_bytes"] == 4096 and s["live_bytes"] == 0
        b = ctx.allocate(4010)  # same bin -> the same slab (arena.rs:28-31)
        assert b.ptr == p
        s = ctx.arena_stats()
        assert s["hits"] == 1 and s["misses"] == 1 and s["live_bytes"] == 4096
        c = ctx.allocate(100)
        assert c.size == 512
        del b, c
        ctx.arena_reset()
        assert ctx.arena_stats()["cached_slabs"] == 0
    finally:
        ctx.close()


def test_invalid_arguments_raise():
    q = torch.zeros(1, 16, 300, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(hx.HxError) as e:
        hx.attn_forward(q, q, q, 1.0)
    assert e.value.status == N.HX_ERR_UNSUPPORTED
    with pytest.raises(ValueError):
        hx.attn_forward(q, q.float(), q, 1.0)
    with pytest.raises(RuntimeError):
        hx.attn_forward(q.cpu(), q.cpu(), q.cpu(), 1.0)


def test_misaligned_operands_take_a_correct_path():
    """Operands that TMA cannot address (16-byte rule) still give the right answer."""
    BH, S, D = 1, 64, 64
    q, k, v = (_host((BH, S, D), 120 + i, torch.bfloat16) for i in range(3))
    buf = [torch.empty(BH * S * D + 1, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    views = []
    for b, a in zip(buf, (q, k, v)):
        t = b[1:].view(BH, S, D)
        t.copy_(torch.from_numpy(a).to(torch.bfloat16))
        views.append(t)
    o, _ = hx.attn_forward(*views, 0.125, False)
    ro, _ = ora.attn_fwd(q, k, v, 0.125, False)
    _check("O", o, ro, torch.bfloat16)


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64)], ids=["bf16", "f32"])
def test_forward_without_lse_stays_on_tcgen05(dtype, D):
    """hx_attn_fwd_strided with lse = NULL (no backward follows): the tcgen05
    kernels take a temporary lse from the arena, so an inference call keeps the
    tensor-core path and gives the same O as the call with an lse buffer."""
    BH, S = 2, 300
    q, k, v = (_dev(_host((BH, S, D), 140 + i, dtype), dtype) for i in range(3))
    ctx = hx.context()
    o_ref, _ = hx.attn_forward(q, k, v, 0.1, True)
    o = torch.empty_like(q)
    shp = hx.attention._shape_of(q)
    code = N.HX_BF16 if dtype == torch.bfloat16 else N.HX_F32
    N.check(N.lib().hx_attn_fwd_strided(ctx.handle, code, ctypes.byref(shp), ctypes.c_void_p(q.data_ptr()),
                                        ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()),
                                        ctypes.c_void_p(o.data_ptr()), None, 0.1, 1), ctx.handle)
    assert ctx.last_path == "tcgen05"
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("layout", ["bshd", "bhsd"])
def test_reassemble_heads_kernel(dtype, layout):
    from haelixe_b200.sharding import reassemble_heads
    n, B, Hs, S, D = 4, 2, 3, 37, 64
    g = torch.randn(n, B, Hs, S, D, device="cuda").to(dtype)
    out = torch.empty((B, S, n * Hs, D) if layout == "bshd" else (B, n * Hs, S, D),
                      device="cuda", dtype=dtype)
    reassemble_heads(g, out, n, layout)
    full = g.permute(1, 0, 2, 3, 4).reshape(B, n * Hs, S, D)
    ref = full.permute(0, 2, 1, 3) if layout == "bshd" else full
    assert torch.equal(out, ref)


ROPE_CASES = [(2, 255, 128), (1, 384, 128), (3, 128, 64), (2, 300, 64), (1, 97, 32)]


def _rope_oracle(q0, k0, v, do, scale, causal, base, dtype):
    """Rotate q, k (stored at the I/O precision), attention, rotate dq, dk back."""
    qr, kr = ora.rope_fwd(q0, base), ora.rope_fwd(k0, base)
    if dtype == torch.bfloat16:
        qr, kr = ora.round_bf16(qr), ora.round_bf16(kr)
    rdq, rdk, rdv = ora.attn_bwd(qr, kr, v, do, scale, causal)
    return ora.rope_bwd(rdq, base), ora.rope_bwd(rdk, base), rdv


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("BH,S,D", ROPE_CASES)
def test_fused_rope_backward_matches_oracle(BH, S, D, causal, dtype):
    """hx_attn_bwd_rope_strided: gradients with respect to q, k before the rotation."""
    base = 10000.0
    seed = 7000 + BH * 100 + S + D
    q0, k0, v, do = (_host((BH, S, D), seed + i, dtype) for i in range(4))
    scale = 1.0 / math.sqrt(D)
    ctx = hx.context()
    expect = "tcgen05" if D in (64, 128) else "simt"  # f32 there: bf16 hi/lo operand planes
    qd, kd = hx.rope_forward(_dev(q0, dtype), base), hx.rope_forward(_dev(k0, dtype), base)
    vd, dod = _dev(v, dtype), _dev(do, dtype)
    o, lse = hx.attn_forward(qd, kd, vd, scale, causal)
    dq, dk, dv = hx.attn_backward(qd, kd, vd, o, lse, dod, scale, causal, rope_base=base)
    assert ctx.last_path == expect
    torch.cuda.synchronize()
    rdq, rdk, rdv = _rope_oracle(q0, k0, v, do, scale, causal, base, dtype)
    _check("dQ", dq, rdq, dtype)
    _check("dK", dk, rdk, dtype)
    _check("dV", dv, rdv, dtype)
    # the fused rotation agrees with the separate rope_backward pass
    g = hx.attn_backward(qd, kd, vd, o, lse, dod, scale, causal)
    sep = (hx.rope_backward(g[0], base), hx.rope_backward(g[1], base))
    for fused, ref in zip((dq, dk), sep):
        a, b = fused.float().cpu().numpy(), ref.float().cpu().numpy()
        assert (np.abs(a - b) <= 2 * _bf16_tol(b, 1e-3 if dtype == torch.float32 else 1e-2)).all()


def test_autograd_node_with_rope():
    """flash_attention(..., rope_base): rotation, attention and the fused backward."""
    BH, S, D, base = 2, 200, 128, 500000.0
    q0, k0, v, do = (_host((BH, S, D), 900 + i, torch.bfloat16) for i in range(4))
    scale = 1.0 / math.sqrt(D)
    qd, kd, vd = (_dev(a, torch.bfloat16).requires_grad_() for a in (q0, k0, v))
    o = hx.flash_attention(qd, kd, vd, scale, causal=True, rope_base=base)
    o.backward(_dev(do, torch.bfloat16))
    rdq, rdk, rdv = _rope_oracle(q0, k0, v, do, scale, True, base, torch.bfloat16)
    _check("dQ", qd.grad, rdq, torch.bfloat16)
    _check("dK", kd.grad, rdk, torch.bfloat16)
    _check("dV", vd.grad, rdv, torch.bfloat16)


def _sampled_full_size(B, H, S, D, causal, rope_base=None, samples=((0, 0),)):
    """Full-size run on the GPU; the oracle on whole sampled (b, h) slices
    (every query row, O, dQ, dK and dV), and gradient identities on every head.

    The oracle is the row-block restatement (oracle.attn_rows: the plain
    oracle's results bit for bit, without S x S buffers). With `rope_base`
    the GPU rotates Q and K (hx.rope_forward) and folds the inverse rotation
    into dQ and dK (attn_backward(..., rope_base)), as the benchmark step does;
    the oracle rotates the same unrotated inputs with its own RoPE
    (src/kernels/rope.rs:5-44), rounds them to bf16 as the GPU stores them,
    and rotates its dQ, dK back (rope.rs:46-82). Returns the max-abs error
    of each checked tensor."""
    torch.manual_seed(0)
    g = torch.Generator(device="cuda").manual_seed(1234)
    q0, k0, v, do = (torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16)
                     for _ in range(4))
    q, k = q0, k0
    if rope_base is not None:
        q = hx.rope_forward(q0, rope_base)
        k = hx.rope_forward(k0, rope_base)
    scale = 1.0 / math.sqrt(D)
    o, lse = hx.attn_forward(q, k, v, scale, causal)
    dq, dk, dv = hx.attn_backward(q, k, v, o, lse, do, scale, causal, rope_base=rope_base)
    torch.cuda.synchronize()
    # identities over every head: sum_j dK_j = 0 (for K as the attention sees
    # it, so not after the inverse rotation), sum_j dV_j = sum_i dO_i
    if rope_base is None:
        dks, dk_l1 = dk.float().sum(2), dk.float().abs().sum(2)
        assert (dks.abs() <= 0.02 * dk_l1 + 1e-3).all(), (dks.abs() / dk_l1).max().item()
    dvs, dos = dv.float().sum(2), do.float().sum(2)
    dv_l1 = dv.float().abs().sum(2)
    assert ((dvs - dos).abs() <= 0.02 * dv_l1 + 1e-2).all(), ((dvs - dos).abs() / dv_l1).max().item()
    errs = {}
    for (b, h) in samples:
        sl = [t[b, h].float().cpu().numpy()[None] for t in (q0, k0, v, do)]
        if rope_base is not None:
            qr, kr = ora.rope_fwd(sl[0], rope_base), ora.rope_fwd(sl[1], rope_base)
            errs[f"RoPE(Q)[{b},{h}]"] = _check(f"RoPE(Q)[{b},{h}]", q[b, h], qr[0], torch.bfloat16)
            errs[f"RoPE(K)[{b},{h}]"] = _check(f"RoPE(K)[{b},{h}]", k[b, h], kr[0], torch.bfloat16)
            sl[0], sl[1] = ora.round_bf16(qr), ora.round_bf16(kr)
        ro, rlse, rdq, rdk, rdv = ora.attn_rows(*sl, scale, causal)
        if rope_base is not None:
            rdq, rdk = ora.rope_bwd(rdq, rope_base), ora.rope_bwd(rdk, rope_base)
        errs[f"O[{b},{h}]"] = _check(f"O[{b},{h}]", o[b, h], ro[0], torch.bfloat16)
        lse_bh = lse.view(B, H, S)[b, h].cpu().numpy()
        errs[f"LSE[{b},{h}]"] = float(np.max(np.abs(lse_bh - rlse[0])))
        assert errs[f"LSE[{b},{h}]"] < 1e-3
        for name, got, ref in zip(("dQ", "dK", "dV"), (dq, dk, dv), (rdq, rdk, rdv)):
            errs[f"{name}[{b},{h}]"] = _check(f"{name}[{b},{h}]", got[b, h], ref[0], torch.bfloat16)
    print(f"max-abs errors B{B} H{H} S{S} D{D} {'causal' if causal else 'full'}"
          f"{'' if rope_base is None else f' rope {rope_base:g}'}: "
          + ", ".join(f"{k}={v:.3g}" for k, v in errs.items()))
    return errs


def test_standalone_op_b8_h16_s2048_d64_causal():
    _sampled_full_size(8, 16, 2048, 64, True, samples=((0, 0), (3, 9), (7, 15)))


def test_llama_layer_b4_h32_s8192_d128_causal_rope():
    """The benchmark step's configuration: RoPE theta 500000 on the GPU against
    the oracle's RoPE at every position of the slice (angles up to 8191 rad),
    then attention, then the fused inverse rotation, on three whole slices."""
    _sampled_full_size(4, 32, 8192, 128, True, rope_base=500000.0, samples=((0, 0), (1, 17), (3, 31)))


def test_long_context_b1_h64_s32768_d128_causal():
    """The long-context configuration at full size (64 heads x 32768): the
    gradient identities on every head, and O, dQ, dK, dV of two whole heads
    (all 32768 query rows) against the oracle."""
    _sampled_full_size(1, 64, 32768, 128, True, samples=((0, 0), (0, 63)))


def test_full_mask_long_sequences():
    """Non-causal at full length on the tcgen05 path, both head dims (every key
    tile of every query tile, no masked tiles skipped)."""
    _sampled_full_size(1, 4, 8192, 128, False, samples=((0, 3),))
    _sampled_full_size(2, 4, 4096, 64, False, samples=((1, 0),))


def test_ragged_lengths_tcgen05():
    """Sequence lengths that leave partial K/V and query tiles at the end."""
    for S, D in ((1000, 128), (2049, 64), (1537, 128)):
        _sampled_full_size(1, 2, S, D, True, samples=((0, 1),))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("shape", [(0, 64, 64), (3, 0, 128), (0, 4, 16, 64), (2, 0, 16, 64)])
def test_empty_inputs_give_empty_outputs(dtype, shape):
    """An empty batch, head count or sequence is a no-op: empty outputs and
    gradients, no error (the attention and RoPE entry points return HX_OK)."""
    q, k, v = (torch.zeros(shape, device="cuda", dtype=dtype).requires_grad_() for _ in range(3))
    o = hx.flash_attention(q, k, v, 0.125, causal=True, rope_base=10000.0)
    assert o.shape == q.shape and o.numel() == 0
    o.backward(torch.zeros_like(o))
    assert all(t.grad is not None and t.grad.shape == q.shape for t in (q, k, v))
    ws = ctypes.c_uint64(1)
    N.check(N.lib().hx_attn_bwd_workspace_size(N.HX_BF16, ctypes.byref(hx.attention._shape_of(q.detach())),
                                               ctypes.byref(ws)))
    assert ws.value == 0
