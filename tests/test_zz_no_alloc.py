"""The allocation-free backward entry point (hx_flash_attention_bwd_noalloc).

Some callers cannot let a library allocate device memory: a runtime that
reserved all of HBM for its own pool at start-up, a latency-critical loop
that cannot risk the synchronisation cudaMalloc/cudaFree can cause, or an
operator callback that must not allocate. This entry point serves them from a
fixed 64 MiB array compiled into the library. These tests call it through the
C ABI and check it against the allocating entry point (hx_flash_attention_bwd)
on the same inputs, on two calls in a row, so a workspace left over from the
previous call cannot leak into the next result; both must report the tcgen05
path, and one shape is also compared with the CPU oracle. The file is named
to be collected last.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

import haelixe_b200 as hx
from haelixe_b200 import _native as N
from oracle import oracle as ora

TCGEN05 = 2  # hx_last_path value of the tcgen05 kernels

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _within_bf16(got, ref):
    got, ref = got.float().cpu().numpy(), ref.float().cpu().numpy()
    spacing = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 1e-30))) - 7)
    bound = np.maximum(2e-2, 2 * spacing)
    return bool((np.abs(got - ref) <= bound).all()), float(np.abs(got - ref).max())


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_noalloc_backward_matches_allocating_entry_point(D, causal):
    L = N.lib()
    BH, S = 4, 1000
    ctx = hx.context(0)
    ctx.use_stream()
    g = torch.Generator(device="cuda").manual_seed(17 + D)
    q, k, v, do = (torch.randn(BH, S, D, device="cuda", generator=g).to(torch.bfloat16)
                   for _ in range(4))
    scale = 1.0 / math.sqrt(D)
    o, lse = hx.attn_forward(q, k, v, scale, causal)
    ref = [torch.empty_like(q) for _ in range(3)]
    N.check(L.hx_flash_attention_bwd(ctx.handle, N.HX_BF16, _p(q), _p(k), _p(v), _p(o), _p(do),
                                     _p(lse), *(_p(t) for t in ref), None, 0, BH, S, D,
                                     scale, int(causal)), ctx.handle)
    assert L.hx_last_path(ctx.handle) == TCGEN05
    torch.cuda.synchronize()
    for call in range(2):
        out = [torch.full_like(q, float("nan")) for _ in range(3)]
        rc = L.hx_flash_attention_bwd_noalloc(ctx.handle, N.HX_BF16, _p(q), _p(k), _p(v), _p(o),
                                              _p(do), _p(lse), *(_p(t) for t in out), BH, S, D,
                                              scale, int(causal))
        N.check(rc, ctx.handle)
        assert L.hx_last_path(ctx.handle) == TCGEN05
        N.check(L.hx_sync(ctx.handle), ctx.handle)
        torch.cuda.synchronize()
        for name, a, b in zip(("dq", "dk", "dv"), out, ref):
            ok, err = _within_bf16(a, b)
            assert ok, f"call {call}: {name} differs from hx_flash_attention_bwd by {err}"


def test_noalloc_rejects_problems_larger_than_its_scratch():
    L = N.lib()
    ctx = hx.context(0)
    t = torch.zeros(16, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(16, device="cuda", dtype=torch.float32)
    # 64 x 32768 rows x (128 + 1) floats of workspace is far beyond 64 MiB;
    # the call must refuse before touching any operand.
    rc = L.hx_flash_attention_bwd_noalloc(ctx.handle, N.HX_BF16, *([_p(t)] * 5), _p(lse),
                                          *([_p(t)] * 3), 64, 32768, 128, 0.088, 1)
    assert rc == N.HX_ERR_INVALID
    assert "64 MiB" in N.last_error(ctx.handle)


def test_noalloc_backward_matches_oracle():
    """The fixed-scratch path checked directly against the CPU oracle (max-abs 2e-2, bf16 I/O)."""
    L = N.lib()
    BH, S, D = 2, 333, 128
    ctx = hx.context(0)
    ctx.use_stream()
    rng = np.random.default_rng(5)
    host = [ora.round_bf16(rng.standard_normal((BH, S, D), dtype=np.float32)) for _ in range(4)]
    q, k, v, do = (torch.from_numpy(a).to(torch.bfloat16).cuda() for a in host)
    scale = 1.0 / math.sqrt(D)
    o, lse = hx.attn_forward(q, k, v, scale, True)
    out = [torch.full_like(q, float("nan")) for _ in range(3)]
    N.check(L.hx_flash_attention_bwd_noalloc(ctx.handle, N.HX_BF16, _p(q), _p(k), _p(v), _p(o),
                                             _p(do), _p(lse), *(_p(t) for t in out), BH, S, D,
                                             scale, 1), ctx.handle)
    assert L.hx_last_path(ctx.handle) == TCGEN05
    N.check(L.hx_sync(ctx.handle), ctx.handle)
    ref = ora.attn_bwd(*host, scale, True)
    for name, got, r in zip(("dq", "dk", "dv"), out, ref):
        err = float(np.abs(got.float().cpu().numpy() - r).max())
        assert err <= 2e-2, f"{name}: max-abs error {err} against the oracle"


def test_noalloc_rejects_bad_scale_and_forced_simt():
    L = N.lib()
    ctx = hx.context(0)
    t = torch.zeros(4 * 64 * 64, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(4 * 64, device="cuda", dtype=torch.float32)
    args = (ctx.handle, N.HX_BF16, *([_p(t)] * 5), _p(lse), *([_p(t)] * 3), 4, 64, 64)
    assert L.hx_flash_attention_bwd_noalloc(*args, float("nan"), 1) == N.HX_ERR_INVALID
    assert "scale" in N.last_error(ctx.handle)
    N.check(L.hx_set_force_simt(ctx.handle, 1), ctx.handle)
    try:
        assert L.hx_flash_attention_bwd_noalloc(*args, 0.125, 1) == N.HX_ERR_UNSUPPORTED
        assert "SIMT" in N.last_error(ctx.handle)
    finally:
        N.check(L.hx_set_force_simt(ctx.handle, 0), ctx.handle)
