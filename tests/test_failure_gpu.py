"""Failure detection and memory-safety checks on the GPU, none of which faults,
traps or hangs the device.

* The bounded-wait path every tcgen05 kernel relies on: hx_selftest_wait_timeout
  runs one CTA whose mbarrier wait never completes; after the 2 s limit it
  records the expiry and exits, hx_sync returns HX_ERR_TIMEOUT naming the wait
  site, and the context keeps working.
* Guard bands: every output is a view into a larger buffer filled with a
  canary value; after the kernels run, the bands around it are unchanged (no
  out-of-bounds writes on the tcgen05, SIMT, fused-RoPE and MHA-op paths).
"""
import math
import time

import pytest
import torch

import haelixe_b200 as hx
from haelixe_b200 import _native as N

pytestmark = pytest.mark.gpu

PAD = 4096  # elements of guard band on each side (16-byte multiples for bf16 and f32)
CANARY = -12345.0


def test_bounded_wait_times_out_and_context_recovers():
    ctx = hx.context()
    ctx.use_stream()
    lib = N.lib()
    torch.cuda.synchronize()
    N.check(lib.hx_selftest_wait_timeout(ctx.handle), ctx.handle)
    t0 = time.time()
    st = lib.hx_sync(ctx.handle)
    waited = time.time() - t0
    assert st == N.HX_ERR_TIMEOUT
    assert "site 99" in N.last_error(ctx.handle)
    assert 1.0 < waited < 60.0
    # the status word was cleared and the context and device still work
    assert lib.hx_sync(ctx.handle) == 0
    q, k, v = (torch.randn(1, 2, 200, 128, device="cuda").to(torch.bfloat16) for _ in range(3))
    o, lse = hx.attn_forward(q, k, v, 0.088, True)
    ctx.sync()
    assert ctx.last_path == "tcgen05" and torch.isfinite(o.float()).all()


def _guarded(shape, dtype):
    n = math.prod(shape)
    buf = torch.full((n + 2 * PAD,), CANARY, dtype=dtype, device="cuda")
    return buf, buf[PAD:PAD + n].view(shape)


def _bands_intact(buf, n):
    return bool((buf[:PAD] == CANARY).all() and (buf[PAD + n:] == CANARY).all())


@pytest.mark.parametrize("dtype,BH,S,D,causal,rope", [
    (torch.bfloat16, 2, 300, 128, True, None),
    (torch.bfloat16, 3, 129, 64, False, None),
    (torch.bfloat16, 2, 257, 128, True, 10000.0),
    (torch.float32, 2, 65, 80, True, None),
    # f32 on the tensor cores (f16 hi/lo planes); S=2200 at D=128 adds the
    # dV/dK accumulation into the outputs in two segments
    (torch.float32, 2, 300, 128, True, None),
    (torch.float32, 3, 129, 64, True, None),
    (torch.float32, 2, 2200, 128, False, 10000.0),
])
def test_kernels_write_only_their_outputs(dtype, BH, S, D, causal, rope):
    shape = (BH, S, D)
    q, k, v, do = (torch.randn(shape, device="cuda").to(dtype) for _ in range(4))
    (ob, o), (lb, lse) = _guarded(shape, dtype), _guarded((BH * S,), torch.float32)
    o, lse = hx.attn_forward(q, k, v, D ** -0.5, causal, out=o, lse=lse)
    grads = [_guarded(shape, dtype) for _ in range(3)]
    hx.attn_backward(q, k, v, o, lse, do, D ** -0.5, causal, dq=grads[0][1], dk=grads[1][1],
                     dv=grads[2][1], rope_base=rope)
    torch.cuda.synchronize()
    n = BH * S * D
    assert _bands_intact(ob, n) and _bands_intact(lb, BH * S)
    for buf, _ in grads:
        assert _bands_intact(buf, n)
    for t in (o, grads[0][1], grads[1][1], grads[2][1]):
        assert torch.isfinite(t.float()).all()


def test_mha_ops_write_only_their_outputs():
    rows, fin, fout = 77, 96, 136
    x = torch.randn(rows, fin, device="cuda")
    w = torch.randn(fin, fout, device="cuda") * 0.1
    b = torch.randn(fout, device="cuda")
    ctx = hx.context()
    ctx.use_stream()
    lib = N.lib()
    yb, y = _guarded((rows, fout), torch.float32)
    N.check(lib.hx_linear_fwd(ctx.handle, N.HX_F32, x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(),
                              rows, fin, fout), ctx.handle)
    dy = torch.randn(rows, fout, device="cuda")
    (dxb, dx), (dwb, dw), (dbb, db) = (_guarded((rows, fin), torch.float32), _guarded((fin, fout), torch.float32),
                                       _guarded((fout,), torch.float32))
    N.check(lib.hx_linear_bwd(ctx.handle, N.HX_F32, x.data_ptr(), w.data_ptr(), dy.data_ptr(), dx.data_ptr(),
                              dw.data_ptr(), db.data_ptr(), rows, fin, fout), ctx.handle)
    nw = torch.rand(fin, device="cuda") + 0.5
    (nb, nrm), (gdb, gdx), (gwb, gdw) = (_guarded((rows, fin), torch.float32), _guarded((rows, fin), torch.float32),
                                         _guarded((fin,), torch.float32))
    N.check(lib.hx_rmsnorm_fwd(ctx.handle, N.HX_F32, x.data_ptr(), nw.data_ptr(), nrm.data_ptr(), rows, fin,
                               1e-5), ctx.handle)
    N.check(lib.hx_rmsnorm_bwd(ctx.handle, N.HX_F32, dx.data_ptr(), x.data_ptr(), nw.data_ptr(), gdx.data_ptr(),
                               gdw.data_ptr(), rows, fin, 1e-5), ctx.handle)
    torch.cuda.synchronize()
    for buf, n in ((yb, rows * fout), (dxb, rows * fin), (dwb, fin * fout), (dbb, fout), (nb, rows * fin),
                   (gdb, rows * fin), (gwb, fin)):
        assert _bands_intact(buf, n)
    assert torch.allclose(y, x @ w + b, atol=1e-4, rtol=1e-4)


def test_arena_limit_reports_oom_and_recovers():
    """Allocator exhaustion simulated with a capped arena: the call fails with
    HX_ERR_OOM (HxError in Python) instead of growing the pool, and works again
    once the cap is lifted."""
    import ctypes
    ctx = hx.context()
    lib = N.lib()
    q, k, v, do = (torch.randn(1, 2, 4096, 128, device="cuda").to(torch.bfloat16) for _ in range(4))
    o, lse = hx.attn_forward(q, k, v, 0.088, True)
    torch.cuda.synchronize()
    ctx.arena_reset()
    ctx.set_arena_limit(1 << 20)
    try:
        p = ctypes.c_void_p()
        assert lib.hx_alloc(ctx.handle, 2 << 20, ctypes.byref(p)) == N.HX_ERR_OOM
        assert "arena limit" in N.last_error(ctx.handle)
        with pytest.raises(N.HxError) as e:  # the backward's workspace (> 4 MB) comes from the arena
            hx.attn_backward(q, k, v, o, lse, do, 0.088, True)
        assert e.value.status == N.HX_ERR_OOM
    finally:
        ctx.set_arena_limit(0)
    dq, dk, dv = hx.attn_backward(q, k, v, o, lse, do, 0.088, True)
    ctx.sync()
    assert torch.isfinite(dq.float()).all()
