"""The tcgen05 GEMM behind the bf16 Linear entry points (gemm_sm100.cu).

y = x W + b (+ residual), dx = dy W^T and dW = x^T dy (src/nn/linear.rs:54-56,
W stored [in, out]) through the C ABI, against an f32 torch product of the
same bf16 inputs. The kernel accumulates in f32 and rounds once to bf16, so
each output may differ from the f32 reference by one bf16 spacing (plus a
little for the different order of the f32 sums). Shapes cover whole tiles,
ragged M/N/K edges, both tile widths (128 and 256 columns), a residual that
aliases the output, and layouts the kernel refuses (rows that are not a
multiple of 8 elements), which must fall back to cuBLAS and still be right.
"""
import ctypes

import pytest
import torch

import haelixe_b200 as hx
from haelixe_b200 import _native as NA

pytestmark = pytest.mark.gpu

TCGEN05, CUBLAS = 2, 1


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _close(got, ref, what, slack=1.0):
    got, ref = got.float(), ref.float()
    spacing = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-20))) - 7)
    bound = slack * (spacing + 1e-3 * ref.abs().max().clamp_min(1.0))
    err = (got - ref).abs()
    assert (err <= bound).all(), f"{what}: max err {err.max().item():.4g}, worst bound {bound.min().item():.3g}"


def _data(M, K, N, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(K, N, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    b = torch.randn(N, device="cuda", generator=g).to(torch.bfloat16)
    r = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
    dy = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
    return x, w, b, r, dy


SHAPES = [(128, 64, 128), (256, 128, 256), (300, 200, 136), (1000, 512, 384), (129, 72, 264), (64, 8, 8),
          (2048, 2048, 2048), (4096, 1024, 3072)]


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_linear_forward_backward_on_tcgen05(M, K, N):
    L = NA.lib()
    ctx = hx.context(0)
    ctx.use_stream()
    x, w, b, r, dy = _data(M, K, N, M + K + N)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    NA.check(L.hx_linear_fwd(ctx.handle, NA.HX_BF16, _p(x), _p(w), _p(b), _p(y), M, K, N), ctx.handle)
    assert L.hx_last_gemm_path(ctx.handle) == TCGEN05
    xf, wf = x.float(), w.float()
    _close(y, xf @ wf + b.float(), "y")
    y2 = r.clone()  # the residual aliases the output
    NA.check(L.hx_linear_residual_fwd(ctx.handle, NA.HX_BF16, _p(x), _p(w), _p(b), _p(y2), _p(y2), M, K, N),
            ctx.handle)
    assert L.hx_last_gemm_path(ctx.handle) == TCGEN05
    _close(y2, r.float() + (xf @ wf + b.float()), "y + residual")
    dx = torch.empty_like(x)
    dw = torch.empty_like(w)
    NA.check(L.hx_linear_bwd(ctx.handle, NA.HX_BF16, _p(x), _p(w), _p(dy), _p(dx), _p(dw), None, M, K, N),
            ctx.handle)
    assert L.hx_last_gemm_path(ctx.handle) == TCGEN05
    torch.cuda.synchronize()
    _close(dx, dy.float() @ wf.t(), "dx")
    _close(dw, xf.t() @ dy.float(), "dw")


def test_tcgen05_and_cublas_agree_and_backend_switch():
    L = NA.lib()
    ctx = hx.context(0)
    ctx.use_stream()
    M, K, N_ = 512, 384, 640
    x, w, b, r, dy = _data(M, K, N_, 11)
    outs = {}
    try:
        for backend, path in ((0, TCGEN05), (1, CUBLAS)):
            NA.check(L.hx_set_gemm_backend(ctx.handle, backend), ctx.handle)
            y = torch.empty(M, N_, device="cuda", dtype=torch.bfloat16)
            NA.check(L.hx_linear_fwd(ctx.handle, NA.HX_BF16, _p(x), _p(w), _p(b), _p(y), M, K, N_), ctx.handle)
            assert L.hx_last_gemm_path(ctx.handle) == path
            outs[path] = y
    finally:
        NA.check(L.hx_set_gemm_backend(ctx.handle, 0), ctx.handle)
    assert L.hx_set_gemm_backend(ctx.handle, 7) == NA.HX_ERR_INVALID
    ref = x.float() @ w.float() + b.float()
    _close(outs[TCGEN05], ref, "tcgen05")
    # cuBLAS adds the bias rows as a beta = 1 operand: its rounding differs, so
    # it is held to twice the bound
    _close(outs[CUBLAS], ref, "cuBLAS", slack=2.0)


def test_layouts_the_kernel_refuses_fall_back_to_cublas():
    L = NA.lib()
    ctx = hx.context(0)
    ctx.use_stream()
    M, K, N_ = 70, 36, 13  # rows of 36 and 13 elements: not 16-byte multiples
    x, w, b, r, dy = _data(M, K, N_, 5)
    y = torch.empty(M, N_, device="cuda", dtype=torch.bfloat16)
    NA.check(L.hx_linear_fwd(ctx.handle, NA.HX_BF16, _p(x), _p(w), _p(b), _p(y), M, K, N_), ctx.handle)
    assert L.hx_last_gemm_path(ctx.handle) == CUBLAS
    _close(y, x.float() @ w.float() + b.float(), "y")


@pytest.mark.parametrize("tile", [2, 3, 4], ids=["128x128", "128x256", "256x256"])
@pytest.mark.parametrize("M,K,N", [(300, 200, 136), (1000, 512, 384), (520, 64, 264), (2048, 1024, 2048)])
def test_every_tile_shape(M, K, N, tile):
    """Each tile configuration (forced with hx_set_gemm_backend) on ragged and whole shapes."""
    L = NA.lib()
    ctx = hx.context(0)
    ctx.use_stream()
    x, w, b, r, dy = _data(M, K, N, 3 * M + K + N + tile)
    try:
        NA.check(L.hx_set_gemm_backend(ctx.handle, tile), ctx.handle)
        y = r.clone()
        NA.check(L.hx_linear_residual_fwd(ctx.handle, NA.HX_BF16, _p(x), _p(w), _p(b), _p(y), _p(y), M, K, N),
                 ctx.handle)
        assert L.hx_last_gemm_path(ctx.handle) == TCGEN05
        dx, dw = torch.empty_like(x), torch.empty_like(w)
        NA.check(L.hx_linear_bwd(ctx.handle, NA.HX_BF16, _p(x), _p(w), _p(dy), _p(dx), _p(dw), None, M, K, N),
                 ctx.handle)
    finally:
        NA.check(L.hx_set_gemm_backend(ctx.handle, 0), ctx.handle)
    torch.cuda.synchronize()
    xf, wf = x.float(), w.float()
    _close(y, r.float() + (xf @ wf + b.float()), "y + residual")
    _close(dx, dy.float() @ wf.t(), "dx")
    _close(dw, xf.t() @ dy.float(), "dw")


def test_gemm_from_a_thread_without_a_current_context():
    """The autograd engine runs backward ops on its own threads: a Linear GEMM
    whose thread has made no CUDA runtime call yet must still encode its
    tensor maps (the entry point makes the device's context current)."""
    import threading
    L = NA.lib()
    ctx = hx.context(0)
    M, K, N_ = 512, 1024, 640
    x, w, b, r, dy = _data(M, K, N_, 23)
    y = torch.empty(M, N_, device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    out = {}

    def run():
        out["rc"] = L.hx_linear_fwd(ctx.handle, NA.HX_BF16, _p(x), _p(w), _p(b), _p(y), M, K, N_)
        out["path"] = L.hx_last_gemm_path(ctx.handle)
        out["err"] = NA.last_error(ctx.handle) if out["rc"] else ""

    t = threading.Thread(target=run)
    t.start()
    t.join(timeout=60)
    assert out.get("rc") == NA.HX_OK, out
    assert out["path"] == TCGEN05
    L.hx_sync(ctx.handle)
    torch.cuda.synchronize()
    _close(y, x.float() @ w.float() + b.float(), "y")
