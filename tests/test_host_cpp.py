"""The C++ host layer (haelixe_b200/host: Device, Tensor, Tensor::to,
Tensor::flash_attention, FlashAttentionOp, the autograd walk) through its own
test program (tests/cpp/test_flash_attention.cpp), which checks it against the
CPU oracle in the style of the reference's tests/tensor_tests.rs.

CPU: the library and the program build, and the tests that need no GPU pass
(shapes, bf16 rounding, the CPU-tensor panic, the autograd walk).
GPU: all of them, including attention parity at the stated tolerances.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tests", "cpp", "build", "test_haelixe_host")


def _build():
    from haelixe_b200 import build as hb
    from oracle import oracle as ora

    hb.build()
    ora.build()
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp")], check=True)
    return BIN


def _run(*args):
    r = subprocess.run([_build(), *args], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAILED" not in r.stdout
    return r.stdout


def test_host_layer_cpu_cases():
    out = _run("--cpu-only")
    assert "5 of 5 passed" in out


def test_host_library_exports_the_mirror():
    """The library carries the C++ types over the C ABI and links the CUDA library."""
    lib = os.path.join(ROOT, "haelixe_b200", "lib", "libhaelixe_host.so")
    _build()
    syms = subprocess.run(["nm", "-DC", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    for name in ("haelixe::Tensor::flash_attention(", "haelixe::FlashAttentionOp::backward(",
                 "haelixe::Tensor::to(", "haelixe::Tensor::backward_with_seed(", "haelixe::CudaContext::get("):
        assert name in syms, name
    needed = subprocess.run(["readelf", "-d", lib], capture_output=True, text=True, check=True).stdout
    assert "libhaelixe_cuda.so" in needed


@pytest.mark.gpu
def test_host_layer_on_gpu():
    out = _run()
    assert "14 of 14 passed" in out
