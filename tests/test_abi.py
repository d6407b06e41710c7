"""CPU checks of the C ABI library: it loads, exports what include/*.h
declares, and its host-only logic (bin sizes, status codes, argument
validation, workspace sizes) behaves as specified - no GPU calls."""
import ctypes
import glob
import os
import re

import pytest

from haelixe_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(hx_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    L = N.lib()
    declared = _declared_functions()
    assert len(declared) >= 25
    missing = [n for n in sorted(declared) if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_covers_declared_functions():
    declared = _declared_functions()
    assert declared <= set(N.SIGNATURES), sorted(declared - set(N.SIGNATURES))


def test_abi_version():
    assert N.lib().hx_abi_version() == 1


@pytest.mark.parametrize("req,expected", [
    (0, 512), (1, 512), (512, 512), (513, 1024), (4000, 4096), (4010, 4096), (4096, 4096),
    (4097, 8192), ((1 << 30) + 1, 1 << 31),
])
def test_bin_size_matches_reference_rule(req, expected):
    # get_bin_size (src/gpu/arena.rs:84-91): 512-byte floor, else next power of two.
    assert N.lib().hx_bin_size(req) == expected


def test_status_strings():
    L = N.lib()
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert L.hx_status_string(code)
    assert L.hx_status_string(-99) == b"unknown status"


def test_null_context_is_rejected_without_device_work():
    L = N.lib()
    shp = N.AttnShape(1, 1, 16, 64, 1024, 1024, 64)
    assert L.hx_attn_fwd_strided(None, N.HX_BF16, ctypes.byref(shp), None, None, None, None,
                                 None, 1.0, 0) == N.HX_ERR_INVALID
    assert L.hx_sync(None) == N.HX_ERR_INVALID
    assert L.hx_alloc(None, 16, ctypes.byref(ctypes.c_void_p())) == N.HX_ERR_INVALID
    assert L.hx_free(None, None) == N.HX_ERR_INVALID


def test_workspace_size():
    L = N.lib()
    out = ctypes.c_uint64()
    shp = N.AttnShape(2, 3, 100, 48, 3 * 100 * 48, 100 * 48, 48)
    assert L.hx_attn_bwd_workspace_size(N.HX_F32, ctypes.byref(shp), ctypes.byref(out)) == 0
    assert out.value >= 2 * 3 * 100 * 4 and out.value % 256 == 0
    bad = N.AttnShape(2, 3, 100, 0, 0, 0, 0)
    assert L.hx_attn_bwd_workspace_size(N.HX_F32, ctypes.byref(bad), ctypes.byref(out)) == N.HX_ERR_INVALID


def test_workspace_size_covers_the_f32_split_path():
    """f32 at head_dim 64/128 runs on f16 hi/lo planes: the backward workspace
    holds a 256-byte statistics block, the hi and lo planes of Q, K, V and dO
    (2 bytes per element each, 256-byte aligned) and the lse / delta tables
    over S padded to 128."""
    L = N.lib()
    out = ctypes.c_uint64()

    def a256(x):
        return (x + 255) // 256 * 256

    for B, H, S, D in ((2, 3, 100, 64), (1, 4, 1000, 128)):
        shp = N.AttnShape(B, H, S, D, H * S * D, S * D, D)
        assert L.hx_attn_bwd_workspace_size(N.HX_F32, ctypes.byref(shp), ctypes.byref(out)) == 0
        s_pad = (S + 127) // 128 * 128
        need = 256 + 8 * a256(B * H * S * D * 2) + 2 * a256(B * H * s_pad * 4)
        assert out.value >= need, (out.value, need)


def test_rust_binding_declares_every_entry_point():
    """The Rust `extern "C"` block of the integration guide binds every function the header declares."""
    import re

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    header = open(os.path.join(root, "include", "haelixe_cuda.h")).read()
    declared = set(re.findall(r"^\s*(?:int|uint64_t|const char\*|void\*)\s+(hx_\w+)\s*\(", header, re.M))
    binding = open(os.path.join(root, "INTEGRATION.md")).read()
    bound = set(re.findall(r"pub fn (hx_\w+)\(", binding))
    assert declared and not (declared - bound), sorted(declared - bound)
