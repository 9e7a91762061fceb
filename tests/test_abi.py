"""The C-ABI library builds, loads without a GPU, and exports every symbol the header declares."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    txt = open(os.path.join(ROOT, "include", "flash_uma_b200.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(fuma_[a-z0-9_]+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    from flash_uma_b200 import build
    path = build.build()
    return ctypes.CDLL(path)


def test_header_declares_entry_points():
    syms = header_symbols()
    assert "fuma_gather_fwd" in syms and "fuma_rotate_scatter_bwd" in syms
    assert len(syms) >= 15


def test_library_exports_every_declared_symbol(lib):
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_header():
    from flash_uma_b200 import _native
    assert sorted(_native.exported_symbols()) == header_symbols()


def test_version_and_error_string(lib):
    lib.fuma_version.restype = ctypes.c_int
    lib.fuma_last_error.restype = ctypes.c_char_p
    assert lib.fuma_version() >= 100
    assert isinstance(lib.fuma_last_error(), bytes)


def test_invalid_arguments_rejected_before_any_launch(lib):
    """Argument validation runs on the host and returns FUMA_E_INVALID without touching
    the device (safe without a GPU)."""
    from flash_uma_b200 import _native
    _native.load()
    f = lib.fuma_gating_fwd
    f.argtypes = _native._SIGS["fuma_gating_fwd"]
    f.restype = ctypes.c_int
    rc = f(None, None, None, 10, 6, None, None, None, None)  # C=6 is not a multiple of 4
    assert rc == -1
    lib.fuma_last_error.restype = ctypes.c_char_p
    assert b"multiple of 4" in lib.fuma_last_error()
    g = lib.fuma_gather_bwd
    g.argtypes = _native._SIGS["fuma_gather_bwd"]
    g.restype = ctypes.c_int
    # a misaligned per-edge pointer is rejected (the scratch arguments are unused: NULL / 0)
    rc = g(*([16] * 3), 16, 16, 16, 16, 16, 16, 16, 16, 16, 16, 5, 7, 8, None, 0, 16, 16, 3, None)
    assert rc == -2 and b"aligned" in lib.fuma_last_error()   # FUMA_E_ALIGN


def test_ops_refuse_cpu_tensors():
    import torch
    from flash_uma_b200 import ops
    x = torch.randn(8, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.layer_norm_silu(x, torch.ones(16), torch.zeros(16))
