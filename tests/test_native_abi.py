"""The C-ABI library loads and exports every symbol include/ictc_cuda.h declares (CPU only)."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "ictc_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(ictc_[a-z_0-9]+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from ictc_o3.backends.cuda import _native
    lib = _native.library()
    names = declared_functions()
    assert "ictc_tp_forward" in names and "ictc_direction_harmonics" in names
    for name in names:
        assert hasattr(lib, name), f"{name} missing from libictc_cuda.so"
    assert set(names) == set(_native.exported_symbols()), "binding table and header disagree"
    assert lib.ictc_version() == _native.ABI_VERSION


def test_header_abi_version_matches_binding():
    from ictc_o3.backends.cuda import _native
    version = int(re.search(r"#define ICTC_ABI_VERSION (\d+)", open(HEADER).read()).group(1))
    assert version == _native.ABI_VERSION


def test_host_argument_validation_without_gpu():
    """Entry points reject bad arguments before touching the device."""
    from ictc_o3.backends.cuda import _native
    lib = _native.library()
    assert lib.ictc_tp_forward(None, None, None, None, None, None, 4, None) == -1
    assert "invalid" in lib.ictc_last_error().decode()
    assert lib.ictc_direction_harmonics(None, None, None, None, None, None, 4, 2, 0, None) == -1
    assert lib.ictc_direction_harmonics(None, None, None, None, None, None, 0, 9, 0, None) == -2
    assert lib.ictc_harmonics_table_size(3) == 3 * 3 + 6 * 5 + 10 * 7
    handle = ctypes.c_void_p()
    assert lib.ictc_tp_plan_create(64, 2, 2, 2, 5, 0, None, None, 0, 0, 0, ctypes.byref(handle)) == -1


def test_operators_reject_host_tensors():
    import torch
    from ictc_o3.operators import EdgeTensorProduct, direction_harmonics
    with pytest.raises(ValueError):
        EdgeTensorProduct.create(channels=64, input_lmax=2, edge_lmax=2, device="cpu")
    with pytest.raises(ValueError):
        direction_harmonics(torch.zeros(4, 3), 2)
