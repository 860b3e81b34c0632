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


def _sw128(rows, r, k):
    """Byte offset of fp32 element (r, k) in a K-major tile with the 128-byte swizzle."""
    atom, kk = divmod(k, 32)
    return atom * rows * 128 + r * 128 + (((kk // 4) ^ (r % 8)) * 16) + (kk % 4) * 4


def test_radial_weight_image_round_trips():
    """ictc_radial_pack (host): every weight equals hi + lo at its swizzled position,
    hi is a TF32 value, and the transposed copies hold the transposes."""
    import numpy as np
    import torch
    from ictc_o3.backends.cuda import radial
    torch.manual_seed(0)
    F, H, G = 6, 64, 192
    ws = [torch.randn(H, F), torch.randn(H, H), torch.randn(H, H), torch.randn(G, H)]
    img = radial.pack_image(ws).numpy()
    assert img.size == _native_size(F, H, G)

    def read(off):
        return np.frombuffer(img[off:off + 4].tobytes(), dtype=np.float32)[0]

    def check(base, rows, value, n, k):
        hi = read(base + _sw128(rows, n, k))
        lo = read(base + 2 * rows * 128 + _sw128(rows, n, k))
        assert np.frombuffer(np.float32(hi).tobytes(), np.uint32)[0] & 0x1FFF == 0
        assert abs((np.float64(hi) + np.float64(lo)) - float(value)) <= 1e-7 * max(1.0, abs(float(value)))

    w1, w2, w3, w4 = (w.numpy() for w in ws)
    for n in range(0, H, 7):
        for k in range(F):
            hi, lo = read(_sw128(H, n, k)), read(_sw128(H, n, 8 + k))
            assert abs(float(hi) + float(lo) - float(w1[n, k])) <= 1e-7 * max(1.0, abs(float(w1[n, k])))
        for k in range(0, H, 5):
            check(8192, H, w2[n, k], n, k)
            check(8192 + 32768, H, w3[n, k], n, k)
            check(8192 + 2 * 32768, H, w3[k, n], n, k)
            check(8192 + 3 * 32768, H, w2[k, n], n, k)
    for n in range(F):
        for k in range(0, H, 3):
            check(8192 + 4 * 32768, 16, w1[k, n], n, k)
    w4_base = 8192 + 4 * 32768 + 8192
    for c in range(G // 64):                    # forward chunks of 64 rows, 32 KB each
        for n in range(0, 64, 5):
            for k in range(0, H, 9):
                check(w4_base + c * 32768, 64, w4[64 * c + n, k], n, k)
    w4t_base = w4_base + G * 512
    for c in range(G // 32):
        for n in range(0, H, 13):
            for k in range(0, 32, 7):
                hi = read(w4t_base + c * 16384 + _sw128(H, n, k))
                lo = read(w4t_base + c * 16384 + 8192 + _sw128(H, n, k))
                want = float(w4[32 * c + k, n])
                assert abs(float(hi) + float(lo) - want) <= 1e-7 * max(1.0, abs(want))


def _native_size(F, H, G):
    from ictc_o3.backends.cuda import _native
    return int(_native.library().ictc_radial_image_bytes(F, H, G))


def test_radial_rejects_unsupported_shapes():
    from ictc_o3.backends.cuda import _native
    lib = _native.library()
    assert lib.ictc_radial_image_bytes(9, 64, 192) == -1
    assert lib.ictc_radial_image_bytes(8, 32, 192) == -1
    assert lib.ictc_radial_image_bytes(8, 64, 100) == -1
    assert lib.ictc_radial_image_bytes(8, 64, 96) == -1
    assert lib.ictc_radial_forward(None, None, None, 10, 8, 64, 192, None, None) == -1


def test_radial_plan_repacks_only_when_weights_change():
    """RadialPlan keeps one packed image per set of weight tensors: the same tensors
    reuse it; an in-place update, a replaced tensor or padded widths repack (host only)."""
    import torch
    from ictc_o3.backends.cuda import radial
    torch.manual_seed(1)
    layers = [torch.nn.Linear(8, 64, bias=False), torch.nn.Linear(64, 64, bias=False),
              torch.nn.Linear(64, 64, bias=False), torch.nn.Linear(64, 88, bias=False)]
    weights = [m.weight for m in layers]
    plan = radial.RadialPlan()
    image, status = plan.get(weights)
    assert plan.get([m.weight for m in layers])[0] is image              # same tensors: reused
    with torch.no_grad():
        layers[2].weight.mul_(0.5)                                        # in-place update
    second, _ = plan.get(weights)
    assert second is not image and not torch.equal(second, image)
    layers[1].weight = torch.nn.Parameter(layers[1].weight.detach().clone())   # replaced tensor
    third, _ = plan.get([m.weight for m in layers])
    assert third is not second and torch.equal(third, second)
    assert radial.padded_gates(88) == 128 and third.numel() == _native_size(8, 64, 128)
