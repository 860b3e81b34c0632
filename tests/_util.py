"""Shared helpers of the test-suite (fixture loading, owners, layout conversion)."""
import os

import numpy as np
import torch

from conftest import GOLDEN


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def make_owner(channels, li, le, lo, weight=None):
    from ictc_o3.basis.ictd_irreps import EdgeWeightedPathPreservingTensorProduct, operator_paths
    owner = EdgeWeightedPathPreservingTensorProduct(
        channels, max(li, le, lo), allowed_paths=operator_paths(li, le, lo))
    with torch.no_grad():
        if weight is None:
            owner.weight.fill_(1.0)
        else:
            owner.weight.copy_(torch.as_tensor(weight))
    owner.weight.requires_grad_(False)
    return owner


def mul_ir_to_ir_mul(packed, channels, degrees):
    """Re-layout a packed [rows, C * sum(2l+1)] tensor whose degree blocks are
    [C][2l+1] into [2l+1][C] blocks; ``degrees`` lists the block degrees."""
    parts, off = [], 0
    rows = packed.shape[0]
    for l in degrees:
        w = channels * (2 * l + 1)
        parts.append(packed[:, off:off + w].reshape(rows, channels, 2 * l + 1).transpose(1, 2).reshape(rows, w))
        off += w
    return torch.cat(parts, 1) if parts else packed


def ir_mul_to_mul_ir(packed, channels, degrees):
    parts, off = [], 0
    rows = packed.shape[0]
    for l in degrees:
        w = channels * (2 * l + 1)
        parts.append(packed[:, off:off + w].reshape(rows, 2 * l + 1, channels).transpose(1, 2).reshape(rows, w))
        off += w
    return torch.cat(parts, 1) if parts else packed


def output_degrees(owner):
    """Degree of each (path block) of the packed output, in output order."""
    degrees = []
    for l in range(owner.lmax + 1):
        degrees += [l] * int(owner.path_counts_by_l.get(l, 0))
    return degrees


def rel_err(a, b):
    a = torch.as_tensor(a, dtype=torch.float64).cpu()
    b = torch.as_tensor(b, dtype=torch.float64).cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def assert_close(actual, expected, rel, atol_scale=None, what=""):
    """FP32 parity check against an FP64 reference.

    * relative L2 error <= rel (1e-5 for TP outputs, 1e-4 for gradients);
    * componentwise |a - b| <= 1e-4 |b| + 2e-5 * max(1, rms(b)), the reference's
      componentwise tolerances (docs/USAGE.md:889-891) with atol scaled by the RMS of
      the quantity, since an FP32 component carries eps * sum|terms|, not eps * |b|.
    ``atol_scale`` is accepted for call-site compatibility; None disables the
    componentwise part.
    """
    a = torch.as_tensor(actual, dtype=torch.float64).cpu()
    b = torch.as_tensor(expected, dtype=torch.float64).cpu()
    assert a.shape == b.shape, f"{what}: shape {tuple(a.shape)} != {tuple(b.shape)}"
    assert torch.isfinite(a).all(), f"{what}: non-finite values"
    err = rel_err(a, b)
    assert err <= rel, f"{what}: relative L2 error {err:.3e} > {rel:.1e}"
    if atol_scale is not None and b.numel():
        rms = float(b.pow(2).mean().sqrt())
        bound = 1e-4 * b.abs() + 2e-5 * max(1.0, rms)
        worst = float(((a - b).abs() - bound).max())
        assert worst <= 0, f"{what}: componentwise error exceeds bound by {worst:.3e}"
