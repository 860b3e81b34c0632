"""Fused edge geometry (unit vectors, Bessel x envelope embedding, cutoff mask) vs the
torch formula in FP64: outputs, the edge-vector gradient, and the second derivative
taken through the differentiable recompute."""
import pytest
import torch

from _util import assert_close

pytestmark = pytest.mark.gpu
R_MAX, BASIS, P = 5.0, 8, 5


def _vectors(device, edges=4000, seed=0):
    gen = torch.Generator().manual_seed(seed)
    v = torch.randn(edges, 3, generator=gen)
    v = v / v.norm(dim=1, keepdim=True) * (torch.rand(edges, 1, generator=gen) * 6.0 + 0.2)
    v[0] = torch.tensor([R_MAX, 0.0, 0.0])          # exactly at the cutoff
    v[1] = torch.tensor([0.0, 5.5, 0.0])            # beyond it
    v[2] = torch.tensor([1e-3, 0.0, 0.0])           # very short
    return v.to(device)


def test_edge_geometry_forward_and_gradient(cuda_device):
    from ictc_o3.backends.cuda.geometry import edge_geometry, edge_geometry_reference
    v = _vectors(cuda_device).requires_grad_(True)
    unit, radial, mask = edge_geometry(v, R_MAX, BASIS, P)
    vd = v.detach().double().cpu().requires_grad_(True)
    ru, rr, rm = edge_geometry_reference(vd, R_MAX, BASIS, P)
    assert_close(unit.detach().cpu(), ru.detach(), 1e-5, 1e-3, "unit")
    assert_close(radial.detach().cpu(), rr.detach(), 1e-5, 1e-3, "radial")
    assert torch.equal(mask.cpu(), rm.float())
    gu, gr = torch.randn_like(unit), torch.randn_like(radial)
    (dv,) = torch.autograd.grad([unit, radial], [v], [gu, gr], retain_graph=True)
    (rdv,) = torch.autograd.grad([ru, rr], [vd], [gu.double().cpu(), gr.double().cpu()], retain_graph=True)
    assert_close(dv.cpu(), rdv, 1e-4, 1e-3, "d vec")
    # Only the radial path carries a cotangent (the unit vector is unused).
    (dv2,) = torch.autograd.grad(radial, [v], gr)
    (rdv2,) = torch.autograd.grad(rr, [vd], gr.double().cpu())
    assert_close(dv2.cpu(), rdv2, 1e-4, 1e-3, "d vec (radial only)")


def test_edge_geometry_second_derivative(cuda_device):
    from ictc_o3.backends.cuda.geometry import edge_geometry, edge_geometry_reference
    v = _vectors(cuda_device, 500, 3).requires_grad_(True)
    unit, radial, _ = edge_geometry(v, R_MAX, BASIS, P)
    gu, gr = torch.randn_like(unit), torch.randn_like(radial)
    (dv,) = torch.autograd.grad([unit, radial], [v], [gu, gr], create_graph=True)
    h = torch.randn_like(dv)
    (hv,) = torch.autograd.grad((dv * h).sum(), [v])
    vd = v.detach().double().cpu().requires_grad_(True)
    ru, rr, _ = edge_geometry_reference(vd, R_MAX, BASIS, P)
    (rdv,) = torch.autograd.grad([ru, rr], [vd], [gu.double().cpu(), gr.double().cpu()], create_graph=True)
    (rhv,) = torch.autograd.grad((rdv * h.double().cpu()).sum(), [vd])
    assert_close(hv.cpu(), rhv, 1e-4, 1e-3, "second derivative")


def test_edge_geometry_empty(cuda_device):
    from ictc_o3.backends.cuda.geometry import edge_geometry
    unit, radial, mask = edge_geometry(torch.empty(0, 3, device=cuda_device), R_MAX, BASIS, P)
    assert unit.shape == (0, 3) and radial.shape == (0, BASIS) and mask.shape == (0,)
