"""The torch restatement of the edge geometry used by the differentiable (second-order)
path equals the model's radial embedding, which the reference-model fixtures pin, in
value and in first and second derivatives (CPU, FP64)."""
import pytest
import torch


@pytest.mark.parametrize("basis_norm", [False, True])
def test_edge_geometry_reference_matches_model_embedding(basis_norm):
    from ictc_o3.backends.cuda.geometry import edge_geometry_reference
    from mace_ictc.models import radial_embedding
    gen = torch.Generator().manual_seed(3)
    r_max, num_basis, p = 5.0, 8, 5
    lengths = torch.cat([torch.rand(200, generator=gen, dtype=torch.float64) * 6.0,
                         torch.tensor([1e-3, 0.5, r_max - 1e-9, r_max, r_max + 1e-9], dtype=torch.float64)])
    dirs = torch.nn.functional.normalize(torch.randn(lengths.numel(), 3, generator=gen, dtype=torch.float64), dim=1)
    vec = (dirs * lengths.unsqueeze(1)).requires_grad_(True)
    unit, radial, mask = edge_geometry_reference(vec, r_max, num_basis, p, basis_norm)
    r = vec.norm(dim=-1)
    want = radial_embedding(r, r_max, num_basis, p, basis_norm)
    torch.testing.assert_close(radial, want, rtol=1e-13, atol=1e-14)
    torch.testing.assert_close(unit, vec / r.unsqueeze(-1), rtol=1e-14, atol=1e-15)
    assert torch.equal(mask, (r <= r_max).double())
    assert bool((radial[lengths > r_max] == 0).all())
    G = torch.randn(radial.shape, generator=gen, dtype=torch.float64)
    (g1,) = torch.autograd.grad(radial, [vec], G, create_graph=True)
    (g2,) = torch.autograd.grad(want, [vec], G, create_graph=True)
    torch.testing.assert_close(g1, g2, rtol=1e-11, atol=1e-12)
    V = torch.randn(vec.shape, generator=gen, dtype=torch.float64)
    (h1,) = torch.autograd.grad((g1 * V).sum(), [vec], retain_graph=True)
    (h2,) = torch.autograd.grad((g2 * V).sum(), [vec])
    torch.testing.assert_close(h1, h2, rtol=1e-9, atol=1e-10)
