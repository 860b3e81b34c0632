"""Torch restatements used by the differentiable (second-order) paths: the edge geometry
and the radial network equal the model formulas the reference-model fixtures pin, in
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


def test_radial_reference_matches_model_network():
    """The radial network's torch restatement (second-order path) is the model's ``fc``
    (Linear, normalised SiLU x 3, Linear; ``pure_cartesian_ictd_fix.py:1545-1553``)."""
    from ictc_o3.backends.cuda.radial import mlp_reference
    from mace_ictc.models import InteractionBlock
    torch.manual_seed(2)
    block = InteractionBlock(channels=8, lmax=2, input_lmax=2, num_elements=3, num_basis=8,
                             avg_num_neighbors=5.0, use_self_connection=True, sc_lmax=2).double()
    linears = [m for m in block.fc if isinstance(m, torch.nn.Linear)]
    feats = torch.randn(50, 8, dtype=torch.float64, requires_grad=True)
    want = block.fc(feats)
    got = mlp_reference(feats, [m.weight for m in linears])
    torch.testing.assert_close(got, want, rtol=1e-13, atol=1e-14)
    G = torch.randn_like(want)
    (g1,) = torch.autograd.grad(got, [feats], G, create_graph=True)
    (g2,) = torch.autograd.grad(want, [feats], G, create_graph=True)
    torch.testing.assert_close(g1, g2, rtol=1e-12, atol=1e-13)
    (h1,) = torch.autograd.grad(g1.sum(), [feats])
    (h2,) = torch.autograd.grad(g2.sum(), [feats])
    torch.testing.assert_close(h1, h2, rtol=1e-11, atol=1e-12)
