"""Reference-named entry points of the CUDA backend against plain torch (FP64) on a GPU."""
import pytest
import torch

from _util import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
def test_channel_linear(degree, cuda_device):
    from ictc_o3.backends.cuda.linear import channel_linear
    gen = torch.Generator().manual_seed(degree)
    m = 2 * degree + 1
    x = torch.randn(2, 37, 24, m, generator=gen)
    w = torch.randn(40, 24, generator=gen) / 24 ** 0.5
    bias = torch.randn(40, generator=gen) if degree == 0 else None
    xd, wd = x.to(cuda_device).requires_grad_(True), w.to(cuda_device).requires_grad_(True)
    out = channel_linear(xd, wd, None if bias is None else bias.to(cuda_device))
    ref = torch.einsum("oi,abim->abom", w.double(), x.double())
    if bias is not None:
        ref = ref + bias.double()[:, None]
    assert_close(out.detach().cpu(), ref, 1e-5, what="channel_linear")
    g = torch.randn(out.shape, generator=gen)
    dx, dw = torch.autograd.grad(out, [xd, wd], g.to(cuda_device))
    assert_close(dx.cpu(), torch.einsum("oi,abom->abim", w.double(), g.double()), 1e-4, what="dx")
    assert_close(dw.cpu(), torch.einsum("abom,abim->oi", g.double(), x.double()), 1e-4, what="dw")


@pytest.mark.parametrize("degree", [0, 2])
def test_species_channel_linear(degree, cuda_device):
    from ictc_o3.backends.cuda.linear import species_channel_linear
    gen = torch.Generator().manual_seed(10 + degree)
    m, n, S = 2 * degree + 1, 301, 3
    x = torch.randn(n, 32, m, generator=gen)
    w = torch.randn(S, 48, 32, generator=gen) / 32 ** 0.5
    species = torch.randint(0, S, (n,), generator=gen)
    bias = torch.randn(S, 48, generator=gen) if degree == 0 else None
    out = species_channel_linear(x.to(cuda_device), w.to(cuda_device), species.to(cuda_device),
                                 None if bias is None else bias.to(cuda_device))
    ref = torch.einsum("noi,nim->nom", w.double()[species], x.double())
    if bias is not None:
        ref = ref + bias.double()[species][:, :, None]
    assert_close(out.cpu(), ref, 1e-5, what="species_channel_linear")


def test_edge_vectors(cuda_device):
    from ictc_o3.backends.cuda.geometry import edge_vectors
    gen = torch.Generator().manual_seed(3)
    n, e, b = 50, 200, 2
    pos = torch.randn(n, 3, generator=gen) * 4
    cell = torch.eye(3).expand(b, 3, 3) * 9 + 0.3 * torch.randn(b, 3, 3, generator=gen)
    batch = torch.randint(0, b, (n,), generator=gen)
    src, dst = torch.randint(0, n, (e,), generator=gen), torch.randint(0, n, (e,), generator=gen)
    shifts = torch.randint(-1, 2, (e, 3), generator=gen).float()
    got = edge_vectors(*(t.to(cuda_device) for t in (pos, cell, shifts, batch, src, dst)))
    want = pos[dst] - pos[src] + torch.einsum("ek,ekj->ej", shifts, cell[batch[src]])
    assert_close(got.cpu(), want.double(), 1e-6, what="edge vectors")
    one = edge_vectors(*(t.to(cuda_device) for t in (pos, cell[:1], shifts, torch.zeros_like(batch), src, dst)))
    assert_close(one.cpu(), (pos[dst] - pos[src] + shifts @ cell[0]).double(), 1e-6, what="single cell")


def test_radial_graph_message_equals_explicit_gates(cuda_device):
    """The reference hook: gates from the block's radial network, then the message."""
    from ictc_o3.backends.cuda.message import graph_message, radial_graph_message
    from mace_ictc.models import InteractionBlock
    torch.manual_seed(0)
    C, L, n, e = 32, 2, 64, 700
    block = InteractionBlock(channels=C, lmax=L, input_lmax=L, num_elements=3, num_basis=8, avg_num_neighbors=10.0,
                             use_self_connection=True, sc_lmax=L).to(cuda_device)
    tp = block.tp
    feats = {l: torch.randn(n, C, 2 * l + 1, device=cuda_device) for l in range(L + 1)}
    from ictc_o3.backends.cuda.geometry import direction_harmonics
    unit = torch.nn.functional.normalize(torch.randn(e, 3, device=cuda_device), dim=1)
    y = direction_harmonics(unit, L)
    harm = {l: y[:, l * l:(l + 1) ** 2].unsqueeze(1) for l in range(L + 1)}
    edge_feats = torch.rand(e, 8, device=cuda_device)
    src = torch.randint(0, n, (e,), device=cuda_device)
    dst = torch.sort(torch.randint(0, n, (e,), device=cuda_device)).values
    got = radial_graph_message(tp, feats, harm, block.fc, edge_feats, src, dst)
    gates = block.fc(edge_feats)                      # the same network in torch ops
    want = graph_message(tp, feats, harm, gates, src, dst)
    for l in want:
        assert_close(got[l].detach().cpu(), want[l].detach().double().cpu(), 1e-5, what=f"l={l}")
    not_streamed = torch.nn.Sequential(torch.nn.Linear(8, tp.num_paths * C)).to(cuda_device)
    assert radial_graph_message(tp, feats, harm, not_streamed, edge_feats, src, dst) is None


def test_runtime_energy_and_forces(cuda_device):
    """mace_ictc.runtime: create, configure, energy_and_forces (lattice shifts, cells,
    atomic numbers) equals the model's own energy and forces."""
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    from mace_ictc.runtime import check_model, configure_model, create_model, energy_and_forces
    from mace_ictc.systems import random_system
    torch.manual_seed(1)
    model = create_model(channels=32, lmax=2, cutoff=5.0, avg_num_neighbors=40.0, device=cuda_device)
    assert model.product_backend == "ictd-bridge-u"                   # as the reference's factory
    assert check_model(model)["supported"]
    info = configure_model(model)
    assert info["selected"] == "generated" and all(m._cuda_hp for m in model.modules())
    pos, species, side = random_system(2000, seed=4, device=cuda_device)
    src, dst, shift, _ = neighbor_list(pos, (side,) * 3, 5.0)
    numbers = torch.tensor([1, 6, 8], device=cuda_device)[species]
    cell = (torch.eye(3, device=cuda_device) * side).unsqueeze(0)
    result = energy_and_forces(model, pos, numbers, torch.zeros_like(species), src, dst, shift / side, cell)
    e_ref, f_ref = model.energy_and_forces(pos, species, src, dst, shift)
    assert_close(result["energy"], e_ref, 1e-5, what="energy")
    assert_close(result["forces"], f_ref, 1e-4, what="forces")
    assert result["atomic_energy"].shape == (2000,)
