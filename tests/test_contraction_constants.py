"""Pin the symmetric-contraction constants and its oracle to the reference (CPU only)."""
import numpy as np
import pytest
import torch

from _util import golden
from oracle import sc_oracle


def test_full_couplings_match_reference():
    from ictc_o3.basis import ictd_irreps as basis
    g = golden("full_cg_l3.npz")
    offset = 0
    for l1, l2, l3 in g["keys"]:
        mine = basis.build_full_cg_tensor_so3(int(l1), int(l2), int(l3)).reshape(-1)
        ref = g["values"][offset:offset + mine.size]
        offset += mine.size
        np.testing.assert_allclose(mine, ref, rtol=0, atol=1e-12, err_msg=str((l1, l2, l3)))
    assert offset == g["values"].size


@pytest.mark.parametrize("lmax", [1, 2, 3])
def test_contraction_u_tensors_match_reference(lmax):
    from ictc_o3.basis import ictd_irreps as basis
    g = golden("u_probes.npz")
    probes = g[f"probes_l{lmax}"]
    for t in range(lmax + 1):
        for nu in (1, 2, 3):
            u = basis.ictd_u_matrix_so3(lmax, t, nu)
            if t == 0:
                u = u[None]
            for a in range(nu):
                u = np.tensordot(u, probes[a], axes=([1], [0]))
            ref = g[f"u_l{lmax}_t{t}_nu{nu}"]
            assert u.shape == ref.shape, (lmax, t, nu)
            np.testing.assert_allclose(u, ref, rtol=1e-10, atol=1e-12, err_msg=str((lmax, t, nu)))


@pytest.mark.parametrize("name", ["contraction_c32_l2.npz", "contraction_c32_l1_t0.npz"])
def test_contraction_oracle_matches_reference(name):
    from ictc_o3.basis import ictd_irreps as basis
    g = golden(name)
    C, L, T, corr = (int(g[k]) for k in ("channels", "lmax", "target_lmax", "correlation"))
    x = torch.from_numpy(g["x"]).double()
    idx = torch.from_numpy(g["idx"])
    feats = sc_oracle.flat_to_mace(x, C, L)
    outs = []
    for t in range(T + 1):
        u = {nu: torch.from_numpy(basis.ictd_u_matrix_so3(L, t, nu)) for nu in range(1, corr + 1)}
        wmax = torch.from_numpy(g[f"w_t{t}_nu{corr}"]).double()
        ws = [torch.from_numpy(g[f"w_t{t}_nu{nu}"]).double() for nu in range(corr - 1, 0, -1)]
        outs.append(sc_oracle.contraction(u, wmax, ws, feats, idx, t))
    np.testing.assert_allclose(torch.cat(outs, -1).numpy(), g["out64"], rtol=1e-11, atol=1e-11)


def test_symmetric_table_reproduces_the_polynomial():
    """Usym evaluated on monomials equals the full U contraction (host constants of the kernel)."""
    from ictc_o3.basis import ictd_irreps as basis
    from ictc_o3.backends.cuda.contraction import monomial_rows, symmetric_table
    rng = np.random.default_rng(0)
    L, corr = 2, 3
    dim = (L + 1) ** 2
    x = rng.standard_normal(dim)
    for t in range(L + 1):
        u = {nu: basis.ictd_u_matrix_so3(L, t, nu) for nu in range(1, corr + 1)}
        sym = symmetric_table(u, t, dim, corr)
        rows = monomial_rows(dim, corr)
        mono = np.array([np.prod([x[i] for i in r]) for r in rows])
        got = np.einsum("r,rmp->mp", mono, sym)
        offset = 0
        for nu in range(corr, 0, -1):
            full = u[nu] if t else u[nu][None]
            for _ in range(nu):
                full = np.tensordot(full, x, axes=([1], [0]))
            np.testing.assert_allclose(got[:, offset:offset + full.shape[-1]], full, rtol=1e-12, atol=1e-12)
            offset += full.shape[-1]


@pytest.mark.parametrize("lmax,target,corr", [(2, 2, 3), (1, 0, 2)])
def test_second_order_polynomial_matches_oracle(lmax, target, corr):
    """The differentiable polynomial of the second-order path equals the recursion,
    and so do its first and mixed second derivatives (FP64, CPU)."""
    from ictc_o3.backends.cuda.contraction import polynomial, species_tiles
    from ictc_o3.ops.symmetric_contraction import ICTDPureUSymmetricContractionSO3
    torch.manual_seed(3)
    S, N, C = 3, 13, 4
    module = ICTDPureUSymmetricContractionSO3(num_elements=S, channels=C, lmax=lmax, target_lmax=target,
                                              correlation=corr).double()
    x = torch.randn(N, C * (lmax + 1) ** 2, dtype=torch.float64, requires_grad=True)
    idx = torch.randint(0, S, (N,))
    # the folded table T_t = Usym_t W_t in FP64 (the kernels fold it on the GPU)
    table = torch.cat([torch.matmul(c.symmetric_table(torch.device("cpu"), torch.float64).unsqueeze(0),
                                    c.stacked_weights()) for c in module.contractions], 1)
    tiles, tile_species = species_tiles(idx, S)
    out = polynomial(x, table.double(), tiles, tile_species, (C, lmax, corr, target))
    feats = sc_oracle.flat_to_mace(x, C, lmax)
    ref = torch.cat([sc_oracle.contraction({nu: torch.from_numpy(c._u64[nu]) for nu in range(1, corr + 1)},
                                           c.weights_max, list(c.weights), feats, idx, t)
                     for t, c in enumerate(module.contractions)], -1)
    assert torch.allclose(out, ref, rtol=1e-10, atol=1e-12)
    G, V = torch.randn_like(out), torch.randn_like(x)
    (dx,) = torch.autograd.grad(out, [x], G, create_graph=True)
    (rdx,) = torch.autograd.grad(ref, [x], G, create_graph=True)
    assert torch.allclose(dx, rdx, rtol=1e-10, atol=1e-12)
    (h,) = torch.autograd.grad((dx * V).sum(), [x])
    (rh,) = torch.autograd.grad((rdx * V).sum(), [x])
    assert torch.allclose(h, rh, rtol=1e-10, atol=1e-12)
