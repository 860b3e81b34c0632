"""Pin the host constants and the CPU oracle to the reference's own outputs (CPU only)."""
import numpy as np
import pytest
import torch

from _util import golden, make_owner, assert_close
from oracle import tp_oracle
from oracle.tp_oracle import harmonic_tables, split_harm, split_mul_ir, pack_out

TP_CASES = ["tp_c64_l2.npz", "tp_c128_l3.npz", "tp_c32_l0e3.npz", "tp_c32_l1_nogate.npz", "tp_c64_l2_unitw.npz"]


@pytest.mark.parametrize("name", TP_CASES)
def test_cg_constants_match_reference(name):
    g = golden(name)
    owner = make_owner(int(g["channels"]), int(g["li"]), int(g["le"]), int(g["lo"]))
    assert np.array_equal(np.array(owner.paths, dtype=np.int32), g["paths"])
    assert list(owner.path_offset) == list(g["path_offset"])
    mine = np.concatenate([c.reshape(-1) for c in owner.cg_f64()])
    np.testing.assert_allclose(mine, g["cg"], rtol=0, atol=1e-13)


@pytest.mark.parametrize("name", TP_CASES)
def test_oracle_forward_matches_reference(name):
    g = golden(name)
    C, li, le = int(g["channels"]), int(g["li"]), int(g["le"])
    owner = make_owner(C, li, le, int(g["lo"]), weight=g["weight"])
    x, y = torch.from_numpy(g["x"]), torch.from_numpy(g["y"])
    gates = torch.from_numpy(g["gates"]) if "gates" in g else None
    rows = x.shape[0]
    gv = None if gates is None else gates.view(rows, owner.num_paths, C)
    out64 = pack_out(owner, tp_oracle.tp_forward(owner, split_mul_ir(x.double(), C, li), split_harm(y.double(), le),
                                                 None if gv is None else gv.double(), dtype=torch.float64))
    np.testing.assert_allclose(out64.numpy(), g["out64"], rtol=1e-12, atol=1e-12)
    out32 = pack_out(owner, tp_oracle.tp_forward(owner, split_mul_ir(x, C, li), split_harm(y, le), gv))
    assert_close(out32, g["out32"], rel=1e-6, what="fp32 oracle vs fp32 reference")


@pytest.mark.parametrize("name", TP_CASES)
def test_oracle_derivatives_match_reference(name):
    g = golden(name)
    C, li, le = int(g["channels"]), int(g["li"]), int(g["le"])
    owner = make_owner(C, li, le, int(g["lo"]), weight=g["weight"])
    use_gates = "gates" in g
    x = torch.from_numpy(g["x"]).double().requires_grad_(True)
    y = torch.from_numpy(g["y"]).double().requires_grad_(True)
    gates = torch.from_numpy(g["gates"]).double().requires_grad_(True) if use_gates else None
    G = torch.from_numpy(g["G"]).double().requires_grad_(True)
    rows = x.shape[0]
    out = pack_out(owner, tp_oracle.tp_forward(owner, split_mul_ir(x, C, li), split_harm(y, le),
                                               None if gates is None else gates.view(rows, owner.num_paths, C),
                                               weight=torch.from_numpy(g["weight"]).double(), dtype=torch.float64))
    targets = [x, y] + ([gates] if use_gates else [])
    firsts = torch.autograd.grad((out * G).sum(), targets, create_graph=True)
    np.testing.assert_allclose(firsts[0].detach().numpy(), g["dx64"], rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(firsts[1].detach().numpy(), g["dy64"], rtol=1e-10, atol=1e-10)
    second = (firsts[0] * torch.from_numpy(g["hx"]).double()).sum() + (firsts[1] * torch.from_numpy(g["hy"]).double()).sum()
    if use_gates:
        np.testing.assert_allclose(firsts[2].detach().numpy(), g["dg64"], rtol=1e-10, atol=1e-10)
        second = second + (firsts[2] * torch.from_numpy(g["hg"]).double()).sum()
    seconds = torch.autograd.grad(second, targets + [G], allow_unused=True)
    np.testing.assert_allclose(seconds[0].numpy(), g["sx64"], rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(seconds[1].numpy(), g["sy64"], rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(seconds[-1].numpy(), g["sG64"], rtol=1e-10, atol=1e-10)
    if use_gates:
        np.testing.assert_allclose(seconds[2].numpy(), g["sg64"], rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("name", ["harmonics_l3.npz", "harmonics_l6.npz"])
def test_oracle_harmonics_match_reference(name):
    g = golden(name)
    lmax = int(g["lmax"])
    tables = harmonic_tables(lmax)
    n = torch.from_numpy(g["n"]).double().requires_grad_(True)
    gy = torch.from_numpy(g["gy"]).double().requires_grad_(True)
    y = torch.cat(tp_oracle.direction_harmonics(n, lmax, tables), -1)
    np.testing.assert_allclose(y.detach().numpy(), g["y64"], rtol=1e-12, atol=1e-12)
    (dn,) = torch.autograd.grad((y * gy).sum(), [n], create_graph=True)
    np.testing.assert_allclose(dn.detach().numpy(), g["dn64"], rtol=1e-11, atol=1e-11)
    sn, sgy = torch.autograd.grad((dn * torch.from_numpy(g["hn"]).double()).sum(), [n, gy])
    np.testing.assert_allclose(sn.numpy(), g["sn64"], rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(sgy.numpy(), g["sgy64"], rtol=1e-10, atol=1e-10)
    y32 = torch.cat(tp_oracle.direction_harmonics(n.detach().float(), lmax, tables), -1)
    assert_close(y32, g["y32"], rel=1e-6, what="fp32 harmonics")


def test_oracle_message_matches_reference():
    g = golden("message_c32_l2.npz")
    C, L, nodes = int(g["channels"]), int(g["lmax"]), int(g["nodes"])
    owner = make_owner(C, L, L, L)
    x = torch.from_numpy(g["x"]).double()
    out = tp_oracle.graph_message(owner, split_mul_ir(x, C, L), split_harm(torch.from_numpy(g["y"]).double(), L),
                                  torch.from_numpy(g["gates"]).double().view(-1, owner.num_paths, C),
                                  torch.from_numpy(g["src"]), torch.from_numpy(g["dst"]),
                                  torch.from_numpy(g["mask"]).double(), nodes=nodes, dtype=torch.float64)
    np.testing.assert_allclose(pack_out(owner, out).numpy(), g["out64"], rtol=1e-12, atol=1e-12)


def test_basis_table_digests():
    from ictc_o3.basis import ictd_irreps as basis
    from ictc_o3.basis.harmonic_basis_pins import BASIS_SHA256
    for l in BASIS_SHA256:
        B = basis.harmonic_basis(l)
        assert B.shape == (basis.sym_dim(l), 2 * l + 1)
    with pytest.raises(ValueError):
        basis.harmonic_basis(max(BASIS_SHA256) + 1)
