"""GPU parity of the symmetric-contraction kernels (forward, feature and weight gradients)."""
import pytest
import torch

from _util import golden, assert_close
from oracle import sc_oracle

pytestmark = pytest.mark.gpu


def _module(g, device):
    from ictc_o3.ops.symmetric_contraction import ICTDPureUSymmetricContractionSO3
    C, L, T, corr, S = (int(g[k]) for k in ("channels", "lmax", "target_lmax", "correlation", "elements"))
    module = ICTDPureUSymmetricContractionSO3(num_elements=S, channels=C, lmax=L, target_lmax=T,
                                              correlation=corr).to(device)
    with torch.no_grad():
        for t, contraction in enumerate(module.contractions):
            contraction.weights_max.copy_(torch.from_numpy(g[f"w_t{t}_nu{corr}"]))
            for j, nu in enumerate(range(corr - 1, 0, -1)):
                contraction.weights[j].copy_(torch.from_numpy(g[f"w_t{t}_nu{nu}"]))
    return module


@pytest.mark.parametrize("name", ["contraction_c32_l2.npz", "contraction_c32_l1_t0.npz"])
def test_contraction_matches_reference(name, cuda_device):
    g = golden(name)
    module = _module(g, cuda_device)
    x = torch.from_numpy(g["x"]).to(cuda_device).requires_grad_(True)
    idx = torch.from_numpy(g["idx"]).to(cuda_device)
    out = module(x, node_type_idx=idx)
    assert_close(out.detach().cpu(), g["out64"], 1e-5, 1e-3, "contraction forward")
    G = torch.from_numpy(g["G"]).float().to(cuda_device)
    params = []
    corr = int(g["correlation"])
    for c in module.contractions:
        params += [c.weights_max, *c.weights]
    grads = torch.autograd.grad(out, [x] + params, G)
    assert_close(grads[0].cpu(), g["dx64"], 1e-4, 1e-3, "contraction dx")
    k = 1
    for t in range(int(g["target_lmax"]) + 1):
        for nu in range(corr, 0, -1):
            assert_close(grads[k].cpu(), g[f"dw_t{t}_nu{nu}"], 1e-4, 1e-3, f"dW t={t} nu={nu}")
            k += 1


@pytest.mark.parametrize("name", ["sc_bridge_c8_l2_t2.npz", "sc_bridge_c4_l3_t1.npz"])
def test_bridge_module_matches_reference_module(name, cuda_device):
    """A state dict of the reference's bridge-U module, loaded into the module of the
    same name, through the CUDA kernels (FP32) against the reference module's FP64
    outputs; the feature gradient against the FP64 recursion over the same couplings."""
    from ictc_o3.operators import configure_symmetric_contraction
    from test_contraction_bridge import _module, _oracle
    g = golden(name)
    module = _module(g).float().to(cuda_device)
    assert configure_symmetric_contraction(module)["backend"] == "cuda"
    x = torch.from_numpy(g["x"]).float().to(cuda_device).requires_grad_(True)
    species = torch.from_numpy(g["species"]).to(cuda_device)
    attrs = torch.nn.functional.one_hot(species, 3).float()
    out = module(x, attrs, species)
    assert_close(out.detach().cpu(), torch.from_numpy(g["out"]), 1e-5, 1e-3, "bridge-U forward")
    assert_close(module(x, attrs).detach().cpu(), torch.from_numpy(g["out_one_hot"]), 1e-5, 1e-3,
                 "bridge-U forward (one-hot attributes)")
    G = torch.randn(out.shape, device=cuda_device, generator=torch.Generator(device=cuda_device).manual_seed(5))
    (dx,) = torch.autograd.grad(out, [x], G)
    x64 = torch.from_numpy(g["x"]).requires_grad_(True)
    ref = _oracle(_module(g), x64, torch.from_numpy(g["species"]))
    (rdx,) = torch.autograd.grad(ref, [x64], G.double().cpu())
    assert_close(dx.cpu(), rdx, 1e-4, 1e-3, "bridge-U dx")


@pytest.mark.parametrize("name", ["sc_bridge_c8_l2_t2.npz", "sc_bridge_c4_l3_t1.npz"])
def test_hook_entry_with_reference_layout_owner(name, cuda_device):
    """``factorized_contractions`` given an object laid out like the reference's own
    bridge-U module (what its hook site passes) and MACE-layout features."""
    from ictc_o3.backends.cuda.contraction import factorized_contractions
    from oracle.sc_oracle import flat_to_mace
    from test_contraction_bridge import reference_layout_module
    g = golden(name)
    owner = reference_layout_module(g).float().to(cuda_device)
    x = flat_to_mace(torch.from_numpy(g["x"]).float(), int(g["channels"]), int(g["lmax"])).to(cuda_device)
    out = factorized_contractions(owner, x.contiguous(), torch.from_numpy(g["species"]).to(cuda_device))
    assert_close(out.detach().cpu(), torch.from_numpy(g["out"]), 1e-5, 1e-3, "hook entry, reference-layout owner")


@pytest.mark.parametrize("lmax,target,corr", [(1, 1, 3), (2, 2, 3), (2, 0, 3), (3, 3, 3), (2, 2, 2), (3, 1, 1)])
@pytest.mark.parametrize("channels", [32, 96, 40])
def test_contraction_random_against_oracle(lmax, target, corr, channels, cuda_device):
    """Channel tails, partial species tiles, an absent species, every supported degree."""
    from ictc_o3.ops.symmetric_contraction import ICTDPureUSymmetricContractionSO3
    torch.manual_seed(lmax * 100 + target * 10 + corr + channels)
    S, N = 4, 29
    module = ICTDPureUSymmetricContractionSO3(num_elements=S, channels=channels, lmax=lmax, target_lmax=target,
                                              correlation=corr).to(cuda_device)
    x = torch.randn(N, channels * (lmax + 1) ** 2, device=cuda_device)
    idx = torch.randint(0, S - 1, (N,), device=cuda_device)  # species S-1 never appears
    xr = x.detach().requires_grad_(True)
    out = module(xr, node_type_idx=idx)
    G = torch.randn_like(out)
    dx = torch.autograd.grad(out, [xr], G)[0]
    xd = x.double().cpu().requires_grad_(True)
    feats = sc_oracle.flat_to_mace(xd, channels, lmax)
    outs = []
    for t, c in enumerate(module.contractions):
        u = {nu: c.U_tensors(nu).double().cpu() for nu in range(1, corr + 1)}
        outs.append(sc_oracle.contraction(u, c.weights_max.detach().double().cpu(),
                                          [w.detach().double().cpu() for w in c.weights], feats, idx.cpu(), t))
    ref = torch.cat(outs, -1)
    (rdx,) = torch.autograd.grad(ref, [xd], G.double().cpu())
    assert_close(out.detach().cpu(), ref.detach(), 1e-5, 1e-3, "forward")
    assert_close(dx.cpu(), rdx, 1e-4, 1e-3, "dx")


@pytest.mark.parametrize("lmax,target,corr", [(2, 2, 3), (2, 0, 3), (1, 1, 2)])
def test_contraction_second_derivatives_against_oracle(lmax, target, corr, cuda_device):
    """Mixed second derivatives (force-loss training): d/d(x, W) of <dx(G), V>."""
    from ictc_o3.ops.symmetric_contraction import ICTDPureUSymmetricContractionSO3
    torch.manual_seed(7 + lmax * 10 + target + corr)
    S, N, channels = 3, 23, 16
    module = ICTDPureUSymmetricContractionSO3(num_elements=S, channels=channels, lmax=lmax, target_lmax=target,
                                              correlation=corr).to(cuda_device)
    params = []
    for c in module.contractions:
        params += [c.weights_max, *c.weights]
    x = torch.randn(N, channels * (lmax + 1) ** 2, device=cuda_device)
    idx = torch.randint(0, S, (N,), device=cuda_device)
    xr = x.detach().requires_grad_(True)
    out = module(xr, node_type_idx=idx)
    G = torch.randn_like(out)
    V = torch.randn_like(x)
    (dx,) = torch.autograd.grad(out, [xr], G, create_graph=True)
    got = torch.autograd.grad((dx * V).sum(), [xr] + params)

    xd = x.double().cpu().requires_grad_(True)
    feats = sc_oracle.flat_to_mace(xd, channels, lmax)
    ref_params, outs = [], []
    for t, c in enumerate(module.contractions):
        u = {nu: c.U_tensors(nu).double().cpu() for nu in range(1, corr + 1)}
        wmax = c.weights_max.detach().double().cpu().requires_grad_(True)
        ws = [w.detach().double().cpu().requires_grad_(True) for w in c.weights]
        ref_params += [wmax, *ws]
        outs.append(sc_oracle.contraction(u, wmax, ws, feats, idx.cpu(), t))
    ref = torch.cat(outs, -1)
    (rdx,) = torch.autograd.grad(ref, [xd], G.double().cpu(), create_graph=True)
    want = torch.autograd.grad((rdx * V.double().cpu()).sum(), [xd] + ref_params)
    assert_close(dx.detach().cpu(), rdx.detach(), 1e-4, 1e-3, "dx")
    for k, (a, b) in enumerate(zip(got, want)):
        assert_close(a.cpu(), b, 1e-4, 1e-3, f"second derivative {k}")


def _ref_fold(module, params, device):
    """The folded table in FP64 torch from (FP64 CPU copies of) the module's weights."""
    k, parts = 0, []
    for c in module.contractions:
        n = len(list(c.parameters()))
        w = torch.cat(params[k:k + n], 1)
        parts.append(torch.matmul(c.symmetric_table(device, torch.float64).cpu().unsqueeze(0), w))
        k += n
    return torch.cat(parts, 1)


def test_weight_fold_kernel_and_its_derivatives(cuda_device):
    """ictc_sc_fold: T_t = Usym_t W_t and dW_t = Usym_t^T dT_t against FP64 torch, the
    second-order path through the adjoint, and the frozen-weight cache."""
    from ictc_o3.backends.cuda.contraction import coefficient_table
    from ictc_o3.ops.symmetric_contraction import ICTDPureUSymmetricContractionSO3
    torch.manual_seed(7)
    module = ICTDPureUSymmetricContractionSO3(num_elements=3, channels=40, lmax=2, target_lmax=2,
                                              correlation=3).to(cuda_device)
    params = list(module.parameters())
    ref_params = [p.detach().double().cpu().requires_grad_(True) for p in params]
    table = coefficient_table(module, cuda_device)
    ref_table = _ref_fold(module, ref_params, cuda_device)
    assert_close(table.detach().cpu(), ref_table.detach(), 1e-6, what="fold")
    G = torch.randn(table.shape, device=cuda_device, requires_grad=True)
    grads = torch.autograd.grad(table, params, G, create_graph=True)
    ref_grads = torch.autograd.grad(ref_table, ref_params, G.detach().double().cpu())
    for g, r in zip(grads, ref_grads):
        assert_close(g.detach().cpu(), r, 1e-5, what="dW")
    # second order: <dW(G), V> is linear in G; its G-gradient is the fold of V
    V = [torch.randn_like(g) for g in grads]
    (dG,) = torch.autograd.grad(sum((g * v).sum() for g, v in zip(grads, V)), [G])
    assert_close(dG.cpu(), _ref_fold(module, [v.double().cpu() for v in V], cuda_device), 1e-5, what="d2")
    # frozen weights: the folded table is kept until a weight changes
    with torch.no_grad():
        first = coefficient_table(module, cuda_device)
        assert coefficient_table(module, cuda_device) is first
        module.contractions[0].weights_max.add_(1.0)
        again = coefficient_table(module, cuda_device)
    assert again is not first and not torch.equal(again, first)


@pytest.mark.parametrize("lmax,target,corr,channels", [(2, 2, 3, 40), (3, 1, 3, 32), (1, 1, 2, 16), (2, 0, 3, 64)])
def test_second_order_kernels(lmax, target, corr, channels, cuda_device):
    """Force-loss training derivatives of the contraction through the kernels
    (directional polynomial, Hessian-vector product, table gradients) against the
    FP64 torch polynomial: dx, then the gradients of <dx, V> with respect to x, the
    output cotangent G and the weights, and the first-order weight gradient."""
    from ictc_o3.backends.cuda.contraction import contract_flat, polynomial, species_tiles
    from ictc_o3.ops.symmetric_contraction import ICTDPureUSymmetricContractionSO3
    torch.manual_seed(lmax * 10 + target)
    S, N = 3, 203
    module = ICTDPureUSymmetricContractionSO3(num_elements=S, channels=channels, lmax=lmax, target_lmax=target,
                                              correlation=corr).to(cuda_device)
    D = (lmax + 1) ** 2
    x = (0.7 * torch.randn(N, channels * D, device=cuda_device)).requires_grad_(True)
    idx = torch.randint(0, S, (N,), device=cuda_device)
    params = list(module.parameters())
    out = contract_flat(module, x, idx)
    G = torch.randn(out.shape, device=cuda_device, requires_grad=True)
    (w1,) = torch.autograd.grad(out, [params[0]], G.detach(), retain_graph=True)   # first-order weight gradient
    (dx,) = torch.autograd.grad(out, [x], G, create_graph=True)
    V = torch.randn_like(dx)
    hx, hG, *hW = torch.autograd.grad((dx * V).sum(), [x, G] + params, allow_unused=True)

    # FP64 reference: the same polynomial in torch, the same folded weights
    spec = (channels, lmax, corr, target)
    tiles, tile_species = species_tiles(idx, S)
    p64 = [p.detach().double().requires_grad_(True) for p in params]
    parts, k = [], 0
    for c in module.contractions:
        n = len(list(c.parameters()))
        parts.append(torch.matmul(c.symmetric_table(cuda_device, torch.float64).unsqueeze(0),
                                  torch.cat(p64[k:k + n], 1)))
        k += n
    table64 = torch.cat(parts, 1)
    x64 = x.detach().double().requires_grad_(True)
    G64 = G.detach().double().requires_grad_(True)
    ref = polynomial(x64, table64, tiles, tile_species, spec)
    assert_close(out.detach(), ref.detach(), 1e-5, what="forward")
    (rw1,) = torch.autograd.grad(ref, [p64[0]], G64.detach(), retain_graph=True)
    (rdx,) = torch.autograd.grad(ref, [x64], G64, create_graph=True)
    assert_close(dx.detach(), rdx.detach(), 1e-4, what="dx")
    rhx, rhG, *rhW = torch.autograd.grad((rdx * V.double()).sum(), [x64, G64] + p64, allow_unused=True)
    assert_close(hx, rhx, 1e-4, what="d<dx,V>/dx (Hessian-vector)")
    assert_close(hG, rhG, 1e-4, what="d<dx,V>/dG (directional)")
    for a, b in zip(hW, rhW):
        assert_close(a, b, 1e-4, what="d<dx,V>/dW (directional table gradient)")
    assert_close(w1, rw1, 1e-4, what="dW (table gradient)")
