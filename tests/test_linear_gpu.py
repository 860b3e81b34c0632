"""Per-degree channel linears (ictc_channel_mix) vs the same linears in FP64 torch."""
import pytest
import torch

from _util import assert_close

pytestmark = pytest.mark.gpu


def _reference(x, weights, lmax, species=None, scale=1.0):
    """y_l[n] = scale * W_{s(n), l} x_l[n] in the flat [channel][2l+1] layout."""
    n = x.shape[0]
    outs, xo = [], 0
    for l in range(lmax + 1):
        w = weights[l]
        m = 2 * l + 1
        cin = w.shape[-1]
        xl = x[:, xo:xo + cin * m].reshape(n, cin, m)
        wn = w[species] if species is not None else w.expand(n, *w.shape[-2:]) if w.dim() == 2 else w[0].expand(n, *w.shape[-2:])
        outs.append(scale * torch.einsum("noi,nim->nom", wn, xl).reshape(n, -1))
        xo += cin * m
    return torch.cat(outs, -1)


@pytest.mark.parametrize("cin,cout,lmax,nodes", [((64, 64, 64), 64, 2, 1000), ((192, 256, 256), 64, 2, 333),
                                                 ((128,) * 4, 128, 3, 77), ((40, 24), 72, 1, 5)])
def test_channel_mix_matches_reference(cin, cout, lmax, nodes, cuda_device):
    from ictc_o3.backends.cuda.linear import channel_mix
    torch.manual_seed(sum(cin) + nodes)
    ws = [(torch.randn(cout, cin[l], device=cuda_device) / cin[l] ** 0.5).requires_grad_(True) for l in range(lmax + 1)]
    width = sum(c * (2 * l + 1) for l, c in enumerate(cin))
    x = torch.randn(nodes, width, device=cuda_device, requires_grad=True)
    y = channel_mix(x, ws, scale=0.25)
    G = torch.randn_like(y)
    grads = torch.autograd.grad(y, [x] + ws, G)
    xd = x.detach().double().cpu().requires_grad_(True)
    wd = [w.detach().double().cpu().requires_grad_(True) for w in ws]
    ref = _reference(xd, wd, lmax, scale=0.25)
    rgrads = torch.autograd.grad(ref, [xd] + wd, G.double().cpu())
    assert_close(y.detach().cpu(), ref.detach(), 1e-5, 1e-3, "y")
    for a, b in zip(grads, rgrads):
        assert_close(a.cpu(), b, 1e-5, 1e-3, "gradient")


def test_species_channel_mix_and_second_order(cuda_device):
    from ictc_o3.backends.cuda.linear import channel_mix
    torch.manual_seed(3)
    S, C, lmax, n = 4, 64, 2, 301
    w = (torch.randn(S, lmax + 1, C, C, device=cuda_device) / C ** 0.5).requires_grad_(True)
    species = torch.randint(0, S - 1, (n,), device=cuda_device)            # species S-1 absent
    x = torch.randn(n, C * (lmax + 1) ** 2, device=cuda_device, requires_grad=True)
    y = channel_mix(x, [w[:, l] for l in range(lmax + 1)], species=species, num_elements=S)
    G = torch.randn_like(y)
    V = torch.randn_like(x)
    (dx, dw) = torch.autograd.grad(y, [x, w], G, create_graph=True)
    (h,) = torch.autograd.grad((dx * V).sum() + (dw ** 2).sum(), [w])
    xd = x.detach().double().cpu().requires_grad_(True)
    wdd = w.detach().double().cpu().requires_grad_(True)
    ref = _reference(xd, [wdd[:, l] for l in range(lmax + 1)], lmax, species=species.cpu())
    (rdx, rdw) = torch.autograd.grad(ref, [xd, wdd], G.double().cpu(), create_graph=True)
    (rh,) = torch.autograd.grad((rdx * V.double().cpu()).sum() + (rdw ** 2).sum(), [wdd])
    assert_close(y.detach().cpu(), ref.detach(), 1e-5, 1e-3, "y")
    assert_close(dx.detach().cpu(), rdx.detach(), 1e-5, 1e-3, "dx")
    assert_close(dw.detach().cpu(), rdw.detach(), 1e-5, 1e-3, "dw")
    assert_close(h.cpu(), rh, 1e-4, 1e-3, "second order")
