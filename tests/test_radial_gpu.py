"""Fused radial MLP (tcgen05, 3xTF32) vs the same network in FP64."""
import pytest
import torch

from _util import assert_close

pytestmark = pytest.mark.gpu


def _net(features, gates, seed):
    torch.manual_seed(seed)
    layers = [torch.nn.Linear(features, 64, bias=False), torch.nn.Linear(64, 64, bias=False),
              torch.nn.Linear(64, 64, bias=False), torch.nn.Linear(64, gates, bias=False)]
    for m in layers:
        torch.nn.init.normal_(m.weight, std=1.0 / m.in_features ** 0.5)
    return layers


def _reference(feats, layers):
    from ictc_o3.backends.cuda.radial import mlp_reference
    return mlp_reference(feats, [m.weight.detach().double().cpu() for m in layers])


@pytest.mark.parametrize("features,gates,edges", [(8, 704, 1000), (8, 192, 4096), (6, 512, 333),
                                                  (8, 2944, 257), (8, 128, 128), (3, 320, 77),
                                                  (8, 96, 500), (8, 24, 129)])
def test_radial_forward_and_embedding_gradient(features, gates, edges, cuda_device):
    from ictc_o3.backends.cuda import radial
    layers = [m.to(cuda_device) for m in _net(features, gates, edges)]
    plan = radial.RadialPlan()
    feats = torch.rand(edges, features, device=cuda_device) * 2.0 - 0.5
    f = feats.clone().requires_grad_(True)
    out = radial.radial_gates(layers, f, plan)
    G = torch.randn_like(out)
    (df,) = torch.autograd.grad(out, [f], G)
    radial.check_status(plan)
    fd = feats.double().cpu().requires_grad_(True)
    ref = _reference(fd, layers)
    (rdf,) = torch.autograd.grad(ref, [fd], G.double().cpu())
    assert_close(out.detach().cpu(), ref.detach(), 1e-5, 1e-3, "gates")
    assert_close(df.cpu(), rdf, 1e-4, 1e-3, "d embedding")


def test_radial_weight_gradients_and_second_order(cuda_device):
    """Weight gradients and create_graph backward go through the differentiable path."""
    from ictc_o3.backends.cuda import radial
    layers = [m.to(cuda_device) for m in _net(8, 192, 3)]
    plan = radial.RadialPlan()
    feats = torch.rand(300, 8, device=cuda_device).requires_grad_(True)
    out = radial.radial_gates(layers, feats, plan)
    G = torch.randn_like(out)
    grads = torch.autograd.grad(out, [feats] + [m.weight for m in layers], G, create_graph=True)
    V = torch.randn_like(feats)
    (h,) = torch.autograd.grad((grads[0] * V).sum(), [feats])
    fd = feats.detach().double().cpu().requires_grad_(True)
    wd = [m.weight.detach().double().cpu().requires_grad_(True) for m in layers]
    ref = radial.mlp_reference(fd, wd)
    rgrads = torch.autograd.grad(ref, [fd] + wd, G.double().cpu(), create_graph=True)
    (rh,) = torch.autograd.grad((rgrads[0] * V.double().cpu()).sum(), [fd])
    for a, b in zip(grads, rgrads):
        assert_close(a.detach().cpu(), b.detach(), 1e-4, 1e-3, "first derivatives")
    assert_close(h.cpu(), rh, 1e-4, 1e-3, "second derivative")


def test_radial_empty_and_weight_update(cuda_device):
    from ictc_o3.backends.cuda import radial
    layers = [m.to(cuda_device) for m in _net(8, 192, 4)]
    plan = radial.RadialPlan()
    empty = radial.radial_gates(layers, torch.empty(0, 8, device=cuda_device), plan)
    assert empty.shape == (0, 192)
    feats = torch.rand(200, 8, device=cuda_device)
    first = radial.radial_gates(layers, feats, plan)
    with torch.no_grad():
        layers[3].weight.mul_(2.0)                      # the plan must repack
    second = radial.radial_gates(layers, feats, plan)
    assert_close(second.cpu(), 2.0 * first.cpu(), 1e-6, None, "repacked weights")
