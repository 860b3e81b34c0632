"""GPU parity of the direction-harmonics kernel and its first/second adjoints."""
import pytest
import torch

from _util import golden, assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["harmonics_l3.npz", "harmonics_l6.npz"])
def test_harmonics_match_reference(name, cuda_device):
    from ictc_o3.backends.cuda.geometry import direction_harmonics
    g = golden(name)
    lmax = int(g["lmax"])
    n = torch.from_numpy(g["n"]).to(cuda_device).requires_grad_(True)
    gy = torch.from_numpy(g["gy"]).to(cuda_device).requires_grad_(True)
    y = direction_harmonics(n, lmax)
    assert_close(y.detach().cpu(), g["y64"], 1e-5, 1e-3, "Y")
    (dn,) = torch.autograd.grad((y * gy).sum(), [n], create_graph=True)
    assert_close(dn.detach().cpu(), g["dn64"], 1e-4, 1e-3, "dY/dn")
    sn, sgy = torch.autograd.grad((dn * torch.from_numpy(g["hn"]).to(cuda_device)).sum(), [n, gy])
    assert_close(sn.cpu(), g["sn64"], 1e-4, 1e-3, "second derivative n")
    assert_close(sgy.cpu(), g["sgy64"], 1e-4, 1e-3, "second derivative gY")


def test_harmonics_public_api_lists(cuda_device):
    from ictc_o3.operators import direction_harmonics
    g = golden("harmonics_l3.npz")
    n = torch.from_numpy(g["n"]).to(cuda_device)
    ys = direction_harmonics(n, 3)
    assert [tuple(v.shape) for v in ys] == [(n.shape[0], 2 * l + 1) for l in range(4)]
    assert_close(torch.cat(ys, -1).cpu(), g["y64"], 1e-5, 1e-3, "list")
    empty = direction_harmonics(torch.zeros(0, 3, device=cuda_device), 2)
    assert [tuple(v.shape) for v in empty] == [(0, 1), (0, 3), (0, 5)]
