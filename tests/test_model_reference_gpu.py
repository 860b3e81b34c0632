"""The CUDA model against the reference's own MACE-ICTC model (FP32 kernels vs the
reference's FP64 outputs; fixtures from ``tests/golden/make_model_golden.py``)."""
import pytest
import torch

from _util import assert_close
from test_model_reference import CASES, load_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,product_backend", [(name, "ictd-pure-u") for name in CASES]
                         + [("model_c8_l2_bridge.npz", "ictd-bridge-u")])
def test_cuda_model_matches_reference_model(name, product_backend, cuda_device):
    model, species, rec = load_case(name, dtype=torch.float32, device=cuda_device, product_backend=product_backend)
    pos = torch.from_numpy(rec["pos"]).float().to(cuda_device).requires_grad_(True)
    src, dst = (torch.from_numpy(rec[k]).to(cuda_device) for k in ("src", "dst"))
    shift = torch.from_numpy(rec["shift"]).float().to(cuda_device)
    atomic = model.node_energies(pos, species, src, dst, shift)
    (grad,) = torch.autograd.grad(atomic.sum(), [pos])
    assert_close(atomic.detach().sum().reshape(1), torch.tensor([rec["atomic_energy"].sum()]), 1e-5,
                 what="energy")
    assert_close(atomic.detach(), torch.from_numpy(rec["atomic_energy"]), 1e-5, what="atomic energies")
    assert_close(-grad, torch.from_numpy(rec["forces"]), 1e-4, what="forces")
