"""The model against the reference's own MACE-ICTC model (CPU, FP64 oracle operators).

Fixtures from ``tests/golden/make_model_golden.py``: the reference
``PureCartesianICTDFix`` (pure-ICTC and bridge-U product backends, reference
defaults for new models, random weights) evaluated by its own forward on small
periodic systems.  Its state dict loads through
``mace_ictc.checkpoint.from_reference_state_dict`` (bridge-U weights through the
exact change of coupling basis); per-atom energies and forces must match to FP64
rounding.
"""
import numpy as np
import pytest
import torch

from conftest import golden

# pure-U at lmax 2 and 3; bridge-U (the reference's default product backend) at lmax 2
CASES = ["model_c8_l2.npz", "model_c8_l3.npz", "model_c8_l2_bridge.npz"]


def load_case(name, ops=None, dtype=torch.float64, device="cpu", product_backend="ictd-pure-u"):
    """(model with the reference weights, species, edges, fixture)."""
    from mace_ictc.checkpoint import from_reference_state_dict
    from mace_ictc.models import MACEICTC
    rec = golden(name)
    state = {k.split(":", 1)[1]: torch.from_numpy(v) for k, v in rec.items()
             if k.startswith("param:") or k.startswith("buffer:")}
    model = MACEICTC(channels=int(rec["channels"]), lmax=int(rec["lmax"]), num_interactions=2, correlation=3,
                     r_max=float(rec["cutoff"]), avg_num_neighbors=float(rec["avg_num_neighbors"]), ops=ops,
                     product_backend=product_backend)
    model = model.to(dtype)
    from_reference_state_dict(model, {k: v.to(dtype) for k, v in state.items()})
    model = model.to(device)
    species = torch.from_numpy(np.searchsorted([1, 6, 8], rec["numbers"])).to(device)
    return model, species, rec


@pytest.mark.parametrize("product_backend", ["ictd-pure-u", "ictd-bridge-u"])
@pytest.mark.parametrize("name", CASES)
def test_model_matches_reference_model(name, product_backend):
    """Every fixture into a model of either product backend (by name, or through the
    change of coupling basis when bridge-U weights meet pure-U blocks)."""
    from oracle.model_ops import OracleOps
    model, species, rec = load_case(name, ops=OracleOps(), product_backend=product_backend)
    assert model.product_backend == product_backend
    assert not model.interactions[0].self_connection is None            # first-layer self-connection
    pos = torch.from_numpy(rec["pos"]).requires_grad_(True)
    src, dst = torch.from_numpy(rec["src"]), torch.from_numpy(rec["dst"])
    shift = torch.from_numpy(rec["shift"])
    atomic = model.node_energies(pos, species, src, dst, shift)
    (grad,) = torch.autograd.grad(atomic.sum(), [pos])
    ref_e = torch.from_numpy(rec["atomic_energy"])
    ref_f = torch.from_numpy(rec["forces"])
    torch.testing.assert_close(atomic.detach(), ref_e, rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(-grad, ref_f, rtol=1e-9, atol=1e-11)
