"""Bridge-U symmetric contraction (the reference's default product block) against
the reference module itself (CPU, FP64).

Fixtures from ``tests/golden/make_model_golden.py``: the reference's
``ICTDBridgeUSymmetricContractionSO3`` with its complete state dict (couplings with
the basis bridge folded in, bridge matrices, weights, zero flags), random flat ICTC
features with species and its outputs.  The state dict must load strictly into the
module of the same name here, and the couplings it carries, turned into the kernel
coefficient table, must give the reference's outputs.
"""
import numpy as np
import pytest
import torch

from conftest import golden

CASES = ["sc_bridge_c8_l2_t2.npz", "sc_bridge_c4_l3_t1.npz"]


def _state(rec):
    return {k.split(":", 1)[1]: torch.from_numpy(np.array(rec[k])) for k in rec if k.startswith("state:")}


def _module(rec, state=None):
    from ictc_o3.ops.symmetric_contraction import ICTDBridgeUSymmetricContractionSO3
    module = ICTDBridgeUSymmetricContractionSO3(num_elements=3, channels=int(rec["channels"]),
                                                lmax=int(rec["lmax"]), target_lmax=int(rec["target_lmax"]),
                                                correlation=3).double()
    module.load_state_dict(_state(rec) if state is None else state, strict=True)
    return module


def _evaluate(module, x, species):
    """The contraction as the kernels evaluate it: per-species coefficient table
    T = Usym W from each block's current couplings, then the per-node polynomial."""
    from ictc_o3.backends.cuda.contraction import polynomial, species_tiles
    table = torch.cat([torch.matmul(c.symmetric_table("cpu", torch.float64).unsqueeze(0), c.stacked_weights())
                       for c in module.contractions], 1)
    tiles, tile_species = species_tiles(species, module.num_elements)
    spec = (module.channels, module.lmax, module.correlation, module.target_lmax)
    return polynomial(x, table, tiles, tile_species, spec)


def _oracle(module, x, species):
    """The reference recursion (``_mace_symmetric_contraction.py:298-346``) over the
    module's couplings and weights."""
    from oracle.sc_oracle import contraction, flat_to_mace
    xm = flat_to_mace(x, module.channels, module.lmax)
    outs = []
    for c in module.contractions:
        u = {nu: c.U_tensors(nu) for nu in range(1, c.correlation + 1)}
        outs.append(contraction(u, c.weights_max, list(c.weights), xm, species, c.output_l))
    return torch.cat(outs, -1)


@pytest.mark.parametrize("name", CASES)
def test_reference_state_dict_loads_strictly_and_round_trips(name):
    rec = golden(name)
    module = _module(rec)
    state = _state(rec)
    own = module.state_dict()
    assert set(own) == set(state)
    for key, value in state.items():
        assert own[key].shape == value.shape, key
        assert torch.equal(own[key].to(value.dtype), value), key


@pytest.mark.parametrize("name", CASES)
def test_matches_reference_module(name):
    rec = golden(name)
    module = _module(rec)
    x = torch.from_numpy(rec["x"])
    species = torch.from_numpy(rec["species"])
    ref = torch.from_numpy(rec["out"])
    torch.testing.assert_close(torch.from_numpy(rec["out_one_hot"]), ref, rtol=1e-12, atol=1e-12)
    with torch.no_grad():
        torch.testing.assert_close(_oracle(module, x, species), ref, rtol=1e-10, atol=1e-11)
        torch.testing.assert_close(_evaluate(module, x, species), ref, rtol=1e-10, atol=1e-11)


@pytest.mark.parametrize("name", CASES)
def test_equals_pure_u_with_mapped_weights(name):
    """The model checkpoint loader's change of coupling basis: the pure-ICTC module
    with the bridge weights mapped onto its couplings gives the same contraction."""
    from ictc_o3.ops.symmetric_contraction import ICTDPureUSymmetricContractionSO3
    from mace_ictc.checkpoint import _bridge_weights
    rec = golden(name)
    bridge = _module(rec)
    pure = ICTDPureUSymmetricContractionSO3(num_elements=3, channels=bridge.channels, lmax=bridge.lmax,
                                            target_lmax=bridge.target_lmax, correlation=3).double()
    state = _state(rec)
    with torch.no_grad():
        for t, block in enumerate(pure.contractions):
            prefix = f"symmetric_contractions.contractions.{t}."
            tensors = {k[len(prefix):]: v for k, v in state.items() if k.startswith(prefix)}
            for key, value in _bridge_weights(block, tensors, name).items():
                block.get_parameter(key).copy_(value)
    x = torch.from_numpy(rec["x"])
    species = torch.from_numpy(rec["species"])
    with torch.no_grad():
        torch.testing.assert_close(_evaluate(pure, x, species), torch.from_numpy(rec["out"]), rtol=1e-9, atol=1e-10)


def test_new_module_uses_ictc_couplings_and_identity_bridge():
    from ictc_o3.basis.ictd_irreps import ictd_u_matrix_so3
    from ictc_o3.ops.symmetric_contraction import ICTDBridgeUSymmetricContractionSO3
    module = ICTDBridgeUSymmetricContractionSO3(num_elements=2, channels=4, lmax=2, target_lmax=1)
    for t, block in enumerate(module.contractions):
        for nu in (1, 2, 3):
            torch.testing.assert_close(block.U_tensors(nu), torch.from_numpy(ictd_u_matrix_so3(2, t, nu)).float())
    for l in range(3):
        assert torch.equal(getattr(module.basis_bridge, f"q_{l}"), torch.eye(2 * l + 1))
    assert not any(k.startswith("contractions.") for k in module.state_dict())


def test_coupling_table_follows_loaded_buffers():
    """A loaded state dict replaces the couplings: the cached table is rebuilt."""
    rec = golden(CASES[0])
    from ictc_o3.ops.symmetric_contraction import ICTDBridgeUSymmetricContractionSO3
    module = ICTDBridgeUSymmetricContractionSO3(num_elements=3, channels=8, lmax=2, target_lmax=2).double()
    before = module.contractions[1].symmetric_table("cpu", torch.float64)
    module.load_state_dict(_state(rec))
    after = module.contractions[1].symmetric_table("cpu", torch.float64)
    assert after is not before and not torch.allclose(after, before)
    assert module.contractions[1].symmetric_table("cpu", torch.float64) is after


def test_zero_flags_hold_weights_at_zero():
    rec = golden(CASES[0])
    state = _state(rec)
    state["symmetric_contractions.contractions.0.weights_1_zeroed"] = torch.tensor(True)
    state["symmetric_contractions.contractions.2.weights_max_zeroed"] = torch.tensor(True)
    module = _module(rec, state)
    w1 = module.contractions[0].weights[1]
    wmax = module.contractions[2].weights_max
    assert not w1.requires_grad and not wmax.requires_grad
    assert float(w1.abs().max()) == 0.0 and float(wmax.abs().max()) == 0.0
    assert module.contractions[0].weights[0].requires_grad


def test_state_dict_with_fewer_couplings_resizes():
    """A state dict whose coupling count differs (the reference's reduced-CG option)
    brings its own U and weight shapes."""
    rec = golden(CASES[0])
    state = _state(rec)
    prefix = "symmetric_contractions.contractions.1."
    state[prefix + "U_matrix_3"] = state[prefix + "U_matrix_3"][..., :15].clone()
    state[prefix + "weights_max"] = state[prefix + "weights_max"][:, :15].clone()
    module = _module(rec, state)
    block = module.contractions[1]
    assert block.U_matrix_3.shape[-1] == 15 and block.weights_max.shape == (3, 15, 8)
    x = torch.from_numpy(rec["x"])
    species = torch.from_numpy(rec["species"])
    with torch.no_grad():
        torch.testing.assert_close(_evaluate(module, x, species), _oracle(module, x, species), rtol=1e-10,
                                   atol=1e-11)


def test_operator_configuration_checks():
    from ictc_o3.operators import configure_symmetric_contraction, create_symmetric_contraction
    from ictc_o3.ops.symmetric_contraction import ICTDBridgeUSymmetricContractionSO3
    with pytest.raises(TypeError, match="bridge-U"):
        configure_symmetric_contraction(torch.nn.Linear(2, 2))
    module = ICTDBridgeUSymmetricContractionSO3(num_elements=2, channels=4, lmax=1, target_lmax=0)
    with pytest.raises((TypeError, ValueError, RuntimeError)):
        configure_symmetric_contraction(module)                     # CPU tensors: no CUDA contraction
    with pytest.raises(ValueError, match="CUDA"):
        create_symmetric_contraction(num_elements=2, lmax=1, device="cpu")


class _ReferenceBlock(torch.nn.Module):
    """The layout of one of the reference's MACE contraction blocks
    (``ictc_o3/ops/_mace_symmetric_contraction.py:87-226``): ``U_matrix_nu`` buffers,
    ``weights_max``, a ``weights`` list, ``correlation``, ``U_tensors(nu)``."""

    def __init__(self, tensors):
        super().__init__()
        self.correlation = sum(1 for k in tensors if k.startswith("U_matrix_"))
        for nu in range(1, self.correlation + 1):
            self.register_buffer(f"U_matrix_{nu}", tensors[f"U_matrix_{nu}"].clone())
        self.weights_max = torch.nn.Parameter(tensors["weights_max"].clone())
        self.weights = torch.nn.ParameterList([torch.nn.Parameter(tensors[f"weights.{i}"].clone())
                                               for i in range(self.correlation - 1)])

    def U_tensors(self, nu):
        return getattr(self, f"U_matrix_{nu}")


def reference_layout_module(rec):
    """An object laid out like the reference's bridge-U module (what its hook site
    passes as ``owner``), filled from the fixture's state dict."""
    state = _state(rec)
    owner = torch.nn.Module()
    owner.channels, owner.lmax, owner.target_lmax = int(rec["channels"]), int(rec["lmax"]), int(rec["target_lmax"])
    blocks = []
    for t in range(owner.target_lmax + 1):
        prefix = f"symmetric_contractions.contractions.{t}."
        blocks.append(_ReferenceBlock({k[len(prefix):]: v for k, v in state.items() if k.startswith(prefix)}))
    owner.symmetric_contractions = torch.nn.Module()
    owner.symmetric_contractions.contractions = torch.nn.ModuleList(blocks)
    return owner


@pytest.mark.parametrize("name", CASES)
def test_reference_layout_owner_gives_the_same_contraction(name):
    """The CUDA entry point reads the reference's own module at its hook site: blocks,
    spec and coefficient tables from that layout equal those of the module here."""
    from ictc_o3.backends.cuda.contraction import (block_table, block_weights, contraction_blocks,
                                                   contraction_spec, polynomial, species_tiles)
    rec = golden(name)
    owner = reference_layout_module(rec)
    module = _module(rec)
    assert contraction_spec(owner) == contraction_spec(module) == (
        module.channels, module.lmax, 3, module.target_lmax, 3)
    for a, b in zip(contraction_blocks(owner), contraction_blocks(module)):
        torch.testing.assert_close(block_table(a, "cpu", torch.float64), block_table(b, "cpu", torch.float64),
                                   rtol=0, atol=0)
        assert block_table(a, "cpu", torch.float64) is block_table(a, "cpu", torch.float64)
    table = torch.cat([torch.matmul(block_table(c, "cpu", torch.float64).unsqueeze(0), block_weights(c))
                       for c in contraction_blocks(owner)], 1)
    species = torch.from_numpy(rec["species"])
    tiles, tile_species = species_tiles(species, 3)
    with torch.no_grad():
        out = polynomial(torch.from_numpy(rec["x"]), table, tiles, tile_species, contraction_spec(owner)[:4])
    torch.testing.assert_close(out, torch.from_numpy(rec["out"]), rtol=1e-10, atol=1e-11)


def test_folded_table_cache(monkeypatch):
    """``coefficient_table``'s cache (host logic; the fold itself replaced by its torch
    definition, T_t = Usym_t W_t, since the kernel needs a GPU): kept for frozen
    weights, rebuilt when a weight changes in place or is replaced, or when a block's
    coupling table is rebuilt; never cached while a weight needs a gradient."""
    from ictc_o3.backends.cuda import contraction as cc

    class TorchFold(torch.autograd.Function):
        @staticmethod
        def forward(ctx, usyms, rows, *weights):
            return torch.cat([torch.matmul(u.unsqueeze(0).to(w.dtype), w) for u, w in zip(usyms, weights)], 1)

    monkeypatch.setattr(cc, "_Fold", TorchFold)
    rec = golden(CASES[0])
    module = _module(rec)
    with torch.no_grad():
        first = cc.coefficient_table(module, torch.device("cpu"))
        assert cc.coefficient_table(module, torch.device("cpu")) is first
        module.contractions[0].weights_max.mul_(2.0)                       # in-place update
        second = cc.coefficient_table(module, torch.device("cpu"))
        assert second is not first and not torch.equal(second, first)
        old = module.contractions[1].weights[0]
        module.contractions[1].weights[0] = torch.nn.Parameter(old.detach().clone())   # new tensor object
        assert cc.coefficient_table(module, torch.device("cpu")) is not second
        third = cc.coefficient_table(module, torch.device("cpu"))
        module.contractions[2].U_matrix_2.mul_(0.5)                          # couplings change
        fourth = cc.coefficient_table(module, torch.device("cpu"))
        assert fourth is not third and not torch.equal(fourth, third)
    live = cc.coefficient_table(module, torch.device("cpu"))                # weights require grad
    assert live.requires_grad and cc.cache_of(module, "_cuda_folded_table")["table"][1] is fourth
