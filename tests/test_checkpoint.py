"""Reference state-dict names and layouts load into the model (CPU, FP64 oracle ops)."""
import math

import pytest
import torch


def _model(seed, product_backend="ictd-pure-u"):
    from mace_ictc.models import MACEICTC
    from oracle.model_ops import OracleOps
    torch.manual_seed(seed)
    return MACEICTC(channels=8, lmax=2, r_max=3.0, avg_num_neighbors=5.0, ops=OracleOps(),
                    product_backend=product_backend).double()


def _system():
    gen = torch.Generator().manual_seed(1)
    side = 8.0
    pos = torch.rand(30, 3, generator=gen, dtype=torch.float64) * side
    species = torch.randint(0, 3, (30,), generator=gen)
    d = pos[:, None, :] - pos[None, :, :]
    shift = -side * torch.round(d / side)
    dist = (d + shift).norm(dim=-1)
    i, j = torch.nonzero((dist < 3.0) & (dist > 0), as_tuple=True)
    return pos, species, j, i, shift[i, j]


def test_reference_names_round_trip():
    from mace_ictc.checkpoint import from_reference_state_dict, to_reference_state_dict
    source, target = _model(1), _model(2)
    ref = to_reference_state_dict(source)
    assert "interactions.0.linear_up.adapters.0.weight" in ref
    assert "products.0.linear.weight" in ref and ref["products.0.linear.weight"].dim() == 1
    from_reference_state_dict(target, ref)
    for (n, a), (m, b) in zip(source.named_parameters(), target.named_parameters()):
        assert n == m and torch.allclose(a, b, rtol=1e-15, atol=1e-15), n   # e3nn scaling round trip
    pos, species, src, dst, shift = _system()
    assert torch.allclose(source.energy(pos, species, src, dst, shift), target.energy(pos, species, src, dst, shift),
                          rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("source_backend,target_backend", [("ictd-bridge-u", "ictd-bridge-u"),
                                                            ("ictd-bridge-u", "ictd-pure-u"),
                                                            ("ictd-pure-u", "ictd-bridge-u")])
def test_product_backends_round_trip(source_backend, target_backend):
    """A bridge-U model writes the reference's bridge-U names (couplings, zero flags,
    basis bridge); checkpoints of either backend load into a model of either."""
    from mace_ictc.checkpoint import from_reference_state_dict, model_metadata, to_reference_state_dict
    source, target = _model(1, source_backend), _model(2, target_backend)
    ref = to_reference_state_dict(source)
    if source_backend == "ictd-bridge-u":
        assert "products.0.symmetric_contractions.symmetric_contractions.contractions.1.U_matrix_3" in ref
        assert "products.0.symmetric_contractions.symmetric_contractions.contractions.0.weights_max_zeroed" in ref
        assert "products.1.symmetric_contractions.basis_bridge.q_0" in ref
    assert model_metadata(target)["ictd_fix_product_backend"] == target_backend
    from_reference_state_dict(target, ref)
    pos, species, src, dst, shift = _system()
    # A new bridge-U block holds the ICTC couplings as FP32-rounded buffers (as the
    # reference's blocks hold theirs); into pure-U blocks they map against the exact
    # couplings, so that direction agrees to the couplings' rounding, not to FP64.
    rtol = 1e-9 if (source_backend, target_backend) == ("ictd-bridge-u", "ictd-pure-u") else 1e-13
    assert torch.allclose(source.energy(pos, species, src, dst, shift), target.energy(pos, species, src, dst, shift),
                          rtol=rtol, atol=0)


def test_bridge_model_rejects_unknown_product_keys():
    from mace_ictc.checkpoint import from_reference_state_dict, to_reference_state_dict
    model = _model(5, "ictd-bridge-u")
    ref = to_reference_state_dict(model)
    ref["products.0.symmetric_contractions.symmetric_contractions.contractions.0.extra"] = torch.zeros(1)
    with pytest.raises(NotImplementedError, match="extra"):
        from_reference_state_dict(model, ref)
    ref = to_reference_state_dict(model)
    del ref["products.1.symmetric_contractions.symmetric_contractions.contractions.0.weights_max"]
    with pytest.raises(KeyError, match="weights_max"):
        from_reference_state_dict(model, ref)
    ref = to_reference_state_dict(model)
    del ref["products.0.symmetric_contractions.symmetric_contractions.contractions.2.U_matrix_3"]
    before = {k: v.clone() for k, v in model.state_dict().items()}
    with pytest.raises(KeyError, match="couplings"):                  # bridge weights without their U
        from_reference_state_dict(model, ref)
    assert all(torch.equal(before[k], v) for k, v in model.state_dict().items() if k.startswith("products."))


def test_e3nn_linear_convention():
    """The product linear follows e3nn's o3.Linear: [mul_in, mul_out] blocks / sqrt(mul_in)."""
    from mace_ictc.checkpoint import from_reference_state_dict, to_reference_state_dict
    model = _model(3)
    ref = to_reference_state_dict(model)
    C = model.channels
    flat = torch.randn(C * C * (model.products[0].linear.lmax + 1), dtype=torch.float64)
    ref["products.0.linear.weight"] = flat
    from_reference_state_dict(model, ref)
    x = torch.randn(5, C, dtype=torch.float64)
    w0 = flat[:C * C].reshape(C, C)                                   # [in, out]
    want = x @ w0 / math.sqrt(C)                                      # e3nn: sum_i x_i w[i, o] / sqrt(C)
    got = x @ model.products[0].linear.weights[0].t()
    assert torch.allclose(got, want)


def test_identity_options_accepted_others_rejected():
    from mace_ictc.checkpoint import from_reference_state_dict, to_reference_state_dict
    model = _model(4)
    ref = to_reference_state_dict(model)
    ref["interactions.0.message_output_scale.log_scale"] = torch.zeros(3, 8, dtype=torch.float64)
    ref["readout_head_scales"] = torch.ones(2, dtype=torch.float64)
    accepted = from_reference_state_dict(model, ref)
    assert "readout_head_scales" in accepted
    ref["interactions.0.message_output_scale.log_scale"] = torch.full((3, 8), 0.1, dtype=torch.float64)
    with pytest.raises(NotImplementedError):
        from_reference_state_dict(model, ref)
    ref = to_reference_state_dict(model)
    ref["interactions.0.attn_q_proj.weight"] = torch.zeros(8, 8, dtype=torch.float64)
    with pytest.raises(NotImplementedError):
        from_reference_state_dict(model, ref)


def test_checkpoint_metadata_is_checked():
    """A reference checkpoint whose metadata differs from the model (e.g. the radial
    embedding's sqrt(num_basis) factor, which no parameter shows) is refused."""
    from mace_ictc.checkpoint import load_reference_checkpoint, model_metadata, to_reference_state_dict
    model = _model(5)
    meta = {k: v for k, v in model_metadata(model).items()}
    ckpt = {"e3trans_state_dict": to_reference_state_dict(model), "model_hyperparameters": meta,
            "dtype": "float32", "tensor_product_mode": "pure-cartesian-ictd-fix"}
    load_reference_checkpoint(model, ckpt)
    bridge = dict(ckpt, model_hyperparameters=dict(meta, ictd_fix_product_backend="ictd-bridge-u"))
    load_reference_checkpoint(model, bridge)      # bridge-U metadata is accepted (weights map exactly)
    for key, value in (("radial_sqrt_num_basis", True), ("ictd_fix_product_backend", "native-mace"),
                       ("ictd_fix_first_layer_self_connection", False), ("avg_num_neighbors", 7.5),
                       ("lmax", 3)):
        bad = dict(ckpt, model_hyperparameters=dict(meta, **{key: value}))
        with pytest.raises(ValueError):
            load_reference_checkpoint(model, bad)
    missing = dict(ckpt, model_hyperparameters={k: v for k, v in meta.items() if k != "radial_sqrt_num_basis"})
    with pytest.raises(ValueError):
        load_reference_checkpoint(model, missing)


def test_model_defaults_follow_the_reference_constructor():
    """Reference defaults for new models: no sqrt(num_basis) radial factor, first-layer
    scalar self-connection (no message selector), atomic numbers H, C, O."""
    from mace_ictc.models import MACEICTC
    model = MACEICTC(channels=8, lmax=2)
    assert model.radial_sqrt_num_basis is False
    assert model.first_layer_self_connection is True
    first = model.interactions[0]
    assert first.self_connection is not None and first.message_selector is None and first.sc_lmax == 0
    assert model.atomic_numbers == (1, 6, 8)
    assert model.atomic_number_to_index.tolist()[:9] == [-1, 0, -1, -1, -1, -1, 1, -1, 2]
