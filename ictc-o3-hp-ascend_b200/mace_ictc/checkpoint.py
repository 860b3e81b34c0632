"""State-dict compatibility with the reference ``PureCartesianICTDFix`` checkpoints.

Maps the parameter names of the reference model
(``mace_ictc/models/pure_cartesian_ictd_fix.py:2058-2765``) onto ``MACEICTC`` for
the configuration this backend implements (residual interaction blocks with the
path-preserving TP, pure-ICTC or bridge-U symmetric contraction product blocks, linear layer
readouts and the MLP last readout):

==============================================================  =====================================
reference key                                                   this model
==============================================================  =====================================
node_embedding.weight                                           node_embedding.weight
interactions.i.linear_up.adapters.l.weight      (:1519)         interactions.i.linear_up.weights.l
interactions.i.tp.weight                        (:1520)         interactions.i.tp.weight
interactions.i.fc.{0,2,4,6}.weight              (:1545-1553)    interactions.i.fc.{0,2,4,6}.weight
interactions.i.message_linear.weights.l         (:629-661)      interactions.i.message_linear.weights.l
interactions.i.self_connection.weights.l        (:335-392)      interactions.i.self_connection.weight[:, l]
interactions.i.message_selector.weights.l                       interactions.i.message_selector.weight[:, l]
products.i.symmetric_contractions.contractions.t.*  (:1202-1395) same names (weights_max, weights.j, U_matrix_nu)
products.i.symmetric_contractions.symmetric_contractions.*      bridge-U model: same names; pure-U model:
  (bridge-U, ops/symmetric_contraction.py:92-206)               weights mapped by ``_bridge_weights``
products.i.linear.weight  (e3nn o3.Linear, :1419)               products.i.linear.weights.l
layer_energy_readouts.i.readout.weight                          layer_readouts.i.weight
last_layer_energy_readout.linear_{1,2}.weight   (:1434-1449)    last_readout.{0,2}.weight
==============================================================  =====================================

The product linear is e3nn's ``o3.Linear`` on ``C x (0e + 1o + 2e + ...)``: its flat
weight holds one ``[mul_in, mul_out]`` block per degree, applied with the
``1/sqrt(mul_in)`` path normalisation, so ``W_l[out, in] = w_l[in, out] / sqrt(C)``.
Optional reference features this model does not implement (normalisations,
per-degree output scales, biases, attention, energy scale/shift, head scales) are
accepted only at their identity values; anything else raises.
"""
from __future__ import annotations

import math
import re
from typing import Dict, List

import torch


# Reference keys of optional features, with the check that makes them an identity.
def _identity(key: str, value: torch.Tensor) -> bool:
    if key.endswith("log_scale"):
        return bool(torch.all(value == 0))
    if re.search(r"\.bias(\.|$)", key):
        return bool(torch.all(value == 0))
    if key.endswith("readout_head_scales"):
        return bool(torch.all(value == 1))
    if key.endswith("energy_output_scale"):
        return value is None or bool(torch.all(value == 1))
    if key.endswith("energy_output_shift"):
        return value is None or bool(torch.all(value == 0))
    return False


def _e3nn_linear_to_blocks(flat: torch.Tensor, channels: int, lmax: int) -> List[torch.Tensor]:
    block = channels * channels
    if flat.numel() != block * (lmax + 1):
        raise ValueError(f"product linear weight has {flat.numel()} values, expected {block * (lmax + 1)}")
    return [flat[l * block:(l + 1) * block].reshape(channels, channels).t() / math.sqrt(channels)
            for l in range(lmax + 1)]


def _blocks_to_e3nn_linear(weights, channels: int) -> torch.Tensor:
    return torch.cat([(w.t() * math.sqrt(channels)).reshape(-1) for w in weights])


def _bridge_weights(module, tensors: Dict[str, torch.Tensor], where: str) -> Dict[str, torch.Tensor]:
    """Weights of one bridge-U contraction expressed in this model's pure-U paths.

    Both parameterisations are complete sets of chained couplings of the same
    degrees, so every bridge-U coupling tensor (the checkpoint's own ``U_matrix_nu``
    buffers, already in the ICTC basis) is an exact combination of the pure-U ones:
    U_bridge = U_pure A.  The contraction sum_p U[..., p] W[s, p, c] is then
    preserved by W_pure = A W_bridge.  A combination that does not reproduce the
    checkpoint's couplings (relative residual above 1e-5) raises."""
    import numpy as np
    out: Dict[str, torch.Tensor] = {}
    corr = module.correlation
    for nu in range(1, corr + 1):
        name = "weights_max" if nu == corr else f"weights.{corr - 1 - nu}"
        if f"U_matrix_{nu}" not in tensors or name not in tensors:
            raise KeyError(f"{where}: bridge-U checkpoint lacks U_matrix_{nu} or {name}")
        u_bridge = tensors[f"U_matrix_{nu}"].detach().double().cpu().numpy()
        u_pure = module._u64[nu]
        if u_bridge.shape[:-1] != u_pure.shape[:-1]:
            raise ValueError(f"{where}: U_matrix_{nu} shape {u_bridge.shape} does not match {u_pure.shape}")
        a = u_pure.reshape(-1, u_pure.shape[-1])
        b = u_bridge.reshape(-1, u_bridge.shape[-1])
        coef = np.linalg.lstsq(a, b, rcond=None)[0]                      # [P_pure, P_bridge]
        residual = np.linalg.norm(a @ coef - b) / max(np.linalg.norm(b), 1e-300)
        if residual > 1e-5:
            raise ValueError(f"{where}: bridge-U couplings of order {nu} are not spanned by this model's "
                             f"(relative residual {residual:.1e})")
        w = tensors[name]
        mapped = torch.einsum("pq,sqc->spc", torch.from_numpy(coef).to(w.dtype), w)
        out["weights_max" if nu == corr else f"weights.{corr - 1 - nu}"] = mapped
    return out


def _require_couplings(module, sub: Dict[str, torch.Tensor], prefix: str):
    lacking = [prefix + n for n in module.state_dict() if ".U_matrix_" in n and n not in sub]
    if lacking:
        raise KeyError(f"bridge-U checkpoint lacks its couplings: {lacking}")


def _load_bridge_module(module, sub: Dict[str, torch.Tensor], prefix: str, strict: bool, unknown: List[str],
                        bridge_named: bool):
    """Load reference product-block tensors (bridge-U names, or pure-U names moved
    under ``symmetric_contractions.``) into a bridge-U product module of this model:
    couplings, weights, zero flags and bridge matrices by name, coupling counts
    resized to the checkpoint's.  Bridge-U weights mean nothing without their own
    couplings, so a bridge-U block must bring every ``U_matrix_nu`` (checked before
    anything is loaded); a pure-U block without them keeps the ICTC couplings, which
    are its own."""
    if bridge_named:
        _require_couplings(module, sub, prefix)
    result = module.load_state_dict(sub, strict=False)
    unknown.extend(prefix + k for k in result.unexpected_keys)
    if strict:
        missing = [prefix + n for n, _ in module.named_parameters() if n not in sub]
        if missing:
            raise KeyError(f"parameters not set by the reference checkpoint: {missing}")


def from_reference_state_dict(model, state: Dict[str, torch.Tensor], strict: bool = True) -> List[str]:
    """Load a reference checkpoint's state dict into ``model`` (a ``MACEICTC``).

    Product blocks: into a pure-U model, pure-U checkpoints load by name and bridge-U
    ones (the reference's default, ``ICTDBridgeUSymmetricContractionSO3``) through
    ``_bridge_weights``; into a bridge-U model (``product_backend="ictd-bridge-u"``)
    both load by name, the couplings with them.  Returns the reference keys accepted
    as identities or as constants this model does not need.  With ``strict``,
    unknown keys and missing parameters raise."""
    from ictc_o3.ops.symmetric_contraction import ICTDBridgeUSymmetricContractionSO3
    own = dict(model.named_parameters())
    own.update(dict(model.named_buffers()))
    target: Dict[str, torch.Tensor] = {}
    accepted: List[str] = []
    unknown: List[str] = []
    element_blocks: Dict[str, Dict[int, torch.Tensor]] = {}
    bridge: Dict[tuple, Dict[str, torch.Tensor]] = {}
    direct: Dict[int, Dict[str, torch.Tensor]] = {}     # product blocks of a bridge-U model, by name
    bridge_named: set = set()                           # ... of those, the ones given under bridge-U names
    loaded: set = set()

    def bridge_model(i: int) -> bool:
        return i < len(model.products) and isinstance(model.products[i].symmetric_contractions,
                                                      ICTDBridgeUSymmetricContractionSO3)

    for key, value in state.items():
        if value is None:
            continue
        m = re.fullmatch(r"products\.(\d+)\.symmetric_contractions\."
                         r"(symmetric_contractions\.contractions\.(\d+)\.(.+)|basis_bridge\.q_\d+)", key)
        if m and bridge_model(int(m[1])):
            direct.setdefault(int(m[1]), {})[m[2]] = value
            if m[3] is not None:
                bridge_named.add(int(m[1]))
            continue
        if m and m[3] is None:
            accepted.append(key)                         # already folded into the U buffers
            continue
        if m:
            if m[4].endswith("_zeroed"):                 # flags of all-zero U orders
                accepted.append(key)
            else:
                bridge.setdefault((int(m[1]), int(m[3])), {})[m[4]] = value
            continue
        m = re.fullmatch(r"products\.(\d+)\.symmetric_contractions\.(contractions\.\d+\..+)", key)
        if m and bridge_model(int(m[1])):
            direct.setdefault(int(m[1]), {})["symmetric_contractions." + m[2]] = value
            continue
        m = re.fullmatch(r"interactions\.(\d+)\.linear_up\.adapters\.(\d+)\.weight", key)
        if m:
            target[f"interactions.{m[1]}.linear_up.weights.{m[2]}"] = value
            continue
        m = re.fullmatch(r"interactions\.(\d+)\.(tp\.weight|fc\.\d+\.weight|message_linear\.weights\.\d+)", key)
        if m:
            target[key] = value
            continue
        m = re.fullmatch(r"interactions\.(\d+)\.(self_connection|message_selector)\.weights\.(\d+)", key)
        if m:
            element_blocks.setdefault(f"interactions.{m[1]}.{m[2]}.weight", {})[int(m[3])] = value
            continue
        if key.startswith("products.") and ".symmetric_contractions.contractions." in key:
            target[key] = value
            continue
        m = re.fullmatch(r"products\.(\d+)\.linear\.weight", key)
        if m:
            lin = model.products[int(m[1])].linear
            for l, w in enumerate(_e3nn_linear_to_blocks(value, lin.out_channels, lin.lmax)):
                target[f"products.{m[1]}.linear.weights.{l}"] = w
            continue
        m = re.fullmatch(r"layer_energy_readouts\.(\d+)\.readout\.weight", key)
        if m:
            target[f"layer_readouts.{m[1]}.weight"] = value
            continue
        m = re.fullmatch(r"last_layer_energy_readout\.linear_([12])\.weight", key)
        if m:
            target[f"last_readout.{0 if m[1] == '1' else 2}.weight"] = value
            continue
        if key == "node_embedding.weight":
            target[key] = value
            continue
        if _identity(key, value):
            accepted.append(key)
            continue
        unknown.append(key)
    for name, blocks in element_blocks.items():
        target[name] = torch.stack([blocks[l] for l in sorted(blocks)], 1)
    for (i, t), tensors in bridge.items():
        module = model.products[i].symmetric_contractions.contractions[t]
        where = f"products.{i}.symmetric_contractions.symmetric_contractions.contractions.{t}"
        for name, value in _bridge_weights(module, tensors, where).items():
            target[f"products.{i}.symmetric_contractions.contractions.{t}.{name}"] = value
    for i in bridge_named:                              # before any block is loaded
        _require_couplings(model.products[i].symmetric_contractions, direct[i], f"products.{i}.symmetric_contractions.")
    for i, sub in direct.items():
        prefix = f"products.{i}.symmetric_contractions."
        _load_bridge_module(model.products[i].symmetric_contractions, sub, prefix, strict, unknown,
                            i in bridge_named)
        loaded.update(prefix + n for n, _ in model.products[i].symmetric_contractions.named_parameters())
    if strict and unknown:
        raise NotImplementedError(f"reference keys without a counterpart in this model: {unknown}")
    with torch.no_grad():
        for name, value in target.items():
            if name not in own:
                if strict:
                    raise KeyError(f"{name} (mapped from the reference checkpoint) is not a parameter of this model")
                continue
            if own[name].shape != value.shape:
                raise ValueError(f"{name}: shape {tuple(value.shape)} does not match {tuple(own[name].shape)}")
            own[name].copy_(value)
    if strict:
        missing = [n for n, p in model.named_parameters() if n not in target and n not in loaded]
        if missing:
            raise KeyError(f"parameters not set by the reference checkpoint: {missing}")
    return accepted


# Architecture metadata a reference checkpoint must carry (the keys the reference's
# multi-device engine requires, ``mace_ictc/interfaces/ascend_lammps.py:50-53``).
# Product backends whose checkpoints load onto this model (either backend): by name,
# or through the exact change of coupling basis (``_bridge_weights``) when a bridge-U
# checkpoint meets pure-U product blocks.
PRODUCT_BACKENDS = ("ictd-pure-u", "ictd-bridge-u")

REQUIRED_METADATA = ("channel_in", "lmax", "num_interaction", "avg_num_neighbors", "radial_sqrt_num_basis",
                     "polynomial_cutoff_p", "ictd_fix_product_backend")


def model_metadata(model) -> Dict[str, object]:
    """The reference metadata values that describe ``model``."""
    return {"channel_in": model.channels, "lmax": model.lmax, "num_interaction": len(model.interactions),
            "avg_num_neighbors": model.avg_num_neighbors, "radial_sqrt_num_basis": model.radial_sqrt_num_basis,
            "polynomial_cutoff_p": model.p, "ictd_fix_product_backend": model.product_backend,
            "ictd_fix_first_layer_self_connection": model.first_layer_self_connection,
            "max_radius": model.r_max, "tensor_product_mode": "pure-cartesian-ictd-fix", "dtype": "float32"}


def check_reference_metadata(model, metadata: Dict[str, object]):
    """Raise unless a reference checkpoint's architecture metadata describes ``model``.

    The state dict alone does not show every choice that changes the energy (the
    radial embedding's sqrt(num_basis) factor has no parameter), so a checkpoint
    whose metadata is missing or differs is refused rather than loaded into a model
    that would give different energies."""
    missing = [k for k in REQUIRED_METADATA if k not in metadata]
    if missing:
        raise ValueError(f"Missing model metadata: {missing}; re-save with the training configuration")
    want = model_metadata(model)
    bad = []
    for key, value in metadata.items():
        if key not in want:
            continue
        mine = want[key]
        if key == "ictd_fix_product_backend":
            same = str(value) in PRODUCT_BACKENDS
        elif isinstance(mine, float) or isinstance(value, float):
            same = abs(float(value) - float(mine)) <= 1e-9 * max(1.0, abs(float(mine)))
        elif isinstance(mine, bool):
            same = bool(value) == mine
        else:
            same = str(value).replace("torch.", "") == str(mine)
        if not same:
            bad.append(f"{key}: checkpoint {value!r}, model {mine!r}")
    if bad:
        raise ValueError("checkpoint does not describe this model: " + "; ".join(bad))


def load_reference_checkpoint(model, checkpoint: Dict[str, object], strict: bool = True) -> List[str]:
    """Load a reference training checkpoint (``Trainer.save_checkpoint``,
    ``mace_ictc/training/train_loop.py:2053-2077``): metadata check, then the weights
    of ``e3trans_state_dict``.  Returns the keys accepted as identities."""
    metadata = dict(checkpoint.get("model_hyperparameters", {}) or {})
    for key in ("dtype", "max_radius", "tensor_product_mode"):
        if key in checkpoint:
            metadata[key] = checkpoint[key]
    check_reference_metadata(model, metadata)
    return from_reference_state_dict(model, checkpoint["e3trans_state_dict"], strict=strict)


def to_reference_state_dict(model) -> Dict[str, torch.Tensor]:
    """The inverse mapping: a state dict with the reference's names and layouts."""
    out: Dict[str, torch.Tensor] = {"node_embedding.weight": model.node_embedding.weight.detach().clone()}
    for i, block in enumerate(model.interactions):
        p = f"interactions.{i}"
        for l, w in enumerate(block.linear_up.weights):
            out[f"{p}.linear_up.adapters.{l}.weight"] = w.detach().clone()
        out[f"{p}.tp.weight"] = block.tp.weight.detach().clone()
        for idx, m in enumerate(block.fc):
            if isinstance(m, torch.nn.Linear):
                out[f"{p}.fc.{idx}.weight"] = m.weight.detach().clone()
        for l, w in enumerate(block.message_linear.weights):
            out[f"{p}.message_linear.weights.{l}"] = w.detach().clone()
        for name in ("self_connection", "message_selector"):
            mod = getattr(block, name)
            if mod is not None:
                for l in range(mod.lmax + 1):
                    out[f"{p}.{name}.weights.{l}"] = mod.weight[:, l].detach().clone()
    for i, prod in enumerate(model.products):
        for k, v in prod.symmetric_contractions.state_dict().items():
            out[f"products.{i}.symmetric_contractions.{k}"] = v.detach().clone()
        out[f"products.{i}.linear.weight"] = _blocks_to_e3nn_linear(list(prod.linear.weights), prod.linear.out_channels)
    for i, r in enumerate(model.layer_readouts):
        out[f"layer_energy_readouts.{i}.readout.weight"] = r.weight.detach().clone()
    out["last_layer_energy_readout.linear_1.weight"] = model.last_readout[0].weight.detach().clone()
    out["last_layer_energy_readout.linear_2.weight"] = model.last_readout[2].weight.detach().clone()
    return out
