"""Model-level API of the CUDA backend: construction, coverage check, configuration
and force evaluation.

Same entry points and arguments as the reference's model runtime
(``mace_ictc/hp/runtime.py``: ``create_model`` :7, ``energy_and_forces`` :84,
``check_model`` :123, ``configure_model`` :132; the device configuration it
delegates to is ``mace_ictc/ascend/runtime.py:10-91``).  The model is
``mace_ictc.models.MACEICTC`` with the reference's defaults for new models.
There is no reference (CPU) path in this package: every operator runs on the
CUDA kernels, and a request for the reference path raises.
"""
from __future__ import annotations

from typing import Optional

import torch

_SUPPORTED_LMAX = (1, 2, 3)


def _positive_int(value, name):
    if not isinstance(value, int) or isinstance(value, bool) or value < 1:
        raise ValueError(f"{name} must be a positive integer")


def create_model(*, channels=64, lmax=3, edge_lmax=None, num_interactions=2, correlation=3, use_reduced_cg=False,
                 atomic_numbers=(1, 6, 8), cutoff=5.0, avg_num_neighbors=50.0, device="cuda",
                 dtype=torch.float32, electrostatics=None):
    """A freshly initialised MACE-ICTC model on the CUDA backend (not a trained potential).

    Bridge-U product blocks, as the reference's factory builds (its couplings are the
    ICTC ones until a reference checkpoint is loaded)."""
    from .models import MACEICTC
    _positive_int(num_interactions, "num_interactions")
    _positive_int(channels, "channels")
    _positive_int(correlation, "correlation")
    if correlation not in (1, 2, 3):
        raise ValueError("correlation must be 1, 2 or 3")
    if not isinstance(use_reduced_cg, bool):
        raise TypeError("use_reduced_cg must be a boolean")
    if use_reduced_cg:
        raise ValueError("the CUDA backend uses the full CG coupling; reduced-basis generation is not enabled")
    if lmax not in _SUPPORTED_LMAX:
        raise ValueError(f"lmax must be one of {_SUPPORTED_LMAX}")
    edge_lmax = lmax if edge_lmax is None else edge_lmax
    if edge_lmax != lmax:
        raise ValueError("the CUDA backend's interaction uses edge_lmax == lmax")
    if electrostatics is not None:
        raise ValueError("long-range electrostatics are not part of the CUDA backend")
    if dtype != torch.float32 or torch.device(device).type != "cuda":
        raise ValueError("the CUDA backend runs FP32 models on CUDA devices")
    model = MACEICTC(channels=channels, lmax=lmax, num_interactions=num_interactions, correlation=correlation,
                     r_max=cutoff, avg_num_neighbors=avg_num_neighbors, atomic_numbers=atomic_numbers,
                     product_backend="ictd-bridge-u")
    return model.to(device)


def check_model(model, *, training=False, capture=False):
    """Coverage of ``model`` by the CUDA kernels, without modifying it."""
    from .models import MACEICTC
    reasons = []
    if not isinstance(model, MACEICTC):
        return {"supported": False, "backend": "cuda", "reasons": ["Expected the MACE-ICTC model"]}
    if any(p.device.type != "cuda" or p.dtype != torch.float32 for p in model.parameters()):
        reasons.append("All model parameters must already be CUDA FP32")
    if model.lmax not in _SUPPORTED_LMAX:
        reasons.append(f"lmax must be one of {_SUPPORTED_LMAX}")
    if model.correlation not in (1, 2, 3):
        reasons.append("The symmetric contraction supports correlation 1, 2 and 3")
    if capture:
        reasons.append("Graph capture is not qualified; use eager execution")
    return {"supported": not reasons, "backend": "cuda", "reasons": reasons}


def configure_model(model, *, training=False, policy="auto", layout="packed", capture=False,
                    message_chunk_edges=None, electrostatics_backend="auto"):
    """Select the CUDA operators for ``model`` (sets ``_cuda_hp`` on every module).

    ``policy``: "auto" selects the kernels when ``check_model`` supports the model,
    "generated" requires them, "reference" is refused (this package has no CPU path).
    ``message_chunk_edges`` is validated and recorded; the message kernels keep no
    per-edge intermediate, so no chunking is needed.  ``layout`` "packed" and
    "fused_pack" both run the packed kernels.  Electrostatics are not part of this
    backend: ``electrostatics_backend`` must be "auto" or "none"."""
    from .models import CudaOps
    if layout not in ("packed", "fused_pack"):
        raise ValueError("layout must be packed or fused_pack")
    if policy not in ("auto", "generated", "reference"):
        raise ValueError("policy must be auto, generated or reference")
    if policy == "reference":
        raise ValueError("the CUDA backend has no reference path; use the reference package for CPU evaluation")
    if electrostatics_backend not in ("auto", "none"):
        raise ValueError("electrostatics are not part of the CUDA backend")
    edge_chunk_size = message_chunk_edges
    if edge_chunk_size is not None and (not isinstance(edge_chunk_size, int) or isinstance(edge_chunk_size, bool)
                                        or edge_chunk_size < 1):
        raise ValueError("edge_chunk_size must be a positive integer or None for automatic sizing")
    coverage = check_model(model, training=training, capture=capture)
    if not coverage["supported"]:
        raise ValueError("CUDA backend unavailable for this model: " + "; ".join(coverage["reasons"]))
    # Destination-sorted CSR views are built on the device without changing the
    # caller's edge order, so the edge order is preserved.
    model.preserve_edge_order = True
    model.ops = CudaOps()
    for module in model.modules():
        module._cuda_hp = True
    for block in model.interactions:
        block._cuda_edge_chunk_size = edge_chunk_size
    return {"requested": policy, "selected": "generated", "backend": "cuda", "reasons": [],
            "arithmetic": "strict FP32 (tensor-core paths use a 3xTF32 split)",
            "edge_chunk_size": "auto" if edge_chunk_size is None else edge_chunk_size,
            "tensor_product_adjoint": "analytic", "counts": {"interactions": len(model.interactions)}}


def energy_and_forces(model, positions, atomic_numbers, batch, edge_src, edge_dst, edge_shifts, cell, *,
                      training=False, owned_mask: Optional[torch.Tensor] = None):
    """Energy [B], forces [N, 3] and atomic energies [N] of a prebuilt graph.

    ``edge_shifts`` are lattice coordinates [E, 3], ``cell`` is [B, 3, 3].  Edge vectors
    are pos[dst] - pos[src] + shift @ cell.  ``training=True`` keeps the graph for
    force-loss training (mixed second derivatives); otherwise results are detached.
    ``owned_mask`` [N] selects the atoms whose energies count (spatial decomposition);
    forces are taken for every supplied coordinate."""
    from ictc_o3.backends.cuda.geometry import edge_vectors
    from ictc_o3.backends.cuda.species import compact_species
    if torch.is_inference_mode_enabled():
        raise ValueError("Full forces require autograd; use no_grad instead of inference_mode")
    if positions.ndim != 2 or positions.shape[1] != 3 or cell.ndim != 3 or cell.shape[1:] != (3, 3):
        raise ValueError("Expected positions [N,3] and cell [B,3,3]")
    n = positions.shape[0]
    if atomic_numbers.shape != (n,) or batch.shape != (n,):
        raise ValueError("Atomic numbers and graph batch must have shape [N]")
    if owned_mask is not None and (owned_mask.shape != (n,) or owned_mask.requires_grad):
        raise ValueError("owned_mask must be a fixed [N] tensor")
    with torch.enable_grad():
        pos = positions if positions.requires_grad else positions.detach().requires_grad_(True)
        species = compact_species(model, atomic_numbers)
        vec = edge_vectors(pos, cell, edge_shifts, batch, edge_src, edge_dst)
        atomic = model.node_energies_from_vectors(vec, species, edge_src, edge_dst).reshape(n)
        selected = atomic if owned_mask is None else atomic * owned_mask.to(atomic)
        energy = selected.new_zeros(cell.shape[0]).index_add(0, batch, selected)
        # keep the coordinate dependency for graphs without edges
        forces = -torch.autograd.grad(energy.sum() + pos.sum() * 0.0, pos, create_graph=training,
                                      retain_graph=training)[0]
    result = {"energy": energy, "forces": forces, "atomic_energy": atomic}
    return result if training else {key: value.detach() for key, value in result.items()}
