"""The drop-in boundary: reference-named backend and model entry points (CPU checks).

Every function a reference hook site calls exists in ``ictc_o3.backends.cuda`` /
``mace_ictc.runtime`` with the reference's parameter names, refuses CPU tensors
(no CPU fallback), and the host-side logic (species mapping, configuration)
behaves as the reference's.  Numerical checks of the same entry points on a GPU
are in ``test_backend_api_gpu.py``.
"""
import inspect

import pytest
import torch

# (module, function, positional parameters, keyword-only parameters) of the reference:
# ictc_o3/backends/ascend/{capacity_message.py:109, tensor_product.py:89,159, geometry.py:6,
# species.py:9,20, linear.py:8,24, contraction.py:8}; mace_ictc/hp/runtime.py:7,84,123,132.
SIGNATURES = [
    ("ictc_o3.backends.cuda.message", "radial_graph_message",
     ["owner", "features", "harmonics", "radial", "edge_features", "src", "dst", "mask"], ["edge_chunk_size"]),
    ("ictc_o3.backends.cuda.message", "graph_message",
     ["owner", "features", "harmonics", "gates", "src", "dst", "mask"], ["edge_chunk_size"]),
    ("ictc_o3.backends.cuda.tensor_product", "tensor_product", ["owner", "features", "harmonics", "gates"], []),
    ("ictc_o3.backends.cuda.geometry", "edge_vectors",
     ["positions", "cell", "shifts", "batch", "source", "destination"], []),
    ("ictc_o3.backends.cuda.species", "validate_species", ["index", "count"], []),
    ("ictc_o3.backends.cuda.species", "compact_species", ["owner", "atomic_numbers"], []),
    ("ictc_o3.backends.cuda.linear", "channel_linear", ["features", "weight", "bias"], []),
    ("ictc_o3.backends.cuda.linear", "species_channel_linear", ["features", "weight", "species", "bias"], []),
    ("ictc_o3.backends.cuda.contraction", "factorized_contractions", ["owner", "x", "index"], []),
    ("mace_ictc.runtime", "create_model", [],
     ["channels", "lmax", "edge_lmax", "num_interactions", "correlation", "use_reduced_cg", "atomic_numbers",
      "cutoff", "avg_num_neighbors", "device", "dtype", "electrostatics"]),
    ("mace_ictc.runtime", "energy_and_forces",
     ["model", "positions", "atomic_numbers", "batch", "edge_src", "edge_dst", "edge_shifts", "cell"],
     ["training", "owned_mask"]),
    ("mace_ictc.runtime", "check_model", ["model"], ["training", "capture"]),
    ("mace_ictc.runtime", "configure_model", ["model"],
     ["training", "policy", "layout", "capture", "message_chunk_edges", "electrostatics_backend"]),
]


# ictc_o3/operators.py:232-234 and mace_ictc/hp/__init__.py of the reference (the mesh
# electrostatics the reference's ictc_o3 package adds are not part of this backend)
PUBLIC_OPERATORS = ["EdgeTensorProduct", "PackedGraphMessage", "GraphMessage", "direction_harmonics",
                    "create_symmetric_contraction", "configure_symmetric_contraction",
                    "channel_linear", "species_channel_linear", "normalized_silu", "strict_fp32"]


def test_public_import_paths():
    """The reference's import paths: ``from ictc_o3 import ...``, ``ictc_o3.operators``,
    ``mace_ictc.hp`` and ``mace_ictc.hp.runtime``."""
    import ictc_o3
    import ictc_o3.operators as operators
    import mace_ictc.hp as hp
    import mace_ictc.hp.runtime as hp_runtime
    import mace_ictc.runtime as runtime
    assert operators.__all__ == PUBLIC_OPERATORS and ictc_o3.__all__ == PUBLIC_OPERATORS
    for name in PUBLIC_OPERATORS:
        assert getattr(ictc_o3, name) is getattr(operators, name)
    assert hp.__all__ == [*PUBLIC_OPERATORS, "check_model", "configure_model", "create_model", "energy_and_forces"]
    for name in ("create_model", "energy_and_forces", "check_model", "configure_model"):
        assert getattr(hp, name) is getattr(runtime, name) is getattr(hp_runtime, name)


@pytest.mark.parametrize("module,name,positional,keyword", SIGNATURES, ids=[s[1] for s in SIGNATURES])
def test_reference_signature(module, name, positional, keyword):
    import importlib
    fn = getattr(importlib.import_module(module), name)
    params = inspect.signature(fn).parameters.values()
    pos = [p.name for p in params if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD)]
    kw = [p.name for p in params if p.kind == p.KEYWORD_ONLY]
    assert pos == positional and kw == keyword


def test_entry_points_refuse_cpu_tensors():
    """No CPU fallback: the CUDA entry points raise on CPU FP32 inputs."""
    from ictc_o3.backends.cuda.geometry import edge_vectors
    from ictc_o3.backends.cuda.linear import channel_linear, species_channel_linear
    x = torch.randn(4, 8, 3)
    with pytest.raises(ValueError):
        channel_linear(x, torch.randn(5, 8))
    with pytest.raises(ValueError):
        species_channel_linear(x, torch.randn(2, 5, 8), torch.zeros(4, dtype=torch.long))
    with pytest.raises(ValueError):
        edge_vectors(torch.randn(3, 3), torch.eye(3)[None], torch.zeros(2, 3), torch.zeros(3, dtype=torch.long),
                     torch.tensor([0, 1]), torch.tensor([1, 2]))


def test_compact_species_maps_and_validates():
    from ictc_o3.backends.cuda.species import compact_species, validate_species
    from mace_ictc.models import MACEICTC
    model = MACEICTC(channels=4, lmax=1, atomic_numbers=(8, 1, 6))
    z = torch.tensor([1, 6, 8, 8, 1])
    index = compact_species(model, z)
    assert index.tolist() == [0, 1, 2, 2, 0]
    assert compact_species(model, z) is index                      # remembered for the same tensor
    z[0] = 6                                                        # a new version is mapped again
    assert compact_species(model, z).tolist()[0] == 1
    for bad in ([2], [9], [-1], [200]):                             # unknown element / outside the table
        with pytest.raises(ValueError):
            compact_species(model, torch.tensor(bad))
    validate_species(torch.tensor([0, 2]), 3)
    with pytest.raises(ValueError):
        validate_species(torch.tensor([0, 3]), 3)


def test_check_and_configure_model_on_cpu_model():
    """A CPU model is reported unsupported; configure refuses it and the reference policy."""
    from mace_ictc.models import MACEICTC
    from mace_ictc.runtime import check_model, configure_model, create_model
    model = MACEICTC(channels=4, lmax=1)
    report = check_model(model, capture=True)
    assert report["backend"] == "cuda" and not report["supported"]
    assert any("CUDA FP32" in r for r in report["reasons"]) and any("capture" in r for r in report["reasons"])
    with pytest.raises(ValueError):
        configure_model(model)
    with pytest.raises(ValueError):
        configure_model(model, policy="reference")
    with pytest.raises(ValueError):
        configure_model(model, layout="dense")
    with pytest.raises(ValueError):
        create_model(device="cpu")
    with pytest.raises(ValueError):
        create_model(device="cuda", correlation=4)
    with pytest.raises(ValueError):
        create_model(device="cuda", use_reduced_cg=True)
