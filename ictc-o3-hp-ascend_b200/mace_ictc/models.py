"""MACE-ICTC model on the CUDA backend (the caller of the hot path).

Structure of the reference model (``mace_ictc/models/pure_cartesian_ictd_fix.py``):

* one-hot species -> ``node_embedding`` (Linear S -> C), scalar node features;
* per interaction layer (``ICTDResidualInteractionBlock.forward`` :1762-2056):
  ``linear_up`` (per-degree channel linear), radial MLP ``fc`` on the Bessel x
  polynomial-cutoff embedding (8 -> 64 -> 64 -> 64 -> P*C, normalised SiLU,
  :1545-1553), the TP graph message summed into receivers, ``message_linear``
  (path-preserving, :629-661) divided by the average neighbour count, and an
  element-conditioned self-connection of the layer input (layers after the first,
  :2381-2440; without it the message goes through an element-conditioned selector);
* product block (:1145-1199): symmetric contraction -> per-degree channel linear
  -> + self-connection (``_add_product_self_connection`` :94-118); product
  targets are lmax for every layer but the last, which targets scalars;
* energy readouts: a linear scalar readout per intermediate layer, an MLP
  readout (C -> 16 -> 1, normalised SiLU) after the last (:1400-1420, :3070-3100);
* forces = -dE/dpos (``mace_ictc/hp/runtime.py:84-121``).

The three hot operators (edge harmonics, TP graph message, symmetric
contraction) are taken from an ``ops`` object; the default is the CUDA backend.
On CUDA tensors the per-degree channel linears run as the backend's channel-mix
kernel and the radial MLP as its fused tensor-core kernels; on CPU tensors (tests
with the oracle ops) the same modules use plain torch matrix products.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ictc_o3.backends.cuda.cache import cache_of
from ictc_o3.basis.ictd_irreps import EdgeWeightedPathPreservingTensorProduct, operator_paths
from ictc_o3.ops.symmetric_contraction import (ICTDBridgeUSymmetricContractionSO3,
                                               ICTDPureUSymmetricContractionSO3)

SILU_SCALE = 1.6791767923989418  # normalised SiLU (pure_cartesian_ictd_fix.py:610-619)


class CudaOps:
    """The hot operators on the CUDA backend."""

    def harmonics(self, n, lmax):
        from ictc_o3.backends.cuda.geometry import direction_harmonics
        return direction_harmonics(n, lmax)

    def edge_geometry(self, vec, r_max, num_basis, p, basis_norm=True):
        """(unit vectors, radial embedding, cutoff mask): one fused kernel each way."""
        from ictc_o3.backends.cuda.geometry import edge_geometry
        return edge_geometry(vec, r_max, num_basis, p, basis_norm)

    def message(self, tp, features, harmonics, gates, src, dst, mask, dst_nodes):
        from ictc_o3.backends.cuda.message import packed_graph_message
        return packed_graph_message(tp, "mul_ir", features, harmonics, gates, src, dst, mask, dst_nodes)

    def contraction(self, module, features, species):
        return module(features, node_type_idx=species)

    def radial(self, fc, feats):
        """Gates of the radial MLP on the fused tensor-core kernels; a shape the kernels do
        not support raises (there is no library fallback)."""
        from ictc_o3.backends.cuda import radial
        linears = [m for m in fc if isinstance(m, nn.Linear)]
        shape = (linears[0].in_features, linears[0].out_features, linears[-1].out_features)
        store = cache_of(fc, "_ictc_radial_plan")
        plan = store.get("plan")
        if plan is None:
            if not radial.supported(*shape):
                raise ValueError(f"radial MLP shape (features, hidden, gates) = {shape} is not supported by the "
                                 "fused radial kernels")
            plan = store["plan"] = radial.RadialPlan()
        return radial.radial_gates(linears, feats, plan)


# ---------------------------------------------------------------------------
# Radial embedding (mace_ictc/models/radial_basis.py:11-92)
# ---------------------------------------------------------------------------

def polynomial_cutoff(r, r_max, p):
    x = r / r_max
    env = (1.0 - ((p + 1.0) * (p + 2.0) / 2.0) * x.pow(p) + p * (p + 2.0) * x.pow(p + 1)
           - (p * (p + 1.0) / 2.0) * x.pow(p + 2))
    return env * (r < r_max).to(r.dtype)


def radial_embedding(r, r_max, num_basis=8, p=5, sqrt_num_basis_norm=True):
    """Bessel basis sqrt(2/r_max) sin(n pi r / r_max) / r times the polynomial envelope."""
    freq = math.pi / r_max * torch.arange(1, num_basis + 1, dtype=r.dtype, device=r.device)
    emb = math.sqrt(2.0 / r_max) * torch.sin(r.unsqueeze(-1) * freq) / r.clamp_min(1e-12).unsqueeze(-1)
    emb = emb * polynomial_cutoff(r, r_max, p).unsqueeze(-1)
    if sqrt_num_basis_norm:
        emb = emb * math.sqrt(num_basis)
    return emb


class NormalizedSiLU(nn.Module):
    _scale = SILU_SCALE

    def forward(self, x):
        return F.silu(x) * SILU_SCALE


# ---------------------------------------------------------------------------
# Equivariant channel linears on flat features (degree blocks [C][2l+1])
# ---------------------------------------------------------------------------

def _blocks(x, widths, lmax):
    n = x.shape[0]
    out, offset = [], 0
    for l in range(lmax + 1):
        w = widths[l] * (2 * l + 1)
        out.append(x[:, offset:offset + w].reshape(n, widths[l], 2 * l + 1))
        offset += w
    return out


def _merge(blocks):
    n = blocks[0].shape[0]
    return torch.cat([b.reshape(n, b.shape[1] * b.shape[2]) for b in blocks], -1)


class ChannelLinearSO3(nn.Module):
    """Per-degree channel mixing, in_l -> out channels (EquivariantChannelLinearSO3 / PathPreservingLinearSO3)."""

    def __init__(self, in_channels, out_channels, lmax, init="normal"):
        super().__init__()
        self.lmax = lmax
        self.in_channels = list(in_channels) if isinstance(in_channels, (list, tuple)) else [in_channels] * (lmax + 1)
        self.out_channels = out_channels
        self.weights = nn.ParameterList()
        for l in range(lmax + 1):
            w = torch.empty(out_channels, self.in_channels[l])
            if init == "identity" and self.in_channels[l] == out_channels:
                nn.init.eye_(w)
            else:
                nn.init.normal_(w, std=1.0 / math.sqrt(max(self.in_channels[l], 1)))
            self.weights.append(nn.Parameter(w))

    def forward(self, x, scale: float = 1.0):
        if x.is_cuda:
            from ictc_o3.backends.cuda.linear import channel_mix
            return channel_mix(x, list(self.weights), scale=scale)
        blocks = _blocks(x, self.in_channels, self.lmax)
        out = _merge([torch.matmul(self.weights[l], b) for l, b in enumerate(blocks)])
        return out if scale == 1.0 else out * scale


class ElementLinearSO3(nn.Module):
    """Per-element, per-degree channel mixing (ElementConditionedLinearSO3)."""

    def __init__(self, num_elements, channels, lmax, init="normal"):
        super().__init__()
        self.lmax, self.channels, self.num_elements = lmax, channels, num_elements
        w = torch.empty(num_elements, lmax + 1, channels, channels)
        if init == "identity":
            w.copy_(torch.eye(channels).expand_as(w))
        else:
            nn.init.normal_(w, std=1.0 / math.sqrt(channels))
        self.weight = nn.Parameter(w)

    def forward(self, x, groups, species=None):
        if x.is_cuda and species is not None:
            from ictc_o3.backends.cuda.linear import channel_mix
            return channel_mix(x, [self.weight[:, l] for l in range(self.lmax + 1)], species=species,
                               num_elements=self.num_elements)
        blocks = _blocks(x, [self.channels] * (self.lmax + 1), self.lmax)
        outs = []
        for l, b in enumerate(blocks):
            out = torch.empty_like(b)
            for s, idx in enumerate(groups):
                if idx.numel():
                    out.index_copy_(0, idx, torch.matmul(self.weight[s, l], b.index_select(0, idx)))
            outs.append(out)
        return _merge(outs)


def species_groups(species: torch.Tensor, num_elements: int):
    """Node indices of every species (cached on the tensor's identity and version)."""
    key = (species._version, num_elements)
    cached = getattr(species, "_ictc_species_groups", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    order = torch.argsort(species, stable=True)
    counts = torch.bincount(species, minlength=num_elements).cpu().tolist()
    groups, start = [], 0
    for c in counts:
        groups.append(order[start:start + c])
        start += c
    species._ictc_species_groups = (key, groups)
    return groups


# ---------------------------------------------------------------------------
# Blocks
# ---------------------------------------------------------------------------

class InteractionBlock(nn.Module):
    def __init__(self, *, channels, lmax, input_lmax, num_elements, num_basis, avg_num_neighbors,
                 use_self_connection, sc_lmax):
        super().__init__()
        self.channels, self.lmax, self.input_lmax = channels, lmax, input_lmax
        self.avg_num_neighbors = avg_num_neighbors
        self.linear_up = ChannelLinearSO3(channels, channels, input_lmax)
        self.tp = EdgeWeightedPathPreservingTensorProduct(channels, lmax,
                                                          allowed_paths=operator_paths(input_lmax, lmax, lmax))
        with torch.no_grad():
            self.tp.weight.fill_(1.0)
        self.tp.weight.requires_grad_(False)
        hidden = 64
        self.fc = nn.Sequential(nn.Linear(num_basis, hidden, bias=False), NormalizedSiLU(),
                                nn.Linear(hidden, hidden, bias=False), NormalizedSiLU(),
                                nn.Linear(hidden, hidden, bias=False), NormalizedSiLU(),
                                nn.Linear(hidden, self.tp.num_paths * channels, bias=False))
        for m in self.fc:
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, std=1.0 / math.sqrt(m.in_features))
        counts = [channels * int(self.tp.path_counts_by_l.get(l, 0)) for l in range(lmax + 1)]
        self.message_linear = ChannelLinearSO3(counts, channels, lmax)
        self.sc_lmax = sc_lmax
        self.self_connection = ElementLinearSO3(num_elements, channels, sc_lmax) if use_self_connection else None
        self.message_selector = None if use_self_connection else ElementLinearSO3(num_elements, channels, lmax,
                                                                                  init="identity")

    def forward(self, ops, node_feats, edge_harmonics, edge_feats, src, dst, mask, groups, owned=None,
                species=None, exchange=None):
        """Messages into the first ``owned`` nodes (all nodes by default); ``groups`` and
        ``species`` (the owned nodes' species) select the element-conditioned weights.

        With ``exchange`` (spatial decomposition), ``node_feats`` holds the owned rows
        only: ``linear_up`` runs on them (it acts row by row, so it commutes with the
        halo copy and no ghost row is transformed), their ghost copies travel to the
        neighbours while the radial MLP runs, and the message reads the local rows."""
        owned = node_feats.shape[0] if owned is None else owned
        x_up = self.linear_up(node_feats)
        pending = exchange(x_up) if exchange is not None else None
        radial = getattr(ops, "radial", None)
        gates = radial(self.fc, edge_feats) if radial is not None else self.fc(edge_feats)
        if pending is not None:
            x_up = pending.finish()
        msg = ops.message(self.tp, x_up, edge_harmonics, gates, src, dst, mask, owned)
        message = self.message_linear(msg, scale=1.0 / max(self.avg_num_neighbors, 1e-8))
        if self.self_connection is None:
            return self.message_selector(message, groups, species), None
        sc_in = node_feats[:owned, :self.channels * (self.sc_lmax + 1) ** 2]
        return message, self.self_connection(sc_in, groups, species)


PRODUCT_MODULES = {"ictd-pure-u": ICTDPureUSymmetricContractionSO3,
                   "ictd-bridge-u": ICTDBridgeUSymmetricContractionSO3}


class ProductBlock(nn.Module):
    def __init__(self, *, channels, lmax, target_lmax, correlation, num_elements, product_backend="ictd-pure-u"):
        super().__init__()
        self.channels, self.target_lmax = channels, target_lmax
        self.symmetric_contractions = PRODUCT_MODULES[product_backend](
            num_elements=num_elements, channels=channels, lmax=lmax, target_lmax=target_lmax,
            correlation=correlation)
        self.linear = ChannelLinearSO3(channels, channels, target_lmax)

    def forward(self, ops, message, sc, species):
        out = self.linear(ops.contraction(self.symmetric_contractions, message, species))
        if sc is not None:
            if sc.shape[-1] == out.shape[-1]:
                out = out + sc
            else:
                out = torch.cat([out[:, :self.channels] + sc[:, :self.channels], out[:, self.channels:]], -1)
        return out


class MACEICTC(nn.Module):
    """MACE-ICTC energy model; ``energy(...)`` and ``energy_and_forces(...)``."""

    def __init__(self, *, num_elements=None, channels=64, lmax=2, num_interactions=2, correlation=3, r_max=5.0,
                 num_basis=8, polynomial_cutoff_p=5, avg_num_neighbors=1.0, readout_hidden=16, ops=None,
                 atomic_numbers=(1, 6, 8), first_layer_self_connection=True, radial_sqrt_num_basis=False,
                 product_backend="ictd-pure-u"):
        """Defaults follow the reference constructor for new models: atomic numbers
        H, C, O (``mace_ictc/hp/runtime.py:7``), an element-conditioned scalar
        self-connection in the first layer (``mace_ictc/models/factory.py:17``,
        ``pure_cartesian_ictd_fix.py:2393-2395``) and the radial embedding without
        the sqrt(num_basis) factor (``radial_sqrt_num_basis=False``, :2191, :2325).
        A ``num_elements`` that differs from ``len(atomic_numbers)`` makes the
        elements anonymous: atomic numbers 1..num_elements.

        ``product_backend`` picks the symmetric-contraction parameterisation of the
        product blocks, with the reference's names (``ictd_fix_product_backend``,
        :2166): "ictd-pure-u" (ICTC couplings) or "ictd-bridge-u" (the reference's
        default; the couplings are buffers that its checkpoints overwrite).  Both run
        the same kernels and span the same couplings; checkpoints of either load
        into a model of either."""
        super().__init__()
        if product_backend not in PRODUCT_MODULES:
            raise ValueError(f"product_backend must be one of {tuple(PRODUCT_MODULES)}")
        self.product_backend = product_backend
        atomic_numbers = tuple(sorted({int(z) for z in atomic_numbers}))
        if not atomic_numbers or atomic_numbers[0] < 0:
            raise ValueError("atomic_numbers must be non-negative and not empty")
        if num_elements is not None and num_elements != len(atomic_numbers):
            atomic_numbers = tuple(range(1, num_elements + 1))   # anonymous elements 1..S
        self.atomic_numbers = atomic_numbers
        num_elements = len(atomic_numbers)
        table = torch.full((max(atomic_numbers) + 1,), -1, dtype=torch.long)
        table[list(atomic_numbers)] = torch.arange(num_elements)
        self.register_buffer("atomic_number_to_index", table, persistent=False)
        self.num_elements, self.channels, self.lmax = num_elements, channels, lmax
        self.r_max, self.num_basis, self.p = float(r_max), num_basis, polynomial_cutoff_p
        self.first_layer_self_connection = bool(first_layer_self_connection)
        self.radial_sqrt_num_basis = bool(radial_sqrt_num_basis)
        self.avg_num_neighbors = float(avg_num_neighbors)
        self.correlation = int(correlation)
        self.preserve_edge_order = False
        self.ops = CudaOps() if ops is None else ops
        self.node_embedding = nn.Linear(num_elements, channels, bias=False)
        self.interactions = nn.ModuleList()
        self.products = nn.ModuleList()
        for layer in range(num_interactions):
            target = lmax if layer < num_interactions - 1 else 0
            first_sc = self.first_layer_self_connection and layer == 0
            self.interactions.append(InteractionBlock(
                channels=channels, lmax=lmax, input_lmax=0 if layer == 0 else lmax, num_elements=num_elements,
                num_basis=num_basis, avg_num_neighbors=avg_num_neighbors, use_self_connection=layer > 0 or first_sc,
                sc_lmax=0 if first_sc else target))
            self.products.append(ProductBlock(channels=channels, lmax=lmax, target_lmax=target,
                                              correlation=correlation, num_elements=num_elements,
                                              product_backend=product_backend))
        self.layer_readouts = nn.ModuleList([nn.Linear(channels, 1, bias=False)
                                             for _ in range(num_interactions - 1)])
        self.last_readout = nn.Sequential(nn.Linear(channels, readout_hidden, bias=False), NormalizedSiLU(),
                                          nn.Linear(readout_hidden, 1, bias=False))

    @staticmethod
    def edge_vectors(pos, src, dst, shift_vectors=None):
        vec = pos[dst] - pos[src]
        return vec if shift_vectors is None else vec + shift_vectors

    def edge_features(self, vec):
        """Harmonics, radial embedding and cutoff mask of edge vectors r_e = pos[dst] - pos[src] + shift."""
        geometry = getattr(self.ops, "edge_geometry", None)
        if geometry is not None:
            n, feats, mask = geometry(vec, self.r_max, self.num_basis, self.p, self.radial_sqrt_num_basis)
        else:
            length = vec.norm(dim=1)
            n = vec / length.clamp_min(1e-8).unsqueeze(-1)
            feats = radial_embedding(length, self.r_max, self.num_basis, self.p, self.radial_sqrt_num_basis)
            mask = (length <= self.r_max).to(vec.dtype).detach()
        harmonics = self.ops.harmonics(n, self.lmax)
        return harmonics, feats, mask

    def edge_inputs(self, pos, src, dst, shift_vectors):
        return self.edge_features(self.edge_vectors(pos, src, dst, shift_vectors))

    def node_energies(self, pos, species, src, dst, shift_vectors=None, layers=None):
        """Per-node energies [N] (sum of the layer readouts)."""
        return self.node_energies_from_vectors(self.edge_vectors(pos, src, dst, shift_vectors), species, src, dst,
                                               layers=layers)

    def node_energies_from_vectors(self, vec, species, src, dst, layers=None, owned=None, exchange=None,
                                   phases=None, owned_species=None):
        """Energies of the first ``owned`` nodes from edge vectors.

        Spatial decomposition (``mace_ictc/interfaces/ascend_lammps.py:286-333``,
        compact owned outputs): rows ``[0, owned)`` are this rank's atoms and the rest
        are ghost copies; every edge's receiver ``dst`` is an owned row.  Messages,
        products and readouts run on owned rows only, and in each later layer
        ``exchange`` starts the copy of the owned rows [owned, W] to the neighbours
        (its ``finish()`` gives all local rows: owned rows followed by the ghosts'
        rows from their owners).  ``phases`` (a ``StepPhases``) receives marks.
        ``owned_species`` may pass the owned rows' species as a tensor that lives
        across steps (its species tiles are then built once, not every step).
        """
        n_local = species.shape[0]
        owned = n_local if owned is None else int(owned)
        if owned != n_local and exchange is None:
            raise ValueError("ghost rows need an exchange to refresh their features")
        own_species = species if owned == n_local else species[:owned]
        if owned_species is not None:
            if owned_species.shape != (owned,):
                raise ValueError("owned_species must hold one species per owned row")
            own_species = owned_species
        # The CUDA linears take species directly; node index groups serve the torch path.
        groups = None if species.is_cuda else species_groups(own_species, self.num_elements)
        mark = (lambda name: phases.mark(name, vec.device)) if phases is not None else (lambda name: None)
        harmonics, feats, mask = self.edge_features(vec)
        mark("edge_geometry")
        h = self.node_embedding.weight.t().index_select(0, species)
        energy = None
        count = len(self.interactions) if layers is None else layers
        for layer in range(count):
            message, sc = self.interactions[layer](self.ops, h, harmonics, feats, src, dst, mask, groups, owned,
                                                   own_species, exchange=exchange if layer else None)
            mark(f"layer{layer}.interaction")
            h = self.products[layer](self.ops, message, sc, own_species)
            readout = (self.layer_readouts[layer](h[:, :self.channels]) if layer < len(self.interactions) - 1
                       else self.last_readout(h[:, :self.channels]))
            energy = readout if energy is None else energy + readout
            mark(f"layer{layer}.product")
        return energy.squeeze(-1)

    def energy(self, pos, species, src, dst, shift_vectors=None, batch=None, num_graphs=1):
        e = self.node_energies(pos, species, src, dst, shift_vectors)
        if batch is None:
            return e.sum().reshape(1)
        return torch.zeros(num_graphs, dtype=e.dtype, device=e.device).index_add(0, batch, e)

    def energy_and_forces(self, pos, species, src, dst, shift_vectors=None, batch=None, num_graphs=1,
                          training=False):
        pos = pos.detach().requires_grad_(True) if not pos.requires_grad else pos
        energy = self.energy(pos, species, src, dst, shift_vectors, batch, num_graphs)
        (grad,) = torch.autograd.grad(energy.sum(), [pos], create_graph=training)
        return energy, -grad
