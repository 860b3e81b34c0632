"""Graph message on the CUDA backend: gather by source, TP, mask, sum into destinations.

Semantics of the reference message (``ictc_o3/backends/ascend/tensor_product.py:159-218``
and ``mace_ictc/models/pure_cartesian_ictd_fix.py:1801-1806,1913-1917``):

    out[n] = sum_{e: dst_e = n} mask_e * TP(x[src_e], Y_e, gates_e)

for the owned destinations n < dst_nodes (``_destination_nodes``,
``tensor_product.py:151-156``).  The CUDA kernels walk a destination-sorted CSR
(forward) and a source-sorted CSR (adjoint), accumulating node rows in registers:
no per-edge intermediate tensor, no atomics.  The CSRs are built once per graph
(stable sort, so every run sums in the same order) and cached on the index
tensors' identity and version.
"""
from __future__ import annotations

import weakref
from typing import Dict, Optional

import torch

from . import _native
from .cache import cache_of
from ._native import ptr, stream_of
from .tensor_product import (_weight_and_gates, _check, get_plan, product, split_output)


# ---------------------------------------------------------------------------
# Graph layout
# ---------------------------------------------------------------------------

class GraphCSR:
    """Destination- and source-sorted CSR views of an edge list (device tensors)."""

    def __init__(self, src: torch.Tensor, dst: torch.Tensor, src_nodes: int, dst_nodes: int):
        self.src, self.dst = src, dst
        self.src_nodes, self.dst_nodes = int(src_nodes), int(dst_nodes)
        self.edges = int(src.numel())
        self.dst_order, self.dst_offsets = _csr(dst, self.dst_nodes)
        self.src_order, self.src_offsets = _csr(src, self.src_nodes)


def mark_grouped(keys: torch.Tensor, grouped: bool):
    """Record that ``keys`` is (or is not) non-decreasing, so CSR views skip the check."""
    keys._ictc_grouped = (keys._version, bool(grouped))


def mark_trusted_graph(src, dst, src_nodes, dst_nodes):
    """Record bounds that the producer of an edge list guarantees (e.g. the neighbour
    search), so ``validate_graph`` needs no device-to-host read for it."""
    src._ictc_cuda_graph_bounds = (weakref.ref(dst), (src._version, dst._version, int(src_nodes), int(dst_nodes)))


def _csr(keys: torch.Tensor, nodes: int):
    """(order, offsets); order is None when the edges are already grouped by key.

    Offsets come from a binary search of the sorted keys (no host synchronisation);
    the grouping check is skipped for keys marked by their producer."""
    mark = getattr(keys, "_ictc_grouped", None)
    if mark is not None and mark[0] == keys._version:
        grouped = mark[1]
    else:
        grouped = keys.numel() == 0 or bool((keys[1:] >= keys[:-1]).all())
    order = None if grouped else torch.argsort(keys, stable=True)
    sorted_keys = keys if order is None else keys.index_select(0, order)
    bounds = torch.arange(nodes + 1, dtype=keys.dtype, device=keys.device)
    offsets = torch.searchsorted(sorted_keys, bounds)
    return order, offsets


def validate_graph(src, dst, src_nodes, dst_nodes, device):
    """Check index dtypes, shapes and bounds once per (tensor, version) (``ascendc/graph.py:7-19``)."""
    if (src.device != device or dst.device != device or src.dtype != torch.int64 or dst.dtype != torch.int64
            or src.ndim != 1 or dst.shape != src.shape):
        raise ValueError("Graph indices must be int64 vectors on the feature device")
    key = (src._version, dst._version, int(src_nodes), int(dst_nodes))
    cached = getattr(src, "_ictc_cuda_graph_bounds", None)
    if cached is not None and cached[0]() is dst and cached[1] == key:
        return
    if src.numel():
        lo_s, hi_s, lo_d, hi_d = torch.stack((src.amin(), src.amax(), dst.amin(), dst.amax())).cpu().tolist()
        if lo_s < 0 or lo_d < 0 or hi_s >= src_nodes or hi_d >= dst_nodes:
            raise ValueError("Graph index is outside the node array")
    src._ictc_cuda_graph_bounds = (weakref.ref(dst), key)


def graph_csr(src, dst, src_nodes, dst_nodes) -> GraphCSR:
    validate_graph(src, dst, src_nodes, dst_nodes, src.device)
    key = (src._version, dst._version, int(src_nodes), int(dst_nodes))
    cached = getattr(src, "_ictc_cuda_csr", None)
    if cached is not None and cached[0]() is dst and cached[1] == key:
        return cached[2]
    csr = GraphCSR(src, dst, src_nodes, dst_nodes)
    src._ictc_cuda_csr = (weakref.ref(dst), key, csr)
    return csr


def destination_nodes(owner, source_nodes: int) -> int:
    """Owned destination count; deployment may aggregate from a larger source halo."""
    nodes = getattr(owner, "_cuda_destination_nodes", source_nodes)
    if not isinstance(nodes, int) or isinstance(nodes, bool) or not 0 <= nodes <= source_nodes:
        raise ValueError("Destination node count must be between zero and the source node count")
    return nodes


# ---------------------------------------------------------------------------
# Operator over a fixed graph: trilinear in (node features, edge harmonics, edge gates)
# ---------------------------------------------------------------------------

class MessageOp:
    def __init__(self, plan, csr: GraphCSR, mask: Optional[torch.Tensor]):
        self.plan, self.csr, self.mask = plan, csr, mask

    def forward(self, x, y, g, w):
        plan, csr = self.plan, self.csr
        out = torch.empty(csr.dst_nodes, plan.output_width, device=x.device, dtype=torch.float32)
        if csr.dst_nodes:
            if csr.edges == 0:
                return out.zero_()
            _check(x, y, g, w, self.mask)
            _native.call("ictc_tp_message_forward", plan.handle, ptr(x), ptr(y), ptr(g), ptr(w), ptr(self.mask),
                         ptr(csr.src), ptr(csr.dst_order), ptr(csr.dst_offsets), ptr(out),
                         int(csr.dst_nodes), stream_of(x))
        return out

    def adjoint(self, x, y, g, w, grad, need):
        plan, csr = self.plan, self.csr
        dx = torch.empty_like(x) if need[0] else None
        dy = torch.empty_like(y) if need[1] else None
        dg = (torch.empty(csr.edges, plan.num_paths * plan.channels, device=x.device, dtype=torch.float32)
              if need[2] else None)
        if not any(need):
            return dx, dy, dg
        if csr.edges == 0:
            return (None if dx is None else dx.zero_()), dy, dg
        _check(x, y, g, w, grad, self.mask)
        _native.call("ictc_tp_message_backward", plan.handle, ptr(x), ptr(y), ptr(g), ptr(w), ptr(self.mask),
                     ptr(csr.dst), ptr(csr.src_order), ptr(csr.src_offsets), ptr(grad),
                     ptr(dx), ptr(dy), ptr(dg), int(csr.src_nodes), stream_of(x))
        return dx, dy, dg


# ---------------------------------------------------------------------------
# Entry points
# ---------------------------------------------------------------------------

def packed_graph_message(owner, layout, features, harmonics, gates, src, dst, mask=None, dst_nodes=None):
    """Packed node features [N, C(Li+1)^2] -> packed messages [dst_nodes, output_width]."""
    src_nodes = features.shape[0]
    dst_nodes = destination_nodes(owner, src_nodes) if dst_nodes is None else int(dst_nodes)
    edges = src.numel()
    if owner.weight.device != features.device:
        raise ValueError("The tensor-product weight must be on the operands' CUDA device")
    plan = get_plan(owner, layout, features.device)
    if features.shape[1] != plan.feature_width or harmonics.shape != (edges, plan.harmonic_width):
        raise ValueError("Packed features/harmonics do not match the message degrees")
    if mask is not None:
        if mask.requires_grad:
            raise ValueError("The CUDA graph message does not differentiate the edge mask")
        if mask.shape not in ((edges,), (edges, 1)) or mask.device != features.device:
            raise ValueError("Expected an edge mask [E] or [E,1] on the feature device")
        mask = mask.reshape(edges).to(torch.float32).contiguous()
    csr = graph_csr(src, dst, src_nodes, dst_nodes)
    w, g = _weight_and_gates(owner, gates, edges)
    if g is not None and g.shape != (edges, plan.num_paths * plan.channels):
        raise ValueError("External graph gates must have shape [E,P*C] or [E,P,C]")
    return product(MessageOp(plan, csr, mask), w, features.contiguous(), harmonics.contiguous(), g)


def graph_message(owner, features: Dict[int, torch.Tensor], harmonics: Dict[int, torch.Tensor], gates,
                  src, dst, mask=None, *, edge_chunk_size=16384) -> Dict[int, torch.Tensor]:
    """Block interface of the hook site (``pure_cartesian_ictd_fix.py:1787-1800``).

    features: l -> [N, C, 2l+1]; harmonics: l -> [E, 1, 2l+1]; gates [E, P, C] or
    [E, P*C]; returns l -> [dst_nodes, count_l*C, 2l+1].  ``edge_chunk_size`` is
    validated for API compatibility; the kernels keep no per-edge intermediate,
    so no chunking is needed.
    """
    if edge_chunk_size is not None and (not isinstance(edge_chunk_size, int) or isinstance(edge_chunk_size, bool)
                                        or edge_chunk_size < 1):
        raise ValueError("Edge chunk size must be a positive integer")
    sample = next(iter(features.values()))
    rows, channels = sample.shape[0], int(owner.channels)
    input_lmax = max(p[0] for p in owner.paths)
    edge_lmax = max(p[1] for p in owner.paths)
    edges = src.numel()
    x = torch.cat([features[l].reshape(rows, channels * (2 * l + 1)) for l in range(input_lmax + 1)], 1)
    y = torch.cat([harmonics[l].reshape(edges, 2 * l + 1) for l in range(edge_lmax + 1)], 1)
    out = packed_graph_message(owner, "mul_ir", x, y, gates, src, dst, mask)
    return split_output(owner, out)


def radial_graph_message(owner, features: Dict[int, torch.Tensor], harmonics: Dict[int, torch.Tensor], radial,
                         edge_features: torch.Tensor, src, dst, mask=None, *, edge_chunk_size=None):
    """Message whose gates come from the interaction's radial network
    (``backends/ascend/capacity_message.py:109``; hook site ``pure_cartesian_ictd_fix.py:1787-1800``).

    ``radial`` is the block's ``fc`` (``nn.Sequential`` of four bias-free Linear layers,
    hidden width 64, with normalised SiLU modules between them: modules whose
    ``_scale`` is 1.6791767923989418, as the reference's ``_Normalize2MomSiLU``).  Its gates are produced
    by the fused tensor-core radial kernels, which keep the hidden activations on
    chip, and fed to ``graph_message``.  Returns None (the caller keeps its own path)
    when ``radial`` is not that network or its last layer does not produce P*C gates,
    as the reference does for networks it does not stream."""
    from . import radial as radial_kernels
    if edge_chunk_size is not None and (not isinstance(edge_chunk_size, int) or isinstance(edge_chunk_size, bool)
                                        or edge_chunk_size < 1):
        raise ValueError("Edge chunk size must be positive")
    if type(radial) is not torch.nn.Sequential or len(radial) == 0:
        return None
    linears = [m for m in radial if isinstance(m, torch.nn.Linear)]
    acts = [m for m in radial if not isinstance(m, torch.nn.Linear)]
    if (len(linears) != 4 or len(acts) != 3 or any(m.bias is not None for m in linears)
            or not isinstance(radial[-1], torch.nn.Linear)
            or any(getattr(m, "_scale", None) != radial_kernels.SILU_SCALE for m in acts)):
        return None
    sample = next(iter(features.values()))
    if linears[-1].out_features != owner.num_paths * sample.shape[1]:
        return None
    shape = (linears[0].in_features, linears[0].out_features, linears[-1].out_features)
    if not radial_kernels.supported(*shape):
        return None
    store = cache_of(radial, "_ictc_radial_plan")
    plan = store.get("plan")
    if plan is None:
        plan = store["plan"] = radial_kernels.RadialPlan()
    gates = radial_kernels.radial_gates(linears, edge_features, plan)
    return graph_message(owner, features, harmonics, gates, src, dst, mask, edge_chunk_size=edge_chunk_size)
