"""Periodic neighbour list on the CUDA backend (cell list, destination-sorted CSR).

Replaces the reference's torch-only PBC radius graph
(``mace_ictc/utils/graph_utils.py:217-297``) for orthorhombic periodic boxes.
"""
import ctypes

import torch

from . import _native
from ._native import ptr, stream_of


def neighbor_list(pos: torch.Tensor, box, cutoff: float, receivers: int = None):
    """Edges (src, dst, shift) with |pos[dst] - pos[src] + shift| < cutoff, grouped by dst.

    ``receivers`` limits the destinations to atoms [0, receivers) (owned atoms of a
    spatial decomposition); sources still range over all atoms.
    Returns (src int64 [E], dst int64 [E], shift fp32 [E, 3], offsets int64 [R + 1]).
    One device-to-host read (the edge count) sizes the outputs.
    """
    if pos.dtype != torch.float32 or pos.device.type != "cuda" or pos.ndim != 2 or pos.shape[1] != 3:
        raise ValueError("neighbor_list requires CUDA FP32 positions [N, 3]")
    pos = pos.contiguous()
    atoms = pos.shape[0]
    rows = atoms if receivers is None else int(receivers)
    if not 0 <= rows <= atoms:
        raise ValueError("receivers must lie in [0, atoms]")
    box_arr = (ctypes.c_float * 3)(*[float(v) for v in box])
    lib = _native.library()
    size = int(lib.ictc_neighbor_workspace_bytes(atoms, box_arr, float(cutoff)))
    if size < 0:
        raise ValueError("neighbor_list needs an orthorhombic box with cutoff < L/2 and >= 3 cells per axis")
    workspace = torch.empty(max(size, 1), dtype=torch.uint8, device=pos.device)
    offsets = torch.empty(rows + 1, dtype=torch.int64, device=pos.device)
    stream = stream_of(pos)
    _native.call("ictc_neighbor_count_receivers", ptr(pos), int(atoms), rows, box_arr, float(cutoff), ptr(workspace),
                 size, ptr(offsets), stream)
    edges = int(offsets[rows].item())
    src = torch.empty(edges, dtype=torch.int64, device=pos.device)
    dst = torch.empty(edges, dtype=torch.int64, device=pos.device)
    shift = torch.empty(edges, 3, dtype=torch.float32, device=pos.device)
    if edges:
        _native.call("ictc_neighbor_fill_receivers", ptr(pos), int(atoms), rows, box_arr, float(cutoff),
                     ptr(workspace), size, ptr(offsets), ptr(src), ptr(dst), ptr(shift), stream)
    # The search guarantees bounds and receiver grouping: message CSR views of this
    # edge list need no device-to-host checks.
    from .message import mark_grouped, mark_trusted_graph
    mark_grouped(dst, True)
    mark_grouped(src, False)
    mark_trusted_graph(src, dst, atoms, rows)
    return src, dst, shift, offsets
