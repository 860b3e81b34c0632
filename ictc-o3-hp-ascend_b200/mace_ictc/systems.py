"""Synthetic atomic systems of the benchmark configurations (benchmark configs 3-5: 0.1 atoms per cubic angstrom).

H/C/O atoms with uniformly random species, placed uniformly at random in a
periodic cube at a given number density with a minimum pair distance (0.9 A):
atoms closer than the minimum to a lower-index atom are redrawn until no pair
violates it.  Generated on the GPU with the cell-list neighbour search.
"""
from __future__ import annotations

import torch


def random_system(atoms: int, *, density: float = 0.1, min_distance: float = 0.9, species: int = 3,
                  seed: int = 0, device="cuda", max_rounds: int = 200):
    """Positions [N, 3] (fp32), species [N] (int64) and the cubic box side."""
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    device = torch.device(device)
    side = (atoms / density) ** (1.0 / 3.0)
    gen = torch.Generator(device=device).manual_seed(seed)
    pos = torch.rand(atoms, 3, device=device, generator=gen, dtype=torch.float32) * side
    box = (side, side, side)
    for _ in range(max_rounds):
        src, dst, _, _ = neighbor_list(pos, box, min_distance)
        bad = torch.unique(torch.maximum(src, dst)) if src.numel() else src
        if bad.numel() == 0:
            break
        pos[bad] = torch.rand(bad.numel(), 3, device=device, generator=gen) * side
    else:
        raise RuntimeError("could not place atoms with the requested minimum distance")
    kinds = torch.randint(0, species, (atoms,), device=device, generator=gen)
    order = locality_order(pos, side)
    return pos[order].contiguous(), kinds[order].contiguous(), side


def locality_order(pos: torch.Tensor, side: float, cell: float = 5.0) -> torch.Tensor:
    """Atom permutation sorting atoms by (z, y, x) cell of width ~cell: neighbours then sit
    close in memory, so gathers of neighbour rows stay in L2."""
    n = max(1, int(side // cell))
    idx = torch.clamp((pos / side * n).long(), 0, n - 1)
    key = (idx[:, 2] * n + idx[:, 1]) * n + idx[:, 0]
    return torch.argsort(key, stable=True)
