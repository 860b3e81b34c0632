"""Equivariant per-degree channel linears on the CUDA backend.

Drop-in for the species-bank / channel linears of the reference
(``ictc_o3/backends/ascend/linear.py:8-46``; model sites
``mace_ictc/models/pure_cartesian_ictd_fix.py:335-392, 629-661, 2381-2440``): for
every degree l the block [C_in][2l+1] of a node row maps to [C_out][2l+1] by a
channel matrix (per species for the element-conditioned linears).  One kernel
launch per degree reads and writes the flat rows in place
(``ictc_channel_mix``).  The input gradient is the same operation with
transposed weights, so derivatives of any order compose; weight gradients use
device einsums.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from ictc_o3.autograd.adjoint_requirements import required_gradients
from . import _native
from ._native import ptr, stream_of


def tile_nodes() -> int:
    return int(_native.library().ictc_channel_mix_tile_nodes())


def species_layout(species: torch.Tensor, num_elements: int):
    """(order, counts): nodes sorted by species (stable) and the node count of each
    species, with a single device-to-host read; cached on the tensor's identity and
    version and shared by every per-species structure built from it."""
    key = (species._version, int(num_elements))
    cached = getattr(species, "_ictc_species_layout", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    index = species.to(torch.int64)
    order = torch.argsort(index, stable=True)
    sorted_species = index.index_select(0, order)
    bounds = torch.arange(num_elements + 1, dtype=torch.int64, device=species.device)
    edges = torch.searchsorted(sorted_species, bounds)
    if index.numel():
        probe = torch.cat([edges, sorted_species[:1], sorted_species[-1:]]).cpu().tolist()
        edges_h, lo, hi = probe[:-2], probe[-2], probe[-1]
        if lo < 0 or hi >= num_elements:
            raise ValueError("Species index is outside the element table")
    else:
        edges_h = [0] * (num_elements + 1)
    counts = [edges_h[s + 1] - edges_h[s] for s in range(num_elements)]
    result = (order, counts)
    try:
        species._ictc_species_layout = (key, result)
    except AttributeError:
        pass
    return result


def species_tiles_of(species: torch.Tensor, num_elements: int, nb: int):
    """Species-homogeneous node tiles [T, nb] (-1 padded) and their species [T] (int32)."""
    order, counts = species_layout(species, num_elements)
    tiles, tspecies, start = [], [], 0
    for s, count in enumerate(counts):
        if count:
            padded = -(-count // nb) * nb
            block = torch.full((padded,), -1, dtype=torch.int64, device=species.device)
            block[:count] = order[start:start + count]
            tiles.append(block.view(-1, nb))
            tspecies.append(torch.full((padded // nb,), s, dtype=torch.int32, device=species.device))
        start += count
    if tiles:
        return torch.cat(tiles).contiguous(), torch.cat(tspecies).contiguous()
    return (torch.empty(0, nb, dtype=torch.int64, device=species.device),
            torch.empty(0, dtype=torch.int32, device=species.device))


def species_node_tiles(species: torch.Tensor, num_elements: int):
    """Tiles of ictc_channel_mix_tile_nodes() nodes (cached on the tensor)."""
    nb = tile_nodes()
    key = (species._version, int(num_elements), nb)
    cached = getattr(species, "_ictc_mix_tiles", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    result = species_tiles_of(species, num_elements, nb)
    try:
        species._ictc_mix_tiles = (key, result)
    except AttributeError:
        pass
    return result


class _Spec:
    """Static part of one linear: species tiles (or None) and the output scale."""

    def __init__(self, tiles, scale: float):
        self.tiles = tiles                    # None or (tiles, tile_species)
        self.scale = float(scale)


def _launch(x, weights, spec: _Spec, out_width: int, cins: List[int], couts: List[int]):
    """One kernel launch per degree; x and the result are flat [N, width] rows."""
    n = x.shape[0]
    y = torch.empty(n, out_width, device=x.device, dtype=torch.float32)
    if n == 0:
        return y
    tiles, tspecies = spec.tiles if spec.tiles is not None else (None, None)
    num_tiles = int(tiles.shape[0]) if tiles is not None else 0
    xo = yo = 0
    stream = stream_of(x)
    for l, w in enumerate(weights):
        m = 2 * l + 1
        _native.call("ictc_channel_mix", ptr(x), int(x.shape[1]), xo, ptr(w), ptr(tiles), ptr(tspecies), num_tiles,
                     ptr(y), int(out_width), yo, int(n), cins[l], couts[l], l, spec.scale, 0, stream)
        xo += cins[l] * m
        yo += couts[l] * m
    return y


class _ChannelMix(torch.autograd.Function):
    """y = mix(x; W_l) for all degrees; weights given as [S, cout, cin_l] tensors."""

    @staticmethod
    def forward(ctx, spec, x, *weights):
        ctx.spec = spec
        ctx.save_for_backward(x, *weights)
        couts = [w.shape[-2] for w in weights]
        cins = [w.shape[-1] for w in weights]
        width = sum(c * (2 * l + 1) for l, c in enumerate(couts))
        return _launch(x, [w.contiguous() for w in weights], spec, width, cins, couts)

    @staticmethod
    def backward(ctx, gy):
        x, *weights = ctx.saved_tensors
        spec = ctx.spec
        need = required_gradients([x] + weights, ctx.needs_input_grad[1:])
        gy = gy.contiguous()
        dx = None
        if need[0]:
            # dx = W^T gy per degree: the same operation with transposed weights.
            dx = _ChannelMix.apply(spec, gy, *[w.transpose(-1, -2) for w in weights])
        dws = []
        xo = yo = 0
        n = x.shape[0]
        for l, w in enumerate(weights):
            m = 2 * l + 1
            cout, cin = w.shape[-2], w.shape[-1]
            if need[1 + l]:
                gl = gy[:, yo:yo + cout * m].reshape(n, cout, m)
                xl = x[:, xo:xo + cin * m].reshape(n, cin, m)
                if spec.tiles is None:
                    dw = spec.scale * torch.einsum("nom,nim->oi", gl, xl).reshape(w.shape)
                else:
                    tiles, tspecies = spec.tiles
                    dw_s = []
                    for s in range(w.shape[0]):
                        nodes = tiles[tspecies == s].reshape(-1)
                        nodes = nodes[nodes >= 0]
                        dw_s.append(spec.scale * torch.einsum("nom,nim->oi", gl.index_select(0, nodes),
                                                              xl.index_select(0, nodes)))
                    dw = torch.stack(dw_s)
                dws.append(dw)
            else:
                dws.append(None)
            xo += cin * m
            yo += cout * m
        return (None, dx, *dws)


def channel_mix(x: torch.Tensor, weights: Sequence[torch.Tensor], scale: float = 1.0,
                species: Optional[torch.Tensor] = None, num_elements: int = 1) -> torch.Tensor:
    """x [N, sum_l cin_l (2l+1)] -> [N, sum_l cout (2l+1)]; weights[l] is [cout, cin_l]
    (shared) or [S, cout, cin_l] (per species, with ``species`` [N])."""
    if x.dtype != torch.float32 or x.device.type != "cuda":
        raise ValueError("the CUDA channel linear requires CUDA FP32 features")
    tiles = None
    if species is not None:
        tiles = species_node_tiles(species, num_elements)
    spec = _Spec(tiles, scale)
    ws = [w if w.dim() == 3 else w.unsqueeze(0) for w in weights]
    out = _ChannelMix.apply(spec, x.contiguous(), *ws)
    return out
