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


def check_species(species: torch.Tensor, num_elements: int):
    """Raise if a species index is outside [0, num_elements) (``backends/ascend/species.py:9-17``).
    One device-to-host read per (tensor, version); later calls on the same tensor are free."""
    key = (species._version, int(num_elements))
    if getattr(species, "_ictc_species_checked", None) == key:
        return
    if species.numel():
        lo, hi = torch.stack([species.amin(), species.amax()]).cpu().tolist()
        if lo < 0 or hi >= num_elements:
            raise ValueError("Species index is outside the element table")
    try:
        species._ictc_species_checked = key
    except AttributeError:
        pass


def species_tiles_of(species: torch.Tensor, num_elements: int, nb: int):
    """Species-homogeneous node tiles [T, nb] (-1 padded) and their species [T] (int32).

    Built on the device without a host read: nodes sorted by species (stable), each
    species' run cut into tiles of nb nodes, the last one padded with -1.  T is the
    bound nodes // nb + num_elements; tiles past the used ones hold only -1 nodes,
    which the kernels skip."""
    check_species(species, num_elements)
    device = species.device
    n, S = species.numel(), int(num_elements)
    T = n // nb + S
    index = species.to(torch.int64)
    order = torch.argsort(index, stable=True)
    bounds = torch.searchsorted(index.index_select(0, order), torch.arange(S + 1, dtype=torch.int64, device=device))
    counts = bounds[1:] - bounds[:-1]
    tiles_per = (counts + nb - 1) // nb
    tile_end = torch.cumsum(tiles_per, 0)
    t = torch.arange(T, dtype=torch.int64, device=device)
    s = torch.searchsorted(tile_end, t, right=True)                 # species of tile t (S: unused tile)
    used = s < S
    s = torch.clamp(s, max=S - 1)
    j = t - (tile_end - tiles_per).index_select(0, s)               # tile number inside the species run
    slot = j.unsqueeze(1) * nb + torch.arange(nb, dtype=torch.int64, device=device)
    valid = used.unsqueeze(1) & (slot < counts.index_select(0, s).unsqueeze(1))
    pos = torch.clamp(bounds.index_select(0, s).unsqueeze(1) + slot, max=max(n - 1, 0))
    nodes = order.index_select(0, pos.flatten()).view(T, nb) if n else torch.zeros(T, nb, dtype=torch.int64,
                                                                                      device=device)
    tiles = torch.where(valid, nodes, torch.full_like(nodes, -1))
    return tiles.contiguous(), s.to(torch.int32).contiguous()


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
    """Static part of one linear: species tiles (or None), the output scale and the
    degree of the first weight (the blocks are degrees degree0, degree0 + 1, ...)."""

    def __init__(self, tiles, scale: float, degree0: int = 0):
        self.tiles = tiles                    # None or (tiles, tile_species)
        self.scale = float(scale)
        self.degree0 = int(degree0)


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
        m = 2 * (l + spec.degree0) + 1
        _native.call("ictc_channel_mix", ptr(x), int(x.shape[1]), xo, ptr(w), ptr(tiles), ptr(tspecies), num_tiles,
                     ptr(y), int(out_width), yo, int(n), cins[l], couts[l], l + spec.degree0, spec.scale, 0, stream)
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
        width = sum(c * (2 * (l + spec.degree0) + 1) for l, c in enumerate(couts))
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
            m = 2 * (l + spec.degree0) + 1
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


# ---------------------------------------------------------------------------
# Reference backend entry points (``ictc_o3/backends/ascend/linear.py:8,24``)
# ---------------------------------------------------------------------------

def _block_degree(features: torch.Tensor) -> int:
    m = features.shape[-1]
    if m % 2 == 0 or m > 7:
        raise ValueError("The angular axis must have 2l+1 components with l <= 3")
    return (m - 1) // 2


def channel_linear(features: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None):
    """features [..., I, M], weight [O, I], optional bias [O] (scalar blocks only) -> [..., O, M].

    One degree block through the channel-mix kernel; first and higher derivatives
    stay live (the weight gradient is a device reduction)."""
    tensors = (features, weight) + (() if bias is None else (bias,))
    if any(t.dtype != torch.float32 or t.device.type != "cuda" for t in tensors):
        raise ValueError("the CUDA channel linear requires CUDA FP32 tensors")
    if features.ndim < 2 or weight.ndim != 2 or features.shape[-2] != weight.shape[1]:
        raise ValueError("Expected features [...,I,M] and weight [O,I]")
    if bias is not None and (features.shape[-1] != 1 or bias.shape != (weight.shape[0],)):
        raise ValueError("Bias is allowed only for scalar angular blocks with shape [O]")
    degree = _block_degree(features)
    lead, (cin, m) = features.shape[:-2], features.shape[-2:]
    flat = features.reshape(-1, cin * m)
    out = _ChannelMix.apply(_Spec(None, 1.0, degree), flat.contiguous(), weight.unsqueeze(0))
    out = out.reshape(*lead, weight.shape[0], m)
    return out if bias is None else out + bias.unsqueeze(-1)


def species_channel_linear(features: torch.Tensor, weight: torch.Tensor, species: torch.Tensor,
                           bias: Optional[torch.Tensor] = None):
    """features [N, I, M], weight bank [S, O, I], species [N], optional bias [S, O] -> [N, O, M].

    Every node uses its species' weights (species-homogeneous node tiles, no [N, O, I]
    temporary and no host sort)."""
    tensors = (features, weight) + (() if bias is None else (bias,))
    if any(t.dtype != torch.float32 or t.device.type != "cuda" for t in tensors):
        raise ValueError("the CUDA species channel linear requires CUDA FP32 tensors")
    if (features.ndim != 3 or weight.ndim != 3 or features.shape[1] != weight.shape[2]
            or species.shape != (features.shape[0],) or species.device != features.device
            or species.dtype not in (torch.int32, torch.int64) or weight.shape[0] < 1):
        raise ValueError("Expected features [N,I,M], weight [S,O,I] and integer species [N]")
    from .species import validate_species
    validate_species(species, weight.shape[0])
    if bias is not None and (features.shape[-1] != 1 or bias.shape != weight.shape[:2]):
        raise ValueError("Bias is allowed only for scalar angular blocks with shape [S,O]")
    degree = _block_degree(features)
    n, cin, m = features.shape
    tiles = species_node_tiles(species, weight.shape[0])
    out = _ChannelMix.apply(_Spec(tiles, 1.0, degree), features.reshape(n, cin * m).contiguous(), weight)
    out = out.reshape(n, weight.shape[1], m)
    return out if bias is None else out + bias.index_select(0, species.to(torch.int64)).unsqueeze(-1)
