"""Direction harmonics on the CUDA backend, with analytic first and second adjoints.

Replaces the generated Triton harmonics of the reference
(``ictc_o3/ops/generated_direction_harmonics.py:43-177``) and evaluates the
same polynomial map as ``direction_harmonics_all``
(``ictc_o3/basis/ictd_irreps.py:1113-1168``).
"""
import numpy as np
import torch

from ictc_o3.autograd.adjoint_requirements import required_gradients
from ictc_o3.basis import ictd_irreps as basis
from . import _native
from ._native import ptr, stream_of

_TABLES = {}


def harmonic_table(lmax: int, device: torch.device) -> torch.Tensor:
    """H_l for l = 1..lmax as one flat FP32 device tensor (cached per device)."""
    key = (int(lmax), str(device))
    table = _TABLES.get(key)
    if table is None:
        flat = np.concatenate([basis.direction_harmonic_table(l).reshape(-1) for l in range(1, lmax + 1)])
        table = torch.from_numpy(flat.astype(np.float32)).to(device)
        _TABLES[key] = table
    return table


def _launch(n, lmax, mode, gy=None, hn=None):
    rows = n.shape[0]
    width = (lmax + 1) ** 2
    out0 = torch.empty(rows, 3 if mode == 1 else width, device=n.device, dtype=torch.float32)
    out1 = torch.empty(rows, 3, device=n.device, dtype=torch.float32) if mode == 2 else None
    if rows:
        table = harmonic_table(lmax, n.device)
        _native.call("ictc_direction_harmonics", ptr(n), ptr(table), ptr(gy), ptr(hn), ptr(out0), ptr(out1),
                     int(rows), int(lmax), int(mode), stream_of(n))
    return out0, out1


class _Harmonics(torch.autograd.Function):
    @staticmethod
    def forward(ctx, n, lmax):
        ctx.lmax = lmax
        ctx.save_for_backward(n)
        return _launch(n, lmax, 0)[0]

    @staticmethod
    def backward(ctx, gy):
        (n,) = ctx.saved_tensors
        if not required_gradients((n,), ctx.needs_input_grad[:1])[0]:
            return None, None
        gy = gy.contiguous()
        if torch.is_grad_enabled():
            return _HarmonicsAdjoint.apply(n, gy, ctx.lmax), None
        return _launch(n, ctx.lmax, 1, gy=gy)[0], None


class _HarmonicsAdjoint(torch.autograd.Function):
    """dn = J(n)^T gY; its backward is the mode-2 kernel (second derivatives)."""

    @staticmethod
    def forward(ctx, n, gy, lmax):
        ctx.lmax = lmax
        ctx.save_for_backward(n, gy)
        return _launch(n, lmax, 1, gy=gy)[0]

    @staticmethod
    def backward(ctx, hn):
        n, gy = ctx.saved_tensors
        need = required_gradients((n, gy), ctx.needs_input_grad[:2])
        if not any(need) or hn is None:
            return None, None, None
        if torch.is_grad_enabled() and any(t.requires_grad for t in (n, gy, hn)):
            raise NotImplementedError("third derivatives of the direction harmonics are not provided")
        d_gy, d_n = _launch(n, ctx.lmax, 2, gy=gy, hn=hn.contiguous())
        return (d_n if need[0] else None), (d_gy if need[1] else None), None


def direction_harmonics(n: torch.Tensor, lmax: int) -> torch.Tensor:
    """Packed Y(n) [..., (lmax+1)^2] for unit vectors n [..., 3]."""
    if n.dtype != torch.float32 or n.device.type != "cuda" or n.shape[-1] != 3:
        raise ValueError("direction harmonics require CUDA FP32 vectors [..., 3]")
    lead = n.shape[:-1]
    flat = n.reshape(-1, 3).contiguous()
    if lmax == 0:
        return torch.ones(*lead, 1, device=n.device, dtype=n.dtype) + 0 * flat.sum()
    if torch.is_grad_enabled() and flat.requires_grad:
        y = _Harmonics.apply(flat, int(lmax))
    else:
        y = _launch(flat, int(lmax), 0)[0]
    return y.reshape(*lead, (lmax + 1) ** 2)


# ---------------------------------------------------------------------------
# Edge geometry: unit vectors, Bessel x polynomial-envelope embedding, cutoff mask
# ---------------------------------------------------------------------------

def edge_geometry_reference(vec, r_max, num_basis, p, basis_norm=True):
    """The same map in torch ops (mace_ictc/models/radial_basis.py:11-91 and the
    model's edge normalisation); differentiable to any order."""
    import math
    r = vec.norm(dim=-1)
    unit = vec / r.clamp_min(1e-8).unsqueeze(-1)
    x = r / r_max
    env = (1.0 - ((p + 1.0) * (p + 2.0) / 2.0) * x.pow(p) + p * (p + 2.0) * x.pow(p + 1)
           - (p * (p + 1.0) / 2.0) * x.pow(p + 2)) * (r < r_max).to(vec.dtype)
    freq = math.pi / r_max * torch.arange(1, num_basis + 1, dtype=vec.dtype, device=vec.device)
    radial = math.sqrt(2.0 / r_max) * torch.sin(r.unsqueeze(-1) * freq) / r.clamp_min(1e-12).unsqueeze(-1)
    radial = radial * env.unsqueeze(-1)
    if basis_norm:
        radial = radial * math.sqrt(num_basis)
    mask = (r <= r_max).to(vec.dtype)
    return unit, radial, mask


def _geometry_args(r_max, num_basis, p, basis_norm):
    return float(r_max), int(num_basis), int(p), int(bool(basis_norm))


class _EdgeGeometry(torch.autograd.Function):
    @staticmethod
    def forward(ctx, vec, r_max, num_basis, p, basis_norm):
        ctx.args = (r_max, num_basis, p, basis_norm)
        ctx.save_for_backward(vec)
        edges = vec.shape[0]
        unit = torch.empty(edges, 3, device=vec.device, dtype=torch.float32)
        radial = torch.empty(edges, num_basis, device=vec.device, dtype=torch.float32)
        mask = torch.empty(edges, device=vec.device, dtype=torch.float32)
        if edges:
            _native.call("ictc_edge_geometry", ptr(vec), int(edges), *_geometry_args(r_max, num_basis, p, basis_norm),
                         ptr(unit), ptr(radial), ptr(mask), stream_of(vec))
        ctx.mark_non_differentiable(mask)
        return unit, radial, mask

    @staticmethod
    def backward(ctx, g_unit, g_radial, _g_mask):
        (vec,) = ctx.saved_tensors
        if not required_gradients((vec,), ctx.needs_input_grad[:1])[0]:
            return None, None, None, None, None
        if torch.is_grad_enabled():
            # The gradient itself is differentiated (force-loss training): recompute
            # through the torch formula so every order is available.
            with torch.enable_grad():
                unit, radial, _ = edge_geometry_reference(vec, *ctx.args)
                outs, grads = [], []
                for o, g in ((unit, g_unit), (radial, g_radial)):
                    if g is not None:
                        outs.append(o)
                        grads.append(g)
                (dv,) = torch.autograd.grad(outs, [vec], grads, create_graph=True)
            return dv, None, None, None, None
        grad_vec = torch.empty_like(vec)
        if vec.shape[0]:
            _native.call("ictc_edge_geometry_backward", ptr(vec),
                         ptr(None if g_unit is None else g_unit.contiguous()),
                         ptr(None if g_radial is None else g_radial.contiguous()), int(vec.shape[0]),
                         *_geometry_args(*ctx.args), ptr(grad_vec), stream_of(vec))
        return grad_vec, None, None, None, None


def edge_geometry(vec: torch.Tensor, r_max: float, num_basis: int, p: int, basis_norm: bool = True):
    """(unit [E, 3], radial [E, num_basis], mask [E]) of CUDA FP32 edge vectors [E, 3]."""
    if vec.dtype != torch.float32 or vec.device.type != "cuda" or vec.dim() != 2 or vec.shape[1] != 3:
        raise ValueError("edge geometry requires CUDA FP32 edge vectors [E, 3]")
    return _EdgeGeometry.apply(vec.contiguous(), float(r_max), int(num_basis), int(p), bool(basis_norm))


def edge_vectors(positions: torch.Tensor, cell: torch.Tensor, shifts: torch.Tensor, batch: torch.Tensor,
                 source: torch.Tensor, destination: torch.Tensor) -> torch.Tensor:
    """r_e = pos[dst] - pos[src] + shifts_e @ cell[batch[src]]  (``backends/ascend/geometry.py:6``,
    hook site ``pure_cartesian_ictd_fix.py:2926-2928``).

    ``shifts`` are lattice coordinates [E, 3] and ``cell`` is [B, 3, 3].  Device
    gathers and a batched 3 x 3 product that autograd differentiates to any order
    in positions and cell (strain derivatives stay live)."""
    if any(t.dtype != torch.float32 or t.device.type != "cuda" for t in (positions, cell, shifts)):
        raise ValueError("edge_vectors requires CUDA FP32 positions, cell and shifts")
    if cell.ndim != 3 or cell.shape[1:] != (3, 3) or shifts.shape != (source.numel(), 3):
        raise ValueError("Expected cell [B,3,3] and lattice shifts [E,3]")
    if cell.shape[0] == 1:
        shift_vectors = shifts @ cell[0]
    else:
        shift_vectors = torch.bmm(shifts.unsqueeze(1), cell.index_select(0, batch.index_select(0, source))).squeeze(1)
    return positions.index_select(0, destination) - positions.index_select(0, source) + shift_vectors
