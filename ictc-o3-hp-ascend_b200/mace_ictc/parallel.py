"""Spatial slab decomposition of a periodic system over ranks, with halo exchange.

Semantics of the reference's multi-device engine
(``mace_ictc/interfaces/ascend_lammps.py``): every rank owns the atoms of one
slab along x and keeps, as ghosts, the atoms within ``halo`` of its slab faces;
after each non-final interaction layer the owned node features that neighbours
hold as ghosts are sent to them (``_FeatureHalo`` :167-179, ``_feature_exchange``
:505-531), the adjoint sends ghost-row gradients back and adds them to the
owners' rows (:573-583), and per-edge force contributions of ghost atoms are
returned to their owners (``_reverse`` :455-483).  Energies are summed over owned
atoms (:632, :646) and the virial is -sum_e r_e (x) dE/dr_e (:660-667).

Transport is ``torch.distributed`` point-to-point (``batch_isend_irecv``): NCCL
over NVLink between GPUs, gloo for CPU tests.  Each exchange packs the rows to
send into contiguous buffers (one per neighbour), so every message is one
transfer.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


@dataclass
class SlabLayout:
    """Local atom layout: [owned | ghosts from the left slab | ghosts from the right slab]."""

    rank: int
    world: int
    owned: int                       # number of owned atoms (first rows)
    local_global: torch.Tensor       # [n_local] global atom index of every local row
    local_shift_x: torch.Tensor      # [n_local] x shift (0 or +-L) that unwraps ghosts next to the slab
    send_left: torch.Tensor          # owned local rows the left neighbour holds as right ghosts
    send_right: torch.Tensor         # owned local rows the right neighbour holds as left ghosts
    ghost_left: slice                # local rows received from the left neighbour
    ghost_right: slice               # local rows received from the right neighbour
    left: int
    right: int
    x0: float
    x1: float

    @property
    def local(self) -> int:
        return int(self.local_global.numel())


def slab_layout(pos: torch.Tensor, side: float, rank: int, world: int, halo: float) -> SlabLayout:
    """Ownership by x slab, ghosts within ``halo`` of the faces (needs slab width >= halo)."""
    width = side / world
    if world > 1 and width < halo:
        raise ValueError("slab width must be at least the halo depth")
    x0, x1 = rank * width, (rank + 1) * width
    if world == 1:                                   # every atom is owned; no ghosts
        owned = torch.arange(pos.shape[0], device=pos.device)
        empty = owned[:0]
        zeros = torch.zeros(owned.numel(), dtype=pos.dtype, device=pos.device)
        return SlabLayout(rank, world, owned.numel(), owned, zeros, empty, empty, slice(owned.numel(), owned.numel()),
                          slice(owned.numel(), owned.numel()), rank, rank, x0, x1)
    x = pos[:, 0] - side * torch.floor(pos[:, 0] / side)
    owner = torch.clamp((x / width).long(), 0, world - 1)
    left, right = (rank - 1) % world, (rank + 1) % world
    n = pos.shape[0]
    # Ghost images sit next to the slab: the left neighbour's atoms within `halo` below
    # x0 (shifted by -L when the slab touches x = 0), the right neighbour's within
    # `halo` above x1 (shifted by +L when it touches x = L).  With two ranks one atom
    # can be both a left and a right ghost (two images), so the sets are separate masks.
    shift_left = -side if rank == 0 else 0.0
    shift_right = side if rank == world - 1 else 0.0
    masks = torch.stack([
        owner == rank,                                                            # owned
        (owner == left) & (x + shift_left >= x0 - halo) & (x + shift_left < x0),   # left ghosts
        (owner == right) & (x + shift_right >= x1) & (x + shift_right < x1 + halo),  # right ghosts
        (owner == rank) & (x < x0 + halo),                                       # left neighbour's right ghosts
        (owner == rank) & (x >= x1 - halo),                                      # right neighbour's left ghosts
    ])
    counts = masks.sum(1).cpu().tolist()                                         # one device-to-host read
    flat = torch.nonzero(masks.reshape(-1)).flatten()
    groups = torch.split(flat, counts)
    owned, gl, gr, mine_left, mine_right = (g - k * n for k, g in enumerate(groups))  # ascending atom ids
    local_of = torch.full((n,), -1, dtype=torch.long, device=pos.device)
    local_of[owned] = torch.arange(owned.numel(), device=pos.device)
    local_global = torch.cat([owned, gl, gr])
    shift = torch.cat([torch.zeros(owned.numel(), dtype=pos.dtype, device=pos.device),
                       torch.full((gl.numel(),), shift_left, dtype=pos.dtype, device=pos.device),
                       torch.full((gr.numel(),), shift_right, dtype=pos.dtype, device=pos.device)])
    n_own = owned.numel()
    return SlabLayout(rank, world, n_own, local_global, shift, local_of[mine_left], local_of[mine_right],
                      slice(n_own, n_own + gl.numel()), slice(n_own + gl.numel(), n_own + gl.numel() + gr.numel()),
                      left, right, x0, x1)


def _exchange(layout: SlabLayout, send_left: torch.Tensor, send_right: torch.Tensor, recv_left_rows: int,
              recv_right_rows: int, width: int, dtype, device):
    """Send rows to both neighbours and receive both ghost blocks.

    Ops are issued as send-right, send-left, recv-left, recv-right on every rank,
    which pairs each send with the right receive even when both neighbours are the
    same rank (two ranks).
    """
    recv_left = torch.empty(recv_left_rows, width, dtype=dtype, device=device)
    recv_right = torch.empty(recv_right_rows, width, dtype=dtype, device=device)
    _p2p([(dist.isend, send_right.contiguous(), layout.right), (dist.isend, send_left.contiguous(), layout.left),
          (dist.irecv, recv_left, layout.left), (dist.irecv, recv_right, layout.right)])
    return recv_left, recv_right


def _p2p(ops):
    """Run one batch of point-to-point ops, leaving out empty messages.

    Sender and receiver derive a message's size from the same global positions, so
    both sides drop the same messages.  Between one pair of ranks messages match in
    issue order, so every rank sends to its right neighbour first and receives from
    its left neighbour first: with two ranks (left == right) each rank's first send
    then meets the other's first receive.
    """
    ops = [dist.P2POp(fn, t, peer) for fn, t, peer in ops if t.numel()]
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


class HaloExchange(torch.autograd.Function):
    """owned rows [n_own, W] -> local rows [n_local, W] (owned, then ghost copies)."""

    @staticmethod
    def forward(ctx, h_own, layout):
        ctx.layout = layout
        gl = layout.ghost_left.stop - layout.ghost_left.start
        gr = layout.ghost_right.stop - layout.ghost_right.start
        left, right = _exchange(layout, h_own.index_select(0, layout.send_left), h_own.index_select(0, layout.send_right),
                                gl, gr, h_own.shape[1], h_own.dtype, h_own.device)
        return torch.cat([h_own, left, right], 0)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        layout = ctx.layout
        grad = grad.contiguous()
        grad_own = grad[:layout.owned].clone()
        # Ghost-row gradients go back to their owners (the reverse of the forward sends):
        # my left ghosts came from my left neighbour's send_right, my right ghosts from
        # my right neighbour's send_left.
        back_left, back_right = _reverse(layout, grad[layout.ghost_left], grad[layout.ghost_right],
                                         layout.send_left.numel(), layout.send_right.numel())
        grad_own.index_add_(0, layout.send_left, back_left)
        grad_own.index_add_(0, layout.send_right, back_right)
        return grad_own, None


def _reverse(layout: SlabLayout, to_left: torch.Tensor, to_right: torch.Tensor, from_left_rows: int,
             from_right_rows: int):
    """Send ghost rows back to their owners; receive the rows my neighbours hold of mine.

    Returns (rows for my send_left list, rows for my send_right list).
    """
    width = to_left.shape[1] if to_left.ndim > 1 else 1
    recv_for_send_left = torch.empty(from_left_rows, width, dtype=to_left.dtype, device=to_left.device)
    recv_for_send_right = torch.empty(from_right_rows, width, dtype=to_left.dtype, device=to_left.device)
    # My right ghosts belong to my right neighbour, which sent them from its send_left
    # list; what arrives from my left neighbour is the cotangent of my send_left rows.
    _p2p([(dist.isend, to_right.contiguous(), layout.right), (dist.isend, to_left.contiguous(), layout.left),
          (dist.irecv, recv_for_send_left, layout.left), (dist.irecv, recv_for_send_right, layout.right)])
    return recv_for_send_left, recv_for_send_right


def reverse_ghost_forces(layout: SlabLayout, forces_local: torch.Tensor) -> torch.Tensor:
    """Owned forces [n_own, 3]: owned rows plus the ghost contributions of neighbours."""
    forces = forces_local[:layout.owned].clone()
    if layout.world == 1:
        return forces
    back_left, back_right = _reverse(layout, forces_local[layout.ghost_left], forces_local[layout.ghost_right],
                                     layout.send_left.numel(), layout.send_right.numel())
    forces.index_add_(0, layout.send_left, back_left)
    forces.index_add_(0, layout.send_right, back_right)
    return forces


def local_positions(layout: SlabLayout, pos_global: torch.Tensor, side: float) -> torch.Tensor:
    """Positions of the local rows: x wrapped into the box, ghosts unwrapped next to the slab."""
    pos = pos_global.index_select(0, layout.local_global).clone()
    x = pos[:, 0]
    pos[:, 0] = x - side * torch.floor(x / side) + layout.local_shift_x
    return pos


def slab_edges(layout: SlabLayout, pos_local: torch.Tensor, side: float, cutoff: float, halo: float):
    """Edges into the owned rows on the GPU: (src, dst, shift) grouped by dst.

    Sources range over owned and ghost rows.  y and z are periodic (minimum image);
    along x the ghosts are already unwrapped, so the search runs in a box whose x
    length exceeds the local extent by the cutoff: no pair is found through that
    artificial x boundary.
    """
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    if layout.world == 1:
        src, dst, shift, _ = neighbor_list(pos_local, (side, side, side), cutoff)
        return src, dst, shift
    pos = pos_local.clone()
    pos[:, 0] -= layout.x0 - halo
    box = ((layout.x1 - layout.x0) + 2.0 * halo + cutoff, side, side)
    src, dst, shift, _ = neighbor_list(pos, box, cutoff, receivers=layout.owned)
    return src, dst, shift


def distributed_energy_forces(model, layout: SlabLayout, pos_local: torch.Tensor, species_local: torch.Tensor,
                              src: torch.Tensor, dst: torch.Tensor, shift: torch.Tensor,
                              virial: bool = True):
    """Energy (summed over all ranks), owned forces and the global virial.

    ``src``/``dst`` are local edges whose receivers are owned rows; gradients are taken
    with respect to the edge vectors, so forces and virial come from per-edge terms
    (``ascend_lammps.py:656-669``).  The virial is the symmetrised
    -sum_e r_e (x) dE/dr_e as (xx, yy, zz, xy, xz, yz)."""
    vec = (pos_local[dst] - pos_local[src] + shift).detach().requires_grad_(True)
    exchange: Optional[Callable] = None
    if layout.world > 1:
        def exchange(h_own):
            return HaloExchange.apply(h_own, layout)
    energy_nodes = model.node_energies_from_vectors(vec, species_local, src, dst, owned=layout.owned,
                                                    exchange=exchange)
    energy = energy_nodes.sum()
    (g,) = torch.autograd.grad(energy, [vec])
    forces_local = torch.zeros(pos_local.shape[0], 3, dtype=g.dtype, device=g.device)
    forces_local.index_add_(0, dst, -g)
    forces_local.index_add_(0, src, g)
    forces = reverse_ghost_forces(layout, forces_local)
    total = energy.detach().reshape(1)
    w = None
    if virial:
        # -sum_e r_e (x) g_e, symmetrised, as three column-product reductions over the
        # edges (a 3 x E by E x 3 matrix product is a poorly shaped GEMM for E ~ 1e7).
        r = vec.detach()
        diag = (r * g).sum(0)                                  # r_x g_x, r_y g_y, r_z g_z
        up = (r * g[:, [1, 2, 0]]).sum(0)                      # r_x g_y, r_y g_z, r_z g_x
        down = (r * g[:, [2, 0, 1]]).sum(0)                    # r_x g_z, r_y g_x, r_z g_y
        w = -torch.stack([diag[0], diag[1], diag[2], 0.5 * (up[0] + down[1]), 0.5 * (down[0] + up[2]),
                          0.5 * (up[1] + down[2])])
    if layout.world > 1:
        dist.all_reduce(total)
        if w is not None:
            dist.all_reduce(w)
    return total, forces, w
