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

Every rank holds only its own atoms (``SlabDomain``: global ids, positions and
species of the owned atoms).  A step (``md_step``) is

1. ``exchange_atoms``: atoms that moved into a neighbouring slab are handed to it
   (ownership changes, reference "changing ownership") and owned atoms within
   ``halo`` of a face are sent, as position and species rows, to the neighbour on
   that side, which keeps them as ghosts -- one message per neighbour, after one
   all_gather of per-rank counts (``migrate`` then ``halo_layout`` is the two-round
   form it falls back to when an atom moved too far for the single round);
2. the owned-receiver neighbour list (``slab_edges``);
3. the model on [owned | left ghosts | right ghosts] with the feature exchange
   before every later layer (``HaloExchange``, overlapped with the radial network)
   and its adjoint;
4. ``reverse_ghost_forces`` and one all-reduce of energy and virial.

Nothing in a step is proportional to the global atom count.  Transport is
``torch.distributed`` point-to-point (``batch_isend_irecv``): NCCL over NVLink
between GPUs, gloo for CPU tests.  Each exchange packs the rows to send into
one contiguous buffer per neighbour, so every message is one transfer; message
sizes are known on both sides from counts read on the host once per step.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist


# ---------------------------------------------------------------------------
# Per-phase timing of a step (CUDA events on the compute stream + host clock)
# ---------------------------------------------------------------------------

class StepPhases:
    """Named marks inside a step.  On CUDA every mark records an event on the current
    stream, so a phase's device time is the stream time between two marks (work plus
    any idle gap, e.g. waiting for the host to launch); the host time is the Python
    time between the same marks.  A phase whose host time exceeds its device time is
    launch-bound.  Disabled objects (the default) record nothing."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self.marks: List[tuple] = []

    def mark(self, name: str, device: Optional[torch.device] = None):
        if not self.enabled:
            return
        event = None
        if device is not None and device.type == "cuda":
            event = torch.cuda.Event(enable_timing=True)
            event.record(torch.cuda.current_stream(device))
        self.marks.append((name, event, time.perf_counter()))

    def reset(self):
        self.marks = []

    def summary(self):
        """[(phase, device_ms or None, host_ms)] between consecutive marks."""
        if self.marks and self.marks[-1][1] is not None:
            self.marks[-1][1].synchronize()
        out = []
        for (_, e0, t0), (name, e1, t1) in zip(self.marks, self.marks[1:]):
            dev = e0.elapsed_time(e1) if (e0 is not None and e1 is not None) else None
            out.append((name, dev, 1e3 * (t1 - t0)))
        return out


NO_PHASES = StepPhases(enabled=False)


# ---------------------------------------------------------------------------
# Domain: the owned atoms of one slab
# ---------------------------------------------------------------------------

@dataclass
class SlabDomain:
    """The atoms rank ``rank`` owns: those with x (wrapped into [0, side)) in its slab."""

    rank: int
    world: int
    side: float
    halo: float
    ids: torch.Tensor        # [n_own] int64 global atom ids (only used to map outputs)
    pos: torch.Tensor        # [n_own, 3] positions, x wrapped into [0, side)
    species: torch.Tensor    # [n_own] int64

    @property
    def width(self) -> float:
        return self.side / self.world

    @property
    def x0(self) -> float:
        return _face(self.side, self.world, self.rank)

    @property
    def x1(self) -> float:
        return _face(self.side, self.world, self.rank + 1)

    @property
    def left(self) -> int:
        return (self.rank - 1) % self.world

    @property
    def right(self) -> int:
        return (self.rank + 1) % self.world

    @property
    def owned(self) -> int:
        return int(self.ids.numel())


def _face(side: float, world: int, k: int) -> float:
    """x of the face between slabs k - 1 and k (one expression, so every rank computes
    bit-identical faces)."""
    return side * k / world


def _signed(x: torch.Tensor, face: float, side: float) -> torch.Tensor:
    """Periodic signed distance x - face in (-side/2, side/2] (FP64)."""
    return torch.remainder(x - face + 0.5 * side, side) - 0.5 * side


def _wrap_x(pos: torch.Tensor, side: float) -> torch.Tensor:
    pos = pos.clone()
    pos[:, 0] = pos[:, 0] - side * torch.floor(pos[:, 0] / side)
    return pos


def _check_slabs(side: float, world: int, halo: float):
    if world > 1 and side / world < halo:
        raise ValueError("slab width must be at least the halo depth (ghosts come from the two neighbour slabs)")


def partition(pos: torch.Tensor, species: torch.Tensor, side: float, rank: int, world: int,
              halo: float) -> SlabDomain:
    """Initial distribution: the atoms of ``rank``'s slab from a global configuration.
    Run once when the system is set up (it reads the global arrays); steps never do."""
    _check_slabs(side, world, halo)
    wrapped = _wrap_x(pos, side)
    slab = torch.clamp((wrapped[:, 0] / (side / world)).long(), 0, world - 1)
    ids = torch.nonzero(slab == rank).flatten()
    return SlabDomain(rank, world, side, halo, ids, wrapped.index_select(0, ids).contiguous(),
                      species.index_select(0, ids).contiguous())


def _p2p(ops):
    """Run one batch of point-to-point ops, leaving out empty messages.

    Both sides of a message know its size (from the exchanged counts), so both drop
    the same empty messages.  Between one pair of ranks messages match in issue order,
    so every rank sends to its right neighbour first and receives from its left
    neighbour first: with two ranks (left == right) each rank's first send then meets
    the other's first receive.  Returns the pending requests."""
    ops = [dist.P2POp(fn, t, peer) for fn, t, peer in ops if t.numel()]
    return dist.batch_isend_irecv(ops) if ops else []


def _wait(requests):
    for req in requests:
        req.wait()


def _swap_counts(domain: SlabDomain, to_left: torch.Tensor, to_right: torch.Tensor):
    """Send a count vector to each neighbour; returns (from_left, from_right)."""
    from_left, from_right = torch.empty_like(to_left), torch.empty_like(to_right)
    _wait(_p2p([(dist.isend, to_right, domain.right), (dist.isend, to_left, domain.left),
                (dist.irecv, from_left, domain.left), (dist.irecv, from_right, domain.right)]))
    return from_left, from_right


def _swap_rows(domain: SlabDomain, to_left: torch.Tensor, to_right: torch.Tensor, from_left_rows: int,
               from_right_rows: int):
    """Send rows to both neighbours and receive both neighbours' rows (same width)."""
    shape = to_left.shape[1:]
    from_left = torch.empty((from_left_rows, *shape), dtype=to_left.dtype, device=to_left.device)
    from_right = torch.empty((from_right_rows, *shape), dtype=to_left.dtype, device=to_left.device)
    reqs = _p2p([(dist.isend, to_right.contiguous(), domain.right), (dist.isend, to_left.contiguous(), domain.left),
                 (dist.irecv, from_left, domain.left), (dist.irecv, from_right, domain.right)])
    return from_left, from_right, reqs


def migrate(domain: SlabDomain) -> SlabDomain:
    """Hand every owned atom whose wrapped x left the slab to the neighbour slab it
    entered.  Atoms may move at most into an adjacent slab between two calls (checked).
    Kept atoms keep their order; arrivals from the left, then from the right, follow."""
    pos = _wrap_x(domain.pos, domain.side)
    if domain.world == 1:
        return SlabDomain(domain.rank, 1, domain.side, domain.halo, domain.ids, pos, domain.species)
    width = domain.width
    slab = torch.clamp((pos[:, 0] / width).long(), 0, domain.world - 1)
    go_left, go_right = slab == domain.left, slab == domain.right
    if domain.world == 2:            # both neighbours are the same rank: one outgoing set
        go_right = go_right & ~go_left
    keep = slab == domain.rank
    far = (~(keep | go_left | go_right)).sum()
    counts = torch.stack([go_left.sum(), go_right.sum(), far])
    from_left, from_right = _swap_counts(domain, counts, counts.clone())
    # one device-to-host read: my outgoing counts and my neighbours' (the left one's
    # right-going atoms and the right one's left-going atoms arrive here)
    n_left, n_right, n_far, _, in_left, far_l, in_right, _, far_r = torch.cat(
        [counts, from_left, from_right]).tolist()
    if n_far or far_l or far_r:
        raise RuntimeError("an atom moved further than one slab between two migrations")
    rows = torch.cat([pos.double(), domain.species.double().unsqueeze(1), domain.ids.double().unsqueeze(1)], 1)
    send_left = torch.nonzero_static(go_left, size=n_left).flatten()
    send_right = torch.nonzero_static(go_right, size=n_right).flatten()
    # from my left neighbour arrive the atoms it sends right, and vice versa
    got_left, got_right, reqs = _swap_rows(domain, rows.index_select(0, send_left),
                                           rows.index_select(0, send_right), in_left, in_right)
    _wait(reqs)
    kept = torch.nonzero_static(keep, size=pos.shape[0] - n_left - n_right).flatten()
    new = torch.cat([rows.index_select(0, kept), got_left, got_right])
    return SlabDomain(domain.rank, domain.world, domain.side, domain.halo, new[:, 4].round().long(),
                      new[:, :3].to(domain.pos.dtype).contiguous(), new[:, 3].round().long())


# ---------------------------------------------------------------------------
# Halo layout of one step
# ---------------------------------------------------------------------------

@dataclass
class SlabLayout:
    """Local atom layout: [owned | ghosts from the left slab | ghosts from the right slab]."""

    rank: int
    world: int
    owned: int                       # number of owned atoms (first rows)
    send_left: torch.Tensor          # owned local rows the left neighbour holds as right ghosts
    send_right: torch.Tensor         # owned local rows the right neighbour holds as left ghosts
    ghost_left: slice                # local rows received from the left neighbour
    ghost_right: slice               # local rows received from the right neighbour
    left: int
    right: int
    x0: float
    x1: float
    halo: float
    side: float
    local_ids: torch.Tensor          # [n_local] global atom id of every local row
    rounds: int = 2                  # message rounds that built it (1: single-round atom exchange)

    @property
    def local(self) -> int:
        return self.ghost_right.stop


def halo_layout(domain: SlabDomain):
    """Ghosts of one step: returns (layout, local positions [n_local, 3], local species).

    Owned rows keep the domain's order.  The left neighbour's atoms within ``halo``
    below x0 arrive as left ghosts and the right neighbour's within ``halo`` above x1
    as right ghosts, with x unwrapped next to the slab (shifted by -L / +L across the
    periodic boundary).  A ghost row travels as (x, y, z, species, global id) in FP64
    (40 B; the ids are only used to map outputs).  One device-to-host read (the four
    ghost counts)."""
    pos, species = domain.pos, domain.species
    n_own = pos.shape[0]
    if domain.world == 1:
        empty = torch.zeros(0, dtype=torch.int64, device=pos.device)
        layout = SlabLayout(domain.rank, 1, n_own, empty, empty, slice(n_own, n_own), slice(n_own, n_own),
                            domain.rank, domain.rank, domain.x0, domain.x1, domain.halo, domain.side, domain.ids)
        return layout, pos, species
    x = pos[:, 0]
    to_left = x < domain.x0 + domain.halo      # my atoms the left neighbour keeps as right ghosts
    to_right = x >= domain.x1 - domain.halo    # my atoms the right neighbour keeps as left ghosts
    counts = torch.stack([to_left.sum(), to_right.sum()])
    from_left, from_right = _swap_counts(domain, counts, counts.clone())
    # my left ghosts are what the left neighbour sends right, and vice versa
    n_left, n_right, gl, gr = torch.cat([counts, from_left[1:], from_right[:1]]).tolist()
    send_left = torch.nonzero_static(to_left, size=n_left).flatten()
    send_right = torch.nonzero_static(to_right, size=n_right).flatten()
    rows = torch.cat([pos.double(), species.double().unsqueeze(1), domain.ids.double().unsqueeze(1)], 1)
    got_left, got_right, reqs = _swap_rows(domain, rows.index_select(0, send_left), rows.index_select(0, send_right),
                                           gl, gr)
    _wait(reqs)
    shift_left = -domain.side if domain.rank == 0 else 0.0
    shift_right = domain.side if domain.rank == domain.world - 1 else 0.0
    got_left[:, 0] += shift_left
    got_right[:, 0] += shift_right
    ghosts = torch.cat([got_left, got_right])
    pos_local = torch.cat([pos, ghosts[:, :3].to(pos.dtype)])
    species_local = torch.cat([species, ghosts[:, 3].round().long()])
    local_ids = torch.cat([domain.ids, ghosts[:, 4].round().long()])
    layout = SlabLayout(domain.rank, domain.world, n_own, send_left, send_right, slice(n_own, n_own + gl),
                        slice(n_own + gl, n_own + gl + gr), domain.left, domain.right, domain.x0, domain.x1,
                        domain.halo, domain.side, local_ids)
    return layout, pos_local, species_local


# ---------------------------------------------------------------------------
# Feature halo and its adjoint
# ---------------------------------------------------------------------------

class PendingHalo:
    """A feature exchange in flight: the owned rows' ghost copies travel while the
    caller launches independent work (the radial MLP); ``finish`` waits and returns
    the local rows [owned | left ghosts | right ghosts] as a differentiable tensor."""

    def __init__(self, layout: SlabLayout, h_own: torch.Tensor):
        self.layout, self.h_own = layout, h_own
        self.reversed = False
        with torch.no_grad():
            send_left = h_own.detach().index_select(0, layout.send_left)
            send_right = h_own.detach().index_select(0, layout.send_right)
        gl = layout.ghost_left.stop - layout.ghost_left.start
        gr = layout.ghost_right.stop - layout.ghost_right.start
        self.left, self.right, self.reqs = _swap_rows(layout, send_left, send_right, gl, gr)

    def finish(self) -> torch.Tensor:
        return HaloExchange.apply(self.h_own, self)


class HaloExchange(torch.autograd.Function):
    """owned rows [n_own, W] -> local rows [n_local, W] (owned, then ghost copies)."""

    @staticmethod
    def forward(ctx, h_own, pending: PendingHalo):
        ctx.layout, ctx.pending = pending.layout, pending
        _wait(pending.reqs)
        return torch.cat([h_own, pending.left, pending.right], 0)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad):
        layout = ctx.layout
        ctx.pending.reversed = True
        grad = grad.contiguous()
        grad_own = grad[:layout.owned].clone()
        # Ghost-row gradients go back to their owners (the reverse of the forward sends):
        # my left ghosts came from my left neighbour's send_right, my right ghosts from
        # my right neighbour's send_left.
        back_left, back_right = _reverse(layout, grad[layout.ghost_left], grad[layout.ghost_right])
        grad_own.index_add_(0, layout.send_left, back_left)
        grad_own.index_add_(0, layout.send_right, back_right)
        return grad_own, None


def _reverse(layout: SlabLayout, to_left: torch.Tensor, to_right: torch.Tensor):
    """Send ghost rows back to their owners; receive the rows my neighbours hold of mine.

    Returns (rows for my send_left list, rows for my send_right list)."""
    # My right ghosts belong to my right neighbour, which sent them from its send_left
    # list; what arrives from my left neighbour is the cotangent of my send_left rows.
    back_left, back_right, reqs = _swap_rows(layout, to_left, to_right, layout.send_left.numel(),
                                             layout.send_right.numel())
    _wait(reqs)
    return back_left, back_right


class HaloExchanges:
    """The model's ``exchange`` hook (owned rows -> ``PendingHalo``; ``.finish()`` gives the
    local rows), remembering every exchange of a forward pass.

    Every rank must take the same communication steps.  Autograd runs an exchange's
    adjoint only where the energy depends on its output, which is not the case on a
    rank that owns no atoms (no receivers, no edges); ``complete_adjoints`` then sends
    zero cotangents for each exchange whose adjoint did not run, latest first (the
    order autograd uses), so the neighbours' reverse exchanges are matched."""

    def __init__(self, layout: SlabLayout):
        self.layout = layout
        self.started: List[PendingHalo] = []

    def __call__(self, h_own):
        pending = PendingHalo(self.layout, h_own)
        self.started.append(pending)
        return pending

    def complete_adjoints(self):
        layout = self.layout
        for pending in reversed(self.started):
            if not pending.reversed:
                width = pending.h_own.shape[1]
                zeros = pending.h_own.new_zeros(layout.local - layout.owned, width)
                _reverse(layout, zeros[:layout.ghost_left.stop - layout.owned],
                         zeros[layout.ghost_left.stop - layout.owned:])
                pending.reversed = True
        self.started = []


def reverse_ghost_forces(layout: SlabLayout, forces_local: torch.Tensor) -> torch.Tensor:
    """Owned forces [n_own, 3]: owned rows plus the ghost contributions of neighbours."""
    forces = forces_local[:layout.owned].clone()
    if layout.world == 1:
        return forces
    back_left, back_right = _reverse(layout, forces_local[layout.ghost_left], forces_local[layout.ghost_right])
    forces.index_add_(0, layout.send_left, back_left)
    forces.index_add_(0, layout.send_right, back_right)
    return forces


def slab_edges(layout: SlabLayout, pos_local: torch.Tensor, cutoff: float):
    """Edges into the owned rows on the GPU: (src, dst, shift) grouped by dst.

    Sources range over owned and ghost rows.  y and z are periodic (minimum image);
    along x the ghosts are already unwrapped, so the search runs in a box whose x
    length exceeds the local extent by the cutoff: no pair is found through that
    artificial x boundary.
    """
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    side = layout.side
    if layout.world == 1:
        src, dst, shift, _ = neighbor_list(pos_local, (side, side, side), cutoff)
        return src, dst, shift
    pos = pos_local.clone()
    pos[:, 0] -= layout.x0 - layout.halo
    box = ((layout.x1 - layout.x0) + 2.0 * layout.halo + cutoff, side, side)
    src, dst, shift, _ = neighbor_list(pos, box, cutoff, receivers=layout.owned)
    return src, dst, shift


def distributed_energy_forces(model, layout: SlabLayout, pos_local: torch.Tensor, species_local: torch.Tensor,
                              src: torch.Tensor, dst: torch.Tensor, shift: torch.Tensor,
                              virial: bool = True, phases: StepPhases = NO_PHASES,
                              owned_species: Optional[torch.Tensor] = None):
    """Energy (summed over all ranks), owned forces and the global virial.

    ``src``/``dst`` are local edges whose receivers are owned rows; gradients are taken
    with respect to the edge vectors, so forces and virial come from per-edge terms
    (``ascend_lammps.py:656-669``).  The virial is the symmetrised
    -sum_e r_e (x) dE/dr_e as (xx, yy, zz, xy, xz, yz)."""
    device = pos_local.device
    vec = (pos_local[dst] - pos_local[src] + shift).detach().requires_grad_(True)
    exchange = HaloExchanges(layout) if layout.world > 1 else None
    energy_nodes = model.node_energies_from_vectors(vec, species_local, src, dst, owned=layout.owned,
                                                    exchange=exchange, phases=phases, owned_species=owned_species)
    energy = energy_nodes.sum()
    # allow_unused: a rank without edges has an energy that does not depend on vec
    (g,) = torch.autograd.grad(energy, [vec], allow_unused=True)
    if g is None:
        g = torch.zeros_like(vec)
    if exchange is not None:
        exchange.complete_adjoints()
    phases.mark("backward", device)
    forces_local = torch.zeros(pos_local.shape[0], 3, dtype=g.dtype, device=g.device)
    forces_local.index_add_(0, dst, -g)
    forces_local.index_add_(0, src, g)
    forces = reverse_ghost_forces(layout, forces_local)
    phases.mark("ghost_forces", device)
    totals = energy.detach().reshape(1)
    if virial:
        # -sum_e r_e (x) g_e, symmetrised, as three column-product reductions over the
        # edges (a 3 x E by E x 3 matrix product is a poorly shaped GEMM for E ~ 1e7).
        r = vec.detach()
        diag = (r * g).sum(0)                                  # r_x g_x, r_y g_y, r_z g_z
        up = (r * torch.roll(g, -1, 1)).sum(0)                 # r_x g_y, r_y g_z, r_z g_x
        down = (r * torch.roll(g, 1, 1)).sum(0)                # r_x g_z, r_y g_x, r_z g_y
        w = -torch.stack([diag[0], diag[1], diag[2], 0.5 * (up[0] + down[1]), 0.5 * (down[0] + up[2]),
                          0.5 * (up[1] + down[2])])
        totals = torch.cat([totals, w])
    if layout.world > 1:
        dist.all_reduce(totals)                                 # energy and virial in one reduction
    phases.mark("reductions", device)
    return totals[:1], forces, (totals[1:] if virial else None)


def exchange_atoms(domain: SlabDomain):
    """Migration and ghost positions of one step with a single count exchange.

    Returns (domain after migration, layout, local positions, local species), the same
    as ``halo_layout(migrate(domain))`` (owned rows: kept atoms, then arrivals from the
    left, then from the right; ghosts as there).  Each rank sends each neighbour one
    message: the atoms it hands over, then its kept atoms within ``halo`` of the shared
    face.  A handed-over atom that lies within ``halo`` of that face is a ghost for the
    sender and a boundary row for the receiver; both apply the same test to the same
    values, so they agree without another round.  This needs every handed-over atom
    to stay clear of its new slab's far halo band (it moved less than width - halo past
    the face); the counts of all ranks travel in one all_gather, and if any rank sees
    an atom that moved further, every rank takes the two-round path.  One
    device-to-host read."""
    side, world, rank, halo = domain.side, domain.world, domain.rank, domain.halo
    if world == 1:
        domain = migrate(domain)
        layout, pos_local, species_local = halo_layout(domain)
        return domain, layout, pos_local, species_local
    width = domain.width
    pos = _wrap_x(domain.pos, side)
    x = pos[:, 0].double()
    # faces as periodic positions in [0, side): a face shared by two ranks has one value
    f0, f1 = _face(side, world, rank), _face(side, world, (rank + 1) % world)
    d0 = _signed(x, f0, side)                             # >= 0 inside the slab
    d1 = _signed(x, f1, side)                             # < 0 inside the slab
    keep = (d0 >= 0) & (d1 < 0)
    go_right = ~keep & (d1 >= 0) & (d1 < width) & ((d0 >= 0) | (d1 < -d0))
    go_left = ~keep & ~go_right & (d0 < 0) & (d0 >= -width)
    far = ~(keep | go_left | go_right)
    too_far = (go_right & (d1 >= width - halo)) | (go_left & (d0 <= halo - width))
    keep_left, keep_right = keep & (d0 < halo), keep & (d1 >= -halo)       # kept boundary rows
    ghost_left, ghost_right = go_left & (d0 >= -halo), go_right & (d1 < halo)  # handed over, still my ghosts
    mine = torch.stack([go_left.sum(), go_right.sum(), keep_left.sum(), keep_right.sum(), ghost_left.sum(),
                        ghost_right.sum(), far.sum(), too_far.sum()])
    gathered = torch.empty(world * mine.numel(), dtype=mine.dtype, device=mine.device)
    dist.all_gather_into_tensor(gathered, mine)
    table = gathered.view(world, -1).tolist()               # the one device-to-host read
    if any(row[6] for row in table):
        raise RuntimeError("an atom moved further than one slab between two steps")
    if any(row[7] for row in table):
        domain = migrate(domain)
        layout, pos_local, species_local = halo_layout(domain)
        return domain, layout, pos_local, species_local
    GL, GR, KL, KR, HL, HR = range(6)
    me, lt, rt = table[rank], table[domain.left], table[domain.right]
    n_kept = pos.shape[0] - me[GL] - me[GR]
    rows = torch.cat([pos.double(), domain.species.double().unsqueeze(1), domain.ids.double().unsqueeze(1)], 1)

    def pick(mask, count):
        return torch.nonzero_static(mask, size=count).flatten()

    to_left = rows.index_select(0, torch.cat([pick(go_left, me[GL]), pick(keep_left, me[KL])]))
    to_right = rows.index_select(0, torch.cat([pick(go_right, me[GR]), pick(keep_right, me[KR])]))
    from_left, from_right, reqs = _swap_rows(domain, to_left, to_right, lt[GR] + lt[KR], rt[GL] + rt[KL])
    kept_idx = pick(keep, n_kept)
    _wait(reqs)
    arrive_left, ghosts_from_left = from_left[:lt[GR]], from_left[lt[GR]:]
    arrive_right, ghosts_from_right = from_right[:rt[GL]], from_right[rt[GL]:]
    if me[GL] or me[GR] or lt[GR] or rt[GL]:
        owned_rows = torch.cat([rows.index_select(0, kept_idx), arrive_left, arrive_right])
        new = SlabDomain(rank, world, side, halo, owned_rows[:, 4].round().long(),
                         owned_rows[:, :3].to(domain.pos.dtype).contiguous(), owned_rows[:, 3].round().long())
    else:                                                   # nobody moved: keep the tensors (caches stay valid)
        new = SlabDomain(rank, world, side, halo, domain.ids, pos, domain.species)
    # boundary rows of the new owned set, in the order the neighbours hold them as ghosts
    ax_left, ax_right = arrive_left[:, 0], arrive_right[:, 0]
    send_left = torch.cat([pick(keep_left.index_select(0, kept_idx), me[KL]),
                           n_kept + pick(_signed(ax_left, f0, side) < halo, lt[HR])])
    send_right = torch.cat([pick(keep_right.index_select(0, kept_idx), me[KR]),
                            n_kept + lt[GR] + pick(_signed(ax_right, f1, side) >= -halo, rt[HL])])
    left_ghosts = torch.cat([ghosts_from_left, rows.index_select(0, pick(ghost_left, me[HL]))])
    right_ghosts = torch.cat([ghosts_from_right, rows.index_select(0, pick(ghost_right, me[HR]))])
    left_ghosts[:, 0] += -side if rank == 0 else 0.0
    right_ghosts[:, 0] += side if rank == world - 1 else 0.0
    ghosts = torch.cat([left_ghosts, right_ghosts])
    n_own, gl, gr = new.owned, left_ghosts.shape[0], right_ghosts.shape[0]
    pos_local = torch.cat([new.pos, ghosts[:, :3].to(new.pos.dtype)])
    species_local = torch.cat([new.species, ghosts[:, 3].round().long()])
    local_ids = torch.cat([new.ids, ghosts[:, 4].round().long()])
    layout = SlabLayout(rank, world, n_own, send_left, send_right, slice(n_own, n_own + gl),
                        slice(n_own + gl, n_own + gl + gr), domain.left, domain.right, domain.x0, domain.x1, halo,
                        side, local_ids, rounds=1)
    return new, layout, pos_local, species_local


def md_step(model, domain: SlabDomain, cutoff: float, virial: bool = True, phases: StepPhases = NO_PHASES):
    """One MD force evaluation on this rank: migration and ghosts, neighbour list, model.

    Returns (domain after migration, energy [1], owned forces [n_own, 3], virial [6]);
    the forces' rows follow the returned domain's atoms (``domain.ids``)."""
    device = domain.pos.device
    phases.mark("start", device)
    domain, layout, pos_local, species_local = exchange_atoms(domain)
    phases.mark("atoms", device)
    src, dst, shift = slab_edges(layout, pos_local, cutoff)
    phases.mark("neighbours", device)
    energy, forces, w = distributed_energy_forces(model, layout, pos_local, species_local, src, dst, shift,
                                                  virial=virial, phases=phases, owned_species=domain.species)
    return domain, energy, forces, w
