"""Slab decomposition with halo exchange (gloo ranks on CPU) vs the single-process model.

Runs the MACE model on the FP64 oracle operators, so the host logic of the
spatial decomposition (ownership, ghost selection, feature exchange and its
adjoint, ghost-force return, virial reduction) is checked without a GPU.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

R_MAX = 3.0


def _system(n_atoms=100, density=0.1, min_dist=0.9, seed=0):
    gen = torch.Generator().manual_seed(seed)
    side = (n_atoms / density) ** (1.0 / 3.0)
    pos = torch.empty(0, 3, dtype=torch.float64)
    while pos.shape[0] < n_atoms:
        cand = torch.rand(1, 3, generator=gen, dtype=torch.float64) * side
        d = pos - cand
        d = d - side * torch.round(d / side)
        if pos.shape[0] == 0 or float(d.norm(dim=1).min()) >= min_dist:
            pos = torch.cat([pos, cand])
    species = torch.randint(0, 3, (n_atoms,), generator=gen)
    return pos, species, side


def _model():
    from mace_ictc.models import MACEICTC
    from oracle.model_ops import OracleOps
    torch.manual_seed(11)
    model = MACEICTC(channels=8, lmax=2, r_max=R_MAX, avg_num_neighbors=5.0, ops=OracleOps())
    return model.double()


def _edges(pos, receivers, side, cutoff, periodic_x):
    """(src, dst, shift) for receivers [0, receivers), minimum image in y, z (and x if periodic_x)."""
    d = pos[:receivers, None, :] - pos[None, :, :]                 # d[i, j] = pos[i] - pos[j]
    shift = -side * torch.round(d / side)
    if not periodic_x:
        shift[..., 0] = 0.0
    dist_ = (d + shift).norm(dim=-1)
    i, j = torch.nonzero(dist_ < cutoff, as_tuple=True)
    keep = i != j
    i, j = i[keep], j[keep]
    return j, i, shift[i, j]


def _single(pos, species, side):
    from mace_ictc.parallel import slab_layout, distributed_energy_forces
    model = _model()
    layout = slab_layout(pos, side, 0, 1, R_MAX)
    src, dst, shift = _edges(pos, pos.shape[0], side, R_MAX, True)
    energy, forces, virial = distributed_energy_forces(model, layout, pos, species, src, dst, shift)
    return energy, forces, virial


def _worker(rank, world, port, out_dir, n_atoms):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from mace_ictc.parallel import slab_layout, local_positions, distributed_energy_forces
        pos, species, side = _system(n_atoms)
        model = _model()
        layout = slab_layout(pos, side, rank, world, R_MAX)
        pos_local = local_positions(layout, pos, side)
        species_local = species.index_select(0, layout.local_global)
        src, dst, shift = _edges(pos_local, layout.owned, side, R_MAX, False)
        energy, forces, virial = distributed_energy_forces(model, layout, pos_local, species_local, src, dst, shift)
        torch.save({"owned": layout.local_global[:layout.owned], "energy": energy, "forces": forces,
                    "virial": virial, "ghosts": layout.local - layout.owned},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_slab_halo_matches_single_process(world, tmp_path):
    n_atoms = 100
    pos, species, side = _system(n_atoms)
    e_ref, f_ref, w_ref = _single(pos, species, side)
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), n_atoms), nprocs=world, join=True,
                       start_method="spawn")
    forces = torch.full_like(f_ref, float("nan"))
    seen = torch.zeros(n_atoms, dtype=torch.long)
    for rank in range(world):
        out = torch.load(tmp_path / f"rank{rank}.pt")
        assert out["ghosts"] > 0
        forces[out["owned"]] = out["forces"]
        seen[out["owned"]] += 1
        torch.testing.assert_close(out["energy"], e_ref, rtol=1e-10, atol=1e-12)
        torch.testing.assert_close(out["virial"], w_ref, rtol=1e-9, atol=1e-11)
    assert bool((seen == 1).all()), "every atom is owned by exactly one rank"
    torch.testing.assert_close(forces, f_ref, rtol=1e-9, atol=1e-11)


def test_slab_layout_send_lists_match_ghosts():
    """The rows a rank sends to a neighbour are, in order, that neighbour's ghost rows."""
    from mace_ictc.parallel import slab_layout
    pos, _, side = _system(200, seed=4)
    world = 4
    halo = 2.5
    layouts = [slab_layout(pos, side, r, world, halo) for r in range(world)]
    for r, lay in enumerate(layouts):
        left, right = layouts[lay.left], layouts[lay.right]
        mine = lay.local_global
        # my left ghosts = my left neighbour's send_right rows
        assert torch.equal(mine[lay.ghost_left], left.local_global[left.send_right])
        assert torch.equal(mine[lay.ghost_right], right.local_global[right.send_left])
        x = pos[mine, 0] - side * torch.floor(pos[mine, 0] / side)
        owned_x = x[:lay.owned]
        assert bool(((owned_x >= lay.x0) & (owned_x < lay.x1)).all())
        unwrapped = pos[mine, 0] - side * torch.floor(pos[mine, 0] / side) + lay.local_shift_x
        ghosts = unwrapped[lay.owned:]
        assert bool((((ghosts >= lay.x0 - halo) & (ghosts < lay.x0)) | ((ghosts >= lay.x1) & (ghosts < lay.x1 + halo))).all())


def test_slab_layout_rejects_thin_slabs():
    from mace_ictc.parallel import slab_layout
    pos, _, side = _system(50, seed=2)
    with pytest.raises(ValueError):
        slab_layout(pos, side, 0, 4, side / 3)
