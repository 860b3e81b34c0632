"""Slab decomposition with halo exchange (gloo ranks on CPU) vs the single-process model.

Runs the MACE model on the FP64 oracle operators, so the host logic of the
spatial decomposition (ownership, migration, ghost selection, feature exchange
and its adjoint, ghost-force return, energy/virial reduction) is checked without
a GPU.  Cases follow the reference's documented multi-device checks: several
rank counts, changing ownership and empty ranks.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

R_MAX = 3.0


def _system(n_atoms=100, density=0.1, min_dist=0.9, seed=0, x_fraction=1.0, faces=0):
    """Random atoms in a periodic cube; ``x_fraction`` < 1 leaves the rest of x empty;
    ``faces`` = world puts atoms exactly on the slab faces (x = k side / world), at
    x = side and just below it."""
    gen = torch.Generator().manual_seed(seed)
    side = (n_atoms / density) ** (1.0 / 3.0)
    scale = torch.tensor([side * x_fraction, side, side], dtype=torch.float64)
    pos = torch.empty(0, 3, dtype=torch.float64)
    while pos.shape[0] < n_atoms:
        cand = torch.rand(1, 3, generator=gen, dtype=torch.float64) * scale
        d = pos - cand
        d = d - side * torch.round(d / side)
        if pos.shape[0] == 0 or float(d.norm(dim=1).min()) >= min_dist:
            pos = torch.cat([pos, cand])
    species = torch.randint(0, 3, (n_atoms,), generator=gen)
    if faces:
        xs = [side * k / faces for k in range(faces + 1)] + [side * (1.0 - 1e-15), 0.5 * side / faces]
        for i, x in enumerate(xs):
            pos[i, 0] = x
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
    """Single process: (energy, forces in global atom order, virial)."""
    from mace_ictc.parallel import distributed_energy_forces, halo_layout, partition
    model = _model()
    domain = partition(pos, species, side, 0, 1, R_MAX)
    layout, p, s = halo_layout(domain)
    src, dst, shift = _edges(p, p.shape[0], side, R_MAX, True)
    energy, forces, virial = distributed_energy_forces(model, layout, p, s, src, dst, shift)
    out = torch.empty_like(forces)
    out[domain.ids] = forces
    return energy, out, virial


def _worker(rank, world, port, out_dir, case):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        from mace_ictc.parallel import (distributed_energy_forces, exchange_atoms, halo_layout, migrate,
                                        partition)
        pos, species, side = _system(**case["system"])
        domain = partition(pos, species, side, rank, world, R_MAX)
        if case.get("displace"):
            # move every atom (ownership changes across faces and the periodic boundary)
            gen = torch.Generator().manual_seed(100 + rank)
            domain.pos = domain.pos + case["displace"] * (2 * torch.rand(domain.pos.shape, generator=gen,
                                                                           dtype=torch.float64) - 1)
        before = domain.owned
        if case.get("two_round"):
            domain = migrate(domain)
            layout, pos_local, species_local = halo_layout(domain)
        else:
            domain, layout, pos_local, species_local = exchange_atoms(domain)
        moved_pos = domain.pos.clone()
        x = pos_local[:, 0]
        ghosts = x[layout.owned:]
        in_band = ((ghosts >= layout.x0 - R_MAX) & (ghosts < layout.x0)) | ((ghosts >= layout.x1) &
                                                                         (ghosts < layout.x1 + R_MAX))
        src, dst, shift = _edges(pos_local, layout.owned, side, R_MAX, False)
        energy, forces, virial = distributed_energy_forces(_model(), layout, pos_local, species_local, src, dst,
                                                           shift)
        torch.save({"ids": domain.ids, "pos": moved_pos, "species": domain.species, "energy": energy,
                    "forces": forces, "virial": virial, "ghosts": layout.local - layout.owned,
                    "ghosts_in_band": bool(in_band.all()), "owned_before": before, "rounds": layout.rounds,
                    "owned_in_slab": bool(((x[:layout.owned] >= layout.x0) & (x[:layout.owned] < layout.x1)).all())},
                   os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, tmp_path, case):
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), case), nprocs=world, join=True,
                       start_method="spawn")
    return [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]


def _check_against_single(outs, n_atoms, side):
    """Every atom owned exactly once; energy, virial and forces equal the single process
    evaluated on the configuration the ranks hold."""
    pos = torch.full((n_atoms, 3), float("nan"), dtype=torch.float64)
    species = torch.full((n_atoms,), -1, dtype=torch.long)
    forces = torch.full((n_atoms, 3), float("nan"), dtype=torch.float64)
    seen = torch.zeros(n_atoms, dtype=torch.long)
    for out in outs:
        assert out["ghosts_in_band"] and out["owned_in_slab"]
        pos[out["ids"]] = out["pos"]
        species[out["ids"]] = out["species"]
        forces[out["ids"]] = out["forces"]
        seen[out["ids"]] += 1
    assert bool((seen == 1).all()), "every atom is owned by exactly one rank"
    e_ref, f_ref, w_ref = _single(pos, species, side)
    for out in outs:
        torch.testing.assert_close(out["energy"], e_ref, rtol=1e-10, atol=1e-12)
        torch.testing.assert_close(out["virial"], w_ref, rtol=1e-9, atol=1e-11)
    torch.testing.assert_close(forces, f_ref, rtol=1e-9, atol=1e-11)


@pytest.mark.parametrize("world,n_atoms,two_round", [(2, 100, False), (3, 100, False), (4, 256, False),
                                                     (3, 100, True)])
def test_slab_halo_matches_single_process(world, n_atoms, two_round, tmp_path):
    case = {"system": {"n_atoms": n_atoms}, "two_round": two_round}
    outs = _run(world, tmp_path, case)
    assert all(out["ghosts"] > 0 for out in outs)
    assert all(out["rounds"] == (2 if two_round else 1) for out in outs)
    _check_against_single(outs, n_atoms, _system(n_atoms)[2])


@pytest.mark.parametrize("world,displace,two_round", [(3, 0.3, False), (2, 0.5, False), (3, 1.5, False),
                                                      (3, 1.0, True)])
def test_migration_changes_ownership(world, displace, two_round, tmp_path):
    """Atoms displaced across slab faces (and the periodic boundary) are handed to their
    new owners; the result equals the single process on the displaced configuration.
    Small moves take the single-round exchange; moves that reach a new slab's far halo
    band make every rank take the two-round path."""
    n_atoms = 150
    outs = _run(world, tmp_path, {"system": {"n_atoms": n_atoms, "seed": 3}, "displace": displace,
                                  "two_round": two_round})
    assert any(out["owned_before"] != out["ids"].numel() for out in outs), "some atom changed owner"
    rounds = {out["rounds"] for out in outs}
    assert len(rounds) == 1, "all ranks took the same path"
    if displace <= 0.5 and not two_round:
        assert rounds == {1}
    if displace >= 1.5 or two_round:
        assert rounds == {2}
    _check_against_single(outs, n_atoms, _system(n_atoms, seed=3)[2])


def test_empty_ranks(tmp_path):
    """Atoms only in the lower half of x: two of four ranks own nothing (one of them
    still holds ghosts); the decomposition still equals the single process."""
    world, n_atoms = 4, 256
    case = {"system": {"n_atoms": n_atoms, "seed": 5, "x_fraction": 0.45}}
    outs = _run(world, tmp_path, case)
    assert sum(out["ids"].numel() == 0 for out in outs) >= 1
    _check_against_single(outs, n_atoms, _system(n_atoms, seed=5)[2])


@pytest.mark.parametrize("world", [2, 3])
def test_atoms_on_slab_faces(world, tmp_path):
    """Atoms exactly on slab faces and on the periodic boundary: each is owned by one
    rank after the step's exchange, and the result equals the single process."""
    n_atoms = 120
    case = {"system": {"n_atoms": n_atoms, "seed": 7, "faces": world}}
    outs = _run(world, tmp_path, case)
    _check_against_single(outs, n_atoms, _system(n_atoms, seed=7)[2])


def test_thin_slabs_are_rejected():
    from mace_ictc.parallel import partition
    pos, species, side = _system(50, seed=2)
    with pytest.raises(ValueError):
        partition(pos, species, side, 0, 4, side / 3)


def test_step_phases_host_only():
    """StepPhases on the CPU records host times and no device times; disabled ones record nothing."""
    from mace_ictc.parallel import NO_PHASES, StepPhases
    phases = StepPhases()
    phases.mark("start")
    phases.mark("work")
    (name, dev, host), = phases.summary()
    assert name == "work" and dev is None and host >= 0.0
    NO_PHASES.mark("ignored")
    assert NO_PHASES.marks == []
