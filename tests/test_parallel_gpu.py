"""Spatial decomposition on GPUs: NCCL ranks (2, 4, 8 B200) against one GPU.

Every rank runs ``md_step`` (migration, ghost positions over NCCL, owned-receiver
neighbour list, model with the feature halo and its adjoint, ghost-force return,
energy/virial all-reduce).  The parent process compares energy, forces and
virial with the single-GPU evaluation of the same configuration, and checks that
the ranks' edges, mapped to global atoms, are exactly the global neighbour list.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _util import assert_close

pytestmark = pytest.mark.gpu

CUTOFF = 5.0


def _model(channels=32):
    from mace_ictc.models import MACEICTC
    torch.manual_seed(5)
    return MACEICTC(channels=channels, lmax=2, r_max=CUTOFF, avg_num_neighbors=40.0)


def _system(n_atoms, seed, device, x_fraction=1.0):
    """Random system; with ``x_fraction`` < 1 only atoms with x below that fraction of the
    box are kept (the rest of x is vacuum, so some slabs own nothing)."""
    from mace_ictc.systems import random_system
    pos, species, side = random_system(n_atoms, seed=seed, device=device)
    if x_fraction < 1.0:
        keep = pos[:, 0] < x_fraction * side
        pos, species = pos[keep].contiguous(), species[keep].contiguous()
    return pos, species, side


def _one_gpu(pos, species, side, model):
    """Single-process reference: energy, forces in atom order, virial, sorted edge keys/vectors."""
    from mace_ictc.parallel import md_step, partition
    domain = partition(pos, species, side, 0, 1, CUTOFF)
    domain, e, f, w = md_step(model, domain, CUTOFF)
    forces = torch.empty_like(f)
    forces[domain.ids] = f
    return e, forces, w


def test_single_rank_decomposition_matches_model(cuda_device):
    """world = 1: md_step equals energy_and_forces of the same model."""
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    pos, species, side = _system(3000, 6, cuda_device)
    model = _model().to(cuda_device)
    src, dst, shift, _ = neighbor_list(pos, (side,) * 3, CUTOFF)
    e_ref, f_ref = model.energy_and_forces(pos, species, src, dst, shift)
    e, f, w = _one_gpu(pos, species, side, model)
    assert_close(e, e_ref, 1e-5, what="energy")
    assert_close(f, f_ref, 1e-4, what="forces")
    assert w.shape == (6,)


def _nccl_worker(rank, world, port, out_dir, n_atoms, x_fraction):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=device)
    try:
        from mace_ictc.parallel import distributed_energy_forces, exchange_atoms, partition, slab_edges
        pos, species, side = _system(n_atoms, 8, device, x_fraction)
        model = _model().to(device)
        domain, layout, p, s = exchange_atoms(partition(pos, species, side, rank, world, CUTOFF))
        src, dst, shift = slab_edges(layout, p, CUTOFF)
        e, f, w = distributed_energy_forces(model, layout, p, s, src, dst, shift, owned_species=domain.species)
        ids = layout.local_ids
        torch.save({"owned": domain.ids.cpu(), "energy": e.cpu(), "forces": f.cpu(), "virial": w.cpu(),
                    "edge_keys": (ids[dst] * pos.shape[0] + ids[src]).cpu(), "edge_vecs": (p[dst] - p[src] + shift).cpu(),
                    "receivers_owned": bool(dst.numel() == 0 or int(dst.max()) < layout.owned)},
                   os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _run_ranks(worker, args, world, deadline_s=300.0):
    """Start ``world`` rank processes and wait for them with a deadline.

    If a rank fails, the others can be left waiting for it inside NCCL; they are
    then ended with SIGKILL (only the processes started here) so that the test fails
    promptly instead of waiting for ever."""
    import signal
    import time
    ctx = mp.start_processes(worker, args=args, nprocs=world, join=False, start_method="spawn")
    start = time.time()
    try:
        while not ctx.join(timeout=5):
            if time.time() - start > deadline_s:
                raise TimeoutError(f"ranks did not finish within {deadline_s:.0f} s")
    except BaseException:
        for pid in ctx.pids():
            try:
                os.kill(pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
        raise


@pytest.mark.multigpu
@pytest.mark.parametrize("world,x_fraction", [(2, 1.0), (4, 1.0), (8, 1.0), (4, 0.45)])
def test_nccl_ranks_match_one_gpu(world, x_fraction, cuda_device, tmp_path):
    """world ranks on world GPUs equal one GPU: energy 1e-5, forces and virial 1e-4, and
    the union of the ranks' edges is the global neighbour list (x_fraction < 1: vacuum,
    some ranks own no atoms)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    n_atoms = 4000 * world
    pos, species, side = _system(n_atoms, 8, cuda_device, x_fraction)
    model = _model().to(cuda_device)
    e_ref, f_ref, w_ref = _one_gpu(pos, species, side, model)
    src, dst, shift, _ = neighbor_list(pos, (side,) * 3, CUTOFF)
    n = pos.shape[0]
    ref_key = dst * n + src
    order = torch.argsort(ref_key)
    ref_key, ref_vec = ref_key[order].cpu(), (pos[dst] - pos[src] + shift)[order].cpu()
    _run_ranks(_nccl_worker, (world, _free_port(), str(tmp_path), n_atoms, x_fraction), world)
    forces = torch.full((n, 3), float("nan"))
    seen = torch.zeros(n, dtype=torch.long)
    keys, vecs, empty = [], [], 0
    for rank in range(world):
        out = torch.load(tmp_path / f"rank{rank}.pt")
        forces[out["owned"]] = out["forces"]
        seen[out["owned"]] += 1
        empty += int(out["owned"].numel() == 0)
        assert out["receivers_owned"]
        keys.append(out["edge_keys"])
        vecs.append(out["edge_vecs"])
        assert_close(out["energy"], e_ref.cpu(), 1e-5, what="energy")
        assert_close(out["virial"], w_ref.cpu(), 1e-4, what="virial")
    assert bool((seen == 1).all()), "every atom owned by exactly one rank"
    if x_fraction < 1.0:
        assert empty >= 1, "the vacuum case has a rank without atoms"
    assert_close(forces, f_ref.cpu(), 1e-4, what="forces")
    key = torch.cat(keys)
    order = torch.argsort(key)
    assert torch.equal(key[order], ref_key)
    torch.testing.assert_close(torch.cat(vecs)[order], ref_vec, rtol=0, atol=2e-4)
