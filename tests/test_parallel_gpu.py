"""Spatial decomposition on the GPU: slab edge lists, and NCCL halo exchange on 2 GPUs."""
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


def _edge_keys(src, dst, vec, n):
    key = dst * n + src
    order = torch.argsort(key)
    return key[order], vec[order]


@pytest.mark.parametrize("world", [2, 3, 4])
def test_slab_edges_cover_global_neighbour_list(world, cuda_device):
    """Every rank's owned-receiver edges, mapped to global atoms, together are exactly the
    global neighbour list, with the same edge vectors."""
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    from mace_ictc.parallel import local_positions, slab_edges, slab_layout
    from mace_ictc.systems import random_system
    n = 6000
    pos, _, side = random_system(n, seed=5, device=cuda_device)
    src, dst, shift, _ = neighbor_list(pos, (side,) * 3, CUTOFF)
    ref_key, ref_vec = _edge_keys(src, dst, pos[dst] - pos[src] + shift, n)
    keys, vecs = [], []
    for rank in range(world):
        layout = slab_layout(pos, side, rank, world, CUTOFF)
        p = local_positions(layout, pos, side)
        s, d, sh = slab_edges(layout, p, side, CUTOFF, CUTOFF)
        assert int(d.max()) < layout.owned
        assert bool((d[1:] >= d[:-1]).all()), "edges grouped by receiver"
        g = layout.local_global
        keys.append(g[d] * n + g[s])
        vecs.append(p[d] - p[s] + sh)
    key = torch.cat(keys)
    order = torch.argsort(key)
    assert torch.equal(key[order], ref_key)
    torch.testing.assert_close(torch.cat(vecs)[order], ref_vec, rtol=0, atol=2e-4)


def _model(channels=32):
    from mace_ictc.models import MACEICTC
    torch.manual_seed(5)
    return MACEICTC(channels=channels, lmax=2, r_max=CUTOFF, avg_num_neighbors=40.0)


def test_single_rank_decomposition_matches_model(cuda_device):
    """world = 1: distributed_energy_forces equals energy_and_forces of the same model."""
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    from mace_ictc.parallel import distributed_energy_forces, local_positions, slab_edges, slab_layout
    from mace_ictc.systems import random_system
    pos, species, side = random_system(3000, seed=6, device=cuda_device)
    model = _model().to(cuda_device)
    src, dst, shift, _ = neighbor_list(pos, (side,) * 3, CUTOFF)
    e_ref, f_ref = model.energy_and_forces(pos, species, src, dst, shift)
    layout = slab_layout(pos, side, 0, 1, CUTOFF)
    p = local_positions(layout, pos, side)
    s, d, sh = slab_edges(layout, p, side, CUTOFF, CUTOFF)
    e, f, w = distributed_energy_forces(model, layout, p, species[layout.local_global], s, d, sh)
    assert_close(e, e_ref, 1e-5, what="energy")
    f_global = torch.empty_like(f)
    f_global[layout.local_global] = f
    assert_close(f_global, f_ref, 1e-4, what="forces")
    assert w.shape == (6,)


def _nccl_worker(rank, world, port, out_dir, n_atoms):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=device)
    try:
        from mace_ictc.parallel import distributed_energy_forces, local_positions, slab_edges, slab_layout
        from mace_ictc.systems import random_system
        pos, species, side = random_system(n_atoms, seed=8, device=device)
        model = _model().to(device)
        layout = slab_layout(pos, side, rank, world, CUTOFF)
        p = local_positions(layout, pos, side)
        s, d, sh = slab_edges(layout, p, side, CUTOFF, CUTOFF)
        e, f, w = distributed_energy_forces(model, layout, p, species[layout.local_global], s, d, sh)
        torch.save({"owned": layout.local_global[:layout.owned].cpu(), "energy": e.cpu(), "forces": f.cpu(),
                    "virial": w.cpu()}, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def test_two_gpu_halo_exchange_matches_one_gpu(cuda_device, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from mace_ictc.parallel import distributed_energy_forces, local_positions, slab_edges, slab_layout
    from mace_ictc.systems import random_system
    n_atoms, world = 8000, 2
    pos, species, side = random_system(n_atoms, seed=8, device=cuda_device)
    model = _model().to(cuda_device)
    layout = slab_layout(pos, side, 0, 1, CUTOFF)
    p = local_positions(layout, pos, side)
    s, d, sh = slab_edges(layout, p, side, CUTOFF, CUTOFF)
    e_ref, f_ref, w_ref = distributed_energy_forces(model, layout, p, species[layout.local_global], s, d, sh)
    mp.start_processes(_nccl_worker, args=(world, _free_port(), str(tmp_path), n_atoms), nprocs=world, join=True,
                       start_method="spawn")
    forces = torch.full((n_atoms, 3), float("nan"))
    f_ref_global = torch.empty(n_atoms, 3)
    f_ref_global[layout.local_global.cpu()] = f_ref.cpu()
    for rank in range(world):
        out = torch.load(tmp_path / f"rank{rank}.pt")
        forces[out["owned"]] = out["forces"]
        assert_close(out["energy"], e_ref.cpu(), 1e-5, what="energy")
        assert_close(out["virial"], w_ref.cpu(), 1e-4, what="virial")
    assert not bool(torch.isnan(forces).any())
    assert_close(forces, f_ref_global, 1e-4, what="forces")
