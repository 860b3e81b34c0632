"""GPU cell-list neighbour search vs a brute-force minimum-image search."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def brute(pos, box, cutoff):
    box = torch.as_tensor(box, dtype=torch.float64, device=pos.device)
    p = pos.double()
    d = p[:, None, :] - p[None, :, :]                 # d[i, j] = pos[i] - pos[j]
    s = -box * torch.round(d / box)
    dist = (d + s).norm(dim=-1)
    i, j = torch.nonzero((dist < cutoff) & ~torch.eye(len(p), dtype=torch.bool, device=p.device), as_tuple=True)
    return j, i, s[i, j]


@pytest.mark.parametrize("atoms,box,cutoff", [(500, (22.0, 17.0, 19.5), 5.0), (4096, (34.4, 34.4, 34.4), 5.0),
                                              (64, (15.1, 15.1, 15.1), 5.0), (0, (16.0, 16.0, 16.0), 5.0),
                                              (30, (40.0, 40.0, 40.0), 0.9)])
def test_neighbor_list_matches_brute_force(atoms, box, cutoff, cuda_device):
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    gen = torch.Generator(device=cuda_device).manual_seed(atoms)
    pos = torch.rand(atoms, 3, device=cuda_device, generator=gen) * torch.tensor(box, device=cuda_device)
    if atoms > 4:
        pos[:4] += torch.tensor(box, device=cuda_device) * torch.tensor([[1.0], [-1.0], [2.0], [0.0]], device=cuda_device)
    src, dst, shift, offsets = neighbor_list(pos, box, cutoff)
    assert offsets.shape == (atoms + 1,) and int(offsets[-1]) == src.numel()
    assert torch.all(dst[1:] >= dst[:-1]), "edges must be grouped by destination"
    if atoms:
        counts = torch.bincount(dst, minlength=atoms)
        assert torch.equal(offsets[1:] - offsets[:-1], counts)
    rs, rd, rshift = brute(pos, box, cutoff)
    assert src.numel() == rs.numel()
    key = dst * max(atoms, 1) + src
    rkey = rd * max(atoms, 1) + rs
    order, rorder = torch.argsort(key), torch.argsort(rkey)
    assert torch.equal(key[order], rkey[rorder])
    vec = pos[dst] - pos[src] + shift
    rvec = pos.double()[rd] - pos.double()[rs] + rshift
    if src.numel():
        assert float((vec[order].double() - rvec[rorder]).abs().max()) < 1e-4
    if src.numel():
        assert float(vec.norm(dim=1).max()) < cutoff
    # Deterministic: a second build is identical.
    src2, dst2, shift2, _ = neighbor_list(pos, box, cutoff)
    assert torch.equal(src, src2) and torch.equal(dst, dst2) and torch.equal(shift, shift2)


def test_neighbor_list_rejects_small_boxes(cuda_device):
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    with pytest.raises(ValueError):
        neighbor_list(torch.zeros(4, 3, device=cuda_device), (9.0, 9.0, 9.0), 5.0)
