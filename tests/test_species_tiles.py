"""Species-homogeneous node tiles (host logic of the symmetric-contraction and
element-linear kernels), checked on the CPU: every node appears exactly once, in
a tile of its own species, tiles are -1 padded, and tile species never decrease
(the table-gradient kernel finds a species' tiles by binary search)."""
import pytest
import torch


@pytest.mark.parametrize("n,S,nb,seed", [(0, 3, 8, 0), (1, 1, 8, 1), (37, 3, 8, 2), (64, 4, 8, 3),
                                         (200, 5, 32, 4), (31, 3, 32, 5)])
def test_tile_invariants(n, S, nb, seed):
    from ictc_o3.backends.cuda.linear import species_tiles_of
    gen = torch.Generator().manual_seed(seed)
    species = torch.randint(0, max(S - 1, 1), (n,), generator=gen)     # the last species absent when S > 1
    tiles, tile_species = species_tiles_of(species, S, nb)
    assert tiles.shape == (n // nb + S, nb) and tiles.dtype == torch.int64
    assert tile_species.shape == (tiles.shape[0],) and tile_species.dtype == torch.int32
    assert bool((tile_species[1:] >= tile_species[:-1]).all())
    assert bool(((tile_species >= 0) & (tile_species < S)).all())
    flat = tiles.flatten()
    nodes = flat[flat >= 0]
    assert torch.equal(torch.sort(nodes).values, torch.arange(n))
    owner = tile_species.to(torch.int64).unsqueeze(1).expand_as(tiles)
    live = tiles >= 0
    assert torch.equal(species[tiles[live]], owner[live])
    # within a tile the live slots come first and keep node order (stable sort)
    for row in tiles:
        live_row = row[row >= 0]
        assert bool((row[:live_row.numel()] >= 0).all())
        assert bool((live_row[1:] > live_row[:-1]).all())


def test_species_outside_table_raises():
    from ictc_o3.backends.cuda.linear import species_tiles_of
    with pytest.raises(ValueError, match="outside"):
        species_tiles_of(torch.tensor([0, 3]), 3, 8)
    with pytest.raises(ValueError, match="outside"):
        species_tiles_of(torch.tensor([-1, 0]), 3, 8)
