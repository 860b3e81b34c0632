"""Host logic of the graph message (CPU): the destination- and source-sorted CSR
views, index validation and the caches keyed on the index tensors."""
import pytest
import torch


def _check_view(keys, order, offsets, nodes):
    """Edges of node n are order[offsets[n]:offsets[n+1]] (or the identity order), in
    ascending edge id (stable), covering every edge once."""
    order = torch.arange(keys.numel()) if order is None else order
    assert offsets.shape == (nodes + 1,) and int(offsets[0]) == 0 and int(offsets[-1]) == keys.numel()
    assert torch.equal(torch.sort(order).values, torch.arange(keys.numel()))
    for n in range(nodes):
        seg = order[int(offsets[n]):int(offsets[n + 1])]
        assert bool((keys[seg] == n).all())
        assert bool((seg[1:] > seg[:-1]).all())


@pytest.mark.parametrize("nodes,edges,dst_nodes,seed", [(10, 50, 10, 0), (7, 0, 7, 1), (30, 200, 12, 2),
                                                        (5, 9, 0, 3), (1, 4, 1, 4)])
def test_csr_views(nodes, edges, dst_nodes, seed):
    from ictc_o3.backends.cuda.message import graph_csr
    gen = torch.Generator().manual_seed(seed)
    src = torch.randint(0, nodes, (edges,), generator=gen)
    dst = torch.randint(0, max(dst_nodes, 1), (edges,), generator=gen) if dst_nodes else torch.zeros(0, dtype=torch.long)
    if not dst_nodes:
        src = src[:0]
    csr = graph_csr(src, dst, nodes, dst_nodes)
    _check_view(dst, csr.dst_order, csr.dst_offsets, dst_nodes)
    _check_view(src, csr.src_order, csr.src_offsets, nodes)
    assert graph_csr(src, dst, nodes, dst_nodes) is csr                 # cached on the index tensors
    if src.numel():
        src.add_(0)                                                     # a new version: rebuilt
        assert graph_csr(src, dst, nodes, dst_nodes) is not csr


def test_grouped_keys_need_no_order():
    from ictc_o3.backends.cuda.message import _csr, mark_grouped
    keys = torch.tensor([0, 0, 1, 3, 3, 3])
    order, offsets = _csr(keys, 5)
    assert order is None and offsets.tolist() == [0, 2, 3, 3, 6, 6]
    shuffled = torch.tensor([3, 0, 3, 1, 0, 3])
    order, offsets = _csr(shuffled, 4)
    assert order.tolist() == [1, 4, 3, 0, 2, 5] and offsets.tolist() == [0, 2, 3, 3, 6]
    mark_grouped(shuffled, False)
    assert _csr(shuffled, 4)[0] is not None
    shuffled.add_(0)                                                    # the mark is per version
    assert getattr(shuffled, "_ictc_grouped")[0] != shuffled._version


def test_validation():
    from ictc_o3.backends.cuda.message import graph_csr, mark_trusted_graph, validate_graph
    src, dst = torch.tensor([0, 1, 2]), torch.tensor([0, 0, 1])
    with pytest.raises(ValueError, match="outside"):
        graph_csr(src, dst, 2, 2)                                       # source 2 of 2 nodes
    with pytest.raises(ValueError, match="outside"):
        graph_csr(torch.tensor([0, 1]), torch.tensor([0, 2]), 3, 2)     # destination past the owned rows
    with pytest.raises(ValueError, match="int64"):
        validate_graph(src.int(), dst, 3, 2, src.device)
    with pytest.raises(ValueError, match="int64"):
        validate_graph(src, dst[:2], 3, 2, src.device)
    good_src, good_dst = torch.tensor([2, 0]), torch.tensor([1, 0])
    mark_trusted_graph(good_src, good_dst, 3, 2)                        # producer-guaranteed bounds
    validate_graph(good_src, good_dst, 3, 2, good_src.device)


def test_destination_nodes():
    from ictc_o3.backends.cuda.message import destination_nodes

    class Owner:
        pass

    owner = Owner()
    assert destination_nodes(owner, 7) == 7
    owner._cuda_destination_nodes = 3
    assert destination_nodes(owner, 7) == 3
    for bad in (8, -1, True, 2.0):
        owner._cuda_destination_nodes = bad
        with pytest.raises(ValueError):
            destination_nodes(owner, 7)
