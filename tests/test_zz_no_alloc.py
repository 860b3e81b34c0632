"""The allocation-free neighbour search, called through the C ABI.

``ictc_neighbor_list_noalloc`` serves callers that cannot allocate device memory
while they run (an MD engine that owns all device buffers, or a host program
using the C library without an allocator for scratch): its scratch is a fixed
array inside the library.  This file is collected last on purpose; only the
multi-GPU rank tests, which run in processes of their own, follow it.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(pos, box, cutoff, max_edges):
    from ictc_o3.backends.cuda import _native
    lib = _native.library()
    atoms = pos.shape[0]
    box_arr = (ctypes.c_float * 3)(*box)
    offsets = torch.full((atoms + 1,), -7, dtype=torch.int64, device=pos.device)
    src = torch.full((max_edges,), -5, dtype=torch.int64, device=pos.device)
    dst = torch.full((max_edges,), -5, dtype=torch.int64, device=pos.device)
    shift = torch.full((max_edges, 3), -5.0, dtype=torch.float32, device=pos.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(pos.device).cuda_stream)
    status = lib.ictc_neighbor_list_noalloc(ctypes.c_void_p(pos.data_ptr()), atoms, box_arr, ctypes.c_float(cutoff),
                                            ctypes.c_void_p(offsets.data_ptr()), ctypes.c_void_p(src.data_ptr()),
                                            ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(shift.data_ptr()),
                                            max_edges, stream)
    torch.cuda.synchronize(pos.device)
    return status, offsets, src, dst, shift


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(cuda_device):
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    box, cutoff = (31.0, 27.5, 29.0), 5.0
    for seed, atoms in ((1, 2500), (2, 1800)):
        gen = torch.Generator(device=cuda_device).manual_seed(seed)
        pos = torch.rand(atoms, 3, device=cuda_device, generator=gen) * torch.tensor(box, device=cuda_device)
        ref_src, ref_dst, ref_shift, ref_offsets = neighbor_list(pos, box, cutoff)
        edges = ref_src.numel()
        status, offsets, src, dst, shift = _noalloc(pos, box, cutoff, edges + 17)
        assert status == 0
        assert torch.equal(offsets, ref_offsets)
        assert torch.equal(src[:edges], ref_src) and torch.equal(dst[:edges], ref_dst)
        assert torch.equal(shift[:edges], ref_shift)
        assert bool((src[edges:] == -5).all())


def test_noalloc_capacity_and_size_limits(cuda_device):
    from ictc_o3.backends.cuda import _native
    box, cutoff = (20.0, 20.0, 20.0), 5.0
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    pos = torch.rand(800, 3, device=cuda_device, generator=gen) * 20.0
    status, offsets, src, _, _ = _noalloc(pos, box, cutoff, 4)
    assert status == 0 and int(offsets[-1]) > 4
    assert bool((src == -5).all()), "nothing is written when the capacity is too small"
    lib = _native.library()
    limit = int(lib.ictc_neighbor_noalloc_scratch_bytes())
    assert limit == 8 << 20
    huge = (ctypes.c_float * 3)(500.0, 500.0, 500.0)
    status = lib.ictc_neighbor_list_noalloc(ctypes.c_void_p(pos.data_ptr()), 5_000_000, huge, ctypes.c_float(5.0),
                                            ctypes.c_void_p(pos.data_ptr()), None, None, None, 0, None)
    assert status == -1 and b"exceed" in lib.ictc_last_error()
