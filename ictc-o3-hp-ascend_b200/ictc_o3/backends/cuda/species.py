"""Species metadata for the CUDA backend, checked once per tensor version.

Entry points of the reference backend's species module
(``ictc_o3/backends/ascend/species.py:9,20``): ``validate_species(index, count)``
and ``compact_species(owner, atomic_numbers)``, which maps atomic numbers to the
model's compact element indices through ``owner.atomic_number_to_index``
(``mace_ictc/models/pure_cartesian_ictd_fix.py:2368-2379``, hook site :2983-2985).
Each check is one boolean read from the device per (tensor, version).
"""
import weakref

import torch

from .cache import cache_of


def validate_species(index: torch.Tensor, count: int):
    """Raise if an element index lies outside [0, count)."""
    stamp = (int(count), index._version)
    if getattr(index, "_ictc_cuda_valid_species", None) == stamp:
        return
    if index.numel() and bool(((index < 0) | (index >= count)).any()):
        raise ValueError("Species index is outside the weight bank")
    index._ictc_cuda_valid_species = stamp


def compact_species(owner, atomic_numbers: torch.Tensor) -> torch.Tensor:
    """Compact element indices [N] (int64) of atomic numbers [N].

    Atomic numbers outside the mapping table, or mapped to -1 (elements the model
    does not know), raise.  The result is remembered on ``owner`` for the same
    atomic-number tensor, table and element count."""
    table = owner.atomic_number_to_index
    stamp = (atomic_numbers._version, table._version, int(owner.num_elements), atomic_numbers.device)
    store = cache_of(owner, "_cuda_species_memo")
    memo = store.get("memo")
    if memo is not None and memo[0]() is atomic_numbers and memo[1] == stamp and memo[2]._version == memo[3]:
        return memo[2]
    z = atomic_numbers.to(torch.int64)
    inside = (z >= 0) & (z < table.numel())
    index = torch.where(inside, table.index_select(0, z.clamp(0, max(table.numel() - 1, 0))),
                        torch.full_like(z, -1))
    if index.numel() and bool(((index < 0) | (index >= owner.num_elements)).any()):
        raise ValueError("Atomic numbers are outside the model's compact mapping")
    index._ictc_cuda_valid_species = (int(owner.num_elements), index._version)
    store["memo"] = (weakref.ref(atomic_numbers), stamp, index, index._version)
    return index
