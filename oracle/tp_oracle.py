"""CPU oracle for the ICTC-O3 hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU, the reference algorithms
the CUDA backend must reproduce.  It is imported only by ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arms,
always as the checker or the timed CPU baseline, never as a product path.

Pinning: the golden fixtures under ``tests/golden/`` were produced by the
reference implementation itself (``tests/golden/make_golden.py`` imports
``ictc_o3`` from the reference tree); ``tests/test_oracle_golden.py`` checks
this oracle against them, so the oracle is pinned to the reference.

Followed reference code (paths inside the reference project):
* TP forward        -- ictc_o3/basis/ictd_irreps.py:2669-2748 (_forward_index_add)
                       and :2278-2283 (_project_group), projector :2239-2263
* graph message     -- ictc_o3/backends/ascend/tensor_product.py:189-218
                       (gather by src, TP, mask, index_add into dst)
* direction harmonics -- ictc_o3/basis/ictd_irreps.py:1113-1168

The owner object supplies the constants (paths, groups, path offsets, CG
list) through the reference attribute names, so the same functions run on a
reference owner and on the backend's owner.
"""
from typing import Dict, List

import numpy as np
import torch


def _cg_list(owner, dtype):
    if hasattr(owner, "cg_f64"):
        return [torch.from_numpy(np.array(c, dtype=np.float64)).to(dtype) for c in owner.cg_f64()]
    return [c.detach().to(dtype) for c in owner._get_cg_list(torch.device("cpu"), dtype)]


def projector_groups(owner, dtype) -> List[torch.Tensor]:
    """U_group [m1*m2, sum m3] per (l1, l2) group (ictd_irreps.py:2239-2263)."""
    cg = _cg_list(owner, dtype)
    groups = []
    for g in owner._groups:
        m1, m2 = 2 * int(g["l1"]) + 1, 2 * int(g["l2"]) + 1
        U = torch.zeros(m1 * m2, int(g["k_total"]), dtype=dtype)
        for p, _l3, s, e in g["segments"]:
            U[:, s:e] = cg[p].reshape(m1 * m2, e - s)
        groups.append(U)
    return groups


def tp_forward(owner, x1: Dict[int, torch.Tensor], x2: Dict[int, torch.Tensor], gates=None,
               weight=None, dtype=torch.float32) -> Dict[int, torch.Tensor]:
    """Path-preserving TP: x1 l -> [E, C, 2l+1], x2 l -> [E, 1, 2l+1], gates [E, P, C]."""
    channels = int(owner.channels)
    sample = next(iter(x1.values()))
    rows = sample.shape[0]
    weight = owner.weight.detach() if weight is None else weight
    weight = weight.to(dtype)
    if gates is not None and gates.shape[-1] == owner.num_paths * channels:
        gates = gates.reshape(rows, owner.num_paths, channels)
    U = projector_groups(owner, dtype)
    out = {l: torch.zeros(rows, channels * int(owner.path_counts_by_l.get(l, 0)), 2 * l + 1, dtype=dtype)
           for l in range(owner.lmax + 1)}
    for g_idx, g in enumerate(owner._groups):
        a, b = x1.get(int(g["l1"])), x2.get(int(g["l2"]))
        if a is None or b is None:
            continue
        a, b = a.to(dtype), b.to(dtype)
        pair = (a.unsqueeze(-1) * b.unsqueeze(-2)).reshape(rows, channels, a.shape[-1] * b.shape[-1])
        y = torch.matmul(pair, U[g_idx])
        for p, l3, s, e in g["segments"]:
            seg = y[..., s:e] * weight[p].view(1, channels, 1)
            if gates is not None:
                seg = seg * gates[:, p, :].to(dtype).unsqueeze(-1)
            c0 = int(owner.path_offset[p]) * channels
            out[l3] = out[l3].index_add(1, torch.arange(c0, c0 + channels), seg)
    return out


def graph_message(owner, x1, x2, gates, src, dst, mask=None, nodes=None, dtype=torch.float32):
    """node_out[dst] += TP(x1[src], x2_e, gates_e) * mask_e."""
    rows = int(src.numel())
    nodes = next(iter(x1.values())).shape[0] if nodes is None else nodes
    edge_x = {l: v.index_select(0, src) for l, v in x1.items()}
    value = tp_forward(owner, edge_x, x2, gates, dtype=dtype)
    out = {}
    for l, block in value.items():
        if mask is not None:
            block = block * mask.to(dtype).reshape(-1, 1, 1)
        out[l] = torch.zeros(nodes, *block.shape[1:], dtype=dtype).index_add(0, dst, block)
    del rows
    return out


def direction_harmonics(n: torch.Tensor, lmax: int, tables) -> List[torch.Tensor]:
    """Y_l(n) = (monomials(n) * multinomials) @ (G_l B_l) * scale_l.

    ``tables[l] = (exponents [D,3] int, multinomials [D], projector [D,2l+1], scale)``.
    """
    out = [torch.ones(*n.shape[:-1], 1, dtype=n.dtype)]
    powers = [torch.stack([torch.ones_like(n[..., c])] + [n[..., c] ** k for k in range(1, lmax + 1)], -1)
              for c in range(3)]
    for l in range(1, lmax + 1):
        exps, coefs, proj, scale = tables[l]
        t = powers[0][..., exps[:, 0]] * powers[1][..., exps[:, 1]] * powers[2][..., exps[:, 2]]
        t = t * coefs.to(n.dtype)
        out.append((t @ proj.to(n.dtype)) * scale)
    return out


def packed_to_blocks(features, channels, lmax, layout):
    """Packed [E, C(L+1)^2] -> l -> [E, C, 2l+1] (ictc_o3/operators.py:88-99)."""
    out, offset = {}, 0
    for l in range(lmax + 1):
        width = channels * (2 * l + 1)
        value = features[:, offset:offset + width]
        out[l] = (value.reshape(-1, 2 * l + 1, channels).transpose(1, 2) if layout == "ir_mul"
                  else value.reshape(-1, channels, 2 * l + 1))
        offset += width
    return out


def blocks_to_packed_output(owner, blocks, layout):
    """l -> [E, count*C, 2l+1] -> packed output (ictc_o3/operators.py:107-115)."""
    rows = next(iter(blocks.values())).shape[0]
    parts = []
    for l in range(owner.lmax + 1):
        count = int(owner.path_counts_by_l.get(l, 0))
        value = blocks[l].reshape(rows, count, owner.channels, 2 * l + 1)
        if layout == "ir_mul":
            value = value.transpose(2, 3)
        parts.append(value.reshape(rows, count * owner.channels * (2 * l + 1)))
    return torch.cat(parts, -1)


def split_mul_ir(packed, channels, lmax):
    return packed_to_blocks(packed, channels, lmax, "mul_ir")


def split_harm(packed, lmax):
    """Packed harmonics [E, (L+1)^2] -> l -> [E, 1, 2l+1] (ictc_o3/operators.py:101-105)."""
    return {l: packed[:, l * l:(l + 1) ** 2].unsqueeze(1) for l in range(lmax + 1)}


def pack_out(owner, blocks):
    return blocks_to_packed_output(owner, blocks, "mul_ir")


def harmonic_tables(lmax):
    """Per-degree constants of ``direction_harmonics`` from the host basis module."""
    from ictc_o3.basis import ictd_irreps as basis
    tables = {}
    for l in range(1, lmax + 1):
        tables[l] = (torch.tensor(basis.counts_list(l), dtype=torch.int64),
                     torch.from_numpy(basis.multinomials(l)),
                     torch.from_numpy(basis.direction_projector(l)),
                     basis.direction_component_scale(l))
    return tables
