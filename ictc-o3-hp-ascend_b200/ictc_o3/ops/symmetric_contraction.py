"""Species-conditioned symmetric contraction in the ICTC basis (CUDA backend).

Mirrors the reference's pure-ICTC contraction (``ICTDPureUSymmetricContractionSO3`` /
``_ICTDPureUContraction``, ``mace_ictc/models/pure_cartesian_ictd_fix.py:1202-1387``):
per target degree t a MACE contraction with U tensors generated from ICTC
couplings only (``ictd_u_matrix_so3``, ``ictc_o3/basis/ictd_irreps.py:1465-1517``)
and trainable per-element weights ``weights_max`` [S, P_corr, C] and
``weights[j]`` [S, P_{corr-1-j}, C] (same buffer and parameter names, so state
dicts carry over).  The reference's bridge-U variant needs e3nn's real
Wigner-3j matrices, which this build does not have; the pure-ICTC U spans the
same intertwiner space.
"""
from __future__ import annotations

from typing import Dict

import numpy as np
import torch
import torch.nn as nn

from ictc_o3.basis.ictd_irreps import ictd_u_matrix_so3


class _ICTDPureUContraction(nn.Module):
    """One target degree: U buffers and per-element weights."""

    def __init__(self, *, u_tensors: Dict[int, np.ndarray], output_l: int, num_elements: int, num_features: int):
        super().__init__()
        self.output_l = int(output_l)
        self.correlation = int(max(u_tensors))
        self.num_elements = int(num_elements)
        self.num_features = int(num_features)
        self._u64 = {nu: np.asarray(u, dtype=np.float64) for nu, u in u_tensors.items()}
        for nu in range(1, self.correlation + 1):
            self.register_buffer(f"U_matrix_{nu}", torch.from_numpy(self._u64[nu].copy()).float())
        num = self.U_tensors(self.correlation).shape[-1]
        self.weights_max = nn.Parameter(torch.randn(num_elements, num, num_features) / max(num, 1))
        self.weights = nn.ParameterList([])
        for nu in range(self.correlation - 1, 0, -1):
            num = self.U_tensors(nu).shape[-1]
            self.weights.append(nn.Parameter(torch.randn(num_elements, num, num_features) / max(num, 1)))
        self._table_cache = {}

    def U_tensors(self, nu: int) -> torch.Tensor:
        return getattr(self, f"U_matrix_{nu}")

    def stacked_weights(self) -> torch.Tensor:
        """[S, sum P, C], weight columns ordered nu = corr, corr-1, ..., 1."""
        return torch.cat([self.weights_max, *self.weights], 1)

    def symmetric_table(self, device, dtype=torch.float32) -> torch.Tensor:
        """Symmetrised U in the kernel's row order, [rows * (2t+1), sum P] (cached per device, dtype)."""
        key = (str(device), dtype)
        table = self._table_cache.get(key)
        if table is None:
            from ictc_o3.backends.cuda.contraction import symmetric_table
            dim = self._u64[1].shape[-2]
            sym = symmetric_table(self._u64, self.output_l, dim, self.correlation)
            table = torch.from_numpy(sym.reshape(-1, sym.shape[-1])).to(device=device, dtype=dtype)
            self._table_cache[key] = table
        return table


class ICTDPureUSymmetricContractionSO3(nn.Module):
    """MACE-style symmetric contraction; forward(node_feats, node_attrs, node_type_idx=None).

    node_feats: [N, C*(lmax+1)^2] flat ICTC features (degree blocks [C][2l+1]);
    returns [N, C*(target_lmax+1)^2] in the same layout.
    """

    def __init__(self, *, num_elements: int, channels: int, lmax: int, target_lmax: int, correlation: int = 3):
        super().__init__()
        if correlation not in (1, 2, 3):
            raise ValueError("The CUDA symmetric contraction supports correlation 1, 2 and 3")
        if not 1 <= lmax <= 3 or not 0 <= target_lmax <= lmax:
            raise ValueError("The CUDA symmetric contraction supports 1 <= lmax <= 3 and target_lmax <= lmax")
        self.num_elements = int(num_elements)
        self.channels = int(channels)
        self.lmax = int(lmax)
        self.target_lmax = int(target_lmax)
        self.correlation = int(correlation)
        self.contractions = nn.ModuleList()
        for t in range(self.target_lmax + 1):
            u = {nu: ictd_u_matrix_so3(self.lmax, t, nu) for nu in range(1, self.correlation + 1)}
            self.contractions.append(_ICTDPureUContraction(u_tensors=u, output_l=t, num_elements=num_elements,
                                                           num_features=channels))

    def forward(self, node_feats: torch.Tensor, node_attrs: torch.Tensor | None = None,
                node_type_idx: torch.Tensor | None = None) -> torch.Tensor:
        from ictc_o3.backends.cuda.contraction import contract_flat
        if node_type_idx is None:
            if node_attrs is None:
                raise ValueError("node_attrs or node_type_idx is required")
            node_type_idx = node_attrs.argmax(-1)
        return contract_flat(self, node_feats, node_type_idx)


SymmetricContraction = ICTDPureUSymmetricContractionSO3
