"""Species-conditioned symmetric contraction in the ICTC basis (CUDA backend).

Mirrors the reference's pure-ICTC contraction (``ICTDPureUSymmetricContractionSO3`` /
``_ICTDPureUContraction``, ``mace_ictc/models/pure_cartesian_ictd_fix.py:1202-1387``):
per target degree t a MACE contraction with U tensors generated from ICTC
couplings only (``ictd_u_matrix_so3``, ``ictc_o3/basis/ictd_irreps.py:1465-1517``)
and trainable per-element weights ``weights_max`` [S, P_corr, C] and
``weights[j]`` [S, P_{corr-1-j}, C] (same buffer and parameter names, so state
dicts carry over).

The reference's default bridge-U contraction (``ICTDBridgeUSymmetricContractionSO3``,
``ictc_o3/ops/symmetric_contraction.py:92-206``) differs only in its coupling
tensors: MACE's e3nn-basis couplings with the ICTC-to-e3nn basis change folded in
at construction, so they act on ICTC features directly.  The class of that name
here evaluates whatever couplings its ``U_matrix_nu`` buffers hold on the same
kernels: the ICTC couplings in a new module (the same intertwiner space), the
reference's own once one of its state dicts is loaded (identical state-dict names
and shapes).
"""
from __future__ import annotations

import weakref
from typing import Dict

import numpy as np
import torch
import torch.nn as nn

from ictc_o3.basis.ictd_irreps import ictd_u_matrix_so3
from ictc_o3.backends.cuda.cache import cache_of


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

    def U_tensors(self, nu: int) -> torch.Tensor:
        return getattr(self, f"U_matrix_{nu}")

    def stacked_weights(self) -> torch.Tensor:
        """[S, sum P, C], weight columns ordered nu = corr, corr-1, ..., 1."""
        return torch.cat([self.weights_max, *self.weights], 1)

    def symmetric_table(self, device, dtype=torch.float32) -> torch.Tensor:
        """Symmetrised U in the kernel's row order, [rows * (2t+1), sum P] (cached per device, dtype)."""
        key = (str(device), dtype)
        cache = cache_of(self, "_table_cache")
        table = cache.get(key)
        if table is None:
            from ictc_o3.backends.cuda.contraction import symmetric_table
            dim = self._u64[1].shape[-2]
            sym = symmetric_table(self._u64, self.output_l, dim, self.correlation)
            table = torch.from_numpy(sym.reshape(-1, sym.shape[-1])).to(device=device, dtype=dtype)
            cache[key] = table
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


def _zero_flags_after_load(module, _incompatible_keys):
    """Runs once the whole block, its weight list included, has loaded."""
    module._apply_zero_flags()


class _BridgeUContraction(_ICTDPureUContraction):
    """One target degree of the bridge-U parameterisation.

    The couplings are this block's ``U_matrix_nu`` buffers as they stand, so the
    kernel table is rebuilt from them whenever they change (a loaded state dict).
    The ``weights_*_zeroed`` flags mirror the reference's
    (``ictc_o3/ops/_mace_symmetric_contraction.py:207-222``, flag ``idx`` guards
    ``weights[idx]``, ``weights_max_zeroed`` guards ``weights_max``): a flagged
    weight is held at zero and is not trained.  A loaded state dict whose coupling
    count P differs from this block's (the reference's reduced-CG option) resizes the
    U buffers and weights to it; the resized weights are new parameter objects, so
    such a state dict is loaded before an optimizer is built over the module.
    """

    def __init__(self, **kwargs):
        super().__init__(**kwargs)
        for idx in range(self.correlation - 1):
            self.register_buffer(f"weights_{idx}_zeroed", torch.tensor(False))
        self.register_buffer("weights_max_zeroed", torch.tensor(False))
        self.register_load_state_dict_post_hook(_zero_flags_after_load)

    def _apply_zero_flags(self):
        with torch.no_grad():
            for name, flag in self._weight_slots():
                if bool(getattr(self, flag)):
                    self._parameter(name).zero_()
                    self._parameter(name).requires_grad_(False)

    def _weight_slots(self):
        """(state-dict name, zero-flag name) of every weight, in ``stacked_weights`` order."""
        return [("weights_max", "weights_max_zeroed")] + [
            (f"weights.{idx}", f"weights_{idx}_zeroed") for idx in range(self.correlation - 1)]

    def _parameter(self, name):
        return self.weights_max if name == "weights_max" else self.weights[int(name.split(".")[1])]

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        for nu in range(1, self.correlation + 1):
            name = f"U_matrix_{nu}"
            incoming = state_dict.get(prefix + name)
            own = self._buffers[name]
            if incoming is not None and incoming.shape[:-1] == own.shape[:-1] and incoming.shape != own.shape:
                self._buffers[name] = own.new_empty(incoming.shape)
        for name, _ in self._weight_slots():
            incoming = state_dict.get(prefix + name)
            param = self._parameter(name)
            if incoming is not None and incoming.shape[::2] == param.shape[::2] and incoming.shape != param.shape:
                resized = nn.Parameter(param.new_empty(incoming.shape), requires_grad=param.requires_grad)
                if name == "weights_max":
                    self.weights_max = resized
                else:
                    self.weights[int(name.split(".")[1])] = resized
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)

    def symmetric_table(self, device, dtype=torch.float32) -> torch.Tensor:
        """Symmetrised couplings of the current buffers, [rows * (2t+1), sum P] (cached
        per device and dtype while the buffers are unchanged)."""
        buffers = [self.U_tensors(nu) for nu in range(1, self.correlation + 1)]
        version = tuple((u.data_ptr(), u._version, tuple(u.shape)) for u in buffers)
        key = (str(device), dtype)
        cache = cache_of(self, "_table_cache")
        cached = cache.get(key)
        if cached is not None and cached[0] == version and all(r() is u for r, u in zip(cached[2], buffers)):
            return cached[1]
        from ictc_o3.backends.cuda.contraction import symmetric_table
        u64 = {nu: u.detach().double().cpu().numpy() for nu, u in zip(range(1, self.correlation + 1), buffers)}
        sym = symmetric_table(u64, self.output_l, u64[1].shape[-2], self.correlation)
        table = torch.from_numpy(sym.reshape(-1, sym.shape[-1])).to(device=device, dtype=dtype)
        cache[key] = (version, table, tuple(weakref.ref(u) for u in buffers))
        return table


class _BasisBridge(nn.Module):
    """The reference's per-degree ICTC-to-e3nn basis change ``q_l`` [2l+1, 2l+1]
    (``ictc_o3/ops/symmetric_contraction.py:24-89``).  Bridge-U couplings already
    contain it (folded in at construction, ``:135-180``), so the contraction never
    applies it; the buffers (identity in a new module) keep state dicts
    interchangeable with the reference's."""

    def __init__(self, lmax: int):
        super().__init__()
        for l in range(int(lmax) + 1):
            self.register_buffer(f"q_{l}", torch.eye(2 * l + 1))


class _Contractions(nn.Module):
    """Holds the per-target blocks under the reference's state-dict path
    (``symmetric_contractions.contractions.<t>``)."""

    def __init__(self, blocks):
        super().__init__()
        self.contractions = nn.ModuleList(blocks)


class ICTDBridgeUSymmetricContractionSO3(nn.Module):
    """The reference's default contraction (same constructor, forward and state-dict
    names as ``ictc_o3/ops/symmetric_contraction.py:92-206``) on the CUDA kernels.

    forward(node_feats [N, C(L+1)^2] flat ICTC features, node_attrs [N, S] one-hot,
    node_type_idx [N] optional) -> [N, C(Lt+1)^2].  The couplings are the block
    buffers: the ICTC couplings in a new module, the reference's bridge-U couplings
    after ``load_state_dict`` of one of its modules or checkpoints.  ``use_reduced_cg``
    is recorded; a reduced-CG state dict brings its own coupling count.
    """

    def __init__(self, *, num_elements: int, channels: int, lmax: int, target_lmax: int, correlation: int = 3,
                 use_reduced_cg: bool = False):
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
        self.use_reduced_cg = bool(use_reduced_cg)
        self.basis_bridge = _BasisBridge(max(self.lmax, self.target_lmax))
        blocks = []
        for t in range(self.target_lmax + 1):
            u = {nu: ictd_u_matrix_so3(self.lmax, t, nu) for nu in range(1, self.correlation + 1)}
            blocks.append(_BridgeUContraction(u_tensors=u, output_l=t, num_elements=num_elements,
                                              num_features=channels))
        self.symmetric_contractions = _Contractions(blocks)

    @property
    def contractions(self) -> nn.ModuleList:
        """The per-target blocks (the interface the CUDA contraction reads)."""
        return self.symmetric_contractions.contractions

    def forward(self, node_feats: torch.Tensor, node_attrs: torch.Tensor | None = None,
                node_type_idx: torch.Tensor | None = None) -> torch.Tensor:
        from ictc_o3.backends.cuda.contraction import contract_flat
        if node_type_idx is None:
            if node_attrs is None:
                raise ValueError("node_attrs or node_type_idx is required")
            node_type_idx = node_attrs.argmax(-1)
        return contract_flat(self, node_feats, node_type_idx)


SymmetricContraction = ICTDPureUSymmetricContractionSO3
