"""Symmetric contraction on the CUDA backend.

Drop-in for ``ictc_o3/backends/ascend/contraction.py`` (``factorized_contractions``).
For every target degree t the reference recursion
(``ictc_o3/ops/_mace_symmetric_contraction.py:298-346``)

    out_t[n, c, m] = sum_nu < U_nu[m, i1..inu, :] W_nu[s_n, :, c], x[n, c, i1] .. x[n, c, inu] >

is a polynomial in the node's features.  The host symmetrises U over its input
axes once (``symmetric_table``), and every call folds the species weights in
with one GEMM, ``T = Usym W``; the kernel evaluates the polynomial per node.
Nodes are grouped into species-homogeneous tiles so every coefficient row is
read once per tile.
"""
from __future__ import annotations

import itertools
import weakref
from functools import lru_cache

import numpy as np
import torch

from ictc_o3.autograd.adjoint_requirements import required_gradients
from . import _native
from .cache import cache_of
from ._native import ptr, stream_of


# ---------------------------------------------------------------------------
# Host constants: symmetrised U in the kernel's row order
# ---------------------------------------------------------------------------

def monomial_rows(dim: int, correlation: int):
    """Monomials in kernel traversal order: for i: (i); for j>=i: (i,j); for k>=j: (i,j,k)."""
    rows = []
    for i in range(dim):
        if correlation >= 1:
            rows.append((i,))
        if correlation >= 2:
            for j in range(i, dim):
                rows.append((i, j))
                if correlation >= 3:
                    for k in range(j, dim):
                        rows.append((i, j, k))
    return rows


def symmetric_table(u_tensors, output_l: int, dim: int, correlation: int) -> np.ndarray:
    """Usym [rows, 2t+1, sum_nu P_nu] with weight columns ordered nu = corr, corr-1, .., 1.

    Row (i, j, k) holds sum over the distinct orderings of (i, j, k) of U_nu[m, ., ., ., p].
    """
    M = 2 * output_l + 1
    blocks = {}
    for nu in range(1, correlation + 1):
        u = np.asarray(u_tensors[nu], dtype=np.float64)
        if output_l == 0:
            u = u[None]
        blocks[nu] = u
    order = list(range(correlation, 0, -1))
    offsets, total = {}, 0
    for nu in order:
        offsets[nu] = total
        total += blocks[nu].shape[-1]
    rows = monomial_rows(dim, correlation)
    table = np.zeros((len(rows), M, total))
    for r, mono in enumerate(rows):
        nu = len(mono)
        u = blocks[nu]
        acc = np.zeros((M, u.shape[-1]))
        for perm in set(itertools.permutations(mono)):
            acc += u[(slice(None),) + perm]
        table[r, :, offsets[nu]:offsets[nu] + u.shape[-1]] = acc
    return table


@lru_cache(maxsize=None)
def _table_rows(lmax: int, correlation: int, target_lmax: int) -> int:
    return int(_native.library().ictc_sc_table_rows(lmax, correlation, target_lmax))


# ---------------------------------------------------------------------------
# The contraction module as the kernels see it
# ---------------------------------------------------------------------------

def contraction_blocks(owner):
    """Per-target blocks in target order: ``owner.contractions`` (this package's
    modules) or ``owner.symmetric_contractions.contractions`` (the reference's
    bridge-U module, ``ictc_o3/ops/symmetric_contraction.py:116-122``, whose blocks
    are MACE contractions holding ``U_matrix_nu`` buffers, ``weights_max`` and
    ``weights``)."""
    try:
        blocks = owner.contractions
    except AttributeError:
        blocks = owner.symmetric_contractions.contractions
    return list(blocks)


def block_weights(block) -> torch.Tensor:
    """[S, sum P, C], weight columns ordered nu = corr, corr-1, ..., 1."""
    return torch.cat([block.weights_max, *block.weights], 1)


def block_table(block, device, dtype=torch.float32) -> torch.Tensor:
    """Symmetrised couplings of one block, [rows * (2t+1), sum P].

    This package's blocks build and cache their own.  A reference block's are
    built from its ``U_matrix_nu`` buffers (output degree from the shape of
    ``U_matrix_1``: [D, P] for degree 0, [2t+1, D, P] otherwise) and kept on the
    block while the buffers are unchanged."""
    own = getattr(block, "symmetric_table", None)
    if own is not None:
        return own(device, dtype)
    corr = int(block.correlation)
    buffers = [block.U_tensors(nu) for nu in range(1, corr + 1)]
    version = tuple((u.data_ptr(), u._version, tuple(u.shape)) for u in buffers)
    cache = cache_of(block, "_cuda_symmetric_tables")
    key = (str(device), dtype)
    hit = cache.get(key)
    if hit is not None and hit[0] == version and all(r() is u for r, u in zip(hit[2], buffers)):
        return hit[1]
    u64 = {nu: u.detach().double().cpu().numpy() for nu, u in zip(range(1, corr + 1), buffers)}
    output_l = 0 if u64[1].ndim == 2 else (u64[1].shape[0] - 1) // 2
    sym = symmetric_table(u64, output_l, u64[1].shape[-2], corr)
    table = torch.from_numpy(sym.reshape(-1, sym.shape[-1])).to(device=device, dtype=dtype)
    cache[key] = (version, table, tuple(weakref.ref(u) for u in buffers))
    return table


def contraction_spec(owner):
    """(channels, lmax, correlation, target_lmax, num_elements) of a contraction module;
    correlation and element count are read from its blocks, which every variant has."""
    blocks = contraction_blocks(owner)
    orders = {int(b.correlation) for b in blocks}
    target = int(owner.target_lmax)
    if len(orders) != 1 or len(blocks) != target + 1:
        raise ValueError("The CUDA symmetric contraction needs one block per target degree, all of one "
                         "correlation order")
    return int(owner.channels), int(owner.lmax), orders.pop(), target, int(blocks[0].weights_max.shape[0])


# ---------------------------------------------------------------------------
# Species tiles
# ---------------------------------------------------------------------------

def species_tiles(index: torch.Tensor, num_elements: int):
    """Species-homogeneous node tiles [T, NB] (-1 padded) and their species [T] (int32)."""
    nb = int(_native.library().ictc_sc_tile_nodes())
    key = (index._version, int(num_elements), nb)
    cached = getattr(index, "_ictc_cuda_sc_tiles", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    from .linear import species_tiles_of
    result = species_tiles_of(index, num_elements, nb)
    index_ref = index
    try:
        index_ref._ictc_cuda_sc_tiles = (key, result)
    except AttributeError:
        pass
    return result


# ---------------------------------------------------------------------------
# Autograd
# ---------------------------------------------------------------------------

def _sc_apply(name, spec, tiles, tile_species, x, table, grad=None, direction=None):
    """One launch of a polynomial kernel over the species tiles.

    ``ictc_sc_forward`` / ``ictc_sc_directional`` return [N, C sum_t M_t];
    ``ictc_sc_backward`` / ``ictc_sc_hvp`` return [N, C D]; unnamed rows are zero."""
    channels, lmax, correlation, target_lmax = spec
    forward_like = name in ("ictc_sc_forward", "ictc_sc_directional")
    width = channels * (target_lmax + 1) ** 2 if forward_like else x.shape[1]
    out = torch.zeros(x.shape[0], width, device=x.device, dtype=torch.float32)
    # No nodes (a rank that owns no atoms): nothing to launch.  The species tiles are
    # never empty (they are padded per species), but an empty tensor has no storage.
    if tiles.shape[0] and x.shape[0]:
        n = int(tiles.shape[0])
        table = table.contiguous()
        stream = stream_of(x)
        if name == "ictc_sc_forward":
            _native.call(name, ptr(x), ptr(table), ptr(tiles), ptr(tile_species), n, ptr(out), channels, lmax,
                         correlation, target_lmax, stream)
        elif name == "ictc_sc_backward":
            _native.call(name, ptr(x), ptr(table), ptr(tiles), ptr(tile_species), n, ptr(grad), ptr(out), channels,
                         lmax, correlation, target_lmax, stream)
        elif name == "ictc_sc_directional":
            _native.call(name, ptr(x), ptr(direction), ptr(table), ptr(tiles), ptr(tile_species), n, ptr(out),
                         channels, lmax, correlation, target_lmax, stream)
        else:
            _native.call(name, ptr(x), ptr(direction), ptr(table), ptr(tiles), ptr(tile_species), n, ptr(grad),
                         ptr(out), channels, lmax, correlation, target_lmax, stream)
    return out


def _sc_table_grad(spec, tiles, tile_species, x, grad, shape, direction=None):
    """dT [S, R, C]: sum over each species' nodes of grad x monomials (directional
    monomials along ``direction`` when given), ``ictc_sc_table_grad``."""
    channels, lmax, correlation, target_lmax = spec
    if x.shape[0] == 0:                                   # no nodes: the sum over them is zero
        return torch.zeros(shape, device=x.device, dtype=torch.float32)
    out = torch.empty(shape, device=x.device, dtype=torch.float32)
    _native.call("ictc_sc_table_grad", ptr(x), ptr(direction), ptr(grad), ptr(tiles), ptr(tile_species),
                 int(tiles.shape[0]), ptr(out), int(shape[0]), channels, lmax, correlation, target_lmax,
                 stream_of(x))
    return out


class _Contraction(torch.autograd.Function):
    """out = poly(x; T) for species tiles; x [N, C*D] mul_ir flat, T [S, R, C]."""

    @staticmethod
    def forward(ctx, spec, tiles, tile_species, x, table):
        ctx.spec = spec
        ctx.save_for_backward(tiles, tile_species, x, table)
        return _sc_apply("ictc_sc_forward", spec, tiles, tile_species, x, table)

    @staticmethod
    def backward(ctx, grad):
        tiles, tile_species, x, table = ctx.saved_tensors
        need = required_gradients((x, table), ctx.needs_input_grad[3:5])
        if not any(need):
            return None, None, None, None, None
        grad = grad.contiguous()
        if torch.is_grad_enabled():
            # The gradient itself will be differentiated (force-loss training): a
            # kernel-backed function whose backward is again kernels.
            dx, dtable = _ContractionGrad.apply(ctx.spec, tiles, tile_species, need, x, table, grad)
            return None, None, None, dx, dtable
        dx = _sc_apply("ictc_sc_backward", ctx.spec, tiles, tile_species, x, table, grad) if need[0] else None
        dtable = _sc_table_grad(ctx.spec, tiles, tile_species, x, grad, table.shape) if need[1] else None
        return None, None, None, dx, dtable


class _ContractionGrad(torch.autograd.Function):
    """(dx, dT) of the polynomial for the output cotangent g, as kernels:
        dx = sc_backward(x; T, g),   dT = table_grad(x, g).
    Its derivatives, for cotangents hx on dx and hT on dT:
        d/dg = directional(x, hx; T) + forward(x; hT)
        d/dx = hvp(x, hx; T, g)      + backward(x; hT, g)
        d/dT = table_grad(x, g, direction hx)
    Differentiating once more (third order) recomputes through the torch
    formulation of the polynomial."""

    @staticmethod
    def forward(ctx, spec, tiles, tile_species, need, x, table, grad):
        ctx.spec, ctx.need = spec, need
        ctx.save_for_backward(tiles, tile_species, x, table, grad)
        dx = _sc_apply("ictc_sc_backward", spec, tiles, tile_species, x, table, grad) if need[0] else None
        dtable = _sc_table_grad(spec, tiles, tile_species, x, grad, table.shape) if need[1] else None
        return dx, dtable

    @staticmethod
    def backward(ctx, hx, htable):
        tiles, tile_species, x, table, grad = ctx.saved_tensors
        spec = ctx.spec
        want = required_gradients((x, table, grad), ctx.needs_input_grad[4:7])
        if not any(want) or (hx is None and htable is None):
            return (None,) * 7
        if torch.is_grad_enabled():
            with torch.enable_grad():
                xs, ts, gs = (t.detach().requires_grad_(True) for t in (x, table, grad))
                dx, dt = _differentiable_gradients(tiles, tile_species, xs, ts, gs, spec, ctx.need)
                outs = [(o, h) for o, h in ((dx, hx), (dt, htable)) if o is not None and h is not None]
                got = list(torch.autograd.grad([o for o, _ in outs], [t for t, w in zip((xs, ts, gs), want) if w],
                                               [h for _, h in outs], create_graph=True, allow_unused=True))
            res = [got.pop(0) if w else None for w in want]
            return (None, None, None, None, *res)
        hx = None if hx is None else hx.contiguous()
        htable = None if htable is None else htable.contiguous()
        gx = gt = gg = None
        if want[0]:
            parts = []
            if hx is not None:
                parts.append(_sc_apply("ictc_sc_hvp", spec, tiles, tile_species, x, table, grad, hx))
            if htable is not None:
                parts.append(_sc_apply("ictc_sc_backward", spec, tiles, tile_species, x, htable, grad))
            gx = sum(parts[1:], parts[0]) if parts else None
        if want[1] and hx is not None:
            gt = _sc_table_grad(spec, tiles, tile_species, x, grad, table.shape, direction=hx)
        if want[2]:
            parts = []
            if hx is not None:
                parts.append(_sc_apply("ictc_sc_directional", spec, tiles, tile_species, x, table, direction=hx))
            if htable is not None:
                parts.append(_sc_apply("ictc_sc_forward", spec, tiles, tile_species, x, htable))
            gg = sum(parts[1:], parts[0]) if parts else None
        return None, None, None, None, gx, gt, gg


def _monomial_factors(dim: int, correlation: int, device):
    rows = monomial_rows(dim, correlation)
    return [torch.tensor([mono[a] if a < len(mono) else dim for mono in rows], device=device)
            for a in range(correlation)], len(rows)


_SELECTIONS = {}


def _selection_matrices(dim: int, correlation: int, device, dtype):
    """One-hot [dim + 1, rows] matrices: column r of matrix a picks the a-th factor of
    monomial r (index dim = the constant 1).  Gathering factors as matrix products
    keeps every derivative of the polynomial a GEMM (an indexed gather would
    differentiate into a sort-based scatter)."""
    key = (dim, correlation, str(device), dtype)
    mats = _SELECTIONS.get(key)
    if mats is None:
        factors, rows = _monomial_factors(dim, correlation, device)
        mats = []
        for idx in factors:
            m = torch.zeros(dim + 1, rows, device=device, dtype=dtype)
            m[idx, torch.arange(rows, device=device)] = 1.0
            mats.append(m)
        _SELECTIONS[key] = mats
    return mats


def polynomial(x, table, tiles, tile_species, spec):
    """The contraction as differentiable device tensor algebra (second-order path).

    Same polynomial as the kernels: monomials of each node's features (index ``dim``
    is the constant 1), contracted with its species' rows of T.  Used only when the
    gradient itself must be differentiated (force-loss training), where autograd
    through this expression supplies the mixed second derivatives.
    """
    channels, lmax, correlation, target_lmax = spec
    dim = (lmax + 1) ** 2
    n = x.shape[0]
    feats = torch.cat([x[:, l * l * channels:(l + 1) ** 2 * channels].reshape(n, channels, 2 * l + 1)
                       for l in range(lmax + 1)], -1)
    f1 = torch.cat([feats, torch.ones_like(feats[:, :, :1])], -1)
    select = _selection_matrices(dim, correlation, x.device, x.dtype)
    rows = select[0].shape[1]
    species = tile_species.to(torch.int64)
    blocks = [x.new_zeros(n, channels, 2 * t + 1) for t in range(target_lmax + 1)]
    for s in torch.unique(species).tolist():
        nodes = tiles[species == s].reshape(-1)
        nodes = nodes[nodes >= 0]
        f = f1.index_select(0, nodes)
        mono = torch.matmul(f, select[0])
        for a in range(1, correlation):
            mono = mono * torch.matmul(f, select[a])                  # [n_s, C, R]
        offset = 0
        for t in range(target_lmax + 1):
            M = 2 * t + 1
            coef = table[s, offset:offset + rows * M].reshape(rows, M, channels)
            blocks[t] = blocks[t].index_copy(0, nodes, torch.einsum("ncr,rmc->ncm", mono, coef))
            offset += rows * M
    return torch.cat([b.reshape(n, -1) for b in blocks], -1)


def _differentiable_gradients(tiles, tile_species, x, table, grad, spec, need):
    """(dx, dT) as functions of (x, T, grad) that autograd can differentiate again."""
    inputs = [t for t, wanted in zip((x, table), need) if wanted]
    if not inputs:
        return None, None
    with torch.enable_grad():
        out = polynomial(x, table, tiles, tile_species, spec)
        grads = list(torch.autograd.grad(out, inputs, grad, create_graph=True, allow_unused=True))
    result = []
    for t, wanted in zip((x, table), need):
        g = grads.pop(0) if wanted else None
        result.append(torch.zeros_like(t) if wanted and g is None else g)
    return tuple(result)


# ---------------------------------------------------------------------------
# Entry point
# ---------------------------------------------------------------------------

class _Fold(torch.autograd.Function):
    """T [S, sum_t R_t, C]: every target's block T_t = Usym_t W_t (``ictc_sc_fold``).

    Linear in the weights: the weight gradient is the adjoint fold, whose own
    derivative is the fold again, so derivatives of every order stay kernels."""

    @staticmethod
    def forward(ctx, usyms, rows, *weights):
        ctx.usyms, ctx.rows = usyms, rows
        S, C = weights[0].shape[0], weights[0].shape[2]
        total = sum(rows)
        table = torch.empty(S, total, C, device=weights[0].device, dtype=torch.float32)
        row0, stream = 0, stream_of(weights[0])
        for usym, w, r in zip(usyms, weights, rows):
            w = w.contiguous()
            _native.call("ictc_sc_fold", ptr(usym), ptr(w), ptr(table), int(r), int(w.shape[1]), int(C), int(S),
                         int(total), int(row0), 0, stream)
            row0 += r
        ctx.shapes = [tuple(w.shape) for w in weights]
        return table

    @staticmethod
    def backward(ctx, grad):
        return (None, None) + tuple(_FoldAdjoint.apply(ctx.usyms, ctx.rows, ctx.shapes, grad.contiguous()))


class _FoldAdjoint(torch.autograd.Function):
    """dW_t [S, P_t, C] = Usym_t^T dT_t for every target block of dT."""

    @staticmethod
    def forward(ctx, usyms, rows, shapes, grad):
        ctx.usyms, ctx.rows, ctx.shapes = usyms, rows, shapes
        total, row0, stream = sum(rows), 0, stream_of(grad)
        out = []
        for usym, shape, r in zip(usyms, shapes, rows):
            dw = torch.empty(shape, device=grad.device, dtype=torch.float32)
            _native.call("ictc_sc_fold", ptr(usym), ptr(dw), ptr(grad), int(r), int(shape[1]), int(shape[2]),
                         int(shape[0]), int(total), int(row0), 1, stream)
            out.append(dw)
            row0 += r
        return tuple(out)

    @staticmethod
    def backward(ctx, *grads):
        grads = [torch.zeros(shape, device=ctx.usyms[0].device) if g is None else g.contiguous()
                 for g, shape in zip(grads, ctx.shapes)]
        return None, None, None, _Fold.apply(ctx.usyms, ctx.rows, *grads)


def coefficient_table(owner, device):
    """T [S, R, C] = Usym W for all targets, folded by ``ictc_sc_fold``.

    Differentiable in the weights.  When no weight needs a gradient (frozen weights,
    or gradients disabled), the folded table is kept and reused until a weight
    changes (same tensors and versions) or a block's coupling table is rebuilt."""
    blocks = contraction_blocks(owner)
    weights = [block_weights(c) for c in blocks]                                # [S, P_t, C] each
    usyms = tuple(block_table(c, device, torch.float32) for c in blocks)
    rows = tuple(int(u.shape[0]) for u in usyms)
    params = [p for c in blocks for p in c.parameters()]
    live = torch.is_grad_enabled() and any(p.requires_grad for p in params)
    if live:
        return _Fold.apply(usyms, rows, *weights)
    key = (str(device), tuple((p.data_ptr(), p._version) for p in params))
    store = cache_of(owner, "_cuda_folded_table")
    cached = store.get("table")
    if (cached is not None and cached[0] == key and all(a is b for a, b in zip(cached[2], usyms))
            and len(cached[3]) == len(params) and all(r() is p for r, p in zip(cached[3], params))):
        return cached[1]
    with torch.no_grad():
        table = _Fold.apply(usyms, rows, *[w.detach() for w in weights])
    store["table"] = (key, table, usyms, tuple(weakref.ref(p) for p in params))
    return table


def contract_flat(owner, node_feats: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """node_feats [N, C(L+1)^2] mul_ir flat -> [N, C(Lt+1)^2] mul_ir flat."""
    if node_feats.dtype != torch.float32 or node_feats.device.type != "cuda":
        raise ValueError("The CUDA symmetric contraction requires CUDA FP32 node features")
    channels, lmax, corr, target, num_elements = contraction_spec(owner)
    table = coefficient_table(owner, node_feats.device)
    if table.shape[1] != _table_rows(lmax, corr, target):
        raise ValueError("coefficient table does not match the kernel row count")
    tiles, tile_species = species_tiles(index.to(node_feats.device), num_elements)
    spec = (channels, lmax, corr, target)
    return _Contraction.apply(spec, tiles, tile_species, node_feats.contiguous(), table)


def factorized_contractions(owner, x: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """Reference signature (``backends/ascend/contraction.py:8``): x [N, C, sum(2l+1)] -> [N, C(Lt+1)^2].

    ``owner`` is a contraction module of this package or the reference's own
    bridge-U module (the object at its hook site, ``ictc_o3/ops/symmetric_contraction.py:189-193``)."""
    n, channels = x.shape[0], owner.channels
    flat = torch.cat([x[:, :, l * l:(l + 1) ** 2].reshape(n, channels * (2 * l + 1))
                      for l in range(owner.lmax + 1)], -1)
    return contract_flat(owner, flat, index)
