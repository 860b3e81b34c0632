"""ICTC harmonic basis, coupling (CG) tensors and the path-preserving TP owner.

Host-side constants for the CUDA backend, restated in float64 numpy from the
mathematics the ICTC-O3 reference documents:

* monomial order ``counts_list``            -- ``ictc_o3/basis/ictd_fast.py:11-18``
* r^{2k} lift                               -- ``ictc_o3/basis/ictd_fast.py:51-77``
* Gaussian-moment Gram matrix on Sym^L      -- ``ictc_o3/basis/ictd_irreps.py:587-629``
* frozen harmonic basis (data, SHA-pinned)  -- ``ictc_o3/basis/ictd_irreps.py:633-694``
* harmonic projectors P_{L->l}              -- ``ictc_o3/basis/ictd_irreps.py:765-791``
* CG tensor (poly product + projection)     -- ``ictc_o3/basis/ictd_irreps.py:1206-1264``
* CG / path normalisation                   -- ``ictc_o3/basis/ictd_irreps.py:101-142``
* direction-harmonic projector and scale    -- ``ictc_o3/basis/ictd_irreps.py:913-959``
* path list, groups, path offsets           -- ``ictc_o3/basis/ictd_irreps.py:2159-2217,2512-2533``

The module-level constants are pure functions of the degrees and are cached.
"""
from __future__ import annotations

import hashlib
import json
import math
import os
from functools import lru_cache
from typing import Dict, List, Tuple

import numpy as np
import torch
import torch.nn as nn

from .harmonic_basis_pins import BASIS_SHA256, BASIS_VERSION


# ---------------------------------------------------------------------------
# Monomials and Gram matrices
# ---------------------------------------------------------------------------

def counts_list(L: int) -> List[Tuple[int, int, int]]:
    """Exponents (a, b, c) with a+b+c = L, a outermost, then b (ICTC order)."""
    return [(a, b, L - a - b) for a in range(L + 1) for b in range(L - a + 1)]


def sym_dim(L: int) -> int:
    return (L + 2) * (L + 1) // 2


def _double_factorial(n: int) -> int:
    value = 1
    while n > 1:
        value *= n
        n -= 2
    return value


def _gaussian_moment(n: int) -> float:
    """E[x^n] for a standard normal x."""
    return 0.0 if n % 2 else float(_double_factorial(n - 1))


def _sphere_moment(a: int, b: int, c: int) -> float:
    """E[x^a y^b z^c] for a uniform unit vector on the 2-sphere."""
    if a % 2 or b % 2 or c % 2:
        return 0.0
    p, q, r = a // 2, b // 2, c // 2
    return (_double_factorial(2 * p - 1) * _double_factorial(2 * q - 1) * _double_factorial(2 * r - 1)
            / _double_factorial(2 * (p + q + r) + 1))


@lru_cache(maxsize=None)
def gram_gaussian(L: int) -> np.ndarray:
    """Rotation-invariant inner product of degree-L monomials under N(0, I_3)."""
    counts = counts_list(L)
    gram = np.zeros((len(counts), len(counts)))
    for i, (a, b, c) in enumerate(counts):
        for j, (a2, b2, c2) in enumerate(counts):
            gram[i, j] = _gaussian_moment(a + a2) * _gaussian_moment(b + b2) * _gaussian_moment(c + c2)
    return gram


@lru_cache(maxsize=None)
def r2k_lift(l: int, k: int) -> np.ndarray:
    """Multiplication by (x^2+y^2+z^2)^k as a map Sym^l -> Sym^{l+2k}."""
    src = counts_list(l)
    if k == 0:
        return np.eye(len(src))
    dst = {t: i for i, t in enumerate(counts_list(l + 2 * k))}
    lift = np.zeros((len(dst), len(src)))
    for col, (a, b, c) in enumerate(src):
        for u in range(k + 1):
            for v in range(k - u + 1):
                w = k - u - v
                coef = math.factorial(k) / (math.factorial(u) * math.factorial(v) * math.factorial(w))
                lift[dst[(a + 2 * u, b + 2 * v, c + 2 * w)], col] += coef
    return lift


# ---------------------------------------------------------------------------
# Frozen harmonic basis (a data format: must match the reference byte for byte)
# ---------------------------------------------------------------------------

_TABLE_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "harmonic_basis_v1.json")


@lru_cache(maxsize=1)
def _basis_table() -> dict:
    with open(_TABLE_PATH) as handle:
        table = json.load(handle)
    if table.get("format") != "ictd-canonical-harmonic-basis" or table.get("version") != BASIS_VERSION:
        raise RuntimeError("harmonic basis table has an unexpected format or version")
    return table


@lru_cache(maxsize=None)
def harmonic_basis(l: int) -> np.ndarray:
    """B_l, shape (Dsym(l), 2l+1): harmonic coordinates -> monomial coefficients.

    Only the frozen degrees are supported; the digest of the float64 bytes is
    checked against the pinned value before use.
    """
    entry = _basis_table()["degrees"].get(str(int(l)))
    if entry is None or int(l) not in BASIS_SHA256:
        raise ValueError(f"ICTC harmonic basis is frozen for l <= {max(BASIS_SHA256)}; got l={l}")
    values = np.array([float.fromhex(v) for v in entry["values"]], dtype=np.float64)
    basis = values.reshape(entry["shape"])
    digest = hashlib.sha256(np.ascontiguousarray(basis).tobytes()).hexdigest()
    if digest != BASIS_SHA256[int(l)] or tuple(basis.shape) != (sym_dim(l), 2 * l + 1):
        raise RuntimeError(f"ICTC harmonic basis integrity check failed for l={l}")
    basis.setflags(write=False)
    return basis


@lru_cache(maxsize=None)
def harmonic_projector(L: int, l: int) -> np.ndarray:
    """P_{L->l}, shape (2l+1, Dsym(L)): Gram-weighted least squares onto r^{L-l} Harm^l."""
    k = (L - l) // 2
    V = r2k_lift(l, k) @ harmonic_basis(l)
    G = gram_gaussian(L)
    return np.linalg.solve(V.T @ G @ V, V.T @ G)


@lru_cache(maxsize=None)
def _poly_mult(l1: int, l2: int) -> np.ndarray:
    """Sym^l1 (x) Sym^l2 -> Sym^{l1+l2}: product of monomials."""
    c1, c2 = counts_list(l1), counts_list(l2)
    dst = {t: i for i, t in enumerate(counts_list(l1 + l2))}
    mult = np.zeros((len(dst), len(c1) * len(c2)))
    for i, (a, b, c) in enumerate(c1):
        for j, (a2, b2, c2_) in enumerate(c2):
            mult[dst[(a + a2, b + b2, c + c2_)], i * len(c2) + j] = 1.0
    return mult


@lru_cache(maxsize=None)
def build_cg_tensor(l1: int, l2: int, l3: int) -> np.ndarray:
    """C[m1, m2, m3]: harmonic product of degrees l1, l2 projected onto l3 (float64)."""
    if not (abs(l1 - l2) <= l3 <= l1 + l2) or (l1 + l2 + l3) % 2:
        return np.zeros((2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1))
    B1, B2 = harmonic_basis(l1), harmonic_basis(l2)
    outer = np.einsum("im,jn->ijmn", B1, B2).reshape(B1.shape[0] * B2.shape[0], -1)
    coords = harmonic_projector(l1 + l2, l3) @ (_poly_mult(l1, l2) @ outer)
    return np.ascontiguousarray(coords.T.reshape(2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1))


def apply_cg_normalization(C: np.ndarray, l_out: int, irrep_normalization: str) -> np.ndarray:
    norm = float(np.sqrt((C * C).sum()))
    if irrep_normalization == "component" and norm > 1e-30:
        return C * (math.sqrt(2 * l_out + 1) / norm)
    if irrep_normalization == "norm" and norm > 1e-30:
        return C * (1.0 / norm)
    return C


def path_normalization_scales(paths, path_normalization: str = "element") -> List[float]:
    """1/sqrt(#paths sharing the output degree) ("element" and "path" coincide at 1 element)."""
    if path_normalization == "none":
        return [1.0] * len(paths)
    counts: Dict[int, int] = {}
    for path in paths:
        counts[int(path[2])] = counts.get(int(path[2]), 0) + 1
    return [1.0 / math.sqrt(float(counts[int(p[2])])) for p in paths]


# ---------------------------------------------------------------------------
# Direction harmonics constants
# ---------------------------------------------------------------------------

@lru_cache(maxsize=None)
def direction_projector(l: int) -> np.ndarray:
    """G_l @ B_l, shape (Dsym(l), 2l+1): monomials of n -> harmonic coordinates."""
    if l == 0:
        return np.ones((1, 1))
    return gram_gaussian(l) @ harmonic_basis(l)


@lru_cache(maxsize=None)
def multinomials(l: int) -> np.ndarray:
    return np.array([math.factorial(l) / (math.factorial(a) * math.factorial(b) * math.factorial(c))
                     for a, b, c in counts_list(l)])


@lru_cache(maxsize=None)
def direction_component_scale(l: int) -> float:
    """Scale that gives each harmonic component unit RMS over the unit sphere."""
    if l == 0:
        return 1.0
    counts, coefs = counts_list(l), multinomials(l)
    sphere = np.zeros((len(counts), len(counts)))
    for i, (a, b, c) in enumerate(counts):
        for j, (a2, b2, c2) in enumerate(counts):
            sphere[i, j] = coefs[i] * coefs[j] * _sphere_moment(a + a2, b + b2, c + c2)
    P = direction_projector(l)
    mean_square = np.trace(P.T @ sphere @ P) / float(2 * l + 1)
    return float(1.0 / math.sqrt(max(mean_square, 1e-30)))


@lru_cache(maxsize=None)
def direction_harmonic_table(l: int) -> np.ndarray:
    """Coefficients H_l[d, m] = multinomial_d * (G_l B_l)[d, m] * scale_l.

    Y_l(n)[m] = sum_d n_x^a n_y^b n_z^c * H_l[d, m] with (a, b, c) = counts_list(l)[d].
    """
    return multinomials(l)[:, None] * direction_projector(l) * direction_component_scale(l)


# ---------------------------------------------------------------------------
# Path structure of the path-preserving tensor product
# ---------------------------------------------------------------------------

def enumerate_paths(lmax: int, allowed=None) -> List[Tuple[int, int, int]]:
    """Triangle- and parity-allowed (l1, l2, l3), l1 outer, l2 middle, l3 inner."""
    paths = [(l1, l2, l3)
             for l1 in range(lmax + 1) for l2 in range(lmax + 1)
             for l3 in range(abs(l1 - l2), min(l1 + l2, lmax) + 1)
             if (l1 + l2 + l3) % 2 == 0]
    if allowed is not None:
        allowed = set(tuple(p) for p in allowed)
        paths = [p for p in paths if p in allowed]
    return paths


def operator_paths(input_lmax: int, edge_lmax: int, output_lmax: int) -> List[Tuple[int, int, int]]:
    """The allowed-path list used by the public operator factory."""
    return [(i, j, k) for i in range(input_lmax + 1) for j in range(edge_lmax + 1)
            for k in range(output_lmax + 1) if abs(i - j) <= k <= i + j and (i + j + k) % 2 == 0]


class EdgeWeightedPathPreservingTensorProduct(nn.Module):
    """Owner of the path-preserving TP constants and its per-(path, channel) weight.

    Mirrors the attribute surface the reference backends read from their owner
    (``ictc_o3/basis/ictd_irreps.py:2125-2533``): ``channels``, ``lmax``,
    ``paths``, ``num_paths``, ``_groups``, ``path_l3``, ``path_offset``,
    ``path_counts_by_l``, ``weight`` [P, C] and ``_get_cg_list``.  ``forward``
    evaluates through the CUDA backend only; there is no host fallback.
    """

    def __init__(self, channels: int, lmax: int, *, allowed_paths=None,
                 irrep_normalization: str = "component", path_normalization: str = "element",
                 internal_compute_dtype: torch.dtype = torch.float32):
        super().__init__()
        self.channels = int(channels)
        self.lmax = int(lmax)
        self._normalization = irrep_normalization
        self._path_normalization = path_normalization
        self.internal_compute_dtype = internal_compute_dtype
        self.paths = enumerate_paths(self.lmax, allowed_paths)
        self.num_paths = len(self.paths)
        self._path_normalization_scales = path_normalization_scales(self.paths, path_normalization)
        self.weight = nn.Parameter(torch.randn(self.num_paths, self.channels) * 0.02)
        groups: Dict[Tuple[int, int], List[Tuple[int, int]]] = {}
        for p, (l1, l2, l3) in enumerate(self.paths):
            groups.setdefault((l1, l2), []).append((p, l3))
        self._groups = []
        for (l1, l2), items in sorted(groups.items()):
            segments, start = [], 0
            for p, l3 in items:
                segments.append((p, l3, start, start + 2 * l3 + 1))
                start += 2 * l3 + 1
            self._groups.append({"l1": l1, "l2": l2, "segments": segments, "k_total": start})
        self.path_l3 = [0] * self.num_paths
        self.path_offset = [0] * self.num_paths
        counts = {l: 0 for l in range(self.lmax + 1)}
        for group in self._groups:
            for p, l3, _s, _e in group["segments"]:
                self.path_l3[p] = l3
                self.path_offset[p] = counts[l3]
                counts[l3] += 1
        self.path_counts_by_l = counts
        self._cg_f64 = None
        self._cg_cache: Dict[Tuple[str, str], List[torch.Tensor]] = {}

    def cg_f64(self) -> List[np.ndarray]:
        """Normalised per-path CG tensors in float64 (path order)."""
        if self._cg_f64 is None:
            tensors = []
            for p, (l1, l2, l3) in enumerate(self.paths):
                C = apply_cg_normalization(build_cg_tensor(l1, l2, l3), l3, self._normalization)
                tensors.append(C * float(self._path_normalization_scales[p]))
            self._cg_f64 = tensors
        return self._cg_f64

    def _get_cg_list(self, device, dtype) -> List[torch.Tensor]:
        key = (str(device), str(dtype))
        if key not in self._cg_cache:
            self._cg_cache[key] = [torch.from_numpy(C.copy()).to(device=device, dtype=dtype)
                                   for C in self.cg_f64()]
        return self._cg_cache[key]

    @property
    def output_width(self) -> int:
        return sum(n * self.channels * (2 * l + 1) for l, n in self.path_counts_by_l.items())

    def forward(self, x1: Dict[int, torch.Tensor], x2: Dict[int, torch.Tensor], gates=None):
        from ictc_o3.backends.cuda.tensor_product import tensor_product
        if gates is not None and gates.shape[-1] == self.num_paths * self.channels:
            gates = gates.view(*gates.shape[:-1], self.num_paths, self.channels)
        return tensor_product(self, x1, x2, gates)


def direction_harmonics_all(n: torch.Tensor, lmax: int) -> List[torch.Tensor]:
    """Direction harmonics Y_l(n), l = 0..lmax, through the CUDA kernel (list of [..., 2l+1])."""
    from ictc_o3.backends.cuda.geometry import direction_harmonics
    packed = direction_harmonics(n, lmax)
    return [packed[..., l * l:(l + 1) ** 2] for l in range(lmax + 1)]


# ---------------------------------------------------------------------------
# Full SO(3) couplings (any parity) and the MACE-style contraction basis
# ---------------------------------------------------------------------------

@lru_cache(maxsize=None)
def monomial_rotation_generator(L: int, axis: str) -> np.ndarray:
    """Infinitesimal rotation about ``axis`` acting on degree-L monomial coefficients.

    Same convention as ``ictc_o3/basis/ictd_irreps.py:1266-1292``: about z,
    x^a y^b z^c -> b x^{a+1} y^{b-1} z^c - a x^{a-1} y^{b+1} z^c (cyclic for x, y).
    """
    counts = counts_list(L)
    index = {t: i for i, t in enumerate(counts)}
    gen = np.zeros((len(counts), len(counts)))
    for col, (a, b, c) in enumerate(counts):
        if axis == "x":
            terms = [(c, (a, b + 1, c - 1)), (-b, (a, b - 1, c + 1))]
        elif axis == "y":
            terms = [(a, (a - 1, b, c + 1)), (-c, (a + 1, b, c - 1))]
        elif axis == "z":
            terms = [(b, (a + 1, b - 1, c)), (-a, (a - 1, b + 1, c))]
        else:
            raise ValueError("axis must be x, y or z")
        for coef, key in terms:
            if coef:
                gen[index[key], col] += coef
    return gen


@lru_cache(maxsize=None)
def harmonic_rotation_generator(l: int, axis: str) -> torch.Tensor:
    """The generator restricted to degree-l harmonics: B^T G M B (``ictd_irreps.py:1295-1301``).

    Evaluated with torch float64 in the same association order as the reference,
    ((B^T G) M) B, so the coupling null vectors below reproduce its bits (their sign
    choice depends on exact ties between entries of equal magnitude).
    """
    B = torch.from_numpy(np.array(harmonic_basis(l)))
    G = torch.from_numpy(gram_gaussian(l))
    M = torch.from_numpy(monomial_rotation_generator(l, axis))
    return (B.T @ G @ M @ B).contiguous()


@lru_cache(maxsize=None)
def build_full_cg_tensor_so3(l1: int, l2: int, l3: int) -> np.ndarray:
    """Unique SO(3) intertwiner l1 x l2 -> l3 in the ICTC basis, any parity of l1+l2+l3.

    Solves J3 C = C (J1 (x) 1 + 1 (x) J2) for x, y, z generators; the 1-D null space is
    sign-fixed so that the entry of largest magnitude is positive
    (``ictc_o3/basis/ictd_irreps.py:1345-1373``).  Shape (2l1+1, 2l2+1, 2l3+1).
    """
    d1, d2, d3 = 2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1
    if not abs(l1 - l2) <= l3 <= l1 + l2:
        return np.zeros((d1, d2, d3))
    eye = lambda n: torch.eye(n, dtype=torch.float64)  # noqa: E731
    rows = []
    for axis in ("x", "y", "z"):
        J1 = harmonic_rotation_generator(l1, axis)
        J2 = harmonic_rotation_generator(l2, axis)
        J3 = harmonic_rotation_generator(l3, axis)
        Jin = torch.kron(J1, eye(d2)) + torch.kron(eye(d1), J2)
        # Unknown Cmat [d3, d1*d2] (row-major): J3 @ Cmat - Cmat @ Jin = 0.
        rows.append(torch.kron(J3, eye(d1 * d2)) - torch.kron(eye(d3), Jin.T.contiguous()))
    A = torch.cat(rows, 0)
    try:
        vh = torch.linalg.svd(A)[2]
    except RuntimeError:  # LAPACK gesdd non-convergence: gesvd through numpy
        vh = torch.from_numpy(np.linalg.svd(A.numpy(), full_matrices=True)[2])
    C = vh[-1].reshape(d3, d1 * d2).T.reshape(d1, d2, d3)
    if C.reshape(-1)[int(C.abs().argmax())] < 0:
        C = -C
    return np.ascontiguousarray(C.numpy())


def _natural_parity(l: int) -> int:
    return 1 if l % 2 == 0 else -1


@lru_cache(maxsize=None)
def coupled_basis(lmax: int, correlation: int, irrep_normalization: str = "component", final_l: int = -1):
    """n-body coupling tensors in the ICTC basis (``ictc_o3/basis/ictd_irreps.py:1389-1446``).

    Returns (l_out, parity, tensor [2l_out+1, D, ..., D]) with D = (lmax+1)^2, built by
    coupling a left chain with one more input degree at a time and sorting by (l, parity)
    after every order, as MACE's chained Wigner construction does.  With
    ``final_l >= 0`` the last order only generates chains ending in degree final_l
    (the entries a later filter on l_out == final_l keeps, in the same order).
    """
    dim = (lmax + 1) ** 2
    eye = np.eye(dim)
    basis = [(l, _natural_parity(l), eye[l * l:(l + 1) ** 2]) for l in range(lmax + 1)]
    for order in range(2, correlation + 1):
        last = order == correlation and final_l >= 0
        following = []
        for l_left, p_left, left in basis:
            flat_left = left.reshape(2 * l_left + 1, -1)
            for l_right in range(lmax + 1):
                for l_out in range(abs(l_left - l_right), l_left + l_right + 1):
                    if last and l_out != final_l:
                        continue
                    cg = apply_cg_normalization(build_full_cg_tensor_so3(l_left, l_right, l_out), l_out,
                                                irrep_normalization)
                    coupled = np.einsum("ar,abq->qrb", flat_left, cg)
                    full = np.zeros((2 * l_out + 1, flat_left.shape[1], dim))
                    full[:, :, l_right * l_right:(l_right + 1) ** 2] = coupled
                    following.append((l_out, p_left * _natural_parity(l_right),
                                      full.reshape(2 * l_out + 1, *left.shape[1:], dim)))
        basis = sorted(following, key=lambda item: (item[0], item[1]))
    return basis


@lru_cache(maxsize=None)
def ictd_u_matrix_so3(lmax: int, output_l: int, correlation: int,
                      irrep_normalization: str = "component") -> np.ndarray:
    """MACE-style symmetric-contraction U in the ICTC basis (``ictd_irreps.py:1465-1517``).

    Shape [2l+1, D x correlation, P] (leading axis dropped for l = 0), float64.
    """
    target = _natural_parity(output_l)
    tensors = [t for l_out, parity, t in coupled_basis(lmax, correlation, irrep_normalization, output_l)
               if l_out == output_l and parity == target]
    dim = (lmax + 1) ** 2
    if not tensors:
        shape = ([dim] * correlation + [1]) if output_l == 0 else ([2 * output_l + 1] + [dim] * correlation + [1])
        return np.zeros(shape)
    if output_l == 0:
        tensors = [t[0] for t in tensors]
    return np.ascontiguousarray(np.stack(tensors, -1))
