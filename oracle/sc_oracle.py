"""CPU oracle of the symmetric contraction -- TEST INFRASTRUCTURE ONLY.

Restates the MACE recursion with element-selected weights
(``ictc_o3/ops/_mace_symmetric_contraction.py:298-346``, ``_forward_selected_elements``)
over caller-provided U tensors, as the reference's pure-ICTC contraction does
(``mace_ictc/models/pure_cartesian_ictd_fix.py:1202-1387``).  Used only by tests.
"""
import torch


def selected_coefficient(u, weight, idx, output_l):
    """sum_p U[..., p] W[s_n, p, c] -> [N, C, (M), D, ..., D]."""
    selected = weight.index_select(0, idx)                   # [N, P, C]
    out = torch.tensordot(selected, u, dims=([1], [u.ndim - 1]))   # [N, C, (M,) D.. ]
    return out


def contraction(u_tensors, weights_max, weights, x, idx, output_l):
    """x [N, C, D]; u_tensors nu -> U_nu; weights_max [S, P_corr, C]; weights: nu = corr-1..1.

    Returns [N, C * (2 output_l + 1)] (channel-major, component-minor).
    """
    corr = max(u_tensors)
    out = selected_coefficient(u_tensors[corr], weights_max, idx, output_l)
    for order, weight in zip(range(corr - 1, 0, -1), weights):
        out = torch.einsum("bc...i,bci->bc...", out, x)
        out = out + selected_coefficient(u_tensors[order], weight, idx, output_l)
    out = torch.einsum("bc...i,bci->bc...", out, x)
    return out.reshape(out.shape[0], out[0].numel() if out.shape[0] else out.shape[1] * (2 * output_l + 1))


def flat_to_mace(flat, channels, lmax):
    """[N, C(L+1)^2] degree blocks [C][2l+1] -> [N, C, (L+1)^2] (reference _so3_flat_to_mace_features)."""
    n = flat.shape[0]
    return torch.cat([flat[:, l * l * channels:(l + 1) ** 2 * channels].reshape(n, channels, 2 * l + 1)
                      for l in range(lmax + 1)], -1)
