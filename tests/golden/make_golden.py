"""Generate the golden fixtures of the ICTC-O3 hot path from the reference itself.

Run in a container that has the reference source tree (it is not needed at
test time; the fixtures are committed):

    PYTHONPATH=<reference root> FSCETP_ICTD_CACHE_DIR=/tmp/ictd \
        python tests/golden/make_golden.py

Every fixture holds seeded FP32 inputs and the outputs of the reference's own
PyTorch modules on them:
* ``EdgeWeightedPathPreservingTensorProduct.forward``
  (ictc_o3/basis/ictd_irreps.py:2750-2795) in FP64 ("truth") and FP32,
  its VJP (autograd) and the mixed second derivatives (double backward);
* ``direction_harmonics_all`` (ictc_o3/basis/ictd_irreps.py:1113-1168) with
  first and second derivatives;
* the full ICTC couplings and the pure-ICTC contraction U tensors
  (ictc_o3/basis/ictd_irreps.py:1305-1517), pinned through seeded probes, and a
  symmetric contraction built from those U tensors with the MACE recursion
  (ictc_o3/ops/_mace_symmetric_contraction.py:298-346);
* the graph message (gather by src, TP, mask, index_add into dst:
  ictc_o3/backends/ascend/tensor_product.py:189-218 and
  mace_ictc/models/pure_cartesian_ictd_fix.py:1801-1806,1913-1917).
Packed tensors use the mul_ir layout ([channel][angular] inside a degree).
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def operator_paths(li, le, lo):
    return [(i, j, k) for i in range(li + 1) for j in range(le + 1) for k in range(lo + 1)
            if abs(i - j) <= k <= i + j and (i + j + k) % 2 == 0]


def make_tp(I, channels, li, le, lo, dtype):
    return I.EdgeWeightedPathPreservingTensorProduct(
        channels=channels, lmax=max(li, le, lo), allowed_paths=operator_paths(li, le, lo),
        internal_compute_dtype=dtype).to(dtype)


def split_mul_ir(packed, channels, lmax):
    out, off = {}, 0
    for l in range(lmax + 1):
        w = channels * (2 * l + 1)
        out[l] = packed[:, off:off + w].reshape(-1, channels, 2 * l + 1)
        off += w
    return out


def split_harm(packed, lmax):
    return {l: packed[:, l * l:(l + 1) ** 2].unsqueeze(1) for l in range(lmax + 1)}


def pack_out(tp, blocks):
    return torch.cat([blocks[l].reshape(blocks[l].shape[0], -1) for l in range(tp.lmax + 1)], 1)


def unit_vectors(gen, rows):
    n = torch.randn(rows, 3, generator=gen, dtype=torch.float64)
    return n / n.norm(dim=1, keepdim=True)


def tp_case(I, name, channels, li, le, lo, rows, seed, use_gates=True, random_weight=True):
    gen = torch.Generator().manual_seed(seed)
    tp64 = make_tp(I, channels, li, le, lo, torch.float64)
    tp32 = make_tp(I, channels, li, le, lo, torch.float32)
    P = tp64.num_paths
    weight = (torch.randn(P, channels, generator=gen) if random_weight else torch.ones(P, channels)).float()
    with torch.no_grad():
        tp64.weight.copy_(weight.double())
        tp32.weight.copy_(weight)
    A = channels * (li + 1) ** 2
    x = torch.randn(rows, A, generator=gen).float()
    n = unit_vectors(gen, rows)
    y = torch.cat(I.direction_harmonics_all(n, le), -1).float()
    gates = (torch.randn(rows, P * channels, generator=gen) / np.sqrt(P)).float() if use_gates else None
    W = sum(c * channels * (2 * l + 1) for l, c in tp64.path_counts_by_l.items())
    G = torch.randn(rows, W, generator=gen).float()
    hx = torch.randn(rows, A, generator=gen).float()
    hy = torch.randn(rows, (le + 1) ** 2, generator=gen).float()
    hg = torch.randn(rows, P * channels, generator=gen).float() if use_gates else None

    # FP32 forward of the reference (its own compute dtype).
    with torch.no_grad():
        out32 = pack_out(tp32, tp32(split_mul_ir(x, channels, li), split_harm(y, le),
                                    None if gates is None else gates.view(rows, P, channels)))

    # FP64 truth with first and mixed second derivatives.
    xd = x.double().requires_grad_(True)
    yd = y.double().requires_grad_(True)
    gd = gates.double().requires_grad_(True) if use_gates else None
    Gd = G.double().requires_grad_(True)
    tp64.weight.requires_grad_(True)
    out = pack_out(tp64, tp64(split_mul_ir(xd, channels, li), split_harm(yd, le),
                              None if gd is None else gd.view(rows, P, channels)))
    inputs = [xd, yd] + ([gd] if use_gates else []) + [tp64.weight]
    firsts = torch.autograd.grad((out * Gd).sum(), inputs, create_graph=True)
    dx, dy = firsts[0], firsts[1]
    dg = firsts[2] if use_gates else None
    dw = firsts[-1]
    second = (dx * hx.double()).sum() + (dy * hy.double()).sum()
    if use_gates:
        second = second + (dg * hg.double()).sum()
    targets = [xd, yd] + ([gd] if use_gates else []) + [Gd]
    seconds = torch.autograd.grad(second, targets, allow_unused=True)
    record = dict(channels=channels, li=li, le=le, lo=lo, rows=rows, x=x.numpy(), y=y.numpy(),
                  weight=weight.numpy(), G=G.numpy(), hx=hx.numpy(), hy=hy.numpy(),
                  out32=out32.numpy(), out64=out.detach().numpy(), dx64=dx.detach().numpy(),
                  dy64=dy.detach().numpy(), dw64=dw.detach().numpy(),
                  sx64=seconds[0].numpy(), sy64=seconds[1].numpy(), sG64=seconds[-1].numpy(),
                  cg=np.concatenate([c.reshape(-1).numpy() for c in
                                     tp64._get_cg_list(torch.device("cpu"), torch.float64)]),
                  paths=np.array(tp64.paths, dtype=np.int32),
                  path_offset=np.array(tp64.path_offset, dtype=np.int32))
    if use_gates:
        record.update(gates=gates.numpy(), hg=hg.numpy(), dg64=dg.detach().numpy(), sg64=seconds[2].numpy())
    np.savez_compressed(os.path.join(HERE, name), **record)
    print("wrote", name)


def harmonics_case(I, name, lmax, rows, seed):
    gen = torch.Generator().manual_seed(seed)
    n = unit_vectors(gen, rows)
    n[:4] = torch.tensor([[1., 0, 0], [0, 1., 0], [0, 0, 1.], [0.6, -0.8, 0.]], dtype=torch.float64)
    nf = n.float()
    W = (lmax + 1) ** 2
    gy = torch.randn(rows, W, generator=gen).float()
    hn = torch.randn(rows, 3, generator=gen).float()
    with torch.no_grad():
        y32 = torch.cat(I.direction_harmonics_all(nf, lmax), -1)
    nd = nf.double().requires_grad_(True)
    gyd = gy.double().requires_grad_(True)
    y = torch.cat(I.direction_harmonics_all(nd, lmax), -1)
    (dn,) = torch.autograd.grad((y * gyd).sum(), [nd], create_graph=True)
    sn, sgy = torch.autograd.grad((dn * hn.double()).sum(), [nd, gyd])
    np.savez_compressed(os.path.join(HERE, name), lmax=lmax, n=nf.numpy(), gy=gy.numpy(), hn=hn.numpy(),
                        y32=y32.numpy(), y64=y.detach().numpy(), dn64=dn.detach().numpy(),
                        sn64=sn.numpy(), sgy64=sgy.numpy())
    print("wrote", name)


def message_case(I, name, channels, lmax, nodes, edges, seed):
    gen = torch.Generator().manual_seed(seed)
    tp = make_tp(I, channels, lmax, lmax, lmax, torch.float64)
    with torch.no_grad():
        tp.weight.fill_(1.0)
    P = tp.num_paths
    A = channels * (lmax + 1) ** 2
    x = torch.randn(nodes, A, generator=gen).float()
    src = torch.randint(0, nodes, (edges,), generator=gen)
    dst = torch.randint(0, nodes - 2, (edges,), generator=gen)  # the last two nodes receive nothing
    n = unit_vectors(gen, edges)
    y = torch.cat(I.direction_harmonics_all(n, lmax), -1).float()
    gates = (torch.randn(edges, P * channels, generator=gen) / np.sqrt(P)).float()
    mask = (torch.rand(edges, generator=gen) > 0.2).float()
    W = sum(c * channels * (2 * l + 1) for l, c in tp.path_counts_by_l.items())
    G = torch.randn(nodes, W, generator=gen).float()
    xd = x.double().requires_grad_(True)
    yd = y.double().requires_grad_(True)
    gd = gates.double().requires_grad_(True)
    blocks = split_mul_ir(xd, channels, lmax)
    edge_blocks = {l: v.index_select(0, src) for l, v in blocks.items()}
    value = tp(edge_blocks, split_harm(yd, lmax), gd.view(edges, P, channels))
    outs = {}
    for l, block in value.items():
        block = block * mask.double().reshape(-1, 1, 1)
        outs[l] = torch.zeros(nodes, *block.shape[1:], dtype=torch.float64).index_add(0, dst, block)
    out = pack_out(tp, outs)
    dx, dy, dg = torch.autograd.grad((out * G.double()).sum(), [xd, yd, gd])
    np.savez_compressed(os.path.join(HERE, name), channels=channels, lmax=lmax, nodes=nodes, x=x.numpy(),
                        y=y.numpy(), gates=gates.numpy(), mask=mask.numpy(), src=src.numpy(), dst=dst.numpy(),
                        G=G.numpy(), out64=out.detach().numpy(), dx64=dx.numpy(), dy64=dy.numpy(),
                        dg64=dg.numpy())
    print("wrote", name)


def full_cg_case(I, name, lmax):
    """Full SO(3) couplings (any parity) of the ICTC basis (ictd_irreps.py:1305-1373)."""
    keys, values = [], []
    for l1 in range(lmax + 1):
        for l2 in range(lmax + 1):
            for l3 in range(abs(l1 - l2), l1 + l2 + 1):
                keys.append((l1, l2, l3))
                values.append(I.build_full_cg_tensor_so3(l1, l2, l3).numpy().reshape(-1))
    np.savez_compressed(os.path.join(HERE, name), keys=np.array(keys, dtype=np.int32),
                        values=np.concatenate(values))
    print("wrote", name)


def u_probe_case(I, name, lmaxes, seed):
    """Pins ictd_u_matrix_so3 (ictd_irreps.py:1465-1517) by contracting every input
    axis with a distinct seeded probe vector: result [2t+1, P] per (lmax, t, nu)."""
    gen = torch.Generator().manual_seed(seed)
    record = {}
    for lmax in lmaxes:
        dim = (lmax + 1) ** 2
        probes = torch.randn(3, dim, generator=gen, dtype=torch.float64)
        record[f"probes_l{lmax}"] = probes.numpy()
        for t in range(lmax + 1):
            for nu in (1, 2, 3):
                u = I.ictd_u_matrix_so3(lmax=lmax, output_l=t, correlation=nu, dtype=torch.float64)
                if t == 0:
                    u = u.unsqueeze(0)
                for a in range(nu):
                    u = torch.tensordot(u, probes[a], dims=([1], [0]))
                record[f"u_l{lmax}_t{t}_nu{nu}"] = u.numpy()
    np.savez_compressed(os.path.join(HERE, name), **record)
    print("wrote", name)


def contraction_case(I, name, channels, lmax, target_lmax, correlation, nodes, elements, seed):
    """Symmetric contraction with the reference's ICTC U tensors and the MACE recursion
    with element-selected weights (_mace_symmetric_contraction.py:298-346), FP64."""
    gen = torch.Generator().manual_seed(seed)
    dim = (lmax + 1) ** 2
    x = torch.randn(nodes, channels * dim, generator=gen).float()
    idx = torch.randint(0, elements, (nodes,), generator=gen)
    record = dict(channels=channels, lmax=lmax, target_lmax=target_lmax, correlation=correlation,
                  elements=elements, x=x.numpy(), idx=idx.numpy())
    xd = x.double().requires_grad_(True)
    blocks = [xd[:, l * l * channels:(l + 1) ** 2 * channels].reshape(nodes, channels, 2 * l + 1)
              for l in range(lmax + 1)]
    feats = torch.cat(blocks, -1)
    outs, weights_all = [], []
    for t in range(target_lmax + 1):
        u = {nu: I.ictd_u_matrix_so3(lmax=lmax, output_l=t, correlation=nu, dtype=torch.float64)
             for nu in range(1, correlation + 1)}
        ws = {}
        for nu in range(correlation, 0, -1):
            p = u[nu].shape[-1]
            w = (torch.randn(elements, p, channels, generator=gen) / max(p, 1)).float()
            record[f"w_t{t}_nu{nu}"] = w.numpy()
            ws[nu] = w.double().requires_grad_(True)
            weights_all.append(ws[nu])

        def coef(order):
            sel = ws[order].index_select(0, idx)
            return torch.tensordot(sel, u[order], dims=([1], [u[order].ndim - 1]))
        out = coef(correlation)
        for order in range(correlation - 1, 0, -1):
            out = torch.einsum("bc...i,bci->bc...", out, feats) + coef(order)
        out = torch.einsum("bc...i,bci->bc...", out, feats)
        outs.append(out.reshape(nodes, -1))
    out = torch.cat(outs, -1)
    G = torch.randn(out.shape, generator=gen, dtype=torch.float64)
    grads = torch.autograd.grad((out * G).sum(), [xd] + weights_all)
    record.update(out64=out.detach().numpy(), G=G.numpy(), dx64=grads[0].numpy())
    k = 1
    for t in range(target_lmax + 1):
        for nu in range(correlation, 0, -1):
            record[f"dw_t{t}_nu{nu}"] = grads[k].numpy()
            k += 1
    np.savez_compressed(os.path.join(HERE, name), **record)
    print("wrote", name)


def main():
    from ictc_o3.basis import ictd_irreps as I
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    tp_case(I, "tp_c64_l2.npz", 64, 2, 2, 2, rows=12, seed=1)
    tp_case(I, "tp_c128_l3.npz", 128, 3, 3, 3, rows=5, seed=2)
    tp_case(I, "tp_c32_l0e3.npz", 32, 0, 3, 3, rows=16, seed=3)
    tp_case(I, "tp_c32_l1_nogate.npz", 32, 1, 1, 1, rows=9, seed=4, use_gates=False)
    tp_case(I, "tp_c64_l2_unitw.npz", 64, 2, 2, 2, rows=7, seed=5, random_weight=False)
    harmonics_case(I, "harmonics_l6.npz", 6, rows=64, seed=6)
    harmonics_case(I, "harmonics_l3.npz", 3, rows=40, seed=7)
    message_case(I, "message_c32_l2.npz", 32, 2, nodes=14, edges=60, seed=8)
    full_cg_case(I, "full_cg_l3.npz", 3)
    u_probe_case(I, "u_probes.npz", (1, 2, 3), seed=9)
    contraction_case(I, "contraction_c32_l2.npz", 32, 2, 2, 3, nodes=23, elements=3, seed=10)
    contraction_case(I, "contraction_c32_l1_t0.npz", 32, 1, 0, 2, nodes=9, elements=2, seed=11)


if __name__ == "__main__":
    sys.exit(main())
