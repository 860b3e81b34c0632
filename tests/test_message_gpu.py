"""GPU parity of the CSR graph-message kernels against the reference (golden) and the oracle."""
import pytest
import torch

from _util import golden, make_owner, assert_close, ir_mul_to_mul_ir, mul_ir_to_ir_mul, output_degrees
from oracle import tp_oracle

pytestmark = pytest.mark.gpu
FWD_TOL, GRAD_TOL = 1e-5, 1e-4


@pytest.mark.parametrize("layout", ["mul_ir", "ir_mul"])
def test_message_matches_reference(layout, cuda_device):
    from ictc_o3.backends.cuda.message import packed_graph_message
    g = golden("message_c32_l2.npz")
    C, L = int(g["channels"]), int(g["lmax"])
    owner = make_owner(C, L, L, L).to(cuda_device)
    x = torch.from_numpy(g["x"])
    if layout == "ir_mul":
        x = mul_ir_to_ir_mul(x, C, range(L + 1))
    x = x.to(cuda_device).contiguous().requires_grad_(True)
    y = torch.from_numpy(g["y"]).to(cuda_device).requires_grad_(True)
    gates = torch.from_numpy(g["gates"]).to(cuda_device).requires_grad_(True)
    src, dst = torch.from_numpy(g["src"]).to(cuda_device), torch.from_numpy(g["dst"]).to(cuda_device)
    mask = torch.from_numpy(g["mask"]).to(cuda_device)
    out = packed_graph_message(owner, layout, x, y, gates, src, dst, mask)
    got = out if layout == "mul_ir" else ir_mul_to_mul_ir(out, C, output_degrees(owner))
    assert_close(got.detach().cpu(), g["out64"], FWD_TOL, 1e-3, "message forward")
    G = torch.from_numpy(g["G"])
    if layout == "ir_mul":
        G = mul_ir_to_ir_mul(G, C, output_degrees(owner))
    dx, dy, dg = torch.autograd.grad(out, [x, y, gates], G.to(cuda_device).contiguous())
    dx = dx if layout == "mul_ir" else ir_mul_to_mul_ir(dx, C, range(L + 1))
    assert_close(dx.cpu(), g["dx64"], GRAD_TOL, 1e-3, "message dx")
    assert_close(dy.cpu(), g["dy64"], GRAD_TOL, 1e-3, "message dY")
    assert_close(dg.cpu(), g["dg64"], GRAD_TOL, 1e-3, "message dgate")


def _random_graph(gen, nodes, edges, dst_nodes):
    src = torch.randint(0, nodes, (edges,), generator=gen)
    dst = torch.randint(0, dst_nodes, (edges,), generator=gen)
    if edges > 4:
        dst[: edges // 4] = 0  # one heavy destination
    return src, dst


@pytest.mark.parametrize("shape", [(64, 2, 2, 2), (128, 3, 3, 3), (64, 0, 2, 2), (96, 1, 1, 1)])
@pytest.mark.parametrize("graph", [(40, 300, 40), (25, 0, 25), (50, 400, 31), (1, 3, 1)])
def test_message_random_against_oracle(shape, graph, cuda_device):
    """Masks, a heavy node, isolated nodes, empty edge lists and owned destinations
    (dst_nodes < src_nodes, the halo layout); first and mixed second derivatives."""
    from ictc_o3.backends.cuda.message import packed_graph_message
    C, li, le, lo = shape
    nodes, edges, dst_nodes = graph
    gen = torch.Generator().manual_seed(nodes * 131 + edges + C)
    owner = make_owner(C, li, le, lo)
    owner._cuda_destination_nodes = dst_nodes
    owner_dev = make_owner(C, li, le, lo).to(cuda_device)
    owner_dev._cuda_destination_nodes = dst_nodes
    P = owner.num_paths
    src, dst = _random_graph(gen, nodes, edges, dst_nodes)
    x = torch.randn(nodes, C * (li + 1) ** 2, generator=gen)
    n = torch.nn.functional.normalize(torch.randn(edges, 3, generator=gen), dim=1)
    y = torch.cat(tp_oracle.direction_harmonics(n.double(), max(le, 1), tp_oracle.harmonic_tables(max(le, 1)))[:le + 1], -1).float()
    gates = torch.randn(edges, P * C, generator=gen) / P ** 0.5
    mask = (torch.rand(edges, generator=gen) > 0.25).float()
    G = torch.randn(dst_nodes, owner.output_width, generator=gen)
    hx = torch.randn_like(x)
    hy = torch.randn_like(y)
    hg = torch.randn_like(gates)

    # FP64 oracle with first and mixed second derivatives.
    xd, yd, gd, Gd = (t.double().requires_grad_(True) for t in (x, y, gates, G))
    ref = tp_oracle.pack_out(owner, tp_oracle.graph_message(
        owner, tp_oracle.split_mul_ir(xd, C, li), tp_oracle.split_harm(yd, le), gd.view(edges, P, C),
        src, dst, mask.double(), nodes=dst_nodes, dtype=torch.float64))
    rdx, rdy, rdg = torch.autograd.grad((ref * Gd).sum(), [xd, yd, gd], create_graph=True, allow_unused=True)
    rdx = torch.zeros_like(xd) if rdx is None else rdx
    rdy = torch.zeros_like(yd) if rdy is None else rdy
    rdg = torch.zeros_like(gd) if rdg is None else rdg
    second = (rdx * hx.double()).sum() + (rdy * hy.double()).sum() + (rdg * hg.double()).sum()
    if second.requires_grad:
        rs = torch.autograd.grad(second, [xd, yd, gd, Gd], allow_unused=True)
        rs = [torch.zeros_like(t) if r is None else r for r, t in zip(rs, (xd, yd, gd, Gd))]
    else:
        rs = [torch.zeros_like(t) for t in (xd, yd, gd, Gd)]

    dev = cuda_device
    for layout in ("mul_ir", "ir_mul"):
        xi = x if layout == "mul_ir" else mul_ir_to_ir_mul(x, C, range(li + 1))
        Gi = G if layout == "mul_ir" else mul_ir_to_ir_mul(G, C, output_degrees(owner))
        hxi = hx if layout == "mul_ir" else mul_ir_to_ir_mul(hx, C, range(li + 1))
        xc = xi.to(dev).contiguous().requires_grad_(True)
        yc = y.to(dev).requires_grad_(True)
        gc = gates.to(dev).requires_grad_(True)
        Gc = Gi.to(dev).contiguous().requires_grad_(True)
        out = packed_graph_message(owner_dev, layout, xc, yc, gc, src.to(dev), dst.to(dev), mask.to(dev))
        assert out.shape == (dst_nodes, owner.output_width)
        got = out if layout == "mul_ir" else ir_mul_to_mul_ir(out, C, output_degrees(owner))
        assert_close(got.detach().cpu(), ref.detach(), FWD_TOL, 1e-3, f"{shape} {graph} {layout} fwd")
        if edges == 0:
            continue
        dx, dy, dg = torch.autograd.grad((out * Gc).sum(), [xc, yc, gc], create_graph=True)
        dxm = dx if layout == "mul_ir" else ir_mul_to_mul_ir(dx, C, range(li + 1))
        assert_close(dxm.detach().cpu(), rdx.detach(), GRAD_TOL, 1e-3, f"{layout} dx")
        assert_close(dy.detach().cpu(), rdy.detach(), GRAD_TOL, 1e-3, f"{layout} dY")
        assert_close(dg.detach().cpu(), rdg.detach(), GRAD_TOL, 1e-3, f"{layout} dg")
        s2 = (dx * hxi.to(dev)).sum() + (dy * hy.to(dev)).sum() + (dg * hg.to(dev)).sum()
        sx, sy, sg, sG = torch.autograd.grad(s2, [xc, yc, gc, Gc], allow_unused=True)
        sx = sx if layout == "mul_ir" else ir_mul_to_mul_ir(sx, C, range(li + 1))
        sG = sG if layout == "mul_ir" else ir_mul_to_mul_ir(sG, C, output_degrees(owner))
        for name, a, b in (("x", sx, rs[0]), ("Y", sy, rs[1]), ("g", sg, rs[2]), ("G", sG, rs[3])):
            if float(b.abs().max()) == 0.0:
                continue
            assert_close(a.cpu(), b, GRAD_TOL, 1e-3, f"{layout} second derivative {name}")


def test_message_block_api_and_public_operator(cuda_device):
    from ictc_o3.operators import GraphMessage, PackedGraphMessage
    g = golden("message_c32_l2.npz")
    C, L = int(g["channels"]), int(g["lmax"])
    op = PackedGraphMessage.create(channels=C, input_lmax=L, edge_lmax=L, layout="mul_ir", device=cuda_device)
    x = torch.from_numpy(g["x"]).to(cuda_device)
    y = torch.from_numpy(g["y"]).to(cuda_device)
    gates = torch.from_numpy(g["gates"]).to(cuda_device)
    src, dst = torch.from_numpy(g["src"]).to(cuda_device), torch.from_numpy(g["dst"]).to(cuda_device)
    mask = torch.from_numpy(g["mask"]).to(cuda_device)
    assert_close(op(x, y, gates, src, dst, mask).cpu(), g["out64"], FWD_TOL, 1e-3, "packed operator")
    blocks = GraphMessage(op.tp, input_lmax=L, edge_lmax=L, layout="mul_ir")(
        tp_oracle.split_mul_ir(x, C, L), tp_oracle.split_harm(y, L), gates.view(-1, op.tp.num_paths, C),
        src, dst, mask)
    assert_close(tp_oracle.pack_out(op.tp, blocks).cpu(), g["out64"], FWD_TOL, 1e-3, "block operator")
    with pytest.raises(ValueError):
        op(x, y, gates, src, dst.clamp_max(0) + x.shape[0], mask)  # out-of-range destination
    with pytest.raises(ValueError):
        op(x, y, gates, src.int(), dst, mask)


def test_message_config3_scale_sampled(cuda_device):
    """Config-3 scale (16,384 atoms, ~52 neighbours, C64/L2): sampled destination rows
    and sampled edge gradients against the oracle."""
    from ictc_o3.backends.cuda.message import packed_graph_message
    C, L, nodes, deg = 64, 2, 16384, 52
    owner = make_owner(C, L, L, L)
    owner_dev = make_owner(C, L, L, L).to(cuda_device)
    dev = cuda_device
    gen = torch.Generator(device=dev).manual_seed(5)
    edges = nodes * deg
    dst = torch.arange(nodes, device=dev).repeat_interleave(deg)
    src = torch.randint(0, nodes, (edges,), device=dev, generator=gen)
    perm = torch.randperm(edges, device=dev, generator=gen)
    src, dst = src[perm], dst[perm]
    x = torch.randn(nodes, C * 9, device=dev, generator=gen, requires_grad=True)
    n = torch.nn.functional.normalize(torch.randn(edges, 3, device=dev, generator=gen), dim=1)
    from ictc_o3.backends.cuda.geometry import direction_harmonics
    y = direction_harmonics(n, L).requires_grad_(True)
    gates = (torch.randn(edges, owner.num_paths * C, device=dev, generator=gen) / 11 ** 0.5).requires_grad_(True)
    out = packed_graph_message(owner_dev, "ir_mul", x, y, gates, src, dst)
    G = torch.randn_like(out)
    dx, dy, dg = torch.autograd.grad(out, [x, y, gates], G)
    rows = torch.randint(0, nodes, (32,), device=dev, generator=gen)
    for r in rows.tolist():
        sel = (dst == r).nonzero().flatten()
        xs = ir_mul_to_mul_ir(x.detach()[src[sel]].double().cpu(), C, range(L + 1))
        ref = tp_oracle.tp_forward(owner, tp_oracle.split_mul_ir(xs, C, L),
                                   tp_oracle.split_harm(y.detach()[sel].double().cpu(), L),
                                   gates.detach()[sel].double().cpu().view(-1, 11, C), dtype=torch.float64)
        ref = tp_oracle.pack_out(owner, ref).sum(0, keepdim=True)
        got = ir_mul_to_mul_ir(out.detach()[r:r + 1].double().cpu(), C, output_degrees(owner))
        assert_close(got, ref, FWD_TOL, 1e-3, f"node {r}")
    # Edge gradients of sampled edges: dY_e and dg_e depend only on x[src], Y_e, g_e and G[dst].
    sample = torch.randint(0, edges, (64,), device=dev, generator=gen)
    xs = ir_mul_to_mul_ir(x.detach()[src[sample]].double().cpu(), C, range(L + 1)).requires_grad_(True)
    ys = y.detach()[sample].double().cpu().requires_grad_(True)
    gs = gates.detach()[sample].double().cpu().requires_grad_(True)
    Gs = ir_mul_to_mul_ir(G[dst[sample]].double().cpu(), C, output_degrees(owner))
    ref = tp_oracle.pack_out(owner, tp_oracle.tp_forward(owner, tp_oracle.split_mul_ir(xs, C, L),
                                                         tp_oracle.split_harm(ys, L), gs.view(-1, 11, C),
                                                         dtype=torch.float64))
    _, rdy, rdg = torch.autograd.grad((ref * Gs).sum(), [xs, ys, gs])
    assert_close(dy[sample].cpu(), rdy, GRAD_TOL, 1e-3, "sampled dY")
    assert_close(dg[sample].cpu(), rdg, GRAD_TOL, 1e-3, "sampled dgate")
    assert torch.isfinite(dx).all()


def test_message_staged_and_direct_paths_agree(cuda_device):
    """C64/lmax2 mul_ir (one warp per node): the adjoint stages each edge's
    output-gradient row and gate row in shared memory by bulk copy, the forward each
    edge's source row and gate row; operands that are not 16-byte aligned take the
    direct-load kernels instead.  Both paths agree, and no staging wait ran out."""
    from ictc_o3.backends.cuda.message import packed_graph_message
    from ictc_o3.backends.cuda.tensor_product import get_plan
    C, L, nodes, edges = 64, 2, 300, 5000
    gen = torch.Generator().manual_seed(17)
    owner = make_owner(C, L, L, L).to(cuda_device)
    src, dst = _random_graph(gen, nodes, edges, nodes)
    src, dst = src.to(cuda_device), dst.to(cuda_device)
    x = torch.randn(nodes, C * (L + 1) ** 2, generator=gen).to(cuda_device).requires_grad_(True)
    n = torch.nn.functional.normalize(torch.randn(edges, 3, generator=gen), dim=1)
    y = torch.cat(tp_oracle.direction_harmonics(n.double(), L, tp_oracle.harmonic_tables(L))[:L + 1], -1)
    y = y.float().to(cuda_device).requires_grad_(True)
    gates = (torch.randn(edges, owner.num_paths * C, generator=gen) / 3.0).to(cuda_device).requires_grad_(True)
    mask = (torch.rand(edges, generator=gen) > 0.2).float().to(cuda_device)
    out = packed_graph_message(owner, "mul_ir", x, y, gates, src, dst, mask)
    G = torch.randn(out.shape, generator=gen).to(cuda_device)
    staged = torch.autograd.grad(out, [x, y, gates], G, retain_graph=True)
    shifted = torch.empty(G.numel() + 1, device=cuda_device)[1:].view_as(G)
    shifted.copy_(G)
    assert shifted.data_ptr() % 16 != 0
    direct = torch.autograd.grad(out, [x, y, gates], shifted)
    for a, b in zip(staged, direct):
        assert torch.equal(a, b)
    # Forward: 16-byte aligned rows take the staged two-channels-per-lane kernel,
    # a shifted feature buffer the one-channel-per-lane kernel with direct loads.
    xs = torch.empty(x.numel() + 1, device=cuda_device)[1:].view_as(x)
    xs.copy_(x.detach())
    assert xs.data_ptr() % 16 != 0
    with torch.no_grad():
        out_direct = packed_graph_message(owner, "mul_ir", xs, y.detach(), gates.detach(), src, dst, mask)
    torch.testing.assert_close(out_direct, out.detach(), rtol=1e-6, atol=1e-6)
    assert get_plan(owner, "mul_ir", cuda_device).status() == 0
