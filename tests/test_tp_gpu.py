"""GPU parity of the CUDA tensor product against the reference (golden) and the oracle.

Tolerances (the project's FP32 parity bar): relative L2 1e-5 on TP outputs, 1e-4 on
gradients and second derivatives, plus the reference's componentwise bound
(rtol 1e-4, atol 2e-5 scaled by the RMS; docs/USAGE.md:889-891); see _util.assert_close.
"""
import pytest
import torch

from _util import golden, make_owner, assert_close, ir_mul_to_mul_ir, mul_ir_to_ir_mul, output_degrees
from oracle import tp_oracle

pytestmark = pytest.mark.gpu

TP_CASES = ["tp_c64_l2.npz", "tp_c128_l3.npz", "tp_c32_l0e3.npz", "tp_c32_l1_nogate.npz", "tp_c64_l2_unitw.npz"]
FWD_TOL, GRAD_TOL = 1e-5, 1e-4


def _inputs(g, layout, device, requires_grad=False):
    C, li = int(g["channels"]), int(g["li"])
    x = torch.from_numpy(g["x"])
    if layout == "ir_mul":
        x = mul_ir_to_ir_mul(x, C, range(li + 1))
    x = x.to(device).contiguous().requires_grad_(requires_grad)
    y = torch.from_numpy(g["y"]).to(device).requires_grad_(requires_grad)
    gates = torch.from_numpy(g["gates"]).to(device).requires_grad_(requires_grad) if "gates" in g else None
    return x, y, gates


def _to_mul_ir(owner, out, layout):
    return out if layout == "mul_ir" else ir_mul_to_mul_ir(out, owner.channels, output_degrees(owner))


@pytest.mark.parametrize("layout", ["ir_mul", "mul_ir"])
@pytest.mark.parametrize("name", TP_CASES)
def test_forward_matches_reference(name, layout, cuda_device):
    from ictc_o3.backends.cuda.tensor_product import packed_product
    g = golden(name)
    owner = make_owner(int(g["channels"]), int(g["li"]), int(g["le"]), int(g["lo"]), weight=g["weight"]).to(cuda_device)
    x, y, gates = _inputs(g, layout, cuda_device)
    out = packed_product(owner, layout, x, y, gates)
    torch.cuda.synchronize()
    assert_close(_to_mul_ir(owner, out, layout).cpu(), g["out64"], FWD_TOL, 1e-3, f"{name} {layout} forward")


@pytest.mark.parametrize("layout", ["ir_mul", "mul_ir"])
@pytest.mark.parametrize("name", TP_CASES)
def test_first_and_second_derivatives_match_reference(name, layout, cuda_device):
    from ictc_o3.backends.cuda.tensor_product import packed_product
    g = golden(name)
    C, li = int(g["channels"]), int(g["li"])
    owner = make_owner(C, li, int(g["le"]), int(g["lo"]), weight=g["weight"]).to(cuda_device)
    x, y, gates = _inputs(g, layout, cuda_device, requires_grad=True)
    G = torch.from_numpy(g["G"])
    if layout == "ir_mul":
        G = mul_ir_to_ir_mul(G, C, output_degrees(owner))
    G = G.to(cuda_device).contiguous().requires_grad_(True)
    out = packed_product(owner, layout, x, y, gates)
    targets = [x, y] + ([gates] if gates is not None else [])
    firsts = torch.autograd.grad((out * G).sum(), targets, create_graph=True)
    dx = firsts[0] if layout == "mul_ir" else ir_mul_to_mul_ir(firsts[0], C, range(li + 1))
    assert_close(dx.detach().cpu(), g["dx64"], GRAD_TOL, 1e-3, "dx")
    assert_close(firsts[1].detach().cpu(), g["dy64"], GRAD_TOL, 1e-3, "dY")
    hx = torch.from_numpy(g["hx"])
    if layout == "ir_mul":
        hx = mul_ir_to_ir_mul(hx, C, range(li + 1))
    second = (firsts[0] * hx.to(cuda_device)).sum() + (firsts[1] * torch.from_numpy(g["hy"]).to(cuda_device)).sum()
    if gates is not None:
        assert_close(firsts[2].detach().cpu(), g["dg64"], GRAD_TOL, 1e-3, "dgate")
        second = second + (firsts[2] * torch.from_numpy(g["hg"]).to(cuda_device)).sum()
    seconds = torch.autograd.grad(second, targets + [G])
    sx = seconds[0] if layout == "mul_ir" else ir_mul_to_mul_ir(seconds[0], C, range(li + 1))
    sG = seconds[-1] if layout == "mul_ir" else ir_mul_to_mul_ir(seconds[-1], C, output_degrees(owner))
    assert_close(sx.cpu(), g["sx64"], GRAD_TOL, 1e-3, "d2 x")
    assert_close(seconds[1].cpu(), g["sy64"], GRAD_TOL, 1e-3, "d2 Y")
    assert_close(sG.cpu(), g["sG64"], GRAD_TOL, 1e-3, "d2 G")
    if gates is not None:
        assert_close(seconds[2].cpu(), g["sg64"], GRAD_TOL, 1e-3, "d2 gate")


def test_block_api_matches_reference(cuda_device):
    from ictc_o3.backends.cuda.tensor_product import tensor_product
    g = golden("tp_c64_l2.npz")
    C, L = int(g["channels"]), int(g["li"])
    owner = make_owner(C, L, L, L, weight=g["weight"]).to(cuda_device)
    x = torch.from_numpy(g["x"]).to(cuda_device)
    y = torch.from_numpy(g["y"]).to(cuda_device)
    gates = torch.from_numpy(g["gates"]).to(cuda_device).view(-1, owner.num_paths, C)
    out = tensor_product(owner, tp_oracle.split_mul_ir(x, C, L), tp_oracle.split_harm(y, L), gates)
    assert sorted(out) == list(range(L + 1))
    assert_close(tp_oracle.pack_out(owner, out).cpu(), g["out64"], FWD_TOL, 1e-3, "block api")


@pytest.mark.parametrize("cpl", [(1, 1), (2, 2), (4, 4), (4, 1)])
@pytest.mark.parametrize("shape", [(128, 3, 3, 3), (64, 2, 2, 2), (64, 0, 2, 2), (96, 1, 1, 1), (256, 2, 2, 2), (16, 2, 2, 2), (40, 3, 3, 3)])
@pytest.mark.parametrize("rows", [1, 37, 1031])
def test_random_against_oracle(shape, rows, cpl, cuda_device):
    """Ragged row counts, every channel-per-lane variant, both layouts, with a live weight."""
    from ictc_o3.backends.cuda.tensor_product import get_plan, raw_backward, raw_forward
    C, li, le, lo = shape
    gen = torch.Generator().manual_seed(rows * 7 + C)
    owner = make_owner(C, li, le, lo, weight=torch.randn(len(make_owner(C, li, le, lo).paths), C, generator=gen))
    P = owner.num_paths
    x = torch.randn(rows, C * (li + 1) ** 2, generator=gen)
    n = torch.nn.functional.normalize(torch.randn(rows, 3, generator=gen), dim=1)
    y = torch.cat(tp_oracle.direction_harmonics(n.double(), le, tp_oracle.harmonic_tables(max(le, 1)))[:le + 1], -1).float()
    gates = torch.randn(rows, P * C, generator=gen)
    G = torch.randn(rows, owner.output_width, generator=gen)
    xd, yd, gd, Gd = (t.double().requires_grad_(True) for t in (x, y, gates, G))
    ref = tp_oracle.pack_out(owner, tp_oracle.tp_forward(owner, tp_oracle.split_mul_ir(xd, C, li),
                                                         tp_oracle.split_harm(yd, le), gd.view(rows, P, C),
                                                         dtype=torch.float64))
    rdx, rdy, rdg = torch.autograd.grad((ref * Gd).sum(), [xd, yd, gd])
    w = owner.weight.detach().reshape(-1).to(cuda_device)
    for layout in ("mul_ir", "ir_mul"):
        plan = get_plan(owner, layout, cuda_device, cpl_forward=cpl[0], cpl_backward=cpl[1])
        xi = x if layout == "mul_ir" else mul_ir_to_ir_mul(x, C, range(li + 1))
        Gi = G if layout == "mul_ir" else mul_ir_to_ir_mul(G, C, output_degrees(owner))
        xc, yc, gc, Gc = (t.to(cuda_device).contiguous() for t in (xi, y, gates, Gi))
        out = raw_forward(plan, xc, yc, gc, w)
        dx, dy, dg = raw_backward(plan, xc, yc, gc, w, Gc, (True, True, True))
        torch.cuda.synchronize()
        out = out.cpu() if layout == "mul_ir" else ir_mul_to_mul_ir(out.cpu(), C, output_degrees(owner))
        dx = dx.cpu() if layout == "mul_ir" else ir_mul_to_mul_ir(dx.cpu(), C, range(li + 1))
        assert_close(out, ref.detach(), FWD_TOL, 1e-3, f"{shape} {layout} fwd")
        assert_close(dx, rdx, GRAD_TOL, 1e-3, f"{shape} {layout} dx")
        assert_close(dy.cpu(), rdy, GRAD_TOL, 1e-3, f"{shape} {layout} dY")
        assert_close(dg.cpu(), rdg, GRAD_TOL, 1e-3, f"{shape} {layout} dg")


def test_empty_rows_and_weight_gradient(cuda_device):
    from ictc_o3.backends.cuda.tensor_product import packed_product
    owner = make_owner(64, 2, 2, 2).to(cuda_device)
    x = torch.zeros(0, 64 * 9, device=cuda_device, requires_grad=True)
    y = torch.zeros(0, 9, device=cuda_device, requires_grad=True)
    out = packed_product(owner, "ir_mul", x, y, None)
    assert out.shape == (0, owner.output_width)
    out.sum().backward()
    assert x.grad.shape == x.shape and y.grad.shape == y.shape
    # A trainable weight receives sum_e gate * dgeff.
    gen = torch.Generator().manual_seed(3)
    rows = 50
    owner.weight.requires_grad_(True)
    x = torch.randn(rows, 64 * 9, generator=gen)
    n = torch.nn.functional.normalize(torch.randn(rows, 3, generator=gen), dim=1)
    y = torch.cat(tp_oracle.direction_harmonics(n.double(), 2, tp_oracle.harmonic_tables(2)), -1).float()
    gates = torch.randn(rows, owner.num_paths * 64, generator=gen)
    out = packed_product(owner, "mul_ir", x.to(cuda_device), y.to(cuda_device), gates.to(cuda_device))
    (dw,) = torch.autograd.grad(out.sum(), [owner.weight])
    wd = owner.weight.detach().cpu().double().requires_grad_(True)
    ref = tp_oracle.tp_forward(owner.cpu(), tp_oracle.split_mul_ir(x.double(), 64, 2), tp_oracle.split_harm(y.double(), 2),
                               gates.double().view(rows, -1, 64), weight=wd, dtype=torch.float64)
    (rdw,) = torch.autograd.grad(sum(v.sum() for v in ref.values()), [wd])
    assert_close(dw.cpu(), rdw, GRAD_TOL, 1e-3, "dweight")


def test_full_size_sampled_rows(cuda_device):
    """Config 2 sizes (C128/L3): 262,144 forward rows and 131,072 fwd+VJP rows,
    checked on sampled rows against the oracle (docs/USAGE.md:859-860 method)."""
    from ictc_o3.backends.cuda.tensor_product import get_plan, raw_backward, raw_forward
    C, L = 128, 3
    owner = make_owner(C, L, L, L)
    plan = get_plan(owner, "ir_mul", cuda_device)
    gen = torch.Generator(device=cuda_device).manual_seed(11)
    for rows, backward in ((262144, False), (131072, True)):
        x = torch.randn(rows, C * 16, device=cuda_device, generator=gen)
        n = torch.nn.functional.normalize(torch.randn(rows, 3, device=cuda_device, generator=gen), dim=1)
        from ictc_o3.backends.cuda.geometry import direction_harmonics
        y = direction_harmonics(n, L)
        gates = torch.randn(rows, owner.num_paths * C, device=cuda_device, generator=gen) / 23 ** 0.5
        out = raw_forward(plan, x, y, gates, None)
        sample = torch.randint(0, rows, (256,), device=cuda_device, generator=gen)
        sample[0], sample[-1] = 0, rows - 1
        xs, ys, gs = (t[sample].double().cpu() for t in (x, y, gates))
        xs_mul = ir_mul_to_mul_ir(xs, C, range(L + 1))
        ref = tp_oracle.pack_out(owner, tp_oracle.tp_forward(owner, tp_oracle.split_mul_ir(xs_mul, C, L),
                                                             tp_oracle.split_harm(ys, L), gs.view(-1, 23, C),
                                                             dtype=torch.float64))
        got = ir_mul_to_mul_ir(out[sample].double().cpu(), C, output_degrees(owner))
        assert_close(got, ref, FWD_TOL, 1e-3, f"sampled forward {rows}")
        if backward:
            G = torch.randn_like(out)
            dx, dy, dg = raw_backward(plan, x, y, gates, None, G, (True, True, True))
            Gs = ir_mul_to_mul_ir(G[sample].double().cpu(), C, output_degrees(owner))
            xr, yr, gr = (t.clone().requires_grad_(True) for t in (xs_mul, ys, gs))
            ref = tp_oracle.pack_out(owner, tp_oracle.tp_forward(owner, tp_oracle.split_mul_ir(xr, C, L),
                                                                 tp_oracle.split_harm(yr, L), gr.view(-1, 23, C),
                                                                 dtype=torch.float64))
            rdx, rdy, rdg = torch.autograd.grad((ref * Gs).sum(), [xr, yr, gr])
            assert_close(ir_mul_to_mul_ir(dx[sample].double().cpu(), C, range(L + 1)), rdx, GRAD_TOL, 1e-3, "dx")
            assert_close(dy[sample].cpu(), rdy, GRAD_TOL, 1e-3, "dY")
            assert_close(dg[sample].cpu(), rdg, GRAD_TOL, 1e-3, "dg")
        del x, y, gates, out
        torch.cuda.empty_cache()
