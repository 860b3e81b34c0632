"""Generate model-level golden fixtures from the reference's own MACE-ICTC model.

Run in a container that has the reference source tree (it is not needed at test
time; the fixtures are committed):

    python tests/golden/make_model_golden.py <reference root>

For each case a small ``PureCartesianICTDFix`` (``mace_ictc/models/pure_cartesian_ictd_fix.py:2058``)
is built by the reference's factory (``mace_ictc/models/factory.py:8``) with the
``ictd-pure-u`` product backend, the factory's defaults for new models
(first-layer self-connection, ``radial_sqrt_num_basis=False``, Bessel radial basis,
polynomial cutoff p = 5) and random weights in FP64, then run by its own forward
on a small periodic system.  The fixture records the model's parameters under the
reference's state-dict names, the system (positions, atomic numbers, edges with
Cartesian and lattice shifts, cell), the per-atom energies and the forces
(-dE/dpos by autograd through the reference).

The reference imports e3nn and opt_einsum_fx, which are not installed here.  This
script registers stand-in modules before importing it:
* ``opt_einsum_fx.optimize_einsums_full(model, example_inputs)`` returns ``model``
  unchanged (that function only reorders the contractions of an einsum graph);
* ``e3nn.o3.Irrep`` / ``Irreps`` parse irreps strings such as ``"8x0e+8x1o"``;
* ``e3nn.o3.Linear`` between equal irreps, the one e3nn operation this model
  executes: for each matching irrep a weight block [mul_in, mul_out] read from one
  flat parameter in irrep order, scaled by 1/sqrt(sum of the feeding mul_in)
  (e3nn's documented path normalisation);
* every other e3nn entry point the import touches raises when called.
So the fixtures pin everything on this path against the reference code itself,
and the product block's linear against the stated o3.Linear semantics.

The bridge-U case (``ictd-bridge-u``, the reference's default product backend) also
runs the reference's e3nn-basis construction: its MACE coupling recursion
(``ictc_o3/basis/_mace_cg.py:41-175``), the basis-bridge fit and the fold of the
bridge into the U tensors (``ictc_o3/ops/symmetric_contraction.py:24-180``).  For
it, ``o3.spherical_harmonics`` and ``o3.wigner_3j`` are stand-ins expressed in a
seeded random orthonormal basis per degree (the ICTC harmonics rotated by it, and
the ICTC couplings rotated the same way, unit Frobenius norm, each with a random
sign): a real basis with its own conventions, as e3nn's is.  The bridge-U couplings
the reference derives from them are stored with the parameters, as in its
checkpoints; the model here must load them through an exact change of coupling
basis whatever those conventions are.

Two contraction cases (``sc_bridge_*.npz``) hold the reference's bridge-U module on
its own, built the same way: its complete state dict (folded couplings, basis
bridge, weights, zero flags), random flat ICTC features with species, and its
outputs through the element-selected and the one-hot forward routes.
"""
import math
import os
import re
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def install_import_stand_ins():
    e3nn = types.ModuleType("e3nn")
    o3 = types.ModuleType("e3nn.o3")
    emath = types.ModuleType("e3nn.math")
    util = types.ModuleType("e3nn.util")
    codegen = types.ModuleType("e3nn.util.codegen")
    jit = types.ModuleType("e3nn.util.jit")

    class Irrep(tuple):
        def __new__(cls, l, p=None):
            if isinstance(l, Irrep):
                return l
            if isinstance(l, str):
                m = re.fullmatch(r"\s*(\d+)([eo])\s*", l)
                l, p = int(m[1]), (1 if m[2] == "e" else -1)
            elif isinstance(l, tuple):
                l, p = l
            return super().__new__(cls, (int(l), int(p)))

        l = property(lambda s: s[0])
        p = property(lambda s: s[1])
        dim = property(lambda s: 2 * s[0] + 1)

        def __repr__(self):
            return f"{self.l}{'e' if self.p == 1 else 'o'}"

    class MulIr(tuple):
        mul = property(lambda s: s[0])
        ir = property(lambda s: s[1])
        dim = property(lambda s: s[0] * s[1].dim)

    class Irreps(tuple):
        def __new__(cls, irreps=None):
            if isinstance(irreps, Irreps):
                return irreps
            items = []
            if isinstance(irreps, str):
                for part in irreps.split("+"):
                    part = part.strip()
                    if part:
                        m = re.fullmatch(r"(?:(\d+)x)?(\d+[eo])", part)
                        items.append(MulIr((int(m[1] or 1), Irrep(m[2]))))
            elif irreps is not None:
                for item in irreps:
                    if isinstance(item, (Irrep, str)):
                        items.append(MulIr((1, Irrep(item))))
                    else:
                        mul, ir = item
                        items.append(MulIr((int(mul), Irrep(ir))))
            return super().__new__(cls, items)

        dim = property(lambda s: sum(x.dim for x in s))
        num_irreps = property(lambda s: sum(x.mul for x in s))
        lmax = property(lambda s: max(x.ir.l for x in s))

        @staticmethod
        def spherical_harmonics(lmax, p=-1):
            return Irreps([(1, (l, p ** l)) for l in range(lmax + 1)])

        def __repr__(self):
            return "+".join(f"{x.mul}x{x.ir!r}" for x in self)

    class Linear(torch.nn.Module):
        def __init__(self, irreps_in, irreps_out, **_):
            super().__init__()
            self.irreps_in, self.irreps_out = Irreps(irreps_in), Irreps(irreps_out)
            self.blocks, n = [], 0
            for o, (mul_o, ir_o) in enumerate(self.irreps_out):
                feeding = [(i, mul_i) for i, (mul_i, ir_i) in enumerate(self.irreps_in) if ir_i == ir_o]
                fan_in = sum(mul_i for _, mul_i in feeding)
                for i, mul_i in feeding:
                    self.blocks.append((i, o, mul_i, mul_o, n, fan_in))
                    n += mul_i * mul_o
            self.weight = torch.nn.Parameter(torch.randn(n))

        def forward(self, x):
            lead = x.shape[:-1]
            parts, off = [], 0
            for mul, ir in self.irreps_in:
                parts.append(x[..., off:off + mul * ir.dim].reshape(*lead, mul, ir.dim))
                off += mul * ir.dim
            outs = [x.new_zeros(*lead, mul, ir.dim) for mul, ir in self.irreps_out]
            for i, o, mul_i, mul_o, n0, fan_in in self.blocks:
                w = self.weight[n0:n0 + mul_i * mul_o].reshape(mul_i, mul_o)
                outs[o] = outs[o] + torch.einsum("...um,uv->...vm", parts[i], w) / math.sqrt(fan_in)
            return torch.cat([t.reshape(*lead, -1) for t in outs], -1)

    def unavailable(name):
        def call(*_, **__):
            raise RuntimeError(f"e3nn.{name} is not available where these fixtures are generated")
        return call

    o3.Irrep, o3.Irreps, o3.Linear = Irrep, Irreps, Linear
    for name in ("TensorProduct", "wigner_3j", "spherical_harmonics", "FullyConnectedTensorProduct", "Norm"):
        setattr(o3, name, unavailable("o3." + name))
    emath.soft_one_hot_linspace = unavailable("math.soft_one_hot_linspace")
    codegen.CodeGenMixin = type("CodeGenMixin", (), {})
    jit.compile_mode = lambda mode: (lambda cls: cls)
    e3nn.o3, e3nn.math, e3nn.util = o3, emath, util
    util.codegen, util.jit = codegen, jit
    e3nn.get_optimization_defaults = lambda: {}
    e3nn.set_optimization_defaults = lambda **_: None
    for name, mod in (("e3nn", e3nn), ("e3nn.o3", o3), ("e3nn.math", emath), ("e3nn.util", util),
                      ("e3nn.util.codegen", codegen), ("e3nn.util.jit", jit)):
        sys.modules[name] = mod
    einsum_fx = types.ModuleType("opt_einsum_fx")
    einsum_fx.optimize_einsums_full = lambda model, example_inputs=None, **_: model
    sys.modules["opt_einsum_fx"] = einsum_fx


def install_basis_stand_ins(seed):
    """e3nn primitives of the bridge-U construction in a seeded random real basis."""
    from ictc_o3.basis import ictd_irreps
    o3 = sys.modules["e3nn.o3"]
    gen = torch.Generator().manual_seed(seed)
    rot = {l: torch.linalg.qr(torch.randn(2 * l + 1, 2 * l + 1, generator=gen, dtype=torch.float64))[0]
           for l in range(8)}
    signs = {}

    def spherical_harmonics(irreps, x, normalize=True, normalization="component"):
        irreps = o3.Irreps(irreps)
        ys = ictd_irreps.direction_harmonics_all(x / x.norm(dim=-1, keepdim=True), irreps.lmax)
        return torch.cat([ys[mul_ir.ir.l].to(torch.float64) @ rot[mul_ir.ir.l] for mul_ir in irreps], -1)

    def wigner_3j(l1, l2, l3, dtype=None, **_):
        c = torch.as_tensor(ictd_irreps.build_full_cg_tensor_so3(l2, l3, l1)).permute(2, 0, 1)
        c = torch.einsum("oab,oi,aj,bk->ijk", c, rot[l1], rot[l2], rot[l3])
        if (l1, l2, l3) not in signs:
            signs[(l1, l2, l3)] = 1.0 if torch.rand(1, generator=gen).item() < 0.5 else -1.0
        return (signs[(l1, l2, l3)] * c / c.norm()).to(dtype or torch.get_default_dtype())

    o3.spherical_harmonics, o3.wigner_3j = spherical_harmonics, wigner_3j


def periodic_system(n, side, cutoff, seed):
    """Random atoms in a cube with a minimum distance of 0.9 A and the minimum-image
    edges within the cutoff: r_e = pos[dst] - pos[src] + shift_e."""
    gen = torch.Generator().manual_seed(seed)
    pos = torch.empty(0, 3, dtype=torch.float64)
    while pos.shape[0] < n:
        cand = torch.rand(1, 3, generator=gen, dtype=torch.float64) * side
        d = pos - cand
        d = d - side * torch.round(d / side)
        if pos.shape[0] == 0 or float(d.norm(dim=1).min()) >= 0.9:
            pos = torch.cat([pos, cand])
    numbers = torch.tensor([1, 6, 8])[torch.randint(0, 3, (n,), generator=gen)]
    d = pos[:, None, :] - pos[None, :, :]
    shift = -side * torch.round(d / side)
    dist = (d + shift).norm(dim=-1)
    i, j = torch.nonzero((dist < cutoff) & (dist > 0), as_tuple=True)
    return pos, numbers, j, i, shift[i, j]


def model_case(name, channels, lmax, n_atoms, side, cutoff, seed, product_backend="ictd-pure-u"):
    from mace_ictc.models.factory import build_baseline_model
    from mace_ictc.utils.config import ModelConfig
    torch.manual_seed(seed)
    dtype = torch.float64
    avg = 5.0
    cfg = ModelConfig(dtype=dtype, internal_compute_dtype=dtype, channel_in=channels,
                      irreps_output_conv_channels=channels, lmax=lmax, max_radius=cutoff, max_radius_main=cutoff,
                      function_type="bessel")
    model = build_baseline_model(cfg, avg_num_neighbors=avg, num_interaction=2, route="baseline",
                                 product_backend=product_backend, correlation=3, use_reduced_cg=False,
                                 freeze_conv_tp_weight=True, radial_sqrt_num_basis=False, edge_lmax=lmax,
                                 attn_heads=0, atomic_numbers=[1, 6, 8], ictd_save_tp_mode="fully-connected",
                                 invariant_channels=32, device=torch.device("cpu"), dtype=dtype)
    with torch.no_grad():                                    # non-trivial values everywhere
        for key, param in model.named_parameters():
            param.copy_(torch.randn(param.shape, dtype=dtype) / math.sqrt(max(param.shape[-1], 1)))
    pos, numbers, src, dst, shift = periodic_system(n_atoms, side, cutoff, seed + 1)
    cell = (torch.eye(3, dtype=dtype) * side).unsqueeze(0)
    p = pos.clone().requires_grad_(True)
    out = model(p, numbers, torch.zeros(n_atoms, dtype=torch.long), src, dst, shift / side, cell)
    atomic = (out[0] if isinstance(out, tuple) else out).reshape(n_atoms)
    (grad,) = torch.autograd.grad(atomic.sum(), [p])
    record = {"channels": channels, "lmax": lmax, "cutoff": cutoff, "side": side, "avg_num_neighbors": avg,
              "pos": pos.numpy(), "numbers": numbers.numpy(), "src": src.numpy(), "dst": dst.numpy(),
              "shift": shift.numpy(), "atomic_energy": atomic.detach().numpy(), "forces": -grad.numpy()}
    for key, param in model.named_parameters():
        record["param:" + key] = param.detach().numpy()
    if product_backend == "ictd-bridge-u":          # its checkpoints carry the folded couplings
        params = dict(model.named_parameters())
        for key, value in model.state_dict().items():
            if key not in params and ".symmetric_contractions." in key and value is not None:
                record["buffer:" + key] = value.detach().numpy()
    record["product_backend"] = product_backend
    np.savez_compressed(os.path.join(HERE, name), **record)
    print(name, "energy", float(atomic.sum()), "edges", src.numel(), "params", len(list(model.parameters())))


def contraction_case(name, channels, lmax, target_lmax, nodes, seed):
    """The reference's bridge-U module alone (``ICTDBridgeUSymmetricContractionSO3``,
    ``ictc_o3/ops/symmetric_contraction.py:92-206``): its whole state dict, random
    flat ICTC features and species, and its outputs through both forward routes
    (element-selected weights and one-hot attributes)."""
    from ictc_o3.ops.symmetric_contraction import ICTDBridgeUSymmetricContractionSO3
    torch.manual_seed(seed)
    dtype = torch.float64
    torch.set_default_dtype(dtype)
    try:
        module = ICTDBridgeUSymmetricContractionSO3(num_elements=3, channels=channels, lmax=lmax,
                                                    target_lmax=target_lmax, correlation=3)
    finally:
        torch.set_default_dtype(torch.float32)
    module = module.to(dtype)
    with torch.no_grad():
        for param in module.parameters():
            param.copy_(torch.randn(param.shape, dtype=dtype) / math.sqrt(param.shape[-2]))
    x = 0.7 * torch.randn(nodes, channels * (lmax + 1) ** 2, dtype=dtype)
    species = torch.randint(0, 3, (nodes,))
    attrs = torch.nn.functional.one_hot(species, 3).to(dtype)
    with torch.no_grad():
        selected = module(x, attrs, species)
        one_hot = module(x, attrs)
    record = {"channels": channels, "lmax": lmax, "target_lmax": target_lmax, "x": x.numpy(),
              "species": species.numpy(), "out": selected.numpy(), "out_one_hot": one_hot.numpy()}
    for key, value in module.state_dict().items():
        record["state:" + key] = value.detach().numpy()
    np.savez_compressed(os.path.join(HERE, name), **record)
    print(name, "out norm", float(selected.norm()), "state keys", len(module.state_dict()))


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ICTC_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_model_golden.py <reference root>")
    os.environ.setdefault("FSCETP_ICTD_CACHE", "0")
    install_import_stand_ins()
    sys.path.insert(0, root)
    model_case("model_c8_l2.npz", channels=8, lmax=2, n_atoms=40, side=8.0, cutoff=3.0, seed=11)
    model_case("model_c8_l3.npz", channels=8, lmax=3, n_atoms=36, side=8.0, cutoff=3.0, seed=21)
    o3 = sys.modules["e3nn.o3"]
    # Irrep products, membership and counts, used by the MACE coupling recursion
    o3.Irrep.__mul__ = lambda a, b: [o3.Irrep(l, a.p * o3.Irrep(b).p)
                                     for l in range(abs(a.l - o3.Irrep(b).l), a.l + o3.Irrep(b).l + 1)]
    o3.Irreps.__contains__ = lambda irreps, ir: o3.Irrep(ir) in [x.ir for x in irreps]
    o3.Irreps.count = lambda irreps, ir: sum(x.mul for x in irreps if x.ir == o3.Irrep(ir))
    install_basis_stand_ins(seed=7)
    model_case("model_c8_l2_bridge.npz", channels=8, lmax=2, n_atoms=40, side=8.0, cutoff=3.0, seed=31,
               product_backend="ictd-bridge-u")
    contraction_case("sc_bridge_c8_l2_t2.npz", channels=8, lmax=2, target_lmax=2, nodes=37, seed=41)
    contraction_case("sc_bridge_c4_l3_t1.npz", channels=4, lmax=3, target_lmax=1, nodes=29, seed=43)


if __name__ == "__main__":
    main()
