"""MACE-ICTC energy/forces on the CUDA backend vs the same model on the CPU oracle (FP64)."""
import math

import pytest
import torch

from _util import assert_close

pytestmark = pytest.mark.gpu


def random_system(n_atoms, density=0.1, min_dist=0.9, seed=0):
    """Uniform random positions in a periodic cube with a minimum pair distance (configs 3-5 recipe)."""
    gen = torch.Generator().manual_seed(seed)
    side = (n_atoms / density) ** (1.0 / 3.0)
    pos = []
    while len(pos) < n_atoms:
        cand = torch.rand(3, generator=gen, dtype=torch.float64) * side
        ok = True
        for p in pos:
            d = cand - p
            d = d - side * torch.round(d / side)
            if float(d.norm()) < min_dist:
                ok = False
                break
        if ok:
            pos.append(cand)
    species = torch.randint(0, 3, (n_atoms,), generator=gen)
    return torch.stack(pos), species, side


def brute_neighbors(pos, side, cutoff):
    """All (src=j, dst=i) pairs with a minimum-image distance below the cutoff, and the
    shift vectors making pos[dst] - pos[src] + shift the minimum image."""
    d = pos[None, :, :] - pos[:, None, :]            # d[i, j] = pos[j] - pos[i]
    shift_img = -side * torch.round(d / side)
    dist = (d + shift_img).norm(dim=-1)
    i, j = torch.nonzero((dist < cutoff) & (dist > 0), as_tuple=True)
    src, dst = j, i
    vec_raw = pos[dst] - pos[src]
    shift = -side * torch.round(vec_raw / side)
    return src, dst, shift


def build_models(channels=32, lmax=2, seed=3):
    from mace_ictc.models import MACEICTC
    from oracle.model_ops import OracleOps
    torch.manual_seed(seed)
    cuda_model = MACEICTC(channels=channels, lmax=lmax, avg_num_neighbors=10.0)
    oracle_model = MACEICTC(channels=channels, lmax=lmax, avg_num_neighbors=10.0, ops=OracleOps())
    oracle_model.load_state_dict(cuda_model.state_dict())
    return cuda_model, oracle_model.double()


@pytest.mark.parametrize("lmax", [2, 3])
def test_energy_and_forces_match_oracle(lmax, cuda_device):
    pos, species, side = random_system(40, seed=lmax)
    src, dst, shift = brute_neighbors(pos, side, 5.0)
    cuda_model, oracle_model = build_models(lmax=lmax)
    cuda_model = cuda_model.to(cuda_device)
    e, f = cuda_model.energy_and_forces(pos.float().to(cuda_device), species.to(cuda_device), src.to(cuda_device),
                                        dst.to(cuda_device), shift.float().to(cuda_device))
    re, rf = oracle_model.energy_and_forces(pos, species, src, dst, shift)
    assert_close(e.detach().cpu(), re.detach(), 1e-5, None, "energy")
    assert_close(f.detach().cpu(), rf.detach(), 1e-4, 1e-3, "forces")


def test_forces_are_rotation_covariant_and_match_finite_differences(cuda_device):
    pos, species, side = random_system(30, seed=7)
    src, dst, shift = brute_neighbors(pos, side, 5.0)
    model, _ = build_models()
    model = model.to(cuda_device)
    # Rotate the unwrapped edge geometry: rotate positions and shift vectors together.
    angle = 0.7
    axis = torch.tensor([1.0, 2.0, 2.0], dtype=torch.float64) / 3.0
    K = torch.tensor([[0, -axis[2], axis[1]], [axis[2], 0, -axis[0]], [-axis[1], axis[0], 0]], dtype=torch.float64)
    R = torch.eye(3, dtype=torch.float64) + math.sin(angle) * K + (1 - math.cos(angle)) * K @ K
    dev = cuda_device
    args = (species.to(dev), src.to(dev), dst.to(dev))
    e0, f0 = model.energy_and_forces(pos.float().to(dev), *args, shift.float().to(dev))
    e1, f1 = model.energy_and_forces((pos @ R.T).float().to(dev), *args, (shift @ R.T).float().to(dev))
    assert abs(float(e0) - float(e1)) <= 1e-5 * max(1.0, abs(float(e0)))
    assert_close(f1.detach().cpu().double(), (f0.detach().cpu().double() @ R.T), 1e-4, None, "rotated forces")
    # Central differences of the FP64 oracle model pin the oracle forces themselves.
    _, oracle = build_models()
    p = pos.clone()
    _, fo = oracle.energy_and_forces(p, species, src, dst, shift)
    h = 1e-5
    for atom, axis_i in ((0, 0), (5, 1), (11, 2)):
        dp = torch.zeros_like(p)
        dp[atom, axis_i] = h
        ep = oracle.energy(p + dp, species, src, dst, shift)
        em = oracle.energy(p - dp, species, src, dst, shift)
        fd = -(ep - em) / (2 * h)
        assert abs(float(fd) - float(fo[atom, axis_i])) <= 1e-6 * max(1.0, abs(float(fd)))


@pytest.mark.parametrize("lmax", [2, 3])
def test_force_loss_training_gradients_match_oracle(lmax, cuda_device):
    """Force-loss training: d(loss)/d(weights) needs the mixed second
    derivatives of every operator (TP message, harmonics, symmetric contraction)."""
    pos, species, side = random_system(28, seed=20 + lmax)
    src, dst, shift = brute_neighbors(pos, side, 5.0)
    cuda_model, oracle_model = build_models(channels=16, lmax=lmax, seed=9)
    cuda_model = cuda_model.to(cuda_device)
    gen = torch.Generator().manual_seed(5)
    e_target = torch.randn(1, generator=gen, dtype=torch.float64)
    f_target = torch.randn(pos.shape[0], 3, generator=gen, dtype=torch.float64)

    def loss_of(model, p, sp, s, d, sh, et, ft):
        p = p.detach().requires_grad_(True)
        energy = model.energy(p, sp, s, d, sh)
        (grad,) = torch.autograd.grad(energy.sum(), [p], create_graph=True)
        return ((energy - et) ** 2).mean() + 100.0 * ((-grad - ft) ** 2).mean()

    dev = cuda_device
    loss = loss_of(cuda_model, pos.float().to(dev), species.to(dev), src.to(dev), dst.to(dev),
                   shift.float().to(dev), e_target.float().to(dev), f_target.float().to(dev))
    names = [n for n, p in cuda_model.named_parameters() if p.requires_grad]
    got = torch.autograd.grad(loss, [dict(cuda_model.named_parameters())[n] for n in names], allow_unused=True)
    ref_loss = loss_of(oracle_model, pos, species, src, dst, shift, e_target, f_target)
    want = torch.autograd.grad(ref_loss, [dict(oracle_model.named_parameters())[n] for n in names],
                               allow_unused=True)
    assert_close(loss.detach().cpu(), ref_loss.detach(), 1e-4, None, "loss")
    for name, a, b in zip(names, got, want):
        if b is None:
            assert a is None or float(a.abs().max()) == 0.0, name
            continue
        assert a is not None, name
        assert_close(a.cpu(), b, 1e-4, None, f"d loss / d {name}")


def test_model_copies_after_running(cuda_device):
    """A model that has run (device plans, packed radial weights, folded tables cached on
    it) deep-copies and saves whole; the copies rebuild their own state and give the
    same energies and forces."""
    import copy
    import io
    pos, species, side = random_system(30, seed=11)
    src, dst, shift = brute_neighbors(pos, side, 5.0)
    args = [t.to(cuda_device) for t in (pos.float(), species, src, dst, shift.float())]
    model, _ = build_models(lmax=2)
    model = model.to(cuda_device)
    e, f = model.energy_and_forces(*args)
    twin = copy.deepcopy(model)
    buf = io.BytesIO()
    torch.save(model, buf)
    buf.seek(0)
    loaded = torch.load(buf, weights_only=False)
    for other in (twin, loaded):
        e2, f2 = other.energy_and_forces(*args)
        assert_close(e2.detach().cpu(), e.detach().cpu(), 1e-6, None, "energy of the copy")
        assert_close(f2.detach().cpu(), f.detach().cpu(), 1e-6, None, "forces of the copy")
