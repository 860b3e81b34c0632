#!/usr/bin/env python
"""Benchmark of the ICTC-O3 hot path on B200: the C128/lmax-3 channelwise tensor product.

Workload (benchmark configs[1]): FP32 path-preserving TP, C=128, lmax 3 (23 paths),
262,144 instances per forward step; forward+VJP (grads of features, harmonics and
per-instance path weights) at 131,072 instances per step.  Inputs are seeded
synthetic tensors with the config's distributions: features N(0,1), harmonics of
uniform random unit vectors, path weights N(0, 1/sqrt(23)), upstream grad N(0,1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun): instances are independent, so every rank runs its own full
batch with no collective on the data path (weak scaling); the timed region is
bracketed by barriers and the reported time is the max over ranks.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PACKAGE_ROOT = os.path.join(REPO, "ictc-o3-hp-ascend_b200")
for _path in (PACKAGE_ROOT, REPO):
    if _path not in sys.path:
        sys.path.insert(0, _path)

import torch  # noqa: E402

C, L, PATHS = 128, 3, 23
FWD_ROWS, VJP_ROWS = 262144, 131072
FEATURE_W, HARM_W, GATE_W, OUT_W = C * 16, 16, PATHS * C, 12672
# Algorithmic bytes per instance: each tensor read or written once per pass.
FWD_BYTES = 4 * (FEATURE_W + HARM_W + GATE_W + OUT_W)                       # 70,720
BWD_BYTES = 4 * (FEATURE_W + HARM_W + GATE_W + OUT_W) + 4 * (FEATURE_W + HARM_W + GATE_W)
VJP_BYTES = FWD_BYTES + BWD_BYTES                                           # 161,472
PUBLISHED_FWD = 2.70e6  # reference, Ascend 910B3, docs/PERFORMANCE.md:19-20
METRIC = "TP instances/s fwd & fwd+VJP; MACE E+F atom-steps/s at 1/2/4/8 B200"
WORKLOAD = "ictc_o3 channelwise TP C128/lmax3 FP32 forward, 262,144 instances/step (configs[1])"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--profile", action="store_true",
                   help="kernel timing only (forward, then forward+VJP) for ncu captures: no e2e, no CPU baseline")
    p.add_argument("--rows", type=int, default=0, help="instances per step in --profile mode (0 = config sizes)")
    p.add_argument("--profile-block", action="store_true",
                   help="time only the configs[2] MACE block step (for ncu launch lists)")
    p.add_argument("--atoms", type=int, default=0,
                   help="atoms of the --profile-block (default 16,384) or --profile-md (default 262,144) system")
    p.add_argument("--profile-md", action="store_true",
                   help="time only the configs[4] MD step (torchrun for several GPUs)")
    p.add_argument("--phases", action="store_true",
                   help="with --profile-md: per-phase CUDA-event breakdown of the step (max over ranks)")
    p.add_argument("--profile-train", action="store_true", help="time only the configs[3] training step")
    p.add_argument("--profile-radial", action="store_true",
                   help="time only the fused radial MLP kernels (forward, backward) at --rows edges, --gates columns")
    p.add_argument("--gates", type=int, default=704, help="gate columns of --profile-radial (11 paths x C64)")
    return p.parse_args()


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------

def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(value, world, device):
    if world == 1:
        return value
    t = torch.tensor([value], device=device, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    QUERY = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device):
        self.proc = None
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", uuid, f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, AttributeError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        for line in out.strip().splitlines():
            parts = [v.strip() for v in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(self.NAMES, parts[3:7]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        loaded = [v for v in sm if smax and v > 0.5 * max(smax)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# Inputs
# ---------------------------------------------------------------------------

def make_inputs(rows, device, seed, requires_grad=False):
    from ictc_o3.operators import direction_harmonics
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(rows, FEATURE_W, device=device, generator=gen)
    n = torch.nn.functional.normalize(torch.randn(rows, 3, device=device, generator=gen), dim=1)
    y = torch.cat(direction_harmonics(n, L), -1).contiguous()
    g = torch.randn(rows, GATE_W, device=device, generator=gen) / PATHS ** 0.5
    if requires_grad:
        x.requires_grad_(True), y.requires_grad_(True), g.requires_grad_(True)
    return x, y, g


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        data = json.load(open(path))
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic(name):
    """Per-instance DRAM bytes from a committed ncu summary (profiles/<name>), or None."""
    path = os.path.join(REPO, "profiles", name)
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("dram_bytes_per_instance:"):
            return float(line.split(":", 1)[1])
    return None


def vjp_traffic():
    """DRAM bytes per instance of one forward + one fused adjoint launch (committed ncu
    summaries of the two kernels), or None."""
    fwd, adj = profiled_traffic("tp_forward_c128_l3.txt"), profiled_traffic("tp_adjoint_c128_l3.txt")
    return None if fwd is None or adj is None else fwd + adj


def roofline(bytes_per_inst, rows, kernel_ms, traffic_per_inst):
    peak, kind = peaks()
    achieved = bytes_per_inst * rows / (kernel_ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_kind": kind,
            "traffic": None if traffic_per_inst is None else round(traffic_per_inst * rows),
            "algorithmic_bytes": bytes_per_inst * rows}


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------

def time_loop(fn, steps, warmup, world, device):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    barrier(world)
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize(device)
    barrier(world)
    return start.elapsed_time(end)


def e2e_forward(op, rows, steps, warmup, device, world):
    """Public API with host buffers: pinned H2D of inputs, forward, D2H of the output,
    pipelined in chunks over three streams (copy-in, compute, copy-out)."""
    chunk = 16384
    gen = torch.Generator().manual_seed(7)
    xh = torch.randn(rows, FEATURE_W, generator=gen).pin_memory()
    nh = torch.nn.functional.normalize(torch.randn(rows, 3, generator=gen), dim=1)
    from ictc_o3.operators import direction_harmonics
    yh = torch.cat(direction_harmonics(nh.to(device), L), -1).cpu().pin_memory()
    gh = (torch.randn(rows, GATE_W, generator=gen) / PATHS ** 0.5).pin_memory()
    oh = torch.empty(rows, OUT_W).pin_memory()
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)
    nbuf = 3
    bufs = [(torch.empty(chunk, FEATURE_W, device=device), torch.empty(chunk, HARM_W, device=device),
             torch.empty(chunk, GATE_W, device=device)) for _ in range(nbuf)]
    done_compute = [torch.cuda.Event() for _ in range(nbuf)]
    done_in = [torch.cuda.Event() for _ in range(nbuf)]

    def step():
        for i, begin in enumerate(range(0, rows, chunk)):
            b = i % nbuf
            end = min(begin + chunk, rows)
            n = end - begin
            xd, yd, gd = bufs[b]
            with torch.cuda.stream(s_in):
                s_in.wait_event(done_compute[b])
                xd[:n].copy_(xh[begin:end], non_blocking=True)
                yd[:n].copy_(yh[begin:end], non_blocking=True)
                gd[:n].copy_(gh[begin:end], non_blocking=True)
                done_in[b].record(s_in)
            compute.wait_event(done_in[b])
            out = op(xd[:n], yd[:n], gd[:n])
            out.record_stream(s_out)
            done_compute[b].record(compute)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done_compute[b])
                oh[begin:end].copy_(out, non_blocking=True)
        compute.wait_stream(s_out)

    ms = time_loop(step, steps, warmup, world, device) / steps
    h2d = rows * 4 * (FEATURE_W + HARM_W + GATE_W)
    d2h = rows * 4 * OUT_W
    check = float(oh[rows - 1, :8].abs().sum())  # the result is read on the host
    del check
    return ms, h2d, d2h


def mace_block(device, steps, warmup, atoms=16384, cpu_seconds=0.0):
    """one non-first MACE interaction block (input lmax 2) and its product
    block, C64/lmax2, correlation 3, 16,384 H/C/O atoms at 0.1/A^3 (5 A cutoff), forward plus
    the force gradient.  Returns the JSON sub-object."""
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    from mace_ictc.models import CudaOps, InteractionBlock, ProductBlock, radial_embedding, species_groups
    from mace_ictc.systems import random_system
    pos, species, side = random_system(atoms, seed=31, device=device)
    src, dst, shift, _ = neighbor_list(pos, (side,) * 3, 5.0)
    edges = src.numel()
    torch.manual_seed(0)
    C, L = 64, 2
    inter = InteractionBlock(channels=C, lmax=L, input_lmax=L, num_elements=3, num_basis=8,
                             avg_num_neighbors=edges / atoms, use_self_connection=True, sc_lmax=L).to(device)
    prod = ProductBlock(channels=C, lmax=L, target_lmax=L, correlation=3, num_elements=3).to(device)
    readout = torch.nn.Linear(C, 1, bias=False).to(device)
    h = torch.randn(atoms, C * (L + 1) ** 2, device=device)
    groups = species_groups(species, 3)
    ops = CudaOps()

    def step():
        p = pos.detach().requires_grad_(True)
        vec = p[dst] - p[src] + shift
        r = vec.norm(dim=1)
        harm = ops.harmonics(vec / r.unsqueeze(-1), L)
        feats = radial_embedding(r, 5.0, 8, 5)
        message, sc = inter(ops, h, harm, feats, src, dst, None, groups, None, species)
        out = prod(ops, message, sc, species)
        energy = readout(out[:, :C]).sum()
        return torch.autograd.grad(energy, [p])[0]

    ms = time_loop(step, steps, warmup, 1, device) / steps
    result = {"value": round(atoms / (ms * 1e-3), 1), "unit": "atom-steps/s", "ms_per_step": round(ms, 3),
              "atoms": atoms, "edges": edges, "neighbours_per_atom": round(edges / atoms, 2),
              "workload": "configs[2]: one MACE interaction block (input lmax 2) + product, C64/lmax2, corr 3, "
                          "forward + force gradient (positions)",
              "gpu_launches_per_step": 6}
    if cpu_seconds > 0:
        result["cpu_baseline"] = mace_block_cpu(cpu_seconds)
    return result


def _cpu_system(atoms, seed, cutoff=5.0):
    """Uniform random periodic system at 0.1 / A^3 with a brute-force minimum-image
    neighbour list (host CPU; needs a box side above twice the cutoff)."""
    gen = torch.Generator().manual_seed(seed)
    side = (atoms / 0.1) ** (1 / 3)
    pos = torch.rand(atoms, 3, generator=gen) * side
    species = torch.randint(0, 3, (atoms,), generator=gen)
    d = pos[None] - pos[:, None]
    s = -side * torch.round(d / side)
    dist = (d + s).norm(dim=-1)
    i, j = torch.nonzero((dist < cutoff) & (dist > 0), as_tuple=True)
    return pos, species, side, j, i, s[i, j]


def mace_md_cpu(seconds, atoms=512):
    """configs[4] step (E, F, virial of the C64/lmax2 model) on the oracle ops, torch CPU
    FP32 with all host threads, on a small system: the port's CPU speed."""
    from mace_ictc.models import MACEICTC
    from mace_ictc.parallel import distributed_energy_forces, halo_layout, partition
    from oracle.model_ops import OracleOps
    torch.set_num_threads(os.cpu_count() or 1)
    pos, species, side, src, dst, shift = _cpu_system(atoms, 9)
    torch.manual_seed(0)
    model = MACEICTC(channels=64, lmax=2, num_interactions=2, correlation=3, r_max=5.0, avg_num_neighbors=52.0,
                     ops=OracleOps(torch.float32))
    layout, p, sp = halo_layout(partition(pos, species, side, 0, 1, 5.0))
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or done == 0:
        distributed_energy_forces(model, layout, p, sp, src, dst, shift)
        done += atoms
    elapsed = time.perf_counter() - t0
    return {"value": round(done / elapsed, 1), "unit": "atom-steps/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{done} atom-steps of a {atoms}-atom system, E+F+virial of the same model "
                                      f"on the oracle ops (torch CPU FP32), {elapsed:.1f} s"}


def mace_train_cpu(seconds, atoms=128):
    """configs[3] training step (C128/lmax3, force loss, Adam) on the oracle ops, torch CPU
    FP32 with all host threads, on one small configuration: the port's CPU speed."""
    from mace_ictc.models import MACEICTC
    from oracle.model_ops import OracleOps
    torch.set_num_threads(os.cpu_count() or 1)
    pos, species, side, src, dst, shift = _cpu_system(atoms, 12)
    torch.manual_seed(0)
    model = MACEICTC(channels=128, lmax=3, num_interactions=2, correlation=3, r_max=5.0,
                     avg_num_neighbors=src.numel() / atoms, ops=OracleOps(torch.float32))
    opt = torch.optim.Adam([p for p in model.parameters() if p.requires_grad], lr=1e-3)
    gen = torch.Generator().manual_seed(77)
    e_target, f_target = torch.randn(1, generator=gen), torch.randn(atoms, 3, generator=gen)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or done == 0:
        opt.zero_grad(set_to_none=True)
        p = pos.detach().requires_grad_(True)
        energy = model.energy(p, species, src, dst, shift)
        (grad,) = torch.autograd.grad(energy.sum(), [p], create_graph=True)
        loss = ((energy / atoms - e_target) ** 2).mean() + 100.0 * ((-grad - f_target) ** 2).mean()
        loss.backward()
        opt.step()
        done += atoms
    elapsed = time.perf_counter() - t0
    return {"value": round(done / elapsed, 1), "unit": "atom-steps/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{done} atom-steps of training on one {atoms}-atom configuration with the "
                                      f"same model on the oracle ops (torch CPU FP32), {elapsed:.1f} s"}


def mace_block_cpu(seconds, atoms=1024):
    """The same block on the oracle ops (torch CPU FP32, all host threads), smaller system."""
    from mace_ictc.models import InteractionBlock, ProductBlock, radial_embedding, species_groups
    from oracle.model_ops import OracleOps
    torch.set_num_threads(os.cpu_count() or 1)
    pos, species, side, src, dst, shift = _cpu_system(atoms, 3)
    torch.manual_seed(0)
    C, L = 64, 2
    ops = OracleOps(torch.float32)
    inter = InteractionBlock(channels=C, lmax=L, input_lmax=L, num_elements=3, num_basis=8,
                             avg_num_neighbors=src.numel() / atoms, use_self_connection=True, sc_lmax=L)
    prod = ProductBlock(channels=C, lmax=L, target_lmax=L, correlation=3, num_elements=3)
    readout = torch.nn.Linear(C, 1, bias=False)
    h = torch.randn(atoms, C * (L + 1) ** 2)
    groups = species_groups(species, 3)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or done == 0:
        p = pos.detach().requires_grad_(True)
        vec = p[dst] - p[src] + shift
        r = vec.norm(dim=1)
        harm = ops.harmonics(vec / r.unsqueeze(-1), L)
        message, sc = inter(ops, h, harm, radial_embedding(r, 5.0, 8, 5), src, dst, None, groups)
        energy = readout(prod(ops, message, sc, species)[:, :C]).sum()
        torch.autograd.grad(energy, [p])
        done += atoms
    elapsed = time.perf_counter() - t0
    return {"value": round(done / elapsed, 1), "unit": "atom-steps/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{done} atom-steps of a {atoms}-atom system with the same block on the "
                                      f"oracle ops (torch CPU FP32), {elapsed:.1f} s"}


def mace_train(device, steps, warmup, configs=4, atoms=2048, cutoff=5.0):
    """force-loss training step of MACE C128/lmax3, 2 interactions,
    correlation 3.  A batch of 4 periodic configurations of 2,048 H/C/O atoms (0.1/A^3,
    minimum distance 0.9 A); synthetic targets: per-atom energy N(0,1) and forces N(0,1).
    loss = mean_c (E_c/N_c - e_c)^2 + 100 mean (F - F_t)^2; each step runs forward, forces
    with create_graph, the backward through the mixed second derivatives, and an Adam step."""
    from ictc_o3.backends.cuda.neighbors import neighbor_list
    from mace_ictc.models import MACEICTC
    from mace_ictc.systems import random_system
    pos_l, spec_l, src_l, dst_l, shift_l, batch_l = [], [], [], [], [], []
    edges = 0
    for c in range(configs):
        pos, species, side = random_system(atoms, seed=100 + c, device=device)
        src, dst, shift, _ = neighbor_list(pos, (side,) * 3, cutoff)
        pos_l.append(pos)
        spec_l.append(species)
        src_l.append(src + c * atoms)
        dst_l.append(dst + c * atoms)
        shift_l.append(shift)
        batch_l.append(torch.full((atoms,), c, dtype=torch.int64, device=device))
        edges += src.numel()
    pos, species = torch.cat(pos_l), torch.cat(spec_l)
    src, dst, shift, batch = torch.cat(src_l), torch.cat(dst_l), torch.cat(shift_l), torch.cat(batch_l)
    gen = torch.Generator(device=device).manual_seed(77)
    e_target = torch.randn(configs, device=device, generator=gen)
    f_target = torch.randn(pos.shape[0], 3, device=device, generator=gen)
    torch.manual_seed(0)
    model = MACEICTC(channels=128, lmax=3, num_interactions=2, correlation=3, r_max=cutoff,
                     avg_num_neighbors=edges / pos.shape[0]).to(device)
    opt = torch.optim.Adam([p for p in model.parameters() if p.requires_grad], lr=1e-3)
    torch.cuda.reset_peak_memory_stats(device)
    losses = []

    def step():
        opt.zero_grad(set_to_none=True)
        p = pos.detach().requires_grad_(True)
        energy = model.energy(p, species, src, dst, shift, batch, configs)
        (grad,) = torch.autograd.grad(energy.sum(), [p], create_graph=True)
        loss = ((energy / atoms - e_target) ** 2).mean() + 100.0 * ((-grad - f_target) ** 2).mean()
        loss.backward()
        opt.step()
        losses.append(loss.detach())

    ms = time_loop(step, steps, warmup, 1, device) / steps
    total = configs * atoms
    return {"value": round(total / (ms * 1e-3), 1), "unit": "atom-steps/s", "ms_per_step": round(ms, 2),
            "configs_per_s": round(configs / (ms * 1e-3), 2), "atoms": total, "edges": edges,
            "peak_device_gb": round(torch.cuda.max_memory_allocated(device) / 1e9, 1),
            "loss_first_last": [round(float(losses[0]), 4), round(float(losses[-1]), 4)],
            "workload": "configs[3]: MACE C128/lmax3, 2 interactions, corr 3, 4 x 2,048 atoms, "
                        "loss = E MSE (per atom) + 100 x F MSE, backward through mixed second derivatives, Adam"}


def mace_md(device, world, rank, steps, warmup, atoms=262144, cutoff=5.0, phases=False):
    """MACE energy + forces + virial MD step, C64/lmax2, 2 interactions,
    correlation 3, 262,144 H/C/O atoms at 0.1/A^3, slab-partitioned along x over the ranks
    with one-cutoff halos.  Each rank holds only its own atoms (distributed once, before
    timing).  Every step migrates atoms between slabs, exchanges ghost positions, rebuilds
    the neighbour list, runs the model with the feature halo exchange before layer 2 (and
    its adjoint) and returns ghost forces to their owners.  Strong scaling: the system
    size is fixed.

    ``value`` times device-resident positions; ``e2e`` adds, every step, the H2D copy of
    each rank's owned positions from pinned host memory and the D2H read of the owned
    forces, energy and virial.  ``phases`` adds a per-phase breakdown (CUDA events on the
    compute stream and host time between marks, median over the timed steps, max over
    ranks)."""
    from mace_ictc.models import MACEICTC
    from mace_ictc.parallel import StepPhases, md_step, partition
    from mace_ictc.systems import random_system
    side = (atoms / 0.1) ** (1.0 / 3.0)
    pos, species, side0 = random_system(atoms, seed=41, device=device)   # same seed on every rank
    assert abs(side0 - side) < 1e-9
    domain = partition(pos, species, side, rank, world, cutoff)
    del pos, species
    torch.manual_seed(0)
    model = MACEICTC(channels=64, lmax=2, num_interactions=2, correlation=3, r_max=cutoff,
                     avg_num_neighbors=52.0).to(device)
    torch.cuda.reset_peak_memory_stats(device)
    stats = {}
    state = {"domain": domain}
    recorder = StepPhases(enabled=phases)
    tables = []

    def step():
        recorder.reset()
        d, energy, forces, virial = md_step(model, state["domain"], cutoff, phases=recorder)
        state["domain"] = d
        if phases:
            tables.append(recorder.summary())
        return energy, forces, virial

    ms = time_loop(step, steps, warmup, world, device) / steps
    ms = max_over_ranks(ms, world, device)
    result_phases = None
    if phases:
        names = [name for name, _, _ in tables[-1]]
        med = torch.tensor([[statistics.median(t[i][1] for t in tables[warmup:]),
                             statistics.median(t[i][2] for t in tables[warmup:])] for i in range(len(names))],
                           device=device, dtype=torch.float64)
        if world > 1:
            torch.distributed.all_reduce(med, op=torch.distributed.ReduceOp.MAX)
        result_phases = {name: {"device_ms": round(float(med[i, 0]), 3), "host_ms": round(float(med[i, 1]), 3)}
                         for i, name in enumerate(names)}
        recorder.enabled = False

    owned_host = state["domain"].pos.cpu().pin_memory()
    pos_dev = torch.empty_like(state["domain"].pos)
    out_host = {}

    def pinned(name, t):
        buf = out_host.get(name)
        if buf is None or buf.shape != t.shape:
            buf = out_host[name] = torch.empty(t.shape, dtype=t.dtype).pin_memory()
        return buf

    def e2e_step():
        pos_dev.copy_(owned_host, non_blocking=True)
        d = state["domain"]
        d.pos = pos_dev
        d, energy, forces, virial = md_step(model, d, cutoff)
        state["domain"] = d
        pinned("forces", forces).copy_(forces, non_blocking=True)
        ev = torch.cat([energy, virial])
        pinned("ev", ev).copy_(ev, non_blocking=True)
        stats.update(owned=d.owned, forces=forces.shape[0])

    e2e_steps = max(2, steps)
    e2e_ms = time_loop(e2e_step, e2e_steps, 1, world, device) / e2e_steps
    e2e_ms = max_over_ranks(e2e_ms, world, device)
    peak_gb = max_over_ranks(torch.cuda.max_memory_allocated(device) / 1e9, world, device)
    from mace_ictc.parallel import halo_layout, slab_edges
    layout, p, _ = halo_layout(state["domain"])
    src, _, _ = slab_edges(layout, p, cutoff)
    ghost_rows = layout.local - layout.owned
    result = {"value": round(atoms / (ms * 1e-3), 1), "unit": "atom-steps/s", "ms_per_step": round(ms, 2),
              "n_gpus": world, "scaling": "strong", "atoms": atoms,
              "per_rank_rank0": {"owned": layout.owned, "ghosts": ghost_rows, "edges": int(src.numel())},
              "halo_bytes_per_exchange_rank0": ghost_rows * 64 * 9 * 4,
              "peak_device_gb": round(peak_gb, 1),
              "workload": "configs[4]: MACE C64/lmax2, 2 interactions, corr 3, E+F+virial, migration, ghost "
                          "positions and neighbour rebuild every step, slab partition along x with 5 A halos, "
                          "NCCL P2P feature exchange",
              "e2e": {"value": round(atoms / (e2e_ms * 1e-3), 1), "unit": "atom-steps/s",
                      "h2d_bytes_per_step": atoms * 12, "d2h_bytes_per_step": atoms * 12 + world * 28}}
    if result_phases is not None:
        result["phases"] = result_phases
    return result


def arm_config(world):
    """The workload description both arms report."""
    return {"workload": WORKLOAD, "channels": C, "lmax": L, "paths": PATHS,
            "instances_per_step": FWD_ROWS, "per_gpu_instances": FWD_ROWS, "layout": "ir_mul",
            "l2": "inputs (7.3 GB) and output (13.3 GB) far exceed the 126 MB L2; no flush needed",
            "parallelism": f"replicas x{world} (independent instances, no collective)"}


def run_ours(args):
    world, rank, local = setup_dist()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from ictc_o3.backends.cuda import _native
    from ictc_o3.operators import EdgeTensorProduct
    _native.library()
    op = EdgeTensorProduct.create(channels=C, input_lmax=L, edge_lmax=L, layout="ir_mul", device=device)

    # Forward at 262,144 instances (inputs 7.3 GB, output 13.3 GB: far above L2).
    x, y, g = make_inputs(FWD_ROWS, device, 1234 + rank)
    sampler = ClockSampler(device)
    with torch.no_grad():
        fwd_ms = time_loop(lambda: op(x, y, g), args.steps, args.warmup, world, device) / args.steps
    fwd_ms = max_over_ranks(fwd_ms, world, device)
    del x, y, g
    torch.cuda.empty_cache()

    # Forward + VJP at 131,072 instances.
    x, y, g = make_inputs(VJP_ROWS, device, 4321 + rank, requires_grad=True)
    G = torch.randn(VJP_ROWS, OUT_W, device=device, generator=torch.Generator(device=device).manual_seed(99))

    def fwd_vjp():
        out = op(x, y, g)
        torch.autograd.grad(out, [x, y, g], G)

    vjp_ms = time_loop(fwd_vjp, args.steps, args.warmup, world, device) / args.steps
    vjp_ms = max_over_ranks(vjp_ms, world, device)
    clocks = sampler.stop()
    del x, y, g, G
    torch.cuda.empty_cache()

    block = mace_block(device, max(3, min(args.steps, 10)), 2,
                       cpu_seconds=(args.cpu_seconds / 2 if world == 1 and rank == 0 else 0.0))
    torch.cuda.empty_cache()
    md = mace_md(device, world, rank, max(3, min(args.steps, 5)), 2)
    torch.cuda.empty_cache()
    train = mace_train(device, 3, 2) if world == 1 else None
    torch.cuda.empty_cache()
    if world == 1 and rank == 0:
        md["cpu_baseline"] = mace_md_cpu(args.cpu_seconds / 3)
        train["cpu_baseline"] = mace_train_cpu(args.cpu_seconds / 3)

    e2e_steps = max(2, min(args.steps, 5))
    e2e_ms, h2d, d2h = e2e_forward(op, FWD_ROWS, e2e_steps, 1, device, world)
    e2e_ms = max_over_ranks(e2e_ms, world, device)

    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    cpu = cpu_baseline(args.cpu_seconds) if world == 1 else None
    value = world * FWD_ROWS / (fwd_ms * 1e-3)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "TP instances/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(fwd_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": round(value / PUBLISHED_FWD, 2),
        "dtype": "f32", "data": "synthetic (seeded; configs[1] distributions)",
        "config": arm_config(world),
        "roofline": roofline(FWD_BYTES, FWD_ROWS, fwd_ms, profiled_traffic("tp_forward_c128_l3.txt")),
        "fwd_vjp": {"value": round(world * VJP_ROWS / (vjp_ms * 1e-3), 1), "unit": "TP instances/s",
                    "instances_per_step": VJP_ROWS, "ms_per_step": round(vjp_ms, 4),
                    "roofline": roofline(VJP_BYTES, VJP_ROWS, vjp_ms, vjp_traffic()),
                    "gpu_launches_per_step": 2},
        "e2e": {"value": round(world * FWD_ROWS / (e2e_ms * 1e-3), 1), "unit": "TP instances/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "ictc_o3.operators.EdgeTensorProduct.forward, pinned host buffers, chunked H2D/compute/D2H"},
        "mace_block": block,
        "mace_md": md,
        "mace_train": train,
        "gpu_launches": args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle port of the reference CPU module
# ---------------------------------------------------------------------------

def _cpu_tp_setup(rows, seed):
    from ictc_o3.basis.ictd_irreps import EdgeWeightedPathPreservingTensorProduct, operator_paths
    from oracle import tp_oracle
    owner = EdgeWeightedPathPreservingTensorProduct(C, L, allowed_paths=operator_paths(L, L, L))
    with torch.no_grad():
        owner.weight.fill_(1.0)
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, FEATURE_W, generator=gen)
    n = torch.nn.functional.normalize(torch.randn(rows, 3, generator=gen), dim=1)
    y = torch.cat(tp_oracle.direction_harmonics(n, L, tp_oracle.harmonic_tables(L)), -1)
    g = torch.randn(rows, GATE_W, generator=gen) / PATHS ** 0.5
    blocks = tp_oracle.split_mul_ir(x, C, L)
    harm = tp_oracle.split_harm(y, L)
    return owner, blocks, harm, g.view(rows, PATHS, C), tp_oracle


def cpu_baseline_port(seconds, rows=2048):
    """Oracle port of the reference CPU TP forward (oracle/tp_oracle.py), all host threads."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    owner, blocks, harm, g, tp_oracle = _cpu_tp_setup(rows, 5)
    with torch.no_grad():
        tp_oracle.tp_forward(owner, blocks, harm, g)
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            tp_oracle.tp_forward(owner, blocks, harm, g)
            done += rows
        elapsed = time.perf_counter() - t0
    return {"value": round(done / elapsed, 1), "unit": "TP instances/s", "cores": threads, "kind": "port",
            "sample": f"{done} instances of C128/lmax3 forward in chunks of {rows} "
                      f"(oracle/tp_oracle.py, torch CPU FP32, {elapsed:.1f} s)"}


def cpu_baseline(seconds):
    """The stock reference module timed in a child process (both packages are named
    ``ictc_o3``, so the reference cannot be imported next to this one); the port as
    a second, labelled number."""
    port = cpu_baseline_port(seconds / 2)
    steps = 4
    proc = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "reference", "--steps", str(steps),
                           "--warmup", "1"], capture_output=True, text=True, timeout=600)
    line = None
    for text in proc.stdout.splitlines():
        if text.startswith("{"):
            line = json.loads(text)
    if proc.returncode != 0 or line is None or "unavailable" in line:
        port["note"] = "reference package unavailable: " + (line or {}).get("unavailable", proc.stderr[-300:])
        return port
    base = dict(line["cpu_baseline"])
    base["port"] = port
    return base


REF_ROOT = os.path.join(REPO, "baseline", "_ref")
REF_ROWS = 4096


def _reference_package():
    """Make ``ictc_o3`` resolve to the installed reference package (baseline/_ref) in
    this process; False when it is not installed."""
    if not os.path.isfile(os.path.join(REF_ROOT, "ictc_o3", "basis", "ictd_irreps.py")):
        return False
    if "ictc_o3" in sys.modules:
        raise RuntimeError("this process already imported the backend's ictc_o3")
    os.environ.setdefault("FSCETP_ICTD_CACHE", "0")        # no disk cache writes from the reference
    while PACKAGE_ROOT in sys.path:
        sys.path.remove(PACKAGE_ROOT)
    sys.path.insert(0, REF_ROOT)
    return True


def _reference_tp(rows, seed):
    """The reference's own module, built as its operator factory builds it
    (``ictc_o3/operators.py:43-66``: operator paths, FP32, path weights fixed to 1),
    on the configs[1] inputs (features N(0,1), harmonics of random unit vectors,
    gates N(0, 1/sqrt(23)))."""
    from ictc_o3.basis.ictd_irreps import EdgeWeightedPathPreservingTensorProduct, direction_harmonics_all
    paths = [(i, j, k) for i in range(L + 1) for j in range(L + 1) for k in range(L + 1)
             if abs(i - j) <= k <= i + j and (i + j + k) % 2 == 0]
    tp = EdgeWeightedPathPreservingTensorProduct(channels=C, lmax=L, allowed_paths=paths,
                                                 internal_compute_dtype=torch.float32)
    with torch.no_grad():
        tp.weight.fill_(1.0)
    tp.weight.requires_grad_(False)
    gen = torch.Generator().manual_seed(seed)
    x = {l: torch.randn(rows, C, 2 * l + 1, generator=gen) for l in range(L + 1)}
    n = torch.nn.functional.normalize(torch.randn(rows, 3, generator=gen), dim=1)
    y = {l: h.unsqueeze(1) for l, h in enumerate(direction_harmonics_all(n, L))}
    g = torch.randn(rows, GATE_W, generator=gen) / PATHS ** 0.5
    return tp, x, y, g


def run_reference(args):
    """Reference arm: the stock ``EdgeWeightedPathPreservingTensorProduct.forward``
    (``ictc_o3/basis/ictd_irreps.py:2750-2795``) from the installed reference package on
    the host cores, each step a bounded sample of the configs[1] workload.  Without
    the installed package, the oracle port (labelled "port")."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if _reference_package():
        rows = REF_ROWS
        tp, x, y, g = _reference_tp(rows, 17)

        def forward():
            tp(x, y, g)
        kind, what = "reference", ("stock ictc_o3 EdgeWeightedPathPreservingTensorProduct.forward "
                                   "(baseline/_ref, torch CPU FP32)")
    else:
        rows = 2048
        owner, blocks, harm, g, tp_oracle = _cpu_tp_setup(rows, 17)

        def forward():
            tp_oracle.tp_forward(owner, blocks, harm, g)
        kind, what = "port", "oracle/tp_oracle.py port (reference package not installed)"
    with torch.no_grad():
        for _ in range(args.warmup):
            forward()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            forward()
        elapsed = time.perf_counter() - t0
    value = args.steps * rows / elapsed
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "TP instances/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * elapsed / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": round(value / PUBLISHED_FWD, 6),
        "dtype": "f32", "data": "synthetic (seeded; configs[1] distributions)", "impl": "reference",
        "config": arm_config(world),
        "cpu_baseline": {"value": round(value, 1), "unit": "TP instances/s", "cores": threads, "kind": kind,
                         "sample": f"each step = {rows} instances of the {FWD_ROWS}-instance workload; {what}"},
        "e2e": {"value": round(value, 1), "unit": "TP instances/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_profile(args):
    """Forward then forward+VJP at one size, printing per-step times (for ncu command lines)."""
    device = torch.device("cuda", 0)
    from ictc_o3.backends.cuda import _native
    from ictc_o3.operators import EdgeTensorProduct
    _native.library()
    op = EdgeTensorProduct.create(channels=C, input_lmax=L, edge_lmax=L, layout="ir_mul", device=device)
    rows_f = args.rows or FWD_ROWS
    rows_v = args.rows or VJP_ROWS
    x, y, g = make_inputs(rows_f, device, 1)
    with torch.no_grad():
        fwd_ms = time_loop(lambda: op(x, y, g), args.steps, args.warmup, 1, device) / args.steps
    del x, y, g
    x, y, g = make_inputs(rows_v, device, 2, requires_grad=True)
    G = torch.randn(rows_v, OUT_W, device=device)

    def fwd_vjp():
        torch.autograd.grad(op(x, y, g), [x, y, g], G)

    vjp_ms = time_loop(fwd_vjp, args.steps, args.warmup, 1, device) / args.steps
    print(json.dumps({"profile": True, "fwd_rows": rows_f, "fwd_ms": round(fwd_ms, 4),
                      "fwd_GBps": round(FWD_BYTES * rows_f / fwd_ms / 1e6, 1), "vjp_rows": rows_v,
                      "vjp_ms": round(vjp_ms, 4), "vjp_GBps": round(VJP_BYTES * rows_v / vjp_ms / 1e6, 1)}))


def run_profile_radial(args):
    """Fused radial MLP alone: seeded weights (8 -> 64 -> 64 -> 64 -> G) and edge embeddings,
    forward and embedding-gradient kernels timed with CUDA events (for ncu command lines)."""
    device = torch.device("cuda", 0)
    from ictc_o3.backends.cuda import radial
    rows = args.rows or 1048576
    g = torch.Generator().manual_seed(11)
    weights = [torch.randn(64, 8, generator=g) / 8 ** 0.5, torch.randn(64, 64, generator=g) / 8.0,
               torch.randn(64, 64, generator=g) / 8.0, torch.randn(args.gates, 64, generator=g) / 8.0]
    plan = radial.RadialPlan()
    image, status = plan.get([w.to(device) for w in weights])
    feats = torch.rand(rows, 8, device=device)
    grad = torch.randn(rows, args.gates, device=device)
    fwd_ms = time_loop(lambda: radial._forward(image, status, feats, args.gates), args.steps, args.warmup, 1,
                       device) / args.steps
    bwd_ms = time_loop(lambda: radial._backward(image, status, feats, grad), args.steps, args.warmup, 1,
                       device) / args.steps
    radial.check_status(plan)
    gate_bytes = rows * args.gates * 4
    print(json.dumps({"profile_radial": True, "rows": rows, "gates": args.gates, "fwd_ms": round(fwd_ms, 4),
                      "fwd_GBps_gates": round(gate_bytes / fwd_ms / 1e6, 1), "bwd_ms": round(bwd_ms, 4),
                      "bwd_GBps_gates": round(gate_bytes / bwd_ms / 1e6, 1)}), flush=True)


def main():
    args = parse_args()
    if args.profile_block:
        device = torch.device("cuda", 0)
        from ictc_o3.backends.cuda import _native
        _native.library()
        print(json.dumps({"profile_block": mace_block(device, args.steps, args.warmup, atoms=args.atoms or 16384)}))
    elif args.profile_radial:
        run_profile_radial(args)
    elif args.profile_train:
        device = torch.device("cuda", 0)
        from ictc_o3.backends.cuda import _native
        _native.library()
        print(json.dumps({"profile_train": mace_train(device, args.steps, args.warmup)}), flush=True)
    elif args.profile_md:
        world, rank, local = setup_dist()
        device = torch.device("cuda", local)
        torch.cuda.set_device(device)
        from ictc_o3.backends.cuda import _native
        _native.library()
        md = mace_md(device, world, rank, args.steps, args.warmup, atoms=args.atoms or 262144, phases=args.phases)
        if rank == 0:
            print(json.dumps({"profile_md": md}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
    elif args.profile:
        run_profile(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
