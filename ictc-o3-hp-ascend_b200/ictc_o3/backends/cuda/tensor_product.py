"""Path-preserving ICTC tensor product on the CUDA backend.

Drop-in for ``ictc_o3/backends/ascend/tensor_product.py`` (same function names
and argument meaning).  The TP is trilinear in (features x, harmonics Y,
effective gate g*w); every derivative of any order is therefore a combination
of the two native kernels:

* ``ictc_tp_forward``   out = T(x, Y, g)
* ``ictc_tp_backward``  (A_x, A_Y, A_g)(., ., ., G): the three first adjoints

The mixed second derivatives follow the reference recursion
(``ictc_o3/backends/ascend/sparse_product.py:226-264``): for cotangents
(hx, hY, hg) of the adjoint outputs, substitute each cotangent for its operand
and apply the other modes, and T(...) gives the gradient of G.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional

import numpy as np
import torch

from ictc_o3.autograd.adjoint_requirements import required_gradients
from . import _native
from .cache import cache_of
from ._native import ptr, stream_of

LAYOUTS = {"ir_mul": 0, "mul_ir": 1}


# ---------------------------------------------------------------------------
# Plans
# ---------------------------------------------------------------------------

class TPPlan:
    """Device-resident constant tables of one TP (one device, one layout)."""

    def __init__(self, owner, layout: str, device: torch.device, cpl_forward: int = 0, cpl_backward: int = 0):
        paths = [tuple(int(v) for v in p) for p in owner.paths]
        self.input_lmax = max(p[0] for p in paths)
        self.edge_lmax = max(p[1] for p in paths)
        self.output_lmax = max(p[2] for p in paths)
        self.channels = int(owner.channels)
        self.num_paths = len(paths)
        self.layout = layout
        self.device = device
        cg = _cg_f64(owner)
        flat = np.ascontiguousarray(np.concatenate([c.reshape(-1) for c in cg]), dtype=np.float64)
        path_arr = np.ascontiguousarray(np.array(paths, dtype=np.int32).reshape(-1))
        handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            _native.call("ictc_tp_plan_create", self.channels, self.input_lmax, self.edge_lmax,
                         self.output_lmax, LAYOUTS[layout], self.num_paths,
                         path_arr.ctypes.data_as(ctypes.c_void_p), flat.ctypes.data_as(ctypes.c_void_p),
                         int(flat.size), int(cpl_forward), int(cpl_backward), ctypes.byref(handle))
        self.handle = handle
        info = (ctypes.c_int64 * 8)()
        _native.call("ictc_tp_plan_info", handle, info, 8)
        (self.np_, self.bond_width, self.output_width, self.feature_width, self.harmonic_width,
         self.cpl_forward, self.cpl_backward, self.grid) = (int(v) for v in info)
        extra = (ctypes.c_int64 * 12)()
        _native.call("ictc_tp_plan_info", handle, extra, 12)
        self.cpl_message_forward, self.cpl_message_backward = int(extra[8]), int(extra[9])

    def status(self, reset: bool = False) -> int:
        """Non-zero when a kernel of this plan gave up on a timed-out wait (one device read)."""
        value = ctypes.c_int32()
        _native.call("ictc_tp_plan_status", self.handle, ctypes.byref(value), int(reset))
        return int(value.value)

    def check_status(self):
        """Raise if a kernel of this plan recorded a timed-out wait.

        Codes: 1 a staged copy did not land in time (the copies in flight drained;
        the context stays usable), 2 a launch the kernel does not support, 3 a staged
        copy did not land and neither did the drain: a bulk copy may still write
        shared memory of a finished CTA, so the CUDA context must be considered lost."""
        code = self.status()
        if code == 3:
            raise RuntimeError("tensor-product kernel reported error 3: a staged copy never completed and its "
                               "drain timed out; treat this CUDA context as lost (restart the process)")
        if code:
            raise RuntimeError(f"tensor-product kernel reported error {code} (timed-out staging wait)")

    def __del__(self):
        handle = getattr(self, "handle", None)
        if handle is not None and _native._lib is not None:
            _native._lib.ictc_tp_plan_destroy(handle)
            self.handle = None


def _cg_f64(owner):
    if hasattr(owner, "cg_f64"):
        return [np.asarray(c, dtype=np.float64) for c in owner.cg_f64()]
    return [c.detach().to("cpu", torch.float64).numpy() for c in
            owner._get_cg_list(torch.device("cpu"), torch.float64)]


def get_plan(owner, layout: str, device: torch.device, cpl_forward: int = 0, cpl_backward: int = 0) -> TPPlan:
    """Cached plan for (owner, device, layout) (pattern of tensor_product.py:12-18)."""
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("The CUDA tensor product requires CUDA tensors")
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, layout, tuple(tuple(p) for p in owner.paths), int(owner.channels), cpl_forward, cpl_backward)
    cache = cache_of(owner, "_cuda_tp_plans")
    plan = cache.get(key)
    if plan is None:
        plan = TPPlan(owner, layout, torch.device("cuda", index), cpl_forward, cpl_backward)
        cache[key] = plan
    return plan


# ---------------------------------------------------------------------------
# Raw kernel calls
# ---------------------------------------------------------------------------

def _check(*tensors):
    for t in tensors:
        if t is not None and (t.dtype != torch.float32 or t.device.type != "cuda" or not t.is_contiguous()):
            raise ValueError("CUDA tensor-product operands must be contiguous FP32 CUDA tensors")


class StandaloneOp:
    """Row-wise TP: out[e] = T(x[e], y[e], g[e])."""

    def __init__(self, plan: TPPlan):
        self.plan = plan

    def forward(self, x, y, g, w):
        plan, rows = self.plan, x.shape[0]
        out = torch.empty(rows, plan.output_width, device=x.device, dtype=torch.float32)
        if rows:
            _check(x, y, g, w)
            _native.call("ictc_tp_forward", plan.handle, ptr(x), ptr(y), ptr(g), ptr(w), ptr(out),
                         int(rows), stream_of(x))
        return out

    def adjoint(self, x, y, g, w, grad, need):
        plan, rows = self.plan, x.shape[0]
        dx = torch.empty_like(x) if need[0] else None
        dy = torch.empty_like(y) if need[1] else None
        dg = (torch.empty(rows, plan.num_paths * plan.channels, device=x.device, dtype=torch.float32)
              if need[2] else None)
        if rows and any(need):
            _check(x, y, g, w, grad)
            _native.call("ictc_tp_backward", plan.handle, ptr(x), ptr(y), ptr(g), ptr(w), ptr(grad),
                         ptr(dx), ptr(dy), ptr(dg), int(rows), stream_of(x))
        return dx, dy, dg


def raw_forward(plan: TPPlan, x, y, g, w):
    return StandaloneOp(plan).forward(x, y, g, w)


def raw_backward(plan: TPPlan, x, y, g, w, grad, need):
    return StandaloneOp(plan).adjoint(x, y, g, w, grad, need)


def _add(a, b):
    if a is None:
        return b
    if b is None:
        return a
    return a + b


# ---------------------------------------------------------------------------
# Autograd (shared by the standalone TP and the graph message: both are
# trilinear in (x, y, g) with every other input fixed)
# ---------------------------------------------------------------------------

class _Product(torch.autograd.Function):
    """out = T(x, y, g); ``w`` is a constant per-(path, channel) factor of g."""

    @staticmethod
    def forward(ctx, op, w, x, y, g):
        ctx.op, ctx.w, ctx.has_g = op, w, g is not None
        ctx.save_for_backward(x, y, g)
        return op.forward(x, y, g, w)

    @staticmethod
    def backward(ctx, grad):
        x, y, g = ctx.saved_tensors
        need = required_gradients((x, y, g), ctx.needs_input_grad[2:5])
        if not any(need):
            return None, None, None, None, None
        grad = grad.contiguous()
        if torch.is_grad_enabled():
            dx, dy, dg = _Adjoint.apply(ctx.op, ctx.w, x, y, g, grad, need)
        else:
            dx, dy, dg = ctx.op.adjoint(x, y, g, ctx.w, grad, need)
        return None, None, dx, dy, (dg if ctx.has_g else None)


def product(op, w, x, y, g):
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (x, y, g)):
        return _Product.apply(op, w, x, y, g)
    return op.forward(x, y, g, w)


def adjoint(op, w, x, y, g, grad, need):
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (x, y, g, grad)):
        return _Adjoint.apply(op, w, x, y, g, grad, tuple(need))
    return op.adjoint(x, y, g, w, grad, need)


class _Adjoint(torch.autograd.Function):
    """(A_x, A_y, A_g) = first adjoints of T at cotangent G; differentiable again."""

    @staticmethod
    def forward(ctx, op, w, x, y, g, grad, need):
        ctx.set_materialize_grads(False)
        ctx.op, ctx.w = op, w
        ctx.save_for_backward(x, y, g, grad)
        return op.adjoint(x, y, g, w, grad, need)

    @staticmethod
    def backward(ctx, hx, hy, hg):
        x, y, g, grad = ctx.saved_tensors
        op, w = ctx.op, ctx.w
        need = required_gradients((x, y, g, grad), ctx.needs_input_grad[2:6])
        hx = None if hx is None else hx.contiguous()
        hy = None if hy is None else hy.contiguous()
        hg = None if hg is None else hg.contiguous()
        gx = gy = gg = gG = None
        # hx: <hx, A_x(y, g, G)> = <G, T(hx, y, g)>
        if hx is not None:
            if need[1] or (need[2] and g is not None):
                _, ay, ag = adjoint(op, w, hx, y, g, grad, (False, need[1], need[2] and g is not None))
                gy, gg = _add(gy, ay), _add(gg, ag)
            if need[3]:
                gG = _add(gG, product(op, w, hx, y, g))
        # hy: <hy, A_y(x, g, G)> = <G, T(x, hy, g)>
        if hy is not None:
            if need[0] or (need[2] and g is not None):
                ax, _, ag = adjoint(op, w, x, hy, g, grad, (need[0], False, need[2] and g is not None))
                gx, gg = _add(gx, ax), _add(gg, ag)
            if need[3]:
                gG = _add(gG, product(op, w, x, hy, g))
        # hg: <hg, A_g(x, y, G)> = <G, T(x, y, hg)>; without gates the third
        # output is the derivative of the effective weight itself.
        if hg is not None:
            wh = w if g is not None else None
            if need[0] or need[1]:
                ax, ay, _ = adjoint(op, wh, x, y, hg, grad, (need[0], need[1], False))
                gx, gy = _add(gx, ax), _add(gy, ay)
            if need[3]:
                gG = _add(gG, product(op, wh, x, y, hg))
        return (None, None, gx if need[0] else None, gy if need[1] else None,
                gg if need[2] else None, gG if need[3] else None, None)


# ---------------------------------------------------------------------------
# Entry points
# ---------------------------------------------------------------------------

def _weight_and_gates(owner, gates, rows):
    """Split owner.weight * gates into (kernel weight, differentiable gates)."""
    weight = owner.weight
    if gates is not None and weight.device != gates.device:
        raise ValueError("The tensor-product weight must be on the operands' CUDA device")
    channels, paths = int(owner.channels), int(owner.num_paths)
    if gates is not None:
        gates = gates.reshape(rows, paths * channels)
    if weight.requires_grad and torch.is_grad_enabled():
        eff = weight.reshape(1, paths * channels)
        gates = eff.expand(rows, -1) if gates is None else gates * eff
        return None, gates.contiguous()
    w = weight.detach().reshape(paths * channels).contiguous()
    return w, (None if gates is None else gates.contiguous())


def packed_product(owner, layout, features, harmonics, gates):
    """Packed public layout: features [E, C(Li+1)^2] -> [E, output_width]."""
    rows = features.shape[0]
    if owner.weight.device != features.device:
        raise ValueError("The tensor-product weight must be on the operands' CUDA device")
    plan = get_plan(owner, layout, features.device)
    w, g = _weight_and_gates(owner, gates, rows)
    if features.shape[1] != plan.feature_width or harmonics.shape != (rows, plan.harmonic_width):
        raise ValueError("Packed features/harmonics do not match the tensor-product degrees")
    return product(StandaloneOp(plan), w, features.contiguous(), harmonics.contiguous(), g)


def tensor_product(owner, features: Dict[int, torch.Tensor], harmonics: Dict[int, torch.Tensor],
                   gates: Optional[torch.Tensor] = None) -> Dict[int, torch.Tensor]:
    """Block interface of the hook site (``ictc_irreps.py:2773-2775``).

    features: l -> [E, C, 2l+1]; harmonics: l -> [E, 1, 2l+1]; gates [E, P, C]
    or [E, P*C].  Returns l -> [E, count_l*C, 2l+1] for l = 0..owner.lmax.
    """
    sample = next(iter(features.values()))
    rows, channels = sample.shape[0], int(owner.channels)
    input_lmax = max(p[0] for p in owner.paths)
    edge_lmax = max(p[1] for p in owner.paths)
    if sorted(features)[:input_lmax + 1] != list(range(input_lmax + 1)):
        raise ValueError("features must hold every degree 0..input_lmax")
    if sorted(harmonics)[:edge_lmax + 1] != list(range(edge_lmax + 1)):
        raise ValueError("harmonics must hold every degree 0..edge_lmax")
    x = torch.cat([features[l].reshape(rows, channels * (2 * l + 1)) for l in range(input_lmax + 1)], 1)
    y = torch.cat([harmonics[l].reshape(rows, 2 * l + 1) for l in range(edge_lmax + 1)], 1)
    out = packed_product(owner, "mul_ir", x, y, gates)
    return split_output(owner, out)


def split_output(owner, out):
    rows, channels = out.shape[0], int(owner.channels)
    result, offset = {}, 0
    for l in range(owner.lmax + 1):
        count = int(owner.path_counts_by_l.get(l, 0))
        span = count * channels * (2 * l + 1)
        result[l] = out[:, offset:offset + span].reshape(rows, count * channels, 2 * l + 1)
        offset += span
    return result
