"""Fused radial MLP (edge embedding -> path gates) on the tensor cores.

The MACE interaction's radial network (``mace_ictc/models/pure_cartesian_ictd_fix.py:1545-1553``):
bias-free Linear F->64, normalised SiLU, 64->64, SiLU, 64->64, SiLU, 64->G.  The
kernels (``csrc/radial.cu``) keep the hidden activations on chip and write only
the gates; the adjoint returns the gradient of the edge embedding.  When the
gradient itself must be differentiated (force-loss training) or the weights need
gradients, the backward recomputes the network with device tensor algebra so
autograd can differentiate it again.
"""
from __future__ import annotations

import ctypes
import weakref

import numpy as np
import torch

from ictc_o3.autograd.adjoint_requirements import required_gradients
from . import _native
from ._native import ptr, stream_of

SILU_SCALE = 1.6791767923989418
HIDDEN = 64


def _silu(x):
    return torch.nn.functional.silu(x) * SILU_SCALE


def mlp_reference(feats, weights):
    """The same network as device tensor algebra (differentiable; used for second order)."""
    w1, w2, w3, w4 = weights
    h = _silu(feats @ w1.t())
    h = _silu(h @ w2.t())
    h = _silu(h @ w3.t())
    return h @ w4.t()


GATE_TILE = 64


def padded_gates(gates: int) -> int:
    """The kernels write gate rows in 64-column chunks; other widths run on W4 padded with
    zero rows to the next multiple of 64 (the extra columns are dropped)."""
    return -(-int(gates) // GATE_TILE) * GATE_TILE


def supported(features: int, hidden: int, gates: int) -> bool:
    return gates > 0 and int(_native.library().ictc_radial_image_bytes(features, hidden, padded_gates(gates))) > 0


def pack_image(weights) -> torch.Tensor:
    """Host-packed TF32 hi/lo image of the four weights, uploaded to the weights' device."""
    w1, w2, w3, w4 = (w.detach().to("cpu", torch.float32).contiguous() for w in weights)
    if w4.shape[0] % GATE_TILE:
        w4 = torch.cat([w4, w4.new_zeros(padded_gates(w4.shape[0]) - w4.shape[0], w4.shape[1])])
    features, gates = w1.shape[1], w4.shape[0]
    lib = _native.library()
    size = int(lib.ictc_radial_image_bytes(features, HIDDEN, gates))
    if size <= 0:
        raise ValueError(f"radial MLP shape not supported (F={features}, G={gates})")
    host = np.zeros(size, dtype=np.uint8)
    _native.call("ictc_radial_pack", ptr(w1), ptr(w2), ptr(w3), ptr(w4), features, HIDDEN, gates,
                 host.ctypes.data_as(ctypes.c_void_p), size)
    return torch.from_numpy(host).to(weights[0].device)


class RadialPlan:
    """Packed image for one set of weights, rebuilt when any weight changes (another
    tensor object, an in-place update, another device)."""

    def __init__(self):
        self.key = None
        self.refs = ()
        self.image = None
        self.status = None

    def get(self, weights):
        key = tuple((w.data_ptr(), w._version, str(w.device)) for w in weights)
        same = key == self.key and len(self.refs) == len(weights) and all(
            r() is w for r, w in zip(self.refs, weights))
        if not same:
            self.image = pack_image(weights)
            self.status = torch.zeros(1, dtype=torch.int32, device=weights[0].device)
            self.key = key
            self.refs = tuple(weakref.ref(w) for w in weights)
        return self.image, self.status


def _forward(image, status, feats, gates_width):
    edges, features = feats.shape
    out = torch.empty(edges, gates_width, device=feats.device, dtype=torch.float32)
    if edges:
        _native.call("ictc_radial_forward", ptr(image), ptr(feats), ptr(out), int(edges), int(features), HIDDEN,
                     int(gates_width), ptr(status), stream_of(feats))
    return out


def _backward(image, status, feats, grad_gates):
    edges, features = feats.shape
    grad_feats = torch.empty_like(feats)
    if edges:
        scratch = torch.empty(edges, HIDDEN, device=feats.device, dtype=torch.float32)
        _native.call("ictc_radial_backward", ptr(image), ptr(feats), ptr(grad_gates), ptr(scratch),
                     ptr(grad_feats), int(edges), int(features), HIDDEN, int(grad_gates.shape[1]), ptr(status),
                     stream_of(feats))
    return grad_feats


class _Radial(torch.autograd.Function):
    @staticmethod
    def forward(ctx, feats, image, status, w1, w2, w3, w4):
        ctx.save_for_backward(feats, image, status, w1, w2, w3, w4)
        gates = w4.shape[0]
        out = _forward(image, status, feats, padded_gates(gates))
        return out if out.shape[1] == gates else out[:, :gates].contiguous()

    @staticmethod
    def backward(ctx, grad):
        feats, image, status, w1, w2, w3, w4 = ctx.saved_tensors
        inputs = (feats, w1, w2, w3, w4)
        need = required_gradients(inputs, (ctx.needs_input_grad[0],) + tuple(ctx.needs_input_grad[3:7]))
        if not any(need):
            return (None,) * 7
        if torch.is_grad_enabled() or any(need[1:]):
            wanted = [t for t, n in zip(inputs, need) if n]
            with torch.enable_grad():
                out = mlp_reference(feats, (w1, w2, w3, w4))
                grads = list(torch.autograd.grad(out, wanted, grad, create_graph=torch.is_grad_enabled(),
                                                 allow_unused=True))
            result = [grads.pop(0) if n else None for n in need]
            return result[0], None, None, result[1], result[2], result[3], result[4]
        grad = grad.contiguous()
        if grad.shape[1] % GATE_TILE:
            grad = torch.nn.functional.pad(grad, (0, padded_gates(grad.shape[1]) - grad.shape[1]))
        return _backward(image, status, feats, grad), None, None, None, None, None, None


def radial_gates(linears, feats: torch.Tensor, plan: RadialPlan) -> torch.Tensor:
    """gates [E, G] of the radial network given its four bias-free linears [out, in]."""
    if feats.dtype != torch.float32 or feats.device.type != "cuda":
        raise ValueError("the CUDA radial MLP requires CUDA FP32 edge features")
    weights = [lin.weight for lin in linears]
    image, status = plan.get(weights)
    return _Radial.apply(feats.contiguous(), image, status, *weights)


def check_status(plan: RadialPlan):
    """Raise if a radial kernel recorded a timed-out wait (reads one int from the device)."""
    if plan.status is not None and int(plan.status.item()) != 0:
        raise RuntimeError(f"radial MLP kernel reported error {int(plan.status.item())}")
