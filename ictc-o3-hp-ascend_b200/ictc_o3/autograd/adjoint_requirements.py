"""Prune adjoint outputs that the running autograd pass will not consume.

``ctx.needs_input_grad`` is fixed when the forward runs; a later
``autograd.grad`` call may target only some inputs (forces need the
coordinates, not the parameters).  This asks the engine whether the gradient
edge of each input will actually execute, as the reference does at
``ictc_o3/autograd/adjoint_requirements.py:12-26``.  Anything the engine cannot
answer (tracing, functorch transforms, missing private API) keeps every
declared gradient.
"""
import torch


def required_gradients(inputs, declared):
    probe = getattr(torch._C, "_will_engine_execute_node", None)
    if probe is None or torch.compiler.is_compiling() or torch._C._are_functorch_transforms_active():
        return tuple(bool(d) for d in declared)
    result = []
    for tensor, needed in zip(inputs, declared):
        if not needed or tensor is None:
            result.append(False)
            continue
        try:
            node = torch.autograd.graph.get_gradient_edge(tensor).node
            result.append(bool(probe(node)))
        except (RuntimeError, AttributeError, AssertionError):
            result.append(True)
    return tuple(result)
