"""Derived state the CUDA backend keeps on modules (plans with device handles, packed
weights, folded tables, weak references) is left out of pickles and deep copies, so
``copy.deepcopy(model)`` (e.g. an EMA copy) and ``torch.save(model)`` work after the
model has run, and the copy rebuilds its own state (CPU checks)."""
import copy
import ctypes
import io
import pickle
import weakref

import torch


class Holder:
    pass


def test_transient_slot():
    from ictc_o3.backends.cuda.cache import Transient, cache_of
    h = Holder()
    cache = cache_of(h, "_state")
    cache["handle"] = ctypes.c_void_p(1234)                      # not picklable by itself
    cache["ref"] = weakref.ref(h)
    assert cache_of(h, "_state") is cache
    for clone in (pickle.loads(pickle.dumps(h)), copy.deepcopy(h)):
        assert isinstance(clone.__dict__["_state"], Transient)
        assert cache_of(clone, "_state") == {}
    assert cache_of(h, "_state") is cache                        # the original keeps its state


def test_modules_with_filled_caches_copy_and_pickle(monkeypatch):
    from ictc_o3.backends.cuda import contraction as cc
    from ictc_o3.backends.cuda import radial
    from ictc_o3.backends.cuda.cache import cache_of
    from ictc_o3.ops.symmetric_contraction import ICTDBridgeUSymmetricContractionSO3

    class TorchFold(torch.autograd.Function):
        @staticmethod
        def forward(ctx, usyms, rows, *weights):
            return torch.cat([torch.matmul(u.unsqueeze(0).to(w.dtype), w) for u, w in zip(usyms, weights)], 1)

    monkeypatch.setattr(cc, "_Fold", TorchFold)
    module = ICTDBridgeUSymmetricContractionSO3(num_elements=2, channels=4, lmax=2, target_lmax=1)
    with torch.no_grad():
        table = cc.coefficient_table(module, torch.device("cpu"))      # fills the coupling and folded caches
    fc = torch.nn.Sequential(torch.nn.Linear(8, 64, bias=False), torch.nn.Linear(64, 64, bias=False),
                             torch.nn.Linear(64, 64, bias=False), torch.nn.Linear(64, 64, bias=False))
    plan = cache_of(fc, "_ictc_radial_plan")["plan"] = radial.RadialPlan()
    plan.get([m.weight for m in fc])                                  # packed image + weak references
    holder = torch.nn.ModuleDict({"sc": module, "fc": fc})
    for clone in (copy.deepcopy(holder), torch.load(_saved(holder), weights_only=False)):
        assert cache_of(clone["fc"], "_ictc_radial_plan") == {}
        assert cache_of(clone["sc"], "_cuda_folded_table") == {}
        with torch.no_grad():
            again = cc.coefficient_table(clone["sc"], torch.device("cpu"))
        torch.testing.assert_close(again, table, rtol=0, atol=0)
    with torch.no_grad():
        assert cc.coefficient_table(module, torch.device("cpu")) is table   # the original's cache is intact


def _saved(obj):
    buf = io.BytesIO()
    torch.save(obj, buf)
    buf.seek(0)
    return buf
