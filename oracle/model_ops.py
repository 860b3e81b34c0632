"""CPU oracle versions of the model's hot operators -- TEST INFRASTRUCTURE ONLY.

Injected into ``mace_ictc.models.MACEICTC(ops=...)`` by tests so the same model
runs on the CPU restatements (FP64) and can be compared with the CUDA path.
"""
import torch

from oracle import sc_oracle, tp_oracle


class OracleOps:
    def __init__(self, dtype=torch.float64):
        self.dtype = dtype

    def harmonics(self, n, lmax):
        return torch.cat(tp_oracle.direction_harmonics(n, lmax, tp_oracle.harmonic_tables(max(lmax, 1)))[:lmax + 1], -1)

    def message(self, tp, features, harmonics, gates, src, dst, mask, dst_nodes):
        li = max(p[0] for p in tp.paths)
        out = tp_oracle.graph_message(tp, tp_oracle.split_mul_ir(features, tp.channels, li),
                                      tp_oracle.split_harm(harmonics, tp.lmax), gates.view(gates.shape[0], tp.num_paths, tp.channels),
                                      src, dst, mask, nodes=dst_nodes, dtype=self.dtype)
        return tp_oracle.pack_out(tp, out)

    def contraction(self, module, features, species):
        feats = sc_oracle.flat_to_mace(features, module.channels, module.lmax)
        outs = []
        for t, c in enumerate(module.contractions):
            u = {nu: c.U_tensors(nu).to(self.dtype) for nu in range(1, module.correlation + 1)}
            outs.append(sc_oracle.contraction(u, c.weights_max.to(self.dtype), [w.to(self.dtype) for w in c.weights],
                                              feats, species, t))
        return torch.cat(outs, -1)
